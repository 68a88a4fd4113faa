// Internal helpers shared by the host-side translation units of
// libsharpinfer_cuda: error reporting, type geometry, argument checks.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/sharpinfer_cuda.h"

namespace si {

// Thread-local last-error message; every failing entry point sets it.
si_status fail(si_status status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

constexpr int kQ8_0Block = 32;
constexpr int kQ8_0Bytes = 34;
constexpr int kQ4KBlock = 256;
constexpr int kQ4KBytes = 144;

inline bool known_type(uint32_t t) {
    return t == SI_TYPE_F32 || t == SI_TYPE_F16 || t == SI_TYPE_Q8_0 || t == SI_TYPE_Q4_K;
}

inline const char *type_name(uint32_t t) {
    switch (t) {
    case SI_TYPE_F32: return "F32";
    case SI_TYPE_F16: return "F16";
    case SI_TYPE_Q8_0: return "Q8_0";
    case SI_TYPE_Q4_K: return "Q4_K";
    default: return "unknown";
    }
}

// Bytes of `elements` elements; returns SI_ERR_INVALID_DATA when a block
// type's count is not a multiple of its block, SI_ERR_UNSUPPORTED for an
// unknown type (GgufModelFile.cs:301-331 throws the same way).
si_status byte_length(uint32_t type, uint64_t elements, uint64_t *bytes);

// IEEE binary16 <-> binary32 (round to nearest even).
float half_to_float(uint16_t h);
uint16_t float_to_half(float f);

}  // namespace si

// Launch wrappers implemented in the .cu files (host side of each kernel).
namespace si::kernels {
si_status matvec_dense(uint32_t wtype, const void *w, uint32_t xtype, const void *x,
                       uint32_t ytype, void *y, int64_t rows, int64_t cols, void *stream);
si_status matvec_quant(uint32_t wtype, const void *w, const float *x, float *y,
                       int64_t rows, int64_t cols, void *stream);
si_status shared_weight_matvec(uint32_t wtype, const void *w, const float *x, const int32_t *control,
                               float *y, int64_t m, int64_t n, int64_t k, void *stream);
si_status batch_shared_matvec(uint32_t wtype, const void *w, const float *in,
                              const int32_t *control, float *out, int64_t batch,
                              int64_t out_features, int64_t in_features, void *stream);
si_status gemm_workspace_bytes(uint32_t wtype, int64_t m, int64_t n, int64_t k, uint64_t *bytes);
si_status gemm_tn(uint32_t wtype, const float *x, const void *w, float *y, int64_t m, int64_t n,
                  int64_t k, void *workspace, uint64_t workspace_bytes, void *stream);
si_status take_error_gemv(int device, uint32_t *code);
si_status take_error_gemm(int device, uint32_t *code);
si_status take_error_gemv_mma(int device, uint32_t *code);
// Row-sharded output exchange of a fused GEMV (see si_rowshard_matvec_peer).
constexpr int kMaxPeerRanks = 8;
struct PeerGather {
    float *ys[kMaxPeerRanks];         // every rank's output vector, as mapped in this process
    uint32_t *flags[kMaxPeerRanks];   // every rank's flag array [nranks]
    uint32_t *ticket;                 // this rank's CTA ticket counter
    uint32_t *epoch;                  // this rank's call counter
    int nranks;                       // 0: not a sharded call
    int rank;
    int64_t row_base;                 // global index of this rank's first row
};
// control/token: batch-shared use, y is written only when token < control[1].
si_status matvec_quant_mma(uint32_t wtype, const void *w, const float *x, float *y, int64_t rows, int64_t cols,
                           void *stream, const PeerGather *peer = nullptr, const int32_t *control = nullptr,
                           int token = 0);
// Q4_K batch on the tensor cores, eight input rows per launch; SI_ERR_UNSUPPORTED
// when the shape or alignment needs another kernel (nothing launched then).
si_status matvec_q4k_batched(const void *w, const float *x, float *y, int64_t m, int64_t rows, int64_t cols,
                             void *stream, const int32_t *control);
}  // namespace si::kernels
