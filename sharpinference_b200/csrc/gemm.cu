// core.matrix-multiply (transpose_right) dispatch: Y[m,n] = X[m,k] W[n,k]^T.
#include <cuda_runtime.h>

#include "si_internal.h"

namespace si::kernels {

si_status gemm_workspace_bytes(uint32_t wtype, int64_t m, int64_t n, int64_t k, uint64_t *bytes) {
    (void)wtype, (void)m, (void)n, (void)k;
    *bytes = 0;
    return SI_OK;
}

si_status gemm_tn(uint32_t wtype, const float *x, const void *w, float *y, int64_t m, int64_t n, int64_t k,
                  void *workspace, uint64_t workspace_bytes, void *stream) {
    (void)workspace, (void)workspace_bytes;
    return shared_weight_matvec(wtype, w, x, nullptr, y, m, n, k, stream);
}

}  // namespace si::kernels
