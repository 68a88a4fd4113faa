// GGUF v3 model file reader (GgufModelFile.Open, GgufModelFile.cs:57-160):
// the file is memory-mapped read-only; the header, the typed metadata and
// the tensor descriptors are parsed with the reference's checks (magic and
// version, counts within int range, non-empty unique keys and tensor names,
// rank 1..8 with no empty dimension, no nested metadata arrays, a legacy
// 32-bit array count accepted, power-of-two general.alignment defaulting to
// 32, every tensor inside the file). Tensor bytes are exposed as pointers
// into the mapping, to be uploaded to the device unchanged.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "si_internal.h"

using si::fail;

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"
constexpr uint32_t kVersion = 3;

enum MetaType : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};

struct MetaValue {
    uint32_t type = 0;
    uint32_t elem_type = 0;   // arrays
    uint64_t count = 0;       // arrays
    double number = 0.0;      // numeric scalars and Bool
    uint64_t bits = 0;        // integer scalars exactly
    std::string text;         // String
    uint64_t data_offset = 0; // arrays: file offset of the first element
};

struct Tensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;
    uint64_t offset = 0;  // absolute file offset
    uint64_t bytes = 0;
};

struct Reader {
    const uint8_t *p;
    uint64_t size;
    uint64_t pos = 0;
    bool ok = true;
    bool need(uint64_t n) {
        if (!ok || n > size - pos) ok = false;
        return ok;
    }
    template <class T>
    T read() {
        T v{};
        if (need(sizeof(T))) {
            std::memcpy(&v, p + pos, sizeof(T));
            pos += sizeof(T);
        }
        return v;
    }
};

}  // namespace

struct si_gguf {
    void *map = nullptr;
    uint64_t size = 0;
    uint32_t alignment = 32;
    uint64_t data_start = 0;
    std::vector<std::string> keys;
    std::unordered_map<std::string, MetaValue> meta;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
};

namespace {

si_status bad(const char *what) { return fail(SI_ERR_INVALID_DATA, "%s", what); }

si_status read_count(Reader &r, const char *kind, uint64_t *out) {
    const uint64_t v = r.read<uint64_t>();
    if (!r.ok) return bad("GGUF file is truncated.");
    if (v > 0x7fffffffull) return fail(SI_ERR_INVALID_DATA, "GGUF %s count %llu is too large.", kind, (unsigned long long)v);
    *out = v;
    return SI_OK;
}

si_status read_string(Reader &r, std::string *out) {
    uint64_t n = 0;
    if (si_status st = read_count(r, "string byte", &n)) return st;
    if (!r.need(n)) return bad("GGUF string is truncated.");
    out->assign(reinterpret_cast<const char *>(r.p + r.pos), size_t(n));
    r.pos += n;
    return SI_OK;
}

uint64_t scalar_size(uint32_t t) {
    switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
    }
}

si_status read_scalar(Reader &r, uint32_t t, MetaValue *v) {
    switch (t) {
    case kU8: v->bits = r.read<uint8_t>(), v->number = double(v->bits); break;
    case kI8: { const int8_t x = r.read<int8_t>(); v->bits = uint64_t(int64_t(x)), v->number = x; break; }
    case kU16: v->bits = r.read<uint16_t>(), v->number = double(v->bits); break;
    case kI16: { const int16_t x = r.read<int16_t>(); v->bits = uint64_t(int64_t(x)), v->number = x; break; }
    case kU32: v->bits = r.read<uint32_t>(), v->number = double(v->bits); break;
    case kI32: { const int32_t x = r.read<int32_t>(); v->bits = uint64_t(int64_t(x)), v->number = x; break; }
    case kF32: v->number = r.read<float>(); break;
    case kU64: v->bits = r.read<uint64_t>(), v->number = double(v->bits); break;
    case kI64: { const int64_t x = r.read<int64_t>(); v->bits = uint64_t(x), v->number = double(x); break; }
    case kF64: v->number = r.read<double>(); break;
    case kBool: {
        const uint8_t b = r.read<uint8_t>();
        if (r.ok && b > 1) return fail(SI_ERR_INVALID_DATA, "Invalid GGUF Boolean value %u.", b);
        v->bits = b, v->number = b;
        break;
    }
    case kString: return read_string(r, &v->text);
    default: return fail(SI_ERR_INVALID_DATA, "Unsupported GGUF metadata type %u.", t);
    }
    return r.ok ? SI_OK : bad("GGUF file is truncated.");
}

si_status read_value(Reader &r, MetaValue *v) {
    v->type = r.read<uint32_t>();
    if (!r.ok) return bad("GGUF file is truncated.");
    if (v->type != kArray) return read_scalar(r, v->type, v);
    v->elem_type = r.read<uint32_t>();
    if (!r.ok) return bad("GGUF file is truncated.");
    if (v->elem_type == kArray) return bad("Nested GGUF metadata arrays are unsupported.");
    uint64_t count = r.read<uint64_t>();
    if (!r.ok) return bad("GGUF file is truncated.");
    if (count > 0x7fffffffull) {
        // Some older converters emitted a 32-bit array count.
        const uint32_t legacy = uint32_t(count);
        if (legacy > 0x7fffffffu)
            return fail(SI_ERR_INVALID_DATA, "GGUF array count %llu is too large.", (unsigned long long)count);
        r.pos -= 4;
        count = legacy;
    }
    v->count = count;
    v->data_offset = r.pos;
    if (v->elem_type == kString) {
        for (uint64_t i = 0; i < count; ++i) {
            std::string s;
            if (si_status st = read_string(r, &s)) return st;
        }
        return SI_OK;
    }
    const uint64_t es = scalar_size(v->elem_type);
    if (!es) return fail(SI_ERR_INVALID_DATA, "Unsupported GGUF array type %u.", v->elem_type);
    if (v->elem_type == kBool) {
        for (uint64_t i = 0; i < count; ++i) {
            const uint8_t b = r.read<uint8_t>();
            if (r.ok && b > 1) return fail(SI_ERR_INVALID_DATA, "Invalid GGUF Boolean value %u.", b);
        }
        return r.ok ? SI_OK : bad("GGUF file is truncated.");
    }
    if (count > (r.size - r.pos) / es) return bad("GGUF array is truncated.");
    r.pos += count * es;
    return SI_OK;
}

si_status parse(si_gguf *g) {
    Reader r{static_cast<const uint8_t *>(g->map), g->size};
    if (r.read<uint32_t>() != kMagic || r.read<uint32_t>() != kVersion || !r.ok)
        return bad("Expected a GGUF v3 model file.");
    uint64_t tensor_count = 0, meta_count = 0;
    if (si_status st = read_count(r, "tensor", &tensor_count)) return st;
    if (si_status st = read_count(r, "metadata", &meta_count)) return st;
    for (uint64_t i = 0; i < meta_count; ++i) {
        std::string key;
        if (si_status st = read_string(r, &key)) return st;
        MetaValue v;
        if (read_value(r, &v) != SI_OK) {
            const std::string msg = si::last_error();
            return fail(SI_ERR_INVALID_DATA, "Invalid GGUF metadata '%s'. (%s)", key.c_str(), msg.c_str());
        }
        bool blank = true;
        for (char c : key) blank = blank && (c == ' ' || c == '\t' || c == '\n' || c == '\r');
        if (blank || g->meta.count(key))
            return fail(SI_ERR_INVALID_DATA, "Empty or duplicate GGUF metadata key '%s'.", key.c_str());
        g->keys.push_back(key);
        g->meta.emplace(key, std::move(v));
    }
    std::vector<Tensor> descs(tensor_count);
    for (uint64_t i = 0; i < tensor_count; ++i) {
        Tensor &t = descs[i];
        if (si_status st = read_string(r, &t.name)) return st;
        bool blank = true;
        for (char c : t.name) blank = blank && (c == ' ' || c == '\t' || c == '\n' || c == '\r');
        if (blank || g->by_name.count(t.name))
            return fail(SI_ERR_INVALID_DATA, "Empty or duplicate GGUF tensor name '%s'.", t.name.c_str());
        g->by_name.emplace(t.name, i);
        const uint32_t rank = r.read<uint32_t>();
        if (!r.ok) return bad("GGUF file is truncated.");
        if (rank < 1 || rank > 8)
            return fail(SI_ERR_INVALID_DATA, "Tensor '%s' has unsupported rank %u.", t.name.c_str(), rank);
        t.dims.resize(rank);
        for (uint32_t d = 0; d < rank; ++d) {
            t.dims[d] = r.read<uint64_t>();
            if (r.ok && t.dims[d] == 0)
                return fail(SI_ERR_INVALID_DATA, "Tensor '%s' has an empty dimension.", t.name.c_str());
        }
        t.type = r.read<uint32_t>();
        t.offset = r.read<uint64_t>();
        if (!r.ok) return bad("GGUF file is truncated.");
    }
    if (auto it = g->meta.find("general.alignment"); it != g->meta.end()) {
        const MetaValue &a = it->second;
        if (a.type == kString || a.type == kArray || a.type == kF32 || a.type == kF64 || a.bits > 0xffffffffull)
            return bad("Invalid GGUF alignment.");
        g->alignment = uint32_t(a.bits);
    }
    if (g->alignment == 0 || (g->alignment & (g->alignment - 1)))
        return fail(SI_ERR_INVALID_DATA, "Invalid GGUF alignment %u.", g->alignment);
    g->data_start = (r.pos + g->alignment - 1) & ~uint64_t(g->alignment - 1);
    for (Tensor &t : descs) {
        uint64_t elements = 1;
        for (uint64_t d : t.dims) {
            if (elements > UINT64_MAX / d) return bad("Tensor element count overflows.");
            elements *= d;
        }
        if (si_status st = si::byte_length(t.type, elements, &t.bytes)) return st;
        if (t.offset > UINT64_MAX - g->data_start) return bad("Tensor offset overflows.");
        const uint64_t abs = g->data_start + t.offset;
        if (abs > g->size || t.bytes > g->size - abs)
            return fail(SI_ERR_INVALID_DATA, "Tensor '%s' exceeds the GGUF file.", t.name.c_str());
        t.offset = abs;
    }
    g->tensors = std::move(descs);
    return SI_OK;
}

void close_map(si_gguf *g) {
    if (g->map && g->map != MAP_FAILED) munmap(g->map, g->size);
    g->map = nullptr;
}

const MetaValue *find_meta(si_gguf *g, const char *key) {
    if (!g || !key) return nullptr;
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

si_status copy_text(const std::string &s, char *buf, size_t cap, size_t *len) {
    if (len) *len = s.size();
    if (buf && cap) {
        const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return SI_OK;
}

}  // namespace

extern "C" {

si_status si_gguf_open(const char *path, si_gguf **out) {
    if (!path || !out || !*path) return fail(SI_ERR_INVALID_ARGUMENT, "a file path is required");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return fail(SI_ERR_INVALID_ARGUMENT, "cannot open '%s': %s", path, std::strerror(errno));
    struct stat stt {};
    if (fstat(fd, &stt) != 0 || stt.st_size <= 0) {
        ::close(fd);
        return fail(SI_ERR_INVALID_DATA, "Expected a GGUF v3 model file.");
    }
    auto *g = new si_gguf();
    g->size = uint64_t(stt.st_size);
    g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (g->map == MAP_FAILED) {
        g->map = nullptr;
        delete g;
        return fail(SI_ERR_INVALID_ARGUMENT, "cannot map '%s'", path);
    }
    if (si_status st = parse(g)) {
        close_map(g);
        delete g;
        return st;
    }
    *out = g;
    return SI_OK;
}

si_status si_gguf_close(si_gguf *g) {
    if (!g) return SI_OK;
    close_map(g);
    delete g;
    return SI_OK;
}

si_status si_gguf_tensor_count(si_gguf *g, int64_t *count) {
    if (!g || !count) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *count = int64_t(g->tensors.size());
    return SI_OK;
}

si_status si_gguf_find_tensor(si_gguf *g, const char *name, int64_t *index) {
    if (!g || !name || !index) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    auto it = g->by_name.find(name);
    if (it == g->by_name.end()) return fail(SI_ERR_INVALID_DATA, "GGUF tensor '%s' is missing.", name);
    *index = int64_t(it->second);
    return SI_OK;
}

si_status si_gguf_tensor_info(si_gguf *g, int64_t index, char *name, size_t name_capacity, uint32_t *type,
                              int32_t *rank, uint64_t *dims, uint64_t *bytes, const void **data) {
    if (!g) return fail(SI_ERR_INVALID_ARGUMENT, "null file");
    if (index < 0 || uint64_t(index) >= g->tensors.size())
        return fail(SI_ERR_INVALID_ARGUMENT, "tensor index %lld out of range", (long long)index);
    const Tensor &t = g->tensors[size_t(index)];
    copy_text(t.name, name, name_capacity, nullptr);
    if (type) *type = t.type;
    if (rank) *rank = int32_t(t.dims.size());
    if (dims)
        for (size_t d = 0; d < 8; ++d) dims[d] = d < t.dims.size() ? t.dims[d] : 0;
    if (bytes) *bytes = t.bytes;
    if (data) *data = static_cast<const uint8_t *>(g->map) + t.offset;
    return SI_OK;
}

si_status si_gguf_metadata_count(si_gguf *g, int64_t *count) {
    if (!g || !count) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    *count = int64_t(g->keys.size());
    return SI_OK;
}

si_status si_gguf_metadata_key(si_gguf *g, int64_t index, char *key, size_t capacity, uint32_t *type,
                               uint32_t *element_type, uint64_t *count) {
    if (!g) return fail(SI_ERR_INVALID_ARGUMENT, "null file");
    if (index < 0 || uint64_t(index) >= g->keys.size())
        return fail(SI_ERR_INVALID_ARGUMENT, "metadata index %lld out of range", (long long)index);
    const std::string &k = g->keys[size_t(index)];
    const MetaValue &v = g->meta[k];
    copy_text(k, key, capacity, nullptr);
    if (type) *type = v.type;
    if (element_type) *element_type = v.type == kArray ? v.elem_type : 0;
    if (count) *count = v.type == kArray ? v.count : 1;
    return SI_OK;
}

si_status si_gguf_metadata_number(si_gguf *g, const char *key, double *value) {
    if (!value) return fail(SI_ERR_INVALID_ARGUMENT, "null argument");
    const MetaValue *v = find_meta(g, key);
    if (!v) return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is missing.", key ? key : "");
    if (v->type == kString || v->type == kArray)
        return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is not a number.", key);
    *value = v->number;
    return SI_OK;
}

si_status si_gguf_metadata_string(si_gguf *g, const char *key, char *buffer, size_t capacity, size_t *length) {
    const MetaValue *v = find_meta(g, key);
    if (!v) return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is missing.", key ? key : "");
    if (v->type != kString) return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is not a String.", key);
    return copy_text(v->text, buffer, capacity, length);
}

si_status si_gguf_metadata_array(si_gguf *g, const char *key, uint32_t *element_type, uint64_t *count,
                                 const void **data) {
    const MetaValue *v = find_meta(g, key);
    if (!v) return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is missing.", key ? key : "");
    if (v->type != kArray) return fail(SI_ERR_INVALID_DATA, "GGUF metadata '%s' is not an Array.", key);
    if (element_type) *element_type = v->elem_type;
    if (count) *count = v->count;
    if (data) *data = static_cast<const uint8_t *>(g->map) + v->data_offset;
    return SI_OK;
}

}  // extern "C"
