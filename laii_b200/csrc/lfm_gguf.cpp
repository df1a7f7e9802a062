/*
 * GGUF binding of lfm2moe checkpoints: the FFN tensors of each block of a
 * GGUF v2/v3 file, uploaded through the library's own upload calls.
 *
 * Behaviour follows the reference's loader and MoE binding:
 *  - header, key/value section and tensor infos as in lfm2_load_gguf_from_fd
 *    (tools/lfm2_loader.c): tensor data starts at the tensor-info end rounded
 *    up to general.alignment (default 32);
 *  - hyperparameters by key suffix (tools/lfm2_loader.c:359-366):
 *    ".expert_used_count" (top-K, default 4), ".expert_count",
 *    ".attention.layer_norm_rms_epsilon" (default 1e-5), ".block_count";
 *  - a block is an lfm2moe layer when blk.l.ffn_gate_exps.weight exists,
 *    else a dense SwiGLU layer (lfm2_bind_moe_layer,
 *    tools/lfm2_moe_checkpoint.c:70-102): ffn_{gate,up,down}_exps,
 *    ffn_gate_inp, exp_probs_b.bias or bare exp_probs_b, E from the experts'
 *    third dimension, norm_topk_prob true, routed_scale 1; dense layers take
 *    ffn_{gate,up,down}.weight; both take ffn_norm.weight.
 * The file is mapped read-only; the upload calls copy the tensors into HBM.
 * Host code only: describing a checkpoint needs no GPU.
 */
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <vector>

#include "lfm_gpu_moe.h"

#define LFM_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u; /* "GGUF" little-endian */
constexpr uint32_t kTypeF32 = 0, kTypeQ4K = 12, kTypeQ6K = 14;
constexpr uint64_t kQ4kBytes = 144, kQ6kBytes = 210;

enum ValueType : uint32_t {
    V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64
};

struct Cursor {
    const uint8_t *p, *end;
    bool ok = true;
    bool take(void *dst, size_t n) {
        if (!ok || (size_t)(end - p) < n) return ok = false;
        memcpy(dst, p, n);
        p += n;
        return true;
    }
    bool skip(uint64_t n) {
        if (!ok || (uint64_t)(end - p) < n) return ok = false;
        p += n;
        return true;
    }
    template <class T> T get() {
        T v{};
        take(&v, sizeof v);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char *>(p), (size_t)n);
        p += n;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
    case V_U8: case V_I8: case V_BOOL: return 1;
    case V_U16: case V_I16: return 2;
    case V_U32: case V_I32: case V_F32: return 4;
    case V_U64: case V_I64: case V_F64: return 8;
    default: return 0;
    }
}

/* An unsigned integer value of any integer type, else false. */
bool read_uint(Cursor &c, uint32_t t, uint64_t *out) {
    switch (t) {
    case V_U8: *out = c.get<uint8_t>(); return c.ok;
    case V_I8: { const int8_t v = c.get<int8_t>(); *out = v < 0 ? 0 : (uint64_t)v; return c.ok; }
    case V_U16: *out = c.get<uint16_t>(); return c.ok;
    case V_I16: { const int16_t v = c.get<int16_t>(); *out = v < 0 ? 0 : (uint64_t)v; return c.ok; }
    case V_U32: *out = c.get<uint32_t>(); return c.ok;
    case V_I32: { const int32_t v = c.get<int32_t>(); *out = v < 0 ? 0 : (uint64_t)v; return c.ok; }
    case V_U64: *out = c.get<uint64_t>(); return c.ok;
    case V_I64: { const int64_t v = c.get<int64_t>(); *out = v < 0 ? 0 : (uint64_t)v; return c.ok; }
    default: return false;
    }
}

bool skip_value(Cursor &c, uint32_t t, int depth = 0) {
    if (t == V_STR) { c.str(); return c.ok; }
    if (t == V_ARR) {
        if (depth > 4) return false;
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (!c.ok) return false;
        const size_t es = scalar_size(et);
        if (es) return c.skip(n * es);
        for (uint64_t i = 0; i < n && c.ok; ++i) skip_value(c, et, depth + 1);
        return c.ok;
    }
    const size_t es = scalar_size(t);
    return es ? c.skip(es) : false;
}

bool ends_with(const std::string &s, const char *suffix) {
    const size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

struct TensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;
    uint64_t offset = 0;
    const uint8_t *data = nullptr;
    uint64_t bytes = 0;
};

struct GgufFile {
    int fd = -1;
    void *map = nullptr;
    size_t size = 0;
    uint32_t alignment = 32;
    uint64_t expert_used = 0, expert_count = 0, block_count = 0;
    float eps = 1e-5f;
    std::vector<TensorInfo> tensors;
    char err[256] = {0};

    ~GgufFile() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
    const TensorInfo *find(const std::string &name) const {
        for (const TensorInfo &t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
    const TensorInfo *block(uint32_t l, const char *suffix) const {
        return find("blk." + std::to_string(l) + "." + suffix);
    }
};

/* Byte size of a tensor from its dims.  Dims come from the file, so every one
 * must be in [1, 2^32) and the products must not wrap: a wrapped size would pass
 * the end-of-file check below while the shapes cast to uint32 describe far more
 * bytes than the mapping holds. */
bool tensor_bytes(TensorInfo &t) {
    uint64_t n = 1;
    for (uint32_t i = 0; i < t.n_dims; ++i) {
        if (t.ne[i] == 0 || t.ne[i] > 0xFFFFFFFFull) return false;
        if (__builtin_mul_overflow(n, t.ne[i], &n)) return false;
    }
    if (t.type == kTypeF32) return !__builtin_mul_overflow(n, (uint64_t)4, &t.bytes);
    if (t.type == kTypeQ4K || t.type == kTypeQ6K) {
        if (t.ne[0] % 256) return false;
        return !__builtin_mul_overflow(n / 256, (uint64_t)(t.type == kTypeQ4K ? kQ4kBytes : kQ6kBytes), &t.bytes);
    }
    t.bytes = 0; /* another type: described, never uploaded */
    return true;
}

bool open_gguf(const char *path, GgufFile &f) {
    f.fd = open(path, O_RDONLY);
    if (f.fd < 0) { snprintf(f.err, sizeof f.err, "cannot open %s", path); return false; }
    struct stat st;
    if (fstat(f.fd, &st) != 0 || st.st_size < 24) { snprintf(f.err, sizeof f.err, "%s: not a GGUF file", path); return false; }
    f.size = (size_t)st.st_size;
    f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
    if (f.map == MAP_FAILED) { f.map = nullptr; snprintf(f.err, sizeof f.err, "cannot map %s", path); return false; }
    const uint8_t *base = static_cast<const uint8_t *>(f.map);
    Cursor c{base, base + f.size};
    const uint32_t magic = c.get<uint32_t>(), version = c.get<uint32_t>();
    if (magic != kGgufMagic || (version != 2 && version != 3)) {
        snprintf(f.err, sizeof f.err, "%s: not a GGUF v2/v3 file", path);
        return false;
    }
    const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) { snprintf(f.err, sizeof f.err, "%s: bad header", path); return false; }
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        const std::string key = c.str();
        const uint32_t t = c.get<uint32_t>();
        if (!c.ok) break;
        uint64_t u = 0;
        if (key == "general.alignment" && read_uint(c, t, &u)) { f.alignment = (uint32_t)u; continue; }
        if (ends_with(key, ".expert_used_count") && read_uint(c, t, &u)) { f.expert_used = u; continue; }
        if (ends_with(key, ".expert_count") && read_uint(c, t, &u)) { f.expert_count = u; continue; }
        if (ends_with(key, ".block_count") && read_uint(c, t, &u)) { f.block_count = u; continue; }
        if (ends_with(key, ".attention.layer_norm_rms_epsilon") && t == V_F32) { f.eps = c.get<float>(); continue; }
        if (!skip_value(c, t)) c.ok = false;
    }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        TensorInfo ti;
        ti.name = c.str();
        ti.n_dims = c.get<uint32_t>();
        if (ti.n_dims == 0 || ti.n_dims > 4) { c.ok = false; break; }
        for (uint32_t d = 0; d < ti.n_dims; ++d) ti.ne[d] = c.get<uint64_t>();
        ti.type = c.get<uint32_t>();
        ti.offset = c.get<uint64_t>();
        if (!c.ok) break;
        if (!tensor_bytes(ti)) { snprintf(f.err, sizeof f.err, "tensor %s: bad shape", ti.name.c_str()); return false; }
        f.tensors.push_back(ti);
    }
    if (!c.ok) { snprintf(f.err, sizeof f.err, "%s: truncated key/value or tensor-info section", path); return false; }
    if (f.alignment == 0 || (f.alignment & (f.alignment - 1))) f.alignment = 32;
    const uint64_t head = (uint64_t)(c.p - base);
    const uint64_t data0 = (head + f.alignment - 1) / f.alignment * f.alignment;
    for (TensorInfo &t : f.tensors) {
        if (data0 > f.size || t.offset > f.size - data0 || t.bytes > f.size - data0 - t.offset) {
            snprintf(f.err, sizeof f.err, "tensor %s: data past the end of the file", t.name.c_str());
            return false;
        }
        t.data = base + data0 + t.offset;
    }
    if (!f.block_count)
        for (const TensorInfo &t : f.tensors) {
            unsigned l = 0;
            if (sscanf(t.name.c_str(), "blk.%u.", &l) == 1 && l + 1 > f.block_count) f.block_count = l + 1;
        }
    return true;
}

bool is(const TensorInfo *t, uint32_t type, uint32_t n_dims, uint64_t ne0, uint64_t ne1 = 1, uint64_t ne2 = 1) {
    return t && t->type == type && t->n_dims == n_dims && t->ne[0] == ne0 && t->ne[1] == ne1 && t->ne[2] == ne2;
}

/* The FFN of block l: kind 0 (none), 1 (dense SwiGLU), 2 (lfm2moe), or -1 with
 * f.err set when tensors are missing, mistyped or misshaped. */
struct BlockFfn {
    int kind = 0;
    uint32_t D = 0, E = 0, K = 0, I = 0;
    const TensorInfo *norm = nullptr, *router = nullptr, *bias = nullptr, *gate = nullptr, *up = nullptr,
                     *down = nullptr;
};

BlockFfn bind_block(GgufFile &f, uint32_t l) {
    BlockFfn b;
    b.norm = f.block(l, "ffn_norm.weight");
    b.gate = f.block(l, "ffn_gate_exps.weight");
    if (b.gate) {
        b.up = f.block(l, "ffn_up_exps.weight");
        b.down = f.block(l, "ffn_down_exps.weight");
        b.router = f.block(l, "ffn_gate_inp.weight");
        b.bias = f.block(l, "exp_probs_b.bias");
        if (!b.bias) b.bias = f.block(l, "exp_probs_b");
        if (!b.up || !b.down || !b.router) {
            snprintf(f.err, sizeof f.err, "block %u has incomplete MoE expert tensors", l);
            b.kind = -1;
            return b;
        }
        b.D = (uint32_t)b.gate->ne[0];
        b.I = (uint32_t)b.gate->ne[1];
        b.E = b.gate->n_dims >= 3 ? (uint32_t)b.gate->ne[2] : (uint32_t)f.expert_count;
        b.K = f.expert_used ? (uint32_t)f.expert_used : 4u;
        /* Q4_K_M files store some ffn_down_exps as Q6_K */
        if (!is(b.gate, kTypeQ4K, 3, b.D, b.I, b.E) || !is(b.up, kTypeQ4K, 3, b.D, b.I, b.E) ||
            !(is(b.down, kTypeQ4K, 3, b.I, b.D, b.E) || is(b.down, kTypeQ6K, 3, b.I, b.D, b.E)) ||
            !is(b.router, kTypeF32, 2, b.D, b.E) ||
            (b.bias && !is(b.bias, kTypeF32, 1, b.E)) || (b.norm && !is(b.norm, kTypeF32, 1, b.D))) {
            snprintf(f.err, sizeof f.err,
                     "block %u: MoE tensors must be Q4_K experts [D,I,E]/[I,D,E] (down Q4_K or Q6_K) with F32 router [D,E], bias [E], norm [D]", l);
            b.kind = -1;
            return b;
        }
        b.kind = 2;
        return b;
    }
    b.gate = f.block(l, "ffn_gate.weight");
    b.up = f.block(l, "ffn_up.weight");
    b.down = f.block(l, "ffn_down.weight");
    if (!b.gate && !b.up && !b.down) return b;
    if (!b.gate || !b.up || !b.down) {
        snprintf(f.err, sizeof f.err, "block %u has an incomplete dense FFN", l);
        b.kind = -1;
        return b;
    }
    b.D = (uint32_t)b.gate->ne[0];
    b.I = (uint32_t)b.gate->ne[1];
    b.E = 1;
    b.K = 1;
    if (!is(b.gate, kTypeQ4K, 2, b.D, b.I) || !is(b.up, kTypeQ4K, 2, b.D, b.I) || !is(b.down, kTypeQ4K, 2, b.I, b.D) ||
        (b.norm && !is(b.norm, kTypeF32, 1, b.D))) {
        snprintf(f.err, sizeof f.err, "block %u: dense FFN tensors must be Q4_K [D,I]/[I,D] with an F32 norm [D]", l);
        b.kind = -1;
        return b;
    }
    b.kind = 1;
    return b;
}

const void *ptr(const TensorInfo *t) { return t ? t->data : nullptr; }

thread_local char g_describe_err[256]; /* per calling thread */

}  // namespace

LFM_API lfm_gpu_status_t lfm_gpu_moe_gguf_describe(const char *path, uint32_t block, lfm_gpu_moe_gguf_block_t *out,
                                                   uint32_t *n_blocks) {
    if (!path || !out) return LFM_GPU_ERR_INVALID_ARG;
    memset(out, 0, sizeof *out);
    GgufFile f;
    if (!open_gguf(path, f)) {
        snprintf(g_describe_err, sizeof g_describe_err, "%s", f.err);
        return LFM_GPU_ERR_INVALID_ARG;
    }
    if (n_blocks) *n_blocks = (uint32_t)f.block_count;
    const BlockFfn b = bind_block(f, block);
    if (b.kind < 0) {
        snprintf(g_describe_err, sizeof g_describe_err, "%s", f.err);
        return LFM_GPU_ERR_UNSUPPORTED;
    }
    out->kind = (uint32_t)b.kind;
    out->D = b.D;
    out->E = b.E;
    out->K = b.K;
    out->I = b.I;
    out->eps = f.eps;
    out->has_bias = b.bias ? 1 : 0;
    out->has_norm = b.norm ? 1 : 0;
    out->down_type = b.kind > 0 ? b.down->type : 0;
    return LFM_GPU_OK;
}

LFM_API const char *lfm_gpu_moe_gguf_last_error(void) { return g_describe_err; }

LFM_API lfm_gpu_status_t lfm_gpu_moe_upload_gguf(lfm_gpu_moe_t *h, const char *path, uint32_t first_block,
                                                 uint32_t n_blocks, uint32_t expert_first, uint32_t n_local,
                                                 uint32_t *n_uploaded) {
    if (!h || !path) return LFM_GPU_ERR_INVALID_ARG;
    if (n_uploaded) *n_uploaded = 0;
    GgufFile f;
    if (!open_gguf(path, f)) {
        snprintf(g_describe_err, sizeof g_describe_err, "%s", f.err);
        return LFM_GPU_ERR_INVALID_ARG;
    }
    if (n_blocks == 0 || first_block + n_blocks > f.block_count) n_blocks = f.block_count > first_block ? (uint32_t)f.block_count - first_block : 0;
    if (n_blocks > LFM_GPU_MOE_MAX_LAYERS) {
        snprintf(g_describe_err, sizeof g_describe_err, "%u blocks above the handle's %d layer slots", n_blocks,
                 LFM_GPU_MOE_MAX_LAYERS);
        return LFM_GPU_ERR_UNSUPPORTED;
    }
    uint32_t done = 0;
    for (uint32_t i = 0; i < n_blocks; ++i) {
        const uint32_t l = first_block + i;
        const BlockFfn b = bind_block(f, l);
        if (b.kind < 0) {
            snprintf(g_describe_err, sizeof g_describe_err, "%s", f.err);
            return LFM_GPU_ERR_UNSUPPORTED;
        }
        if (b.kind == 0) continue;
        lfm_gpu_status_t st;
        if (b.kind == 1) {
            st = lfm_gpu_moe_upload_dense(h, i, b.D, b.I, f.eps, static_cast<const float *>(ptr(b.norm)), ptr(b.gate),
                                          ptr(b.up), ptr(b.down), kTypeQ4K);
        } else if (n_local == 0) {
            st = lfm_gpu_moe_upload_layer_typed(h, i, b.D, b.E, b.K, b.I, f.eps, static_cast<const float *>(ptr(b.norm)),
                                                static_cast<const float *>(ptr(b.router)),
                                                static_cast<const float *>(ptr(b.bias)), ptr(b.gate), ptr(b.up),
                                                ptr(b.down), kTypeQ4K, b.down->type, 1, 1.0f);
        } else if (b.down->type != kTypeQ4K) {
            snprintf(g_describe_err, sizeof g_describe_err,
                     "block %u: an expert shard needs Q4_K down experts (this file's are type %u)", l, b.down->type);
            return LFM_GPU_ERR_UNSUPPORTED;
        } else {
            if (expert_first + n_local > b.E) {
                snprintf(g_describe_err, sizeof g_describe_err, "block %u: experts [%u, %u) past E=%u", l, expert_first,
                         expert_first + n_local, b.E);
                return LFM_GPU_ERR_INVALID_ARG;
            }
            const uint64_t per_gu = (uint64_t)b.I * (b.D / 256) * kQ4kBytes, per_dn = (uint64_t)b.D * (b.I / 256) * kQ4kBytes;
            st = lfm_gpu_moe_upload_layer_shard(
                h, i, b.D, b.E, b.K, b.I, f.eps, static_cast<const float *>(ptr(b.norm)),
                static_cast<const float *>(ptr(b.router)), static_cast<const float *>(ptr(b.bias)),
                b.gate->data + expert_first * per_gu, b.up->data + expert_first * per_gu, b.down->data + expert_first * per_dn,
                kTypeQ4K, 1, 1.0f, expert_first, n_local);
        }
        if (st != LFM_GPU_OK) {
            snprintf(g_describe_err, sizeof g_describe_err, "block %u: %s", l, lfm_gpu_moe_last_error(h));
            return st;
        }
        ++done;
        if (n_uploaded) *n_uploaded = done;
    }
    return LFM_GPU_OK;
}
