// gguf.cu -- GGUF ingest: a bounds-checked reader of GGUF v2/v3 files (mapped
// read-only), device decoders of the GGUF tensor types the reference's loader
// reads, the reference's Q8_0 re-quantiser on the device, and
// x100q_model_load_gguf.
//
// The reference reads a file with gguf_open (qwen_moe_q3k.c:1098-1126): the
// header counts, metadata (only the qwen3moe.* dimensions, the rope base and
// the token list are kept; other values are skipped by type), the tensor
// infos, and the data start (the info table's end rounded up to 32 bytes).
// It trusts every length in the file.  This reader walks the same structure
// but checks each read against the file size, caps counts and nesting, honours
// general.alignment when present (32 otherwise, which is what real Qwen3 files
// use and all the reference supports) and reports X100_E_FORMAT instead of
// exiting.
#include <cuda_fp16.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/x100q.h"
#include "moe.h"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace gguf {

constexpr uint64_t kMaxCount = 1u << 24;   // tensors, metadata entries, array items
constexpr int kMaxDepth = 4;               // nested arrays

// Metadata value types of the GGUF format.
enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

struct Kv {
    std::string key;
    uint32_t type = 0;
    uint64_t off = 0;     // value position in the file
    std::string sval;     // T_STR values
};

struct Tensor {
    std::string name;
    uint32_t type = 0;
    int nd = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t off = 0;     // relative to the data start
    uint64_t n = 0, bytes = 0;
};

// Elements and bytes per block of a ggml type (0, 0: size unknown).
void type_block(uint32_t t, uint64_t &be, uint64_t &bb) {
    be = bb = 0;
    switch (t) {
    case 0: be = 1, bb = 4; break;     // F32
    case 1: be = 1, bb = 2; break;     // F16
    case 2: be = 32, bb = 18; break;   // Q4_0
    case 3: be = 32, bb = 20; break;   // Q4_1
    case 6: be = 32, bb = 22; break;   // Q5_0
    case 7: be = 32, bb = 24; break;   // Q5_1
    case 8: be = 32, bb = 34; break;   // Q8_0
    case 9: be = 32, bb = 36; break;   // Q8_1
    case 10: be = 256, bb = 84; break;   // Q2_K
    case 11: be = 256, bb = 110; break;  // Q3_K
    case 12: be = 256, bb = 144; break;  // Q4_K
    case 13: be = 256, bb = 176; break;  // Q5_K
    case 14: be = 256, bb = 210; break;  // Q6_K
    case 15: be = 256, bb = 292; break;  // Q8_K
    case 24: be = 1, bb = 1; break;      // I8
    case 25: be = 1, bb = 2; break;      // I16
    case 26: be = 1, bb = 4; break;      // I32
    case 27: be = 1, bb = 8; break;      // I64
    case 28: be = 1, bb = 8; break;      // F64
    case 30: be = 1, bb = 2; break;      // BF16
    default: break;
    }
}

bool decodable(int t) {
    return t == X100Q_F32 || t == X100Q_F16 || t == X100Q_Q4_0 || t == X100Q_Q4_1 || t == X100Q_Q8_0 ||
           t == X100Q_Q3_K || t == X100Q_Q4_K || t == X100Q_Q5_K || t == X100Q_Q6_K;
}

// Cursor over the mapped file; any read past the end clears ok.
struct Cur {
    const uint8_t *p;
    uint64_t size, o = 0;
    bool ok = true;
    bool need(uint64_t n) {
        if (!ok || o > size || n > size - o) ok = false;
        return ok;
    }
    uint32_t u32() {
        uint32_t v = 0;
        if (need(4)) memcpy(&v, p + o, 4), o += 4;
        return v;
    }
    uint64_t u64() {
        uint64_t v = 0;
        if (need(8)) memcpy(&v, p + o, 8), o += 8;
        return v;
    }
    bool str(std::string *out) {
        const uint64_t n = u64();
        if (!need(n)) return false;
        if (out) out->assign(reinterpret_cast<const char *>(p + o), n);
        o += n;
        return true;
    }
    bool skip(uint32_t t, int depth) {
        switch (t) {
        case T_U8: case T_I8: case T_BOOL: return need(1) && (o += 1, true);
        case T_U16: case T_I16: return need(2) && (o += 2, true);
        case T_U32: case T_I32: case T_F32: return need(4) && (o += 4, true);
        case T_U64: case T_I64: case T_F64: return need(8) && (o += 8, true);
        case T_STR: return str(nullptr);
        case T_ARR: {
            if (depth >= kMaxDepth) return ok = false;
            const uint32_t et = u32();
            const uint64_t n = u64();
            if (!ok || n > kMaxCount) return ok = false;
            for (uint64_t i = 0; i < n && ok; ++i) skip(et, depth + 1);
            return ok;
        }
        default: return ok = false;
        }
    }
};

}  // namespace gguf
}  // namespace x100

using namespace x100;
using namespace x100::gguf;

struct x100q_gguf {
    uint8_t *map = nullptr;
    uint64_t size = 0;
    uint64_t data_start = 0, alignment = 32;
    std::vector<Kv> kv;
    std::vector<Tensor> tensors;
    std::vector<std::string> tokens;

    ~x100q_gguf() {
        if (map) munmap(map, size);
    }
    const Kv *find_kv(const char *key) const {
        for (const Kv &e : kv)
            if (e.key == key) return &e;
        return nullptr;
    }
    const Tensor *find(const char *name) const {
        for (const Tensor &t : tensors)
            if (t.name == name) return &t;
        return nullptr;
    }
    bool get_int(const char *key, int64_t *out) const {
        const Kv *e = find_kv(key);
        if (!e) return false;
        const uint8_t *v = map + e->off;
        switch (e->type) {
        case T_U8: *out = v[0]; return true;
        case T_BOOL: *out = v[0] != 0; return true;
        case T_I8: *out = (int8_t)v[0]; return true;
        case T_U16: { uint16_t x; memcpy(&x, v, 2); *out = x; return true; }
        case T_I16: { int16_t x; memcpy(&x, v, 2); *out = x; return true; }
        case T_U32: { uint32_t x; memcpy(&x, v, 4); *out = x; return true; }
        case T_I32: { int32_t x; memcpy(&x, v, 4); *out = x; return true; }
        case T_U64: { uint64_t x; memcpy(&x, v, 8); if (x > (uint64_t)INT64_MAX) return false; *out = (int64_t)x; return true; }
        case T_I64: { int64_t x; memcpy(&x, v, 8); *out = x; return true; }
        default: return false;
        }
    }
    bool get_f32(const char *key, float *out) const {
        const Kv *e = find_kv(key);
        if (!e) return false;
        if (e->type == T_F32) {
            memcpy(out, map + e->off, 4);
            return true;
        }
        if (e->type == T_F64) {
            double x;
            memcpy(&x, map + e->off, 8);
            *out = (float)x;
            return true;
        }
        return false;
    }
};

namespace {

int fail(int code) {
    set_error(code);
    return code;
}

bool parse(x100q_gguf *g) {
    Cur c{g->map, g->size};
    if (!c.need(4) || memcmp(g->map, "GGUF", 4) != 0) return false;
    c.o = 4;
    const uint32_t version = c.u32();
    if (version != 2 && version != 3) return false;
    const uint64_t nt = c.u64(), nkv = c.u64();
    if (!c.ok || nt > kMaxCount || nkv > kMaxCount) return false;
    g->kv.reserve(nkv);
    for (uint64_t i = 0; i < nkv; ++i) {
        Kv e;
        if (!c.str(&e.key)) return false;
        e.type = c.u32();
        e.off = c.o;
        if (!c.ok) return false;
        if (e.type == T_STR) {
            if (!c.str(&e.sval)) return false;
        } else if (e.type == T_ARR && e.key == "tokenizer.ggml.tokens") {
            const uint32_t et = c.u32();
            const uint64_t n = c.u64();
            if (!c.ok || n > kMaxCount) return false;
            if (et == T_STR) {
                g->tokens.resize(n);
                for (uint64_t j = 0; j < n; ++j)
                    if (!c.str(&g->tokens[j])) return false;
            } else {
                for (uint64_t j = 0; j < n; ++j)
                    if (!c.skip(et, 1)) return false;
            }
        } else if (!c.skip(e.type, 0)) {
            return false;
        }
        g->kv.push_back(std::move(e));
    }
    int64_t al = 0;
    if (g->get_int("general.alignment", &al)) {
        if (al <= 0 || (al & (al - 1)) || al > (1 << 20)) return false;
        g->alignment = (uint64_t)al;
    }
    g->tensors.resize(nt);
    for (uint64_t i = 0; i < nt; ++i) {
        Tensor &t = g->tensors[i];
        if (!c.str(&t.name)) return false;
        const uint32_t nd = c.u32();
        if (!c.ok || nd < 1 || nd > 4) return false;
        t.nd = (int)nd;
        t.n = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            t.dims[d] = c.u64();
            if (!c.ok || t.dims[d] == 0 || t.dims[d] > (1ull << 40) / t.n) return false;   // no overflow, no empties
            t.n *= t.dims[d];
        }
        t.type = c.u32();
        t.off = c.u64();
        if (!c.ok) return false;
        uint64_t be, bb;
        type_block(t.type, be, bb);
        if (be) {
            if (t.dims[0] % be) return false;   // rows hold whole blocks
            t.bytes = t.n / be * bb;
        }
    }
    g->data_start = (c.o + g->alignment - 1) / g->alignment * g->alignment;
    for (const Tensor &t : g->tensors) {
        if (g->data_start > g->size || t.off > g->size - g->data_start) return false;
        if (t.bytes > g->size - g->data_start - t.off) return false;
    }
    return true;
}

}  // namespace

// ---- device decoders ---------------------------------------------------------

namespace x100 {
namespace gguf {

// Exact fp16 -> fp32 from the bits (NaN payloads kept).
__device__ __forceinline__ float h2f(const uint8_t *p) {
    const uint32_t h = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
    const uint32_t s = (h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t b;
    if (e == 0) {
        if (m == 0) {
            b = s;
        } else {   // subnormal: normalise
            int ee = -14;
            uint32_t mm = m;
            while (!(mm & 0x400)) {
                mm <<= 1;
                --ee;
            }
            b = s | ((uint32_t)(ee + 127) << 23) | ((mm & 0x3FF) << 13);
        }
    } else if (e == 0x1F) {
        b = s | 0x7F800000u | (m << 13);
    } else {
        b = s | ((e + 112) << 23) | (m << 13);
    }
    return __uint_as_float(b);
}

// The 6-bit scale and min j (0..7) of a Q4_K / Q5_K block.
__device__ __forceinline__ void kq_scale_min(int j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Element j of one block.  Every product and sum is rounded separately, as
// the scalar reference computes it (no fused multiply-add).
template <int T>
__device__ __forceinline__ float dq(const uint8_t *b, int j) {
    if constexpr (T == X100Q_F32) {
        return __uint_as_float((uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) |
                               ((uint32_t)b[3] << 24));
    } else if constexpr (T == X100Q_F16) {
        return h2f(b);
    } else if constexpr (T == X100Q_Q4_0 || T == X100Q_Q4_1) {
        const uint8_t *qs = b + (T == X100Q_Q4_0 ? 2 : 4);
        const int nib = j < 16 ? (qs[j] & 0xF) : (qs[j - 16] >> 4);
        if constexpr (T == X100Q_Q4_0) return __fmul_rn((float)(nib - 8), h2f(b));
        else return __fadd_rn(__fmul_rn((float)nib, h2f(b)), h2f(b + 2));
    } else if constexpr (T == X100Q_Q8_0) {
        return __fmul_rn((float)(int8_t)b[2 + j], h2f(b));
    } else if constexpr (T == X100Q_Q3_K) {
        // element 128h + 32t + l: 2-bit value (qs[32h + l] >> 2t) & 3, minus 4
        // when bit 4h + t of hmask[l] is clear; scale 8h + 2t + (l >= 16)
        const int h = j >> 7, t = (j >> 5) & 3, l = j & 31, i = 8 * h + 2 * t + (l >> 4);
        const uint8_t *s12 = b + 96;
        const int lo = i < 8 ? (s12[i] & 0xF) : (s12[i - 8] >> 4);
        const int hi = (s12[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
        const int sc = (int)(int8_t)(uint8_t)(lo | (hi << 4)) - 32;
        const int q = (int)((b[32 + 32 * h + l] >> (2 * t)) & 3) - ((b[l] >> (4 * h + t)) & 1 ? 0 : 4);
        return __fmul_rn(__fmul_rn(h2f(b + 108), (float)sc), (float)q);
    } else if constexpr (T == X100Q_Q4_K || T == X100Q_Q5_K) {
        // 64-element chunk c: scale/min 2c (low nibbles), 2c + 1 (high nibbles)
        const int c = j >> 6, hi = (j >> 5) & 1, l = j & 31;
        const uint8_t *qs = b + (T == X100Q_Q4_K ? 16 : 48);
        int sc, m;
        kq_scale_min(2 * c + hi, b + 4, sc, m);
        int q = hi ? (qs[32 * c + l] >> 4) : (qs[32 * c + l] & 0xF);
        if constexpr (T == X100Q_Q5_K) q += ((b[16 + l] >> (2 * c + hi)) & 1) * 16;
        const float d1 = __fmul_rn(h2f(b), (float)sc), m1 = __fmul_rn(h2f(b + 2), (float)m);
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    } else {   // Q6_K: half h, quarter t, l < 32
        const int h = j >> 7, t = (j >> 5) & 3, l = j & 31;
        const int lo = b[64 * h + l + 32 * (t & 1)];
        const int q = ((t < 2 ? (lo & 0xF) : (lo >> 4)) | (((b[128 + 32 * h + l] >> (2 * t)) & 3) << 4)) - 32;
        const float ds = __fmul_rn(h2f(b + 208), (float)(int8_t)b[192 + 8 * h + 2 * t + (l >> 4)]);
        return __fmul_rn(ds, (float)q);
    }
}

template <int T, int BE, int BB>
__global__ void dequant_kernel(const uint8_t *__restrict__ data, long n, float *__restrict__ out) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        out[i] = dq<T>(data + (i / BE) * BB, (int)(i % BE));
}

// One warp per 32 values: amax from 1e-6, d = amax / 127, q = round-to-
// nearest-even(w * (1 / d)) clamped to int8, d stored as truncated fp16.
__global__ void quantize_q8_0_kernel(const float *__restrict__ x, long nblocks, uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const long warps = (long)gridDim.x * (blockDim.x >> 5);
    for (long b = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); b < nblocks; b += warps) {
        const float w = x[32 * b + lane];
        float amax = fmaxf(fabsf(w), 1e-6f);
        for (int s = 16; s; s >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, s));
        const float d = __fdiv_rn(amax, 127.0f);
        const float inv = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int q = __float2int_rn(__fmul_rn(w, inv));
        q = q > 127 ? 127 : (q < -128 ? -128 : q);
        uint8_t *blk = out + 34 * b;
        blk[2 + lane] = (uint8_t)(int8_t)q;
        if (lane == 0) {   // truncating fp32 -> fp16 of d
            const uint32_t u = __float_as_uint(d);
            const uint32_t sign = (u >> 16) & 0x8000u, mant = u & 0x7FFFFFu;
            const int ex = (int)((u >> 23) & 0xFF) - 127 + 15;
            uint32_t h;
            if (ex <= 0) h = ex < -10 ? sign : sign | ((mant | 0x800000u) >> (14 - ex));
            else if (ex >= 31) h = sign | 0x7C00u;
            else h = sign | ((uint32_t)ex << 10) | (mant >> 13);
            blk[0] = (uint8_t)h;
            blk[1] = (uint8_t)(h >> 8);
        }
    }
}

int launch_dequant(DevCtx *c, int type, const void *data, long n, float *out, cudaStream_t s) {
    const int grid = c->sm_count * 8, threads = 256;
    const uint8_t *d = static_cast<const uint8_t *>(data);
    switch (type) {
    case X100Q_F32: dequant_kernel<X100Q_F32, 1, 4><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_F16: dequant_kernel<X100Q_F16, 1, 2><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q4_0: dequant_kernel<X100Q_Q4_0, 32, 18><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q4_1: dequant_kernel<X100Q_Q4_1, 32, 20><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q8_0: dequant_kernel<X100Q_Q8_0, 32, 34><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q3_K: dequant_kernel<X100Q_Q3_K, 256, 110><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q4_K: dequant_kernel<X100Q_Q4_K, 256, 144><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q5_K: dequant_kernel<X100Q_Q5_K, 256, 176><<<grid, threads, 0, s>>>(d, n, out); break;
    case X100Q_Q6_K: dequant_kernel<X100Q_Q6_K, 256, 210><<<grid, threads, 0, s>>>(d, n, out); break;
    default: return fail(X100_E_FORMAT);
    }
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_quantize_q8_0(DevCtx *c, const float *x, long n, void *blocks, cudaStream_t s) {
    quantize_q8_0_kernel<<<c->sm_count * 8, 256, 0, s>>>(x, n / 32, static_cast<uint8_t *>(blocks));
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

// ---- loader ------------------------------------------------------------------

// Device buffers of one layer's converted tensors, freed together.
struct Arena {
    std::vector<void *> bufs;
    void *alloc(size_t bytes) {
        void *p = nullptr;
        if (cudaMalloc(&p, bytes < 256 ? 256 : bytes) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            return nullptr;
        }
        bufs.push_back(p);
        return p;
    }
    ~Arena() {
        for (void *p : bufs) cudaFree(p);
    }
};

struct Loader {
    const x100q_gguf *g;
    DevCtx *c;
    int st = X100_OK;

    const Tensor *need(const char *name, uint64_t n) {
        const Tensor *t = g->find(name);
        if (!t || t->n != n || !t->bytes) {
            if (getenv("X100_VERBOSE"))
                fprintf(stderr, "[x100] gguf: tensor %s %s\n", name, t ? "has the wrong size or type" : "missing");
            st = fail(X100_E_FORMAT);
            return nullptr;
        }
        return t;
    }
    const uint8_t *host(const Tensor *t) { return g->map + g->data_start + t->off; }

    // fp32 values of a tensor: the mapped data when it is F32, else decoded on
    // the device into the arena.
    const float *f32(Arena &a, const char *name, uint64_t n) {
        const Tensor *t = need(name, n);
        if (!t) return nullptr;
        if (t->type == X100Q_F32) return reinterpret_cast<const float *>(host(t));
        if (!decodable((int)t->type)) {
            st = fail(X100_E_FORMAT);
            return nullptr;
        }
        void *raw = a.alloc(t->bytes);
        float *out = static_cast<float *>(a.alloc(n * 4));
        if (!raw || !out) return st = X100_E_ALLOC, nullptr;
        if ((st = check_cuda(cudaMemcpyAsync(raw, host(t), t->bytes, cudaMemcpyHostToDevice, c->stream), X100_E_COPY)) ||
            (st = launch_dequant(c, (int)t->type, raw, (long)n, out, c->stream)))
            return nullptr;
        return out;
    }

    // Blocks of type `slot` for a weight tensor: the mapped data when the
    // file holds that type, else Q8_0 re-quantised on the device.
    const void *weight(Arena &a, const char *name, uint64_t n, int slot) {
        const Tensor *t = need(name, n);
        if (!t) return nullptr;
        if ((int)t->type == slot) return host(t);
        if (slot != X100Q_Q8_0 || !decodable((int)t->type)) {
            if (getenv("X100_VERBOSE"))
                fprintf(stderr, "[x100] gguf: %s is type %u, the model slot takes type %d\n", name, t->type, slot);
            st = fail(X100_E_FORMAT);
            return nullptr;
        }
        void *raw = a.alloc(t->bytes);
        float *f = static_cast<float *>(a.alloc(n * 4));
        void *q = a.alloc(n / 32 * 34);
        if (!raw || !f || !q) return st = X100_E_ALLOC, nullptr;
        if ((st = check_cuda(cudaMemcpyAsync(raw, host(t), t->bytes, cudaMemcpyHostToDevice, c->stream), X100_E_COPY)) ||
            (st = launch_dequant(c, (int)t->type, raw, (long)n, f, c->stream)) ||
            (st = launch_quantize_q8_0(c, f, (long)n, q, c->stream)))
            return nullptr;
        return q;
    }
    int sync() {
        if (!st) st = check_cuda(cudaStreamSynchronize(c->stream), X100_E_LAUNCH);
        return st;
    }
};

bool gemv_type(int t) { return t == X100Q_Q8_0 || t == X100Q_Q4_0 || t == X100Q_Q4_K || t == X100Q_Q3_K; }

}  // namespace gguf
}  // namespace x100

extern "C" {

x100q_gguf *x100q_gguf_open(const char *path) {
    set_error(X100_OK);
    if (!path) return fail(X100_E_ARG), nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(X100_E_ARG), nullptr;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
        close(fd);
        return fail(X100_E_FORMAT), nullptr;
    }
    x100q_gguf *g = new x100q_gguf();
    g->size = (uint64_t)sb.st_size;
    void *m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
        g->size = 0;
        delete g;
        return fail(X100_E_ALLOC), nullptr;
    }
    g->map = static_cast<uint8_t *>(m);
    if (!parse(g)) {
        delete g;
        return fail(X100_E_FORMAT), nullptr;
    }
    return g;
}

void x100q_gguf_close(x100q_gguf *g) { delete g; }

int x100q_gguf_n_tensors(const x100q_gguf *g) { return g ? (int)g->tensors.size() : 0; }

static void fill_info(const x100q_gguf *g, const Tensor &t, x100q_gguf_tensor *out) {
    out->name = t.name.c_str();
    out->type = (int)t.type;
    out->n_dims = t.nd;
    for (int d = 0; d < 4; ++d) out->dims[d] = d < t.nd ? t.dims[d] : 1;
    out->n_elems = t.n;
    out->bytes = t.bytes;
    out->data = g->map + g->data_start + t.off;
}

int x100q_gguf_tensor_at(const x100q_gguf *g, int i, x100q_gguf_tensor *out) {
    set_error(X100_OK);
    if (!g || !out || i < 0 || i >= (int)g->tensors.size()) return fail(X100_E_ARG);
    fill_info(g, g->tensors[i], out);
    return X100_OK;
}

int x100q_gguf_find(const x100q_gguf *g, const char *name, x100q_gguf_tensor *out) {
    set_error(X100_OK);
    if (!g || !name || !out) return fail(X100_E_ARG);
    const Tensor *t = g->find(name);
    if (!t) return fail(X100_E_FORMAT);
    fill_info(g, *t, out);
    return X100_OK;
}

uint64_t x100q_gguf_data_offset(const x100q_gguf *g) { return g ? g->data_start : 0; }

int x100q_gguf_n_tokens(const x100q_gguf *g) { return g ? (int)g->tokens.size() : 0; }

const char *x100q_gguf_token(const x100q_gguf *g, int id) {
    if (!g || id < 0 || id >= (int)g->tokens.size()) return nullptr;
    return g->tokens[id].c_str();
}

int x100q_gguf_get_int(const x100q_gguf *g, const char *key, int64_t *out) {
    set_error(X100_OK);
    if (!g || !key || !out) return fail(X100_E_ARG);
    return g->get_int(key, out) ? X100_OK : fail(X100_E_FORMAT);
}

int x100q_gguf_get_f32(const x100q_gguf *g, const char *key, float *out) {
    set_error(X100_OK);
    if (!g || !key || !out) return fail(X100_E_ARG);
    return g->get_f32(key, out) ? X100_OK : fail(X100_E_FORMAT);
}

int x100q_gguf_get_str(const x100q_gguf *g, const char *key, const char **out) {
    set_error(X100_OK);
    if (!g || !key || !out) return fail(X100_E_ARG);
    const Kv *e = g->find_kv(key);
    if (!e || e->type != T_STR) return fail(X100_E_FORMAT);
    *out = e->sval.c_str();
    return X100_OK;
}

int x100q_gguf_model_cfg(const x100q_gguf *g, x100q_model_cfg *cfg) {
    set_error(X100_OK);
    if (!g || !cfg) return fail(X100_E_ARG);
    auto geti = [&](const char *k, int dflt, bool required, int *v) {
        int64_t x;
        if (!g->get_int(k, &x)) {
            *v = dflt;
            return !required;
        }
        if (x <= 0 || x > (1 << 30)) return false;
        *v = (int)x;
        return true;
    };
    x100q_model_cfg c{};
    bool ok = geti("qwen3moe.block_count", 0, true, &c.n_layers) &&
              geti("qwen3moe.embedding_length", 0, true, &c.d) &&
              geti("qwen3moe.attention.head_count", 0, true, &c.n_heads) &&
              geti("qwen3moe.attention.head_count_kv", 0, true, &c.n_kv_heads) &&
              geti("qwen3moe.attention.key_length", 0, true, &c.head_dim) &&
              geti("qwen3moe.expert_count", 128, false, &c.n_exp) &&
              geti("qwen3moe.expert_used_count", 8, false, &c.n_act) &&
              geti("qwen3moe.expert_feed_forward_length", 768, false, &c.moe_ffn);
    if (!ok) return fail(X100_E_FORMAT);
    c.rope_base = 1e6f;
    g->get_f32("qwen3moe.rope.freq_base", &c.rope_base);
    c.eps = 1e-6f;   // the reference's model_load fixes it (qwen_moe_q3k.c:1744)
    const Tensor *emb = g->find("token_embd.weight");
    if (!emb || emb->nd < 2 || emb->dims[0] != (uint64_t)c.d || emb->dims[1] > (1u << 30)) return fail(X100_E_FORMAT);
    c.vocab = (int)emb->dims[1];
    // one type per slot: the type every layer's tensors share, if usable
    auto common = [&](const char *const *sufs, int nsuf) {
        int t = -1;
        char nm[96];
        for (int l = 0; l < c.n_layers; ++l)
            for (int s = 0; s < nsuf; ++s) {
                snprintf(nm, sizeof nm, "blk.%d.%s", l, sufs[s]);
                const Tensor *x = g->find(nm);
                if (!x) return -2;
                if (t == -1) t = (int)x->type;
                else if (t != (int)x->type) return -1;
            }
        return t;
    };
    static const char *const attn[] = {"attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight"};
    static const char *const exps[] = {"ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"};
    const int ta = common(attn, 4), te = common(exps, 3);
    if (ta == -2 || te == -2) return fail(X100_E_FORMAT);
    c.attn_qtype = gemv_type(ta) ? ta : X100Q_Q8_0;
    c.expert_qtype = (gemv_type(te) && moe_shapes_ok(c.d, c.n_exp, c.n_act, c.moe_ffn, te)) ? te : X100Q_Q8_0;
    const Tensor *lm = g->find("output.weight");
    c.lm_qtype = (lm && gemv_type((int)lm->type)) ? (int)lm->type : X100Q_Q8_0;
    c.ctx = 4096;
    c.max_batch = 1;
    c.expert_lo = 0;
    c.expert_hi = c.n_exp;
    *cfg = c;
    return X100_OK;
}

x100q_model *x100q_model_load_gguf(const x100q_gguf *g, const x100q_model_cfg *cfg) {
    set_error(X100_OK);
    if (!g || !cfg) return fail(X100_E_ARG), nullptr;
    x100q_model_cfg file;
    if (x100q_gguf_model_cfg(g, &file)) return nullptr;
    const x100q_model_cfg &c = *cfg;
    if (c.n_layers != file.n_layers || c.d != file.d || c.n_heads != file.n_heads || c.n_kv_heads != file.n_kv_heads ||
        c.head_dim != file.head_dim || c.vocab != file.vocab || c.n_exp != file.n_exp || c.moe_ffn != file.moe_ffn)
        return fail(X100_E_ARG), nullptr;
    DevCtx *dc = ctx();
    if (!dc) return nullptr;
    x100q_model *m = x100q_model_create(cfg);
    if (!m) return nullptr;
    Loader L{g, dc};
    const uint64_t d = c.d, qd = (uint64_t)c.n_heads * c.head_dim, kvd = (uint64_t)c.n_kv_heads * c.head_dim;
    const uint64_t E = c.n_exp, F = c.moe_ffn, hd = c.head_dim;
    char nm[12][96];
    for (int l = 0; l < c.n_layers && !L.st; ++l) {
        static const char *const sufs[12] = {"attn_norm.weight", "attn_q.weight", "attn_k.weight", "attn_v.weight",
                                             "attn_q_norm.weight", "attn_k_norm.weight", "attn_output.weight",
                                             "ffn_norm.weight", "ffn_gate_inp.weight", "ffn_gate_exps.weight",
                                             "ffn_up_exps.weight", "ffn_down_exps.weight"};
        for (int i = 0; i < 12; ++i) snprintf(nm[i], sizeof nm[i], "blk.%d.%s", l, sufs[i]);
        Arena a;
        const float *an = L.f32(a, nm[0], d);
        const void *wq = L.weight(a, nm[1], qd * d, c.attn_qtype);
        const void *wk = L.weight(a, nm[2], kvd * d, c.attn_qtype);
        const void *wv = L.weight(a, nm[3], kvd * d, c.attn_qtype);
        const float *qn = L.f32(a, nm[4], hd), *kn = L.f32(a, nm[5], hd);
        const void *wo = L.weight(a, nm[6], d * qd, c.attn_qtype);
        const float *fn = L.f32(a, nm[7], d), *router = L.f32(a, nm[8], E * d);
        const void *gate = L.weight(a, nm[9], E * F * d, c.expert_qtype);
        const void *up = L.weight(a, nm[10], E * F * d, c.expert_qtype);
        const void *down = L.weight(a, nm[11], E * d * F, c.expert_qtype);
        if (L.sync()) break;
        L.st = x100q_model_set_layer(m, l, an, wq, wk, wv, qn, kn, wo, fn, router, gate, up, down);
    }
    if (!L.st) {
        Arena a;
        const float *emb = L.f32(a, "token_embd.weight", (uint64_t)c.vocab * d);
        const float *on = L.f32(a, "output_norm.weight", d);
        const void *lm = nullptr;
        if (g->find("output.weight")) {
            lm = L.weight(a, "output.weight", (uint64_t)c.vocab * d, c.lm_qtype);
        } else if (c.lm_qtype != X100Q_Q8_0) {
            L.st = fail(X100_E_FORMAT);
        } else if (emb) {   // tied: Q8_0 of the fp32 embeddings
            const float *src = emb;
            if (!is_device_ptr(emb)) {
                float *dev = static_cast<float *>(a.alloc((uint64_t)c.vocab * d * 4));
                if (!dev || (L.st = check_cuda(cudaMemcpyAsync(dev, emb, (uint64_t)c.vocab * d * 4,
                                                               cudaMemcpyHostToDevice, dc->stream),
                                               X100_E_COPY)))
                    dev = nullptr;
                src = dev;
            }
            void *q = a.alloc((uint64_t)c.vocab * d / 32 * 34);
            if (src && q && !(L.st = launch_quantize_q8_0(dc, src, (long)((uint64_t)c.vocab * d), q, dc->stream)))
                lm = q;
        }
        if (!L.st && !L.sync()) L.st = x100q_model_set_output(m, emb, on, lm);
    }
    if (L.st) {
        x100q_model_destroy(m);
        set_error(L.st);
        return nullptr;
    }
    return m;
}

int x100q_gguf_dequant_dev(int type, const void *data, long n, float *out, void *stream) {
    set_error(X100_OK);
    uint64_t be, bb;
    type_block((uint32_t)type, be, bb);
    if (!data || !out || n <= 0 || !decodable(type) || n % (long)be) return fail(X100_E_ARG);
    DevCtx *c = ctx();
    if (!c) return get_error();
    return launch_dequant(c, type, data, n, out, static_cast<cudaStream_t>(stream));
}

int x100q_quantize_q8_0_dev(const float *x, long n, void *blocks, void *stream) {
    set_error(X100_OK);
    if (!x || !blocks || n <= 0 || n % 32) return fail(X100_E_ARG);
    DevCtx *c = ctx();
    if (!c) return get_error();
    return launch_quantize_q8_0(c, x, n, blocks, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
