// qformats.cuh -- device-side block formats of the quantised decode path and
// the per-unit dot products shared by the dequant-GEMV and the MoE kernels.
//
// Weights keep the reference's GGUF block arithmetic (decoders restated from
// qwen_moe.c:162-165, qwen_moe_q3k.c:534-577, repack.cpp:222-283), laid out
// on the device so every weight load is a 16-byte vector load:
//   Q4_0  qs plane [N][K/32][16 B] + fp16 d plane [N][K/32]        (18 B/32)
//   Q8_0  qs plane [N][K/32][32 B] + fp16 d plane [N][K/32]        (34 B/32)
//   Q4_K  native 144-byte superblocks (already 9 x 16 B)           (144 B/256)
//   Q3_K  110-byte superblocks padded to 112 B and reordered as
//         [qs 64][hmask 32][scales 12][d 2][pad 2]                (112 B/256)
//
// Activations: each 32-element block of the fp32 activation x is written as
// x ~= s * (256 h + l) with s = max|x|/32639 and int8 planes h, l (error at
// most s/2, ~1.5e-5 of the block maximum), plus exact fp32 sums of the block
// and of its two 16-element halves.  A "unit" is 32 weights of one row; its
// dot product with x is formed from int32 dp4a sums (exact) and one fp32
// scale per block or sub-block.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace x100 {
namespace q {

enum { F32 = 0, Q4_0 = 2, Q8_0 = 8, Q3_K = 11, Q4_K = 12 };

// One 32-element activation block: h and l planes, 8 words each.
struct __align__(16) XBlk {
    uint4 h0, h1;   // h bytes of elements 0-15, 16-31
    uint4 l0, l1;   // l bytes of elements 0-15, 16-31
};
// {s, sum of the 32 elements, sum of elements 0-15, sum of 16-31}
using XF = float4;

constexpr int kXScale = 32639;   // |256 h + l| <= 32639 keeps h in [-127, 127]

// Units per row: 32 weights per unit, except Q3_K whose unit covers 64
// weights (one 16-byte qs slice and one 16-byte hmask slice, see load_unit).
__host__ __device__ constexpr int units_per_row(int qt, int K) { return qt == Q3_K ? K / 64 : K / 32; }
__host__ __device__ constexpr long row_bytes_dev(int qt, int K) {
    return qt == Q4_0 ? (long)(K / 32) * 16
         : qt == Q8_0 ? (long)(K / 32) * 32
         : qt == Q4_K ? (long)(K / 256) * 144
         : qt == Q3_K ? (long)(K / 256) * 112
         : 0;
}

// Device view of a resident quantised matrix.
struct QView {
    int qt;              // Q4_0 / Q8_0 / Q4_K / Q3_K
    const uint8_t *w;    // weight plane / superblocks
    const __half *d;     // Q4_0 / Q8_0 block scales (nullptr for K-quants)
    long wstride;        // bytes per row in w
    int dstride;         // scales per row in d
    int N, K;
};

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// 256 * sum(w.h) + sum(w.l) over 16 unsigned weight bytes.
__device__ __forceinline__ int dot16_u(uint4 w, uint4 h, uint4 l) {
    int sh = dp4a_us(w.x, h.x, 0);
    sh = dp4a_us(w.y, h.y, sh);
    sh = dp4a_us(w.z, h.z, sh);
    sh = dp4a_us(w.w, h.w, sh);
    int sl = dp4a_us(w.x, l.x, 0);
    sl = dp4a_us(w.y, l.y, sl);
    sl = dp4a_us(w.z, l.z, sl);
    sl = dp4a_us(w.w, l.w, sl);
    return sh * 256 + sl;
}
__device__ __forceinline__ int dot16_s(uint4 w, uint4 h, uint4 l) {
    int sh = dp4a_ss(w.x, h.x, 0);
    sh = dp4a_ss(w.y, h.y, sh);
    sh = dp4a_ss(w.z, h.z, sh);
    sh = dp4a_ss(w.w, h.w, sh);
    int sl = dp4a_ss(w.x, l.x, 0);
    sl = dp4a_ss(w.y, l.y, sl);
    sl = dp4a_ss(w.z, l.z, sl);
    sl = dp4a_ss(w.w, l.w, sl);
    return sh * 256 + sl;
}
__device__ __forceinline__ uint4 nib_lo(uint4 q) {
    return make_uint4(q.x & 0x0F0F0F0Fu, q.y & 0x0F0F0F0Fu, q.z & 0x0F0F0F0Fu, q.w & 0x0F0F0F0Fu);
}
__device__ __forceinline__ uint4 nib_hi(uint4 q) {
    return make_uint4((q.x >> 4) & 0x0F0F0F0Fu, (q.y >> 4) & 0x0F0F0F0Fu, (q.z >> 4) & 0x0F0F0F0Fu,
                      (q.w >> 4) & 0x0F0F0F0Fu);
}
__device__ __forceinline__ uint4 ldg16(const uint8_t *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

// K-quant 6-bit scale/min pair j (restates qwen_moe_q3k.c:534-538 /
// repack.cpp:222-233) from the 12 scale bytes held in three words.
__device__ __forceinline__ void kq_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, int &sc, int &m) {
    auto byte = [&](int i) -> int {
        uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
        return (w >> (8 * (i & 3))) & 0xFF;
    };
    if (j < 4) {
        sc = byte(j) & 63;
        m = byte(j + 4) & 63;
    } else {
        sc = (byte(j + 4) & 0xF) | ((byte(j - 4) >> 6) << 4);
        m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
}
// Q3_K scale i (0..15), biased by 32 (restates qwen_moe_q3k.c:560-564).
__device__ __forceinline__ int q3k_scale(int i, uint32_t s0, uint32_t s1, uint32_t s2) {
    auto byte = [&](int k) -> int {
        uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
        return (w >> (8 * (k & 3))) & 0xFF;
    };
    int lo = i < 8 ? (byte(i) & 0xF) : (byte(i - 8) >> 4);
    int hi = (byte(8 + (i & 3)) >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

// ---- one unit (32 weights) of one row, in registers -------------------------
template <int QT> struct WUnit;
template <> struct WUnit<Q4_0> { uint4 q; float d; };
template <> struct WUnit<Q8_0> { uint4 q0, q1; float d; };
template <> struct WUnit<Q4_K> { uint4 q; float da, ma, db, mb; };
template <> struct WUnit<Q3_K> { uint4 q, hm; float ds[4]; };

template <int QT> __device__ __forceinline__ WUnit<QT> load_unit(const QView &W, int row, int u);

template <> __device__ __forceinline__ WUnit<Q4_0> load_unit<Q4_0>(const QView &W, int row, int u) {
    WUnit<Q4_0> r;
    r.q = ldg16(W.w + (long)row * W.wstride + (long)u * 16);
    r.d = __half2float(W.d[(long)row * W.dstride + u]);
    return r;
}
template <> __device__ __forceinline__ WUnit<Q8_0> load_unit<Q8_0>(const QView &W, int row, int u) {
    WUnit<Q8_0> r;
    const uint8_t *p = W.w + (long)row * W.wstride + (long)u * 32;
    r.q0 = ldg16(p);
    r.q1 = ldg16(p + 16);
    r.d = __half2float(W.d[(long)row * W.dstride + u]);
    return r;
}
// Q4_K unit u: superblock u/8, 16 qs bytes (u%8): chunk c = (u%8)/2 holds
// sub-blocks 2c (low nibbles) and 2c+1 (high nibbles); half = u%2.
template <> __device__ __forceinline__ WUnit<Q4_K> load_unit<Q4_K>(const QView &W, int row, int u) {
    WUnit<Q4_K> r;
    const uint8_t *sb = W.w + (long)row * W.wstride + (long)(u >> 3) * 144;
    const int v = u & 7, c = v >> 1;
    r.q = ldg16(sb + 16 + 16 * v);
    const uint4 hd = ldg16(sb);
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    int sc, m;
    kq_scale_min(2 * c, hd.y, hd.z, hd.w, sc, m);
    r.da = d * (float)sc;
    r.ma = dmin * (float)m;
    kq_scale_min(2 * c + 1, hd.y, hd.z, hd.w, sc, m);
    r.db = d * (float)sc;
    r.mb = dmin * (float)m;
    return r;
}
// Q3_K unit u: superblock u/4, v = u%4: hh = v/2 selects elements 128..255,
// lh = v%2 selects l in 16..31; covers elements 128hh + 32j + 16lh + i for
// j < 4, i < 16 (scales 8hh + 2j + lh).
template <> __device__ __forceinline__ WUnit<Q3_K> load_unit<Q3_K>(const QView &W, int row, int u) {
    WUnit<Q3_K> r;
    const uint8_t *sb = W.w + (long)row * W.wstride + (long)(u >> 2) * 112;
    const int v = u & 3, hh = v >> 1, lh = v & 1;
    r.q = ldg16(sb + 32 * hh + 16 * lh);
    r.hm = ldg16(sb + 64 + 16 * lh);
    const uint4 hd = ldg16(sb + 96);
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.w & 0xFFFF)));
#pragma unroll
    for (int j = 0; j < 4; ++j) r.ds[j] = d * (float)q3k_scale(8 * hh + 2 * j + lh, hd.x, hd.y, hd.z);
    return r;
}

// ---- unit . x ------------------------------------------------------------------
// xq/xf: the activation blocks of one batch column (nxb = K/32 entries).
template <int QT>
__device__ __forceinline__ float dot_unit(const WUnit<QT> &w, const XBlk *xq, const XF *xf, int u);

template <> __device__ __forceinline__ float dot_unit<Q4_0>(const WUnit<Q4_0> &w, const XBlk *xq, const XF *xf, int u) {
    const XBlk &x = xq[u];
    const XF f = xf[u];
    const int dot = dot16_u(nib_lo(w.q), x.h0, x.l0) + dot16_u(nib_hi(w.q), x.h1, x.l1);
    return w.d * (f.x * (float)dot - 8.0f * f.y);   // (nib - 8) * d
}
template <> __device__ __forceinline__ float dot_unit<Q8_0>(const WUnit<Q8_0> &w, const XBlk *xq, const XF *xf, int u) {
    const XBlk &x = xq[u];
    const XF f = xf[u];
    const int dot = dot16_s(w.q0, x.h0, x.l0) + dot16_s(w.q1, x.h1, x.l1);
    return w.d * (f.x * (float)dot);
}
template <> __device__ __forceinline__ float dot_unit<Q4_K>(const WUnit<Q4_K> &w, const XBlk *xq, const XF *xf, int u) {
    const int v = u & 7, c = v >> 1, half = v & 1;
    const int xa = (u >> 3) * 8 + 2 * c;                     // x block of sub-block 2c
    const XBlk &a = xq[xa];
    const XBlk &b = xq[xa + 1];
    const XF fa = xf[xa], fb = xf[xa + 1];
    const int da = dot16_u(nib_lo(w.q), half ? a.h1 : a.h0, half ? a.l1 : a.l0);
    const int db = dot16_u(nib_hi(w.q), half ? b.h1 : b.h0, half ? b.l1 : b.l0);
    const float sa = half ? fa.w : fa.z, sbm = half ? fb.w : fb.z;
    return w.da * (fa.x * (float)da) - w.ma * sa + w.db * (fb.x * (float)db) - w.mb * sbm;
}
template <> __device__ __forceinline__ float dot_unit<Q3_K>(const WUnit<Q3_K> &w, const XBlk *xq, const XF *xf, int u) {
    const int v = u & 3, hh = v >> 1, lh = v & 1;
    const int x0 = (u >> 2) * 8 + 4 * hh;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int hs = 4 * hh + j;
        uint4 vv;
        vv.x = ((w.q.x >> (2 * j)) & 0x03030303u) | (((w.hm.x >> hs) & 0x01010101u) << 2);
        vv.y = ((w.q.y >> (2 * j)) & 0x03030303u) | (((w.hm.y >> hs) & 0x01010101u) << 2);
        vv.z = ((w.q.z >> (2 * j)) & 0x03030303u) | (((w.hm.z >> hs) & 0x01010101u) << 2);
        vv.w = ((w.q.w >> (2 * j)) & 0x03030303u) | (((w.hm.w >> hs) & 0x01010101u) << 2);
        const XBlk &x = xq[x0 + j];
        const XF f = xf[x0 + j];
        const int dot = dot16_u(vv, lh ? x.h1 : x.h0, lh ? x.l1 : x.l0);   // v in [0,7]; q = v - 4
        acc += w.ds[j] * (f.x * (float)dot - 4.0f * (lh ? f.w : f.z));
    }
    return acc;
}

// ---- activation preparation -----------------------------------------------------
// Eight consecutive threads (t = lane % 8) convert one 32-element block
// x[0..31] into (xq, xf).  Every lane of the warp must call it together (it
// shuffles across the whole warp); lanes whose group has no block pass
// active = false and write nothing.
__device__ __forceinline__ void xprep_block(const float *x, XBlk *xq, XF *xf, int t, bool active) {
    const float4 v = active ? *reinterpret_cast<const float4 *>(x + 4 * t) : make_float4(0.f, 0.f, 0.f, 0.f);
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    float s16 = (v.x + v.y) + (v.z + v.w);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
    s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
    const float s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 4);
    const float other16 = __shfl_xor_sync(0xffffffffu, s16, 4);
    const float s = amax > 0.f ? amax / (float)kXScale : 0.f;
    const float inv = amax > 0.f ? (float)kXScale / amax : 0.f;
    const float e[4] = {v.x, v.y, v.z, v.w};
    uint32_t hw = 0, lw = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int X = __float2int_rn(e[k] * inv);
        X = max(-kXScale, min(kXScale, X));
        const int h = (X + 128) >> 8;
        const int l = X - 256 * h;
        hw |= (uint32_t)(h & 0xFF) << (8 * k);
        lw |= (uint32_t)(l & 0xFF) << (8 * k);
    }
    if (!active) return;
    uint32_t *hwords = reinterpret_cast<uint32_t *>(&xq->h0);
    uint32_t *lwords = reinterpret_cast<uint32_t *>(&xq->l0);
    hwords[t] = hw;
    lwords[t] = lw;
    if (t == 0) *xf = make_float4(s, s32, s16, other16);
}

}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// The whole CTA prepares `batch` activation rows x[c*K .. c*K+K) into
// xq/xf[c*(K/32) + j]; warp-uniform trip counts keep the shuffles legal.
__device__ __forceinline__ void xprep_all(const float *x, int K, int batch, XBlk *xq, XF *xf) {
    const int nxb = K / 32;
    const int total = batch * nxb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int b0 = warp * 4; b0 < total; b0 += nwarps * 4) {
        const int blk = b0 + (lane >> 3);
        const bool active = blk < total;
        const int c = active ? blk / nxb : 0, j = active ? blk - c * nxb : 0;
        xprep_block(x + (long)c * K + j * 32, &xq[c * nxb + j], &xf[c * nxb + j], lane & 7, active);
    }
}
}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// ---- 256-element slices -----------------------------------------------------------
// A slice is 256 consecutive weights of one row: one K-quant superblock, or
// eight Q4_0 / Q8_0 blocks.  The slice GEMV kernels give each warp one slice
// of 32 rows (one row per lane), so a lane reads its slice with consecutive
// 16-byte loads and every lane of the warp reads the same activation blocks
// (shared-memory broadcast).
template <int QT> struct WSlice;
template <> struct WSlice<Q4_0> { uint4 q[8]; uint4 dh; };
template <> struct WSlice<Q8_0> { uint4 q[16]; uint4 dh; };
template <> struct WSlice<Q4_K> { uint4 hdr; uint4 q[8]; };
template <> struct WSlice<Q3_K> { uint4 q[4]; uint4 hm[2]; uint4 hdr; };

__device__ __forceinline__ uint4 ld16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
// kG: global memory (read-only path) or, when false, any address space.
template <bool kG> __device__ __forceinline__ uint4 ldq(const uint8_t *p) { return kG ? ldg16(p) : ld16(p); }

template <int QT, bool kG = true> __device__ __forceinline__ void load_slice(const QView &W, int row, int s, WSlice<QT> &r);
template <int QT, bool kG> struct SliceLoader;
template <bool kG> struct SliceLoader<Q4_0, kG> {
static __device__ __forceinline__ void run(const QView &W, int row, int s, WSlice<Q4_0> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 128;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = ldq<kG>(p + 16 * i);
    r.dh = ldq<kG>(reinterpret_cast<const uint8_t *>(W.d + (long)row * W.dstride + s * 8));
}};
template <bool kG> struct SliceLoader<Q8_0, kG> {
static __device__ __forceinline__ void run(const QView &W, int row, int s, WSlice<Q8_0> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 256;
#pragma unroll
    for (int i = 0; i < 16; ++i) r.q[i] = ldq<kG>(p + 16 * i);
    r.dh = ldq<kG>(reinterpret_cast<const uint8_t *>(W.d + (long)row * W.dstride + s * 8));
}};
template <bool kG> struct SliceLoader<Q4_K, kG> {
static __device__ __forceinline__ void run(const QView &W, int row, int s, WSlice<Q4_K> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 144;
    r.hdr = ldq<kG>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = ldq<kG>(p + 16 + 16 * i);
}};
template <bool kG> struct SliceLoader<Q3_K, kG> {
static __device__ __forceinline__ void run(const QView &W, int row, int s, WSlice<Q3_K> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 112;
#pragma unroll
    for (int i = 0; i < 4; ++i) r.q[i] = ldq<kG>(p + 16 * i);
    r.hm[0] = ldq<kG>(p + 64);
    r.hm[1] = ldq<kG>(p + 80);
    r.hdr = ldq<kG>(p + 96);
}};
template <int QT, bool kG> __device__ __forceinline__ void load_slice(const QView &W, int row, int s, WSlice<QT> &r) {
    SliceLoader<QT, kG>::run(W, row, s, r);
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
__device__ __forceinline__ uint32_t u4_word(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// slice . x, with xq / xf pointing at the slice's 8 activation blocks.
template <int QT> __device__ __forceinline__ float dot_slice(const WSlice<QT> &w, const XBlk *xq, const XF *xf);

template <> __device__ __forceinline__ float dot_slice<Q4_0>(const WSlice<Q4_0> &w, const XBlk *xq, const XF *xf) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const XBlk x = xq[b];
        const XF f = xf[b];
        const int dot = dot16_u(nib_lo(w.q[b]), x.h0, x.l0) + dot16_u(nib_hi(w.q[b]), x.h1, x.l1);
        const uint32_t dw = u4_word(w.dh, b >> 1);
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (f.x * (float)dot - 8.0f * f.y);
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_slice<Q8_0>(const WSlice<Q8_0> &w, const XBlk *xq, const XF *xf) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const XBlk x = xq[b];
        const XF f = xf[b];
        const int dot = dot16_s(w.q[2 * b], x.h0, x.l0) + dot16_s(w.q[2 * b + 1], x.h1, x.l1);
        const uint32_t dw = u4_word(w.dh, b >> 1);
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (f.x * (float)dot);
    }
    return acc;
}
// Q4_K: qs 16-byte slice v (chunk c = v/2, half = v%2) holds elements
// 64c + 16half + i (low nibbles, sub-block 2c) and 64c + 32 + 16half + i
// (high nibbles, sub-block 2c + 1).
template <> __device__ __forceinline__ float dot_slice<Q4_K>(const WSlice<Q4_K> &w, const XBlk *xq, const XF *xf) {
    const float d = half_lo(w.hdr.x), dmin = half_hi(w.hdr.x);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int sc0, m0, sc1, m1;
        kq_scale_min(2 * c, w.hdr.y, w.hdr.z, w.hdr.w, sc0, m0);
        kq_scale_min(2 * c + 1, w.hdr.y, w.hdr.z, w.hdr.w, sc1, m1);
        const XBlk xa = xq[2 * c], xb = xq[2 * c + 1];
        const XF fa = xf[2 * c], fb = xf[2 * c + 1];
        const int da = dot16_u(nib_lo(w.q[2 * c]), xa.h0, xa.l0) + dot16_u(nib_lo(w.q[2 * c + 1]), xa.h1, xa.l1);
        const int db = dot16_u(nib_hi(w.q[2 * c]), xb.h0, xb.l0) + dot16_u(nib_hi(w.q[2 * c + 1]), xb.h1, xb.l1);
        acc += d * (float)sc0 * (fa.x * (float)da) - dmin * (float)m0 * fa.y;
        acc += d * (float)sc1 * (fb.x * (float)db) - dmin * (float)m1 * fb.y;
    }
    return acc;
}
// Q3_K: qs 16-byte slice 2hh + lh and hmask slice lh hold elements
// 128hh + 32j + 16lh + i (j < 4), two bits at shift 2j and the bit 4hh + j.
template <> __device__ __forceinline__ float dot_slice<Q3_K>(const WSlice<Q3_K> &w, const XBlk *xq, const XF *xf) {
    const float d = half_lo(w.hdr.w);
    float acc = 0.f;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const XBlk x = xq[4 * hh + j];
            const XF f = xf[4 * hh + j];
            const int hs = 4 * hh + j;
            int dots[2];
#pragma unroll
            for (int lh = 0; lh < 2; ++lh) {
                const uint4 q = w.q[2 * hh + lh], hm = w.hm[lh];
                uint4 vv;
                vv.x = ((q.x >> (2 * j)) & 0x03030303u) | (((hm.x >> hs) & 0x01010101u) << 2);
                vv.y = ((q.y >> (2 * j)) & 0x03030303u) | (((hm.y >> hs) & 0x01010101u) << 2);
                vv.z = ((q.z >> (2 * j)) & 0x03030303u) | (((hm.z >> hs) & 0x01010101u) << 2);
                vv.w = ((q.w >> (2 * j)) & 0x03030303u) | (((hm.w >> hs) & 0x01010101u) << 2);
                dots[lh] = dot16_u(vv, lh ? x.h1 : x.h0, lh ? x.l1 : x.l0);
            }
            const float s0 = d * (float)q3k_scale(8 * hh + 2 * j, w.hdr.x, w.hdr.y, w.hdr.z);
            const float s1 = d * (float)q3k_scale(8 * hh + 2 * j + 1, w.hdr.x, w.hdr.y, w.hdr.z);
            acc += s0 * (f.x * (float)dots[0] - 4.0f * f.z) + s1 * (f.x * (float)dots[1] - 4.0f * f.w);
        }
    }
    return acc;
}
}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// ---- programmatic dependent launch -------------------------------------------------
// Kernels launched with the programmatic-serialization attribute may start
// while the previous kernel of the stream is still running.  They first issue
// loads that do not depend on it (weights), then allow their own dependents
// to launch, and wait for the previous grid (its writes become visible)
// before reading its outputs.  Without the attribute both calls are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- half slices -------------------------------------------------------------------
// Half h of a 256-element slice: Q4_0 / Q8_0 blocks 4h..4h+3, Q4_K chunks
// 2h and 2h+1, Q3_K elements 128h..128h+127; in every format it covers the
// slice's activation blocks 4h..4h+3.
template <int QT> struct WHalf;
template <> struct WHalf<Q4_0> { uint4 q[4]; uint2 dh; };
template <> struct WHalf<Q8_0> { uint4 q[8]; uint2 dh; };
template <> struct WHalf<Q4_K> { uint4 hdr; uint4 q[4]; };
template <> struct WHalf<Q3_K> { uint4 q[2]; uint4 hm[2]; uint4 hdr; };

__device__ __forceinline__ uint2 ldg8(const uint8_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }

template <int QT> __device__ __forceinline__ void load_half(const QView &W, int row, int s, int h, WHalf<QT> &r);
template <> __device__ __forceinline__ void load_half<Q4_0>(const QView &W, int row, int s, int h, WHalf<Q4_0> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 128 + 64 * h;
#pragma unroll
    for (int i = 0; i < 4; ++i) r.q[i] = ldg16(p + 16 * i);
    r.dh = ldg8(reinterpret_cast<const uint8_t *>(W.d + (long)row * W.dstride + s * 8 + 4 * h));
}
template <> __device__ __forceinline__ void load_half<Q8_0>(const QView &W, int row, int s, int h, WHalf<Q8_0> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 256 + 128 * h;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.q[i] = ldg16(p + 16 * i);
    r.dh = ldg8(reinterpret_cast<const uint8_t *>(W.d + (long)row * W.dstride + s * 8 + 4 * h));
}
template <> __device__ __forceinline__ void load_half<Q4_K>(const QView &W, int row, int s, int h, WHalf<Q4_K> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 144;
    r.hdr = ldg16(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) r.q[i] = ldg16(p + 16 + 64 * h + 16 * i);
}
template <> __device__ __forceinline__ void load_half<Q3_K>(const QView &W, int row, int s, int h, WHalf<Q3_K> &r) {
    const uint8_t *p = W.w + (long)row * W.wstride + (long)s * 112;
    r.q[0] = ldg16(p + 32 * h);
    r.q[1] = ldg16(p + 32 * h + 16);
    r.hm[0] = ldg16(p + 64);
    r.hm[1] = ldg16(p + 80);
    r.hdr = ldg16(p + 96);
}

// half-slice . x; xq / xf point at the slice's activation block 4h.
template <int QT> __device__ __forceinline__ float dot_half(const WHalf<QT> &w, int h, const XBlk *xq, const XF *xf);
template <> __device__ __forceinline__ float dot_half<Q4_0>(const WHalf<Q4_0> &w, int, const XBlk *xq, const XF *xf) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XBlk x = xq[b];
        const XF f = xf[b];
        const int dot = dot16_u(nib_lo(w.q[b]), x.h0, x.l0) + dot16_u(nib_hi(w.q[b]), x.h1, x.l1);
        const uint32_t dw = (b >> 1) ? w.dh.y : w.dh.x;
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (f.x * (float)dot - 8.0f * f.y);
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_half<Q8_0>(const WHalf<Q8_0> &w, int, const XBlk *xq, const XF *xf) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XBlk x = xq[b];
        const XF f = xf[b];
        const int dot = dot16_s(w.q[2 * b], x.h0, x.l0) + dot16_s(w.q[2 * b + 1], x.h1, x.l1);
        const uint32_t dw = (b >> 1) ? w.dh.y : w.dh.x;
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (f.x * (float)dot);
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_half<Q4_K>(const WHalf<Q4_K> &w, int h, const XBlk *xq, const XF *xf) {
    const float d = half_lo(w.hdr.x), dmin = half_hi(w.hdr.x);
    float acc = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * h + cc;
        int sc0, m0, sc1, m1;
        kq_scale_min(2 * c, w.hdr.y, w.hdr.z, w.hdr.w, sc0, m0);
        kq_scale_min(2 * c + 1, w.hdr.y, w.hdr.z, w.hdr.w, sc1, m1);
        const XBlk xa = xq[2 * cc], xb = xq[2 * cc + 1];
        const XF fa = xf[2 * cc], fb = xf[2 * cc + 1];
        const int da = dot16_u(nib_lo(w.q[2 * cc]), xa.h0, xa.l0) + dot16_u(nib_lo(w.q[2 * cc + 1]), xa.h1, xa.l1);
        const int db = dot16_u(nib_hi(w.q[2 * cc]), xb.h0, xb.l0) + dot16_u(nib_hi(w.q[2 * cc + 1]), xb.h1, xb.l1);
        acc += d * (float)sc0 * (fa.x * (float)da) - dmin * (float)m0 * fa.y;
        acc += d * (float)sc1 * (fb.x * (float)db) - dmin * (float)m1 * fb.y;
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_half<Q3_K>(const WHalf<Q3_K> &w, int h, const XBlk *xq, const XF *xf) {
    const float d = half_lo(w.hdr.w);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const XBlk x = xq[j];
        const XF f = xf[j];
        const int hs = 4 * h + j;
        int dots[2];
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            const uint4 q = w.q[lh], hm = w.hm[lh];
            uint4 vv;
            vv.x = ((q.x >> (2 * j)) & 0x03030303u) | (((hm.x >> hs) & 0x01010101u) << 2);
            vv.y = ((q.y >> (2 * j)) & 0x03030303u) | (((hm.y >> hs) & 0x01010101u) << 2);
            vv.z = ((q.z >> (2 * j)) & 0x03030303u) | (((hm.z >> hs) & 0x01010101u) << 2);
            vv.w = ((q.w >> (2 * j)) & 0x03030303u) | (((hm.w >> hs) & 0x01010101u) << 2);
            dots[lh] = dot16_u(vv, lh ? x.h1 : x.h0, lh ? x.l1 : x.l0);
        }
        const float s0 = d * (float)q3k_scale(8 * h + 2 * j, w.hdr.x, w.hdr.y, w.hdr.z);
        const float s1 = d * (float)q3k_scale(8 * h + 2 * j + 1, w.hdr.x, w.hdr.y, w.hdr.z);
        acc += s0 * (f.x * (float)dots[0] - 4.0f * f.z) + s1 * (f.x * (float)dots[1] - 4.0f * f.w);
    }
    return acc;
}
}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// ---- row tiles staged in shared memory by bulk copies ---------------------------------
// Each of 32 rows (one per lane) is copied with one cp.async.bulk into its own
// shared-memory row whose stride is an odd multiple of 16 bytes, so the 8
// lanes of a quarter-warp that read the same column of 8 different rows hit
// 8 distinct bank groups.
__host__ __device__ constexpr int bulk_stride(int bytes) { return ((bytes / 16) & 1) ? bytes : bytes + 16; }
__host__ __device__ constexpr int qscale_row_bytes(int qt, int K) { return (qt == Q4_0 || qt == Q8_0) ? K / 16 : 0; }
// bytes of shared memory for `rows` staged rows of a K-wide matrix
__host__ __device__ constexpr int tile_bytes(int qt, int K, int rows) {
    return rows * (bulk_stride((int)row_bytes_dev(qt, K)) +
                   (qscale_row_bytes(qt, K) ? bulk_stride(qscale_row_bytes(qt, K)) : 0));
}
// View of a staged tile: row r of the tile is row r of the view.
__device__ __forceinline__ QView tile_view(int qt, int K, uint8_t *base, int rows) {
    QView v;
    v.qt = qt;
    v.K = K;
    v.N = rows;
    v.wstride = bulk_stride((int)row_bytes_dev(qt, K));
    v.w = base;
    const int sb = qscale_row_bytes(qt, K);
    v.d = sb ? reinterpret_cast<const __half *>(base + rows * v.wstride) : nullptr;
    v.dstride = sb ? bulk_stride(sb) / 2 : 0;
    return v;
}
// Lane `lane` (< rows) copies global row `grow` of W into tile row `lane`.
// Returns the bytes it requested (to be announced with expect_tx).
__device__ __forceinline__ void tile_issue_row(const QView &W, long grow, uint8_t *base, int rows, int lane,
                                               uint64_t *bar) {
    const int wb = (int)row_bytes_dev(W.qt, W.K), sb = qscale_row_bytes(W.qt, W.K);
    const int ws = bulk_stride(wb);
    bulk_load(base + lane * ws, W.w + grow * W.wstride, wb, bar);
    if (sb) bulk_load(base + rows * ws + lane * bulk_stride(sb), W.d + grow * W.dstride, sb, bar);
}
__host__ __device__ constexpr int tile_row_tx(int qt, int K) { return (int)row_bytes_dev(qt, K) + qscale_row_bytes(qt, K); }
}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// ---- cooperative async staging (cp.async, 16 bytes per request) -----------------------
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(gsrc))
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// All threads of the CTA copy rows [grow0, grow0 + rows) of W (weights and,
// for Q4_0 / Q8_0, scale rows) into a tile laid out as tile_view expects
// (tile_rows rows, padded strides).  Consecutive threads copy consecutive
// 16-byte chunks of a row, so every warp reads 512 contiguous bytes.  The
// copies are asynchronous; cp_async_wait_all + __syncthreads complete them.
__device__ __forceinline__ void tile_cp_async(const QView &W, long grow0, int rows, uint8_t *base, int tile_rows) {
    const int wb = (int)row_bytes_dev(W.qt, W.K), sb = qscale_row_bytes(W.qt, W.K);
    const int ws = bulk_stride(wb), ds = sb ? bulk_stride(sb) : 0;
    const int cw = wb / 16, cs = sb / 16, per_row = cw + cs;
    const int total = rows * per_row;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int r = i / per_row;
        int c = i - r * per_row;
        if (c < cw) {
            cp_async16(base + r * ws + c * 16, W.w + (grow0 + r) * W.wstride + c * 16);
        } else {
            c -= cw;
            cp_async16(base + tile_rows * ws + r * ds + c * 16,
                       reinterpret_cast<const uint8_t *>(W.d + (grow0 + r) * W.dstride) + c * 16);
        }
    }
}
}  // namespace q
}  // namespace x100

namespace x100 {
namespace q {
// ---- row tiles staged by 2-D TMA boxes --------------------------------------------------
// A tile holds 32 consecutive rows as boxes of 32 rows x 128 bytes (4 KB each,
// 1024-byte aligned, 128-byte swizzle): weight boxes first, then scale boxes.
// The 16-byte chunk c of tile row r sits in box c / 8, line r, at chunk
// position (c % 8) ^ (r % 8) -- the TMA 128-byte swizzle, which also makes
// the 8 lanes of a quarter-warp (8 consecutive rows, same c) hit 8 distinct
// bank groups.
__host__ __device__ constexpr int tma_wboxes(int qt, int K) { return ((int)row_bytes_dev(qt, K) + 127) / 128; }
__host__ __device__ constexpr int tma_dboxes(int qt, int K) { return (qscale_row_bytes(qt, K) + 127) / 128; }
__host__ __device__ constexpr int tma_tile_bytes(int qt, int K) { return (tma_wboxes(qt, K) + tma_dboxes(qt, K)) * 4096; }

__device__ __forceinline__ const uint8_t *swz(const uint8_t *tile, int r, int c) {
    return tile + (c >> 3) * 4096 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}
// One thread: issue the boxes of rows [row0, row0 + 32) of one matrix into
// `tile`; returns the transaction bytes to announce on `bar`.
__device__ __forceinline__ uint32_t tma_issue_tile(const CUtensorMap *mw, const CUtensorMap *md, int qt, int K,
                                                   int row0, uint8_t *tile, uint64_t *bar) {
    const int nw = tma_wboxes(qt, K), nd = tma_dboxes(qt, K);
    for (int b = 0; b < nw; ++b) tma_load_2d(tile + b * 4096, mw, b * 128, row0, bar);
    for (int b = 0; b < nd; ++b) tma_load_2d(tile + (nw + b) * 4096, md, b * 128, row0, bar);
    return (uint32_t)(nw + nd) * 4096u;
}

// slice s of tile row r (swizzled) -> registers
template <int QT> __device__ __forceinline__ void load_slice_swz(const uint8_t *tile, int nwb, int r, int s, WSlice<QT> &w);
template <> __device__ __forceinline__ void load_slice_swz<Q4_0>(const uint8_t *tile, int nwb, int r, int s, WSlice<Q4_0> &w) {
#pragma unroll
    for (int i = 0; i < 8; ++i) w.q[i] = ld16(swz(tile, r, 8 * s + i));
    w.dh = ld16(swz(tile + nwb * 4096, r, s));
}
template <> __device__ __forceinline__ void load_slice_swz<Q8_0>(const uint8_t *tile, int nwb, int r, int s, WSlice<Q8_0> &w) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w.q[i] = ld16(swz(tile, r, 16 * s + i));
    w.dh = ld16(swz(tile + nwb * 4096, r, s));
}
template <> __device__ __forceinline__ void load_slice_swz<Q4_K>(const uint8_t *tile, int, int r, int s, WSlice<Q4_K> &w) {
    w.hdr = ld16(swz(tile, r, 9 * s));
#pragma unroll
    for (int i = 0; i < 8; ++i) w.q[i] = ld16(swz(tile, r, 9 * s + 1 + i));
}
template <> __device__ __forceinline__ void load_slice_swz<Q3_K>(const uint8_t *tile, int, int r, int s, WSlice<Q3_K> &w) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w.q[i] = ld16(swz(tile, r, 7 * s + i));
    w.hm[0] = ld16(swz(tile, r, 7 * s + 4));
    w.hm[1] = ld16(swz(tile, r, 7 * s + 5));
    w.hdr = ld16(swz(tile, r, 7 * s + 6));
}
}  // namespace q
}  // namespace x100
