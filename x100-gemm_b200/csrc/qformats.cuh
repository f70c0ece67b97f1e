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
