// qformats.cuh -- device-side block formats of the quantised decode path and
// the slice dot products shared by the dequant-GEMV and the MoE kernels.
//
// Weights keep the reference's GGUF block arithmetic (decoders restated from
// qwen_moe.c:162-165, qwen_moe_q3k.c:534-577, repack.cpp:222-283).  On the
// device every row is a sequence of 256-weight SLICES; a slice is an odd
// number of 16-byte chunks, so a lane reading chunk i of slice p and its
// neighbours reading chunk i of slices p+1..p+7 hit 8 distinct bank groups
// when a run of rows is staged contiguously in shared memory:
//   Q4_0  [8 fp16 block scales][8 x 16 B nibbles]          144 B =  9 chunks
//   Q8_0  [8 fp16 block scales][8 x 32 B int8]             272 B = 17 chunks
//   Q4_K  the native 144-byte superblock                    144 B =  9 chunks
//   Q3_K  [8 x 12 B values][scales 12][d 2][pad 2]          112 B =  7 chunks
//         (values v = q + 4 in 3 bits, packed for cheap unpacking: q3k_groups)
// A row of K weights holds ceil(K/256) slices; for Q4_0 / Q8_0 the blocks
// past K are zero (scale 0), so rows stay whole slices.  Rows are contiguous,
// so a run of rows is one contiguous byte range (one bulk copy).
//
// Activations: each 32-element block of the fp32 activation x is written as
// x ~= s * (256 h + l) with s = max|x|/32639 and int8 planes h, l (error at
// most s/2, ~1.5e-5 of the block maximum), plus exact fp32 sums of the block
// and of its two 16-element halves.  A slice's dot product with x is formed
// from int32 dp4a sums (exact) and one fp32 scale per block or sub-block.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace x100 {
namespace q {

enum { F32 = 0, Q4_0 = 2, Q8_0 = 8, Q3_K = 11, Q4_K = 12 };

// ---- layout ----------------------------------------------------------------------
__host__ __device__ constexpr int slice_bytes(int qt) {
    return qt == Q4_0 ? 144 : qt == Q8_0 ? 272 : qt == Q4_K ? 144 : qt == Q3_K ? 112 : 0;
}
__host__ __device__ constexpr int slices_per_row(int K) { return (K + 255) / 256; }
__host__ __device__ constexpr long row_bytes_dev(int qt, int K) { return (long)slices_per_row(K) * slice_bytes(qt); }

// One 32-element activation block: h and l planes (8 words each) and its
// fp32 terms {s, sum of the 32 elements, sum of elements 0-15, sum of 16-31}.
struct __align__(16) XB {
    uint4 h0, h1;   // h bytes of elements 0-15, 16-31
    uint4 l0, l1;   // l bytes of elements 0-15, 16-31
    float4 f;
};

constexpr int kXScale = 32639;   // |256 h + l| <= 32639 keeps h in [-127, 127]

// Prepared activations in shared memory.  A token's slice s holds its 8
// blocks as two halves of 4 (one per thread that dots the slice): half h at
// byte (s * 50 + h * 25) * 16.  The strides (50 = 2 mod 8 and 25 = 1 mod 8
// sixteen-byte chunks) put the 8 lanes of a quarter-warp -- four consecutive
// slices x two halves -- on 8 distinct bank groups.
constexpr int kXSlice = 800, kXHalf = 400;
__host__ __device__ constexpr int xbuf_bytes(int ns, int ntok) { return ntok * ns * kXSlice; }
struct XBuf {
    uint8_t *base;
    int ns;   // slices per token
    __device__ __forceinline__ const XB *half(int t, int s, int h) const {
        return reinterpret_cast<const XB *>(base + (t * ns + s) * kXSlice + h * kXHalf);
    }
    __device__ __forceinline__ XB *block(int t, int j) const {   // block j of token t
        return reinterpret_cast<XB *>(base + (t * ns + (j >> 3)) * kXSlice + ((j >> 2) & 1) * kXHalf + (j & 3) * 80);
    }
};
__device__ __forceinline__ XBuf xbuf_at(uint8_t *base, int ns) {
    XBuf x;
    x.base = base;
    x.ns = ns;
    return x;
}
// Block-major prepared activations for the tensor-core GEMV: block j of
// token t at (j * ntok + t) * 80 bytes, so the 8 tokens of an MMA column tile
// sit 80 bytes apart (8 distinct 16-byte bank groups for ldmatrix).
struct XBufBM {
    uint8_t *base;
    int ns;     // slices per token
    int ntok;   // tokens per block row (a multiple of 8)
    __device__ __forceinline__ XB *block(int t, int j) const {
        return reinterpret_cast<XB *>(base + ((long)j * ntok + t) * 80);
    }
};

// ---- integer dot products ----------------------------------------------------------
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
// Q3_K values of one 32-element block, v = q + 4 in [0, 7] (qwen_moe_q3k.c:
// 568-577), in three words W0, W1, W2 whose byte i holds element 4g + i of
// the block's 4-element groups g: bits 0-2 of W0 / W1 / W2 groups 0 / 2 / 4,
// bits 3-5 groups 1 / 3 / 5, bits 6-7 of W0 / W1 the low two bits of groups
// 6 / 7 and bits 6 / 7 of W2 their high bits.  a (groups 0-3) and b (4-7)
// come out as dp4a-ready bytes, four elements a word.
__device__ __forceinline__ void q3k_groups(uint32_t W0, uint32_t W1, uint32_t W2, uint4 &a, uint4 &b) {
    a.x = W0 & 0x07070707u;
    a.y = (W0 >> 3) & 0x07070707u;
    a.z = W1 & 0x07070707u;
    a.w = (W1 >> 3) & 0x07070707u;
    b.x = W2 & 0x07070707u;
    b.y = (W2 >> 3) & 0x07070707u;
    b.z = ((W0 >> 6) & 0x03030303u) | ((W2 >> 4) & 0x04040404u);
    b.w = ((W1 >> 6) & 0x03030303u) | ((W2 >> 5) & 0x04040404u);
}
// The unbiased 6-bit scales of sub-blocks 8h .. 8h+3 (c = 0) or 8h+4 ..
// 8h+7 (c = 1) as the four bytes of a word (0 .. 63; the scale is byte - 32)
// from the 12 scale bytes s0, s1, s2 (the packing of qwen_moe_q3k.c:560-564:
// low nibbles in bytes 0-7, high nibbles for scales 8-15, top two bits in
// bytes 8-11).
__device__ __forceinline__ uint32_t q3k_scale_word(int h, int c, uint32_t s0, uint32_t s1, uint32_t s2) {
    const uint32_t lo = ((c ? s1 : s0) >> (4 * h)) & 0x0F0F0F0Fu;
    const uint32_t hi = h ? (c ? s2 >> 2 : s2) : (c ? s2 << 2 : s2 << 4);
    return lo | (hi & 0x30303030u);
}

// ---- half a slice in registers ------------------------------------------------------
// Half h of a slice covers its activation blocks 4h .. 4h+3 (128 weights).
template <int QT> struct WHalf;
template <> struct WHalf<Q4_0> { uint4 dh; uint4 q[4]; };          // scales + blocks 4h..4h+3
template <> struct WHalf<Q8_0> { uint4 dh; uint4 q[8]; };
template <> struct WHalf<Q4_K> { uint4 hdr; uint4 q[4]; };         // header + qs chunks of pairs 2h, 2h+1
template <> struct WHalf<Q3_K> { uint4 v[3]; uint4 hdr; };        // blocks 4h..4h+3: 12 words; scales + d

__device__ __forceinline__ uint4 ld16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// p: the slice's first byte (16-byte aligned, any address space)
template <int QT> __device__ __forceinline__ void load_half(const uint8_t *p, int h, WHalf<QT> &w);
template <> __device__ __forceinline__ void load_half<Q4_0>(const uint8_t *p, int h, WHalf<Q4_0> &w) {
    w.dh = ld16(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) w.q[i] = ld16(p + 16 * (1 + 4 * h + i));
}
template <> __device__ __forceinline__ void load_half<Q8_0>(const uint8_t *p, int h, WHalf<Q8_0> &w) {
    w.dh = ld16(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) w.q[i] = ld16(p + 16 * (1 + 8 * h + i));
}
template <> __device__ __forceinline__ void load_half<Q4_K>(const uint8_t *p, int h, WHalf<Q4_K> &w) {
    w.hdr = ld16(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) w.q[i] = ld16(p + 16 * (1 + 4 * h + i));
}
template <> __device__ __forceinline__ void load_half<Q3_K>(const uint8_t *p, int h, WHalf<Q3_K> &w) {
#pragma unroll
    for (int i = 0; i < 3; ++i) w.v[i] = ld16(p + 48 * h + 16 * i);
    w.hdr = ld16(p + 96);
}

__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
__device__ __forceinline__ uint32_t u4_word(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// half h of a slice . x, with x pointing at the half's 4 activation blocks.
template <int QT> __device__ __forceinline__ float dot_half(const WHalf<QT> &w, int h, const XB *x);

template <> __device__ __forceinline__ float dot_half<Q4_0>(const WHalf<Q4_0> &w, int h, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XB &xb = x[b];
        const int dot = dot16_u(nib_lo(w.q[b]), xb.h0, xb.l0) + dot16_u(nib_hi(w.q[b]), xb.h1, xb.l1);
        const uint32_t dw = u4_word(w.dh, 2 * h + (b >> 1));
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (xb.f.x * (float)dot - 8.0f * xb.f.y);   // (nib - 8) * d, qwen_moe.c:164-165
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_half<Q8_0>(const WHalf<Q8_0> &w, int h, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XB &xb = x[b];
        const int dot = dot16_s(w.q[2 * b], xb.h0, xb.l0) + dot16_s(w.q[2 * b + 1], xb.h1, xb.l1);
        const uint32_t dw = u4_word(w.dh, 2 * h + (b >> 1));
        const float d = (b & 1) ? half_hi(dw) : half_lo(dw);
        acc += d * (xb.f.x * (float)dot);                    // q * d, qwen_moe.c:162-163
    }
    return acc;
}
// Q4_K: qs chunk v (pair c = v/2, part = v%2) holds elements 64c + 16part + i
// (low nibbles, sub-block 2c) and 64c + 32 + 16part + i (high nibbles,
// sub-block 2c + 1); half h holds pairs 2h and 2h+1.
template <> __device__ __forceinline__ float dot_half<Q4_K>(const WHalf<Q4_K> &w, int h, const XB *x) {
    const float d = half_lo(w.hdr.x), dmin = half_hi(w.hdr.x);
    float acc = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * h + cc;
        int sc0, m0, sc1, m1;
        kq_scale_min(2 * c, w.hdr.y, w.hdr.z, w.hdr.w, sc0, m0);
        kq_scale_min(2 * c + 1, w.hdr.y, w.hdr.z, w.hdr.w, sc1, m1);
        const XB &xa = x[2 * cc], &xb = x[2 * cc + 1];
        const int da = dot16_u(nib_lo(w.q[2 * cc]), xa.h0, xa.l0) + dot16_u(nib_lo(w.q[2 * cc + 1]), xa.h1, xa.l1);
        const int db = dot16_u(nib_hi(w.q[2 * cc]), xb.h0, xb.l0) + dot16_u(nib_hi(w.q[2 * cc + 1]), xb.h1, xb.l1);
        acc += d * (float)sc0 * (xa.f.x * (float)da) - dmin * (float)m0 * xa.f.y;
        acc += d * (float)sc1 * (xb.f.x * (float)db) - dmin * (float)m1 * xb.f.y;
    }
    return acc;
}
// Q3_K: block j of the half in words 3j .. 3j+2 of w.v (q3k_groups); its
// sub-blocks 8h + 2j + lh take scale byte 2j + lh of the half's two scale
// words.
__device__ __forceinline__ uint32_t q3k_w(const uint4 (&v)[3], int k) { return u4_word(v[k >> 2], k & 3); }
__device__ __forceinline__ float q3k_s(uint32_t scw, int byte, float d) {
    return d * (float)((int)((scw >> (8 * byte)) & 0xFFu) - 32);
}
template <> __device__ __forceinline__ float dot_half<Q3_K>(const WHalf<Q3_K> &w, int h, const XB *x) {
    const float d = half_lo(w.hdr.w);
    const uint32_t sc0 = q3k_scale_word(h, 0, w.hdr.x, w.hdr.y, w.hdr.z),
                   sc1 = q3k_scale_word(h, 1, w.hdr.x, w.hdr.y, w.hdr.z);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const XB &xb = x[j];
        uint4 a, b;
        q3k_groups(q3k_w(w.v, 3 * j), q3k_w(w.v, 3 * j + 1), q3k_w(w.v, 3 * j + 2), a, b);
        const int d0 = dot16_u(a, xb.h0, xb.l0), d1 = dot16_u(b, xb.h1, xb.l1);   // v in [0,7]; q = v - 4
        const uint32_t scw = j < 2 ? sc0 : sc1;
        const float s0 = q3k_s(scw, (2 * j) & 3, d), s1 = q3k_s(scw, (2 * j + 1) & 3, d);
        acc += s0 * (xb.f.x * (float)d0 - 4.0f * xb.f.z) + s1 * (xb.f.x * (float)d1 - 4.0f * xb.f.w);
    }
    return acc;
}

// ---- half a slice unpacked once for many tokens ----------------------------------------------
// UHalf holds a half slice with its weight bytes already in dp4a form and
// its scales decoded, so a kernel that dots the same weights with several
// tokens pays the unpacking once; dot_uhalf(u, x) evaluates exactly the
// expression of dot_half(w, h, x) (same operations, same order).
template <int QT> struct UHalf;
template <> struct UHalf<Q4_0> { uint4 lo[4], hi[4]; float d[4]; };
template <> struct UHalf<Q8_0> { uint4 q[8]; float d[4]; };
template <> struct UHalf<Q4_K> { uint4 lo[4], hi[4]; float ds[4], dm[4]; };   // sub-blocks 4h .. 4h+3
template <> struct UHalf<Q3_K> { uint4 v[4][2]; float s[4][2]; };             // [j][lh]

template <int QT> __device__ __forceinline__ void unpack_half(const WHalf<QT> &w, int h, UHalf<QT> &u);
template <> __device__ __forceinline__ void unpack_half<Q4_0>(const WHalf<Q4_0> &w, int h, UHalf<Q4_0> &u) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        u.lo[b] = nib_lo(w.q[b]);
        u.hi[b] = nib_hi(w.q[b]);
        const uint32_t dw = u4_word(w.dh, 2 * h + (b >> 1));
        u.d[b] = (b & 1) ? half_hi(dw) : half_lo(dw);
    }
}
template <> __device__ __forceinline__ void unpack_half<Q8_0>(const WHalf<Q8_0> &w, int h, UHalf<Q8_0> &u) {
#pragma unroll
    for (int i = 0; i < 8; ++i) u.q[i] = w.q[i];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const uint32_t dw = u4_word(w.dh, 2 * h + (b >> 1));
        u.d[b] = (b & 1) ? half_hi(dw) : half_lo(dw);
    }
}
template <> __device__ __forceinline__ void unpack_half<Q4_K>(const WHalf<Q4_K> &w, int h, UHalf<Q4_K> &u) {
    const float d = half_lo(w.hdr.x), dmin = half_hi(w.hdr.x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        u.lo[i] = nib_lo(w.q[i]);
        u.hi[i] = nib_hi(w.q[i]);
    }
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * h + cc;
        int sc0, m0, sc1, m1;
        kq_scale_min(2 * c, w.hdr.y, w.hdr.z, w.hdr.w, sc0, m0);
        kq_scale_min(2 * c + 1, w.hdr.y, w.hdr.z, w.hdr.w, sc1, m1);
        u.ds[2 * cc] = d * (float)sc0;
        u.dm[2 * cc] = dmin * (float)m0;
        u.ds[2 * cc + 1] = d * (float)sc1;
        u.dm[2 * cc + 1] = dmin * (float)m1;
    }
}
template <> __device__ __forceinline__ void unpack_half<Q3_K>(const WHalf<Q3_K> &w, int h, UHalf<Q3_K> &u) {
    const float d = half_lo(w.hdr.w);
    const uint32_t sc0 = q3k_scale_word(h, 0, w.hdr.x, w.hdr.y, w.hdr.z),
                   sc1 = q3k_scale_word(h, 1, w.hdr.x, w.hdr.y, w.hdr.z);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        q3k_groups(q3k_w(w.v, 3 * j), q3k_w(w.v, 3 * j + 1), q3k_w(w.v, 3 * j + 2), u.v[j][0], u.v[j][1]);
        const uint32_t scw = j < 2 ? sc0 : sc1;
        u.s[j][0] = q3k_s(scw, (2 * j) & 3, d);
        u.s[j][1] = q3k_s(scw, (2 * j + 1) & 3, d);
    }
}

template <int QT> __device__ __forceinline__ float dot_uhalf(const UHalf<QT> &u, const XB *x);
template <> __device__ __forceinline__ float dot_uhalf<Q4_0>(const UHalf<Q4_0> &u, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XB &xb = x[b];
        const int dot = dot16_u(u.lo[b], xb.h0, xb.l0) + dot16_u(u.hi[b], xb.h1, xb.l1);
        acc += u.d[b] * (xb.f.x * (float)dot - 8.0f * xb.f.y);
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_uhalf<Q8_0>(const UHalf<Q8_0> &u, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const XB &xb = x[b];
        const int dot = dot16_s(u.q[2 * b], xb.h0, xb.l0) + dot16_s(u.q[2 * b + 1], xb.h1, xb.l1);
        acc += u.d[b] * (xb.f.x * (float)dot);
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_uhalf<Q4_K>(const UHalf<Q4_K> &u, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const XB &xa = x[2 * cc], &xb = x[2 * cc + 1];
        const int da = dot16_u(u.lo[2 * cc], xa.h0, xa.l0) + dot16_u(u.lo[2 * cc + 1], xa.h1, xa.l1);
        const int db = dot16_u(u.hi[2 * cc], xb.h0, xb.l0) + dot16_u(u.hi[2 * cc + 1], xb.h1, xb.l1);
        acc += u.ds[2 * cc] * (xa.f.x * (float)da) - u.dm[2 * cc] * xa.f.y;
        acc += u.ds[2 * cc + 1] * (xb.f.x * (float)db) - u.dm[2 * cc + 1] * xb.f.y;
    }
    return acc;
}
template <> __device__ __forceinline__ float dot_uhalf<Q3_K>(const UHalf<Q3_K> &u, const XB *x) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const XB &xb = x[j];
        const int d0 = dot16_u(u.v[j][0], xb.h0, xb.l0), d1 = dot16_u(u.v[j][1], xb.h1, xb.l1);
        acc += u.s[j][0] * (xb.f.x * (float)d0 - 4.0f * xb.f.z) + u.s[j][1] * (xb.f.x * (float)d1 - 4.0f * xb.f.w);
    }
    return acc;
}

// ---- activation preparation -----------------------------------------------------------
// Eight consecutive threads (t = lane % 8) convert one 32-element block, held
// as one float4 per thread, into *o.  Every lane of the warp calls it
// together (it shuffles across the warp); lanes whose group has no block pass
// active = false and write nothing.  The scale s = amax / 32639 is formed as
// amax * (1/32639) and the quantiser's 1/s by a fast reciprocal: any x = s *
// X with |X| <= 32639 is represented to within s/2 + 1e-6 amax.
__device__ __forceinline__ void xprep_vals(const float4 v, XB *o, int t, bool active) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    float s16 = (v.x + v.y) + (v.z + v.w);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
    s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
    const float other16 = __shfl_xor_sync(0xffffffffu, s16, 4);
    const float s32 = s16 + other16;
    const float s = amax * (1.0f / (float)kXScale);
    const float inv = amax > 0.f ? __fdividef((float)kXScale, amax) : 0.f;
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
    reinterpret_cast<uint32_t *>(&o->h0)[t] = hw;
    reinterpret_cast<uint32_t *>(&o->l0)[t] = lw;
    // lanes 0-3 hold elements 0-15 (s16 = their sum), lanes 4-7 elements 16-31
    if (t == 0) o->f = make_float4(s, s32, s16, other16);
}

// "A8" preparation: the activations quantised as the reference packs them
// for its IME kernels, held in the same XB form (h = q, l = 0, s = scale /
// 256, so 256 s h = scale q exactly and the dot products need no change;
// the sums are scale * the integer sums of q).  xprep_vals_i8 is pack_A_i8
// (qwen_moe_q3k.c:420-426) for one 32-element block held as in xprep_vals:
// scale = max(|x|, 1e-6) / 127, q = round-to-nearest-even(x * (1 / scale))
// clamped to int8, both divisions correctly rounded.
__device__ __forceinline__ void xprep_vals_i8(const float4 v, XB *o, int t, bool active) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
    amax = fmaxf(amax, 1e-6f);
    const float scale = __fdiv_rn(amax, 127.0f);
    const float inv = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
    const float e[4] = {v.x, v.y, v.z, v.w};
    uint32_t hw = 0;
    int s4 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int q = max(-128, min(127, __float2int_rn(__fmul_rn(e[k], inv))));
        hw |= (uint32_t)(q & 0xFF) << (8 * k);
        s4 += q;
    }
    int s16 = s4 + __shfl_xor_sync(0xffffffffu, s4, 1);
    s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
    const int other16 = __shfl_xor_sync(0xffffffffu, s16, 4);
    if (!active) return;
    reinterpret_cast<uint32_t *>(&o->h0)[t] = hw;
    reinterpret_cast<uint32_t *>(&o->l0)[t] = 0u;
    if (t == 0) o->f = make_float4(scale * (1.0f / 256.0f), scale * (float)(s16 + other16), scale * (float)s16,
                                   scale * (float)other16);
}

// pack_A_q3k (qwen_moe_q3k.c:613-623) into XB blocks: one warp per
// 256-element superblock of a row, 8 elements per lane; scale = max|x| / 127
// over the superblock, q = roundf(x * (1 / scale)) clamped to int8.  K must be
// a multiple of 256.
template <class RowPtr, class XBT>
__device__ __forceinline__ void xprep_rows_q3k8(RowPtr row, int K, int nrows, const XBT &xb) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int nsb = K / 256, total = nrows * nsb, u4 = lane & 3;
    for (int u = warp; u < total; u += nwarps) {   // warp-uniform
        const int c = nrows == 1 ? 0 : u / nsb, sb = u - c * nsb;
        const float4 *a = reinterpret_cast<const float4 *>(row(c) + sb * 256 + lane * 8);
        const float4 p0 = __ldcg(a), p1 = __ldcg(a + 1);
        const float e[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(e[k]));
#pragma unroll
        for (int m = 16; m; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        const float scale = __fdiv_rn(amax, 127.0f);
        const float rep = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
        uint32_t w0 = 0, w1 = 0;
        int s8 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = max(-128, min(127, (int)roundf(__fmul_rn(e[k], rep))));
            (k < 4 ? w0 : w1) |= (uint32_t)(q & 0xFF) << (8 * (k & 3));
            s8 += q;
        }
        const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);   // lanes 4j, 4j+1: elements 0-15 of block j
        const int s16b = __shfl_xor_sync(0xffffffffu, s16, 2);       // lanes 4j+2, 4j+3: elements 16-31
        XB *o = xb.block(c, sb * 8 + (lane >> 2));
        uint32_t *h = reinterpret_cast<uint32_t *>(&o->h0), *l = reinterpret_cast<uint32_t *>(&o->l0);
        h[2 * u4] = w0;
        h[2 * u4 + 1] = w1;
        l[2 * u4] = 0u;
        l[2 * u4 + 1] = 0u;
        if (u4 == 0) o->f = make_float4(scale * (1.0f / 256.0f), scale * (float)(s16 + s16b), scale * (float)s16,
                                        scale * (float)s16b);
    }
}

// fp32 -> fp16 bits by truncation, the conversion of the reference's int4
// "HP" engine (qwen_moe_hp.c:71-79): mantissa bits below the fp16 precision
// are dropped, subnormal results shifted out, overflow to infinity.
__host__ __device__ __forceinline__ uint16_t f32_to_f16_trunc(float f) {
#ifdef __CUDA_ARCH__
    const uint32_t x = __float_as_uint(f);
#else
    uint32_t x;
    memcpy(&x, &f, 4);
#endif
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int exp = (int)((x >> 23) & 0xffu) - 127 + 15;
    uint32_t mant = x & 0x7fffffu;
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        return (uint16_t)(sign | (mant >> (14 - exp)));
    }
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

// The scales of one 256-element record of pack_A_hp (qwen_moe_hp.c:131-180)
// for the calling lane, whose 8 elements e[] are elements 8 lane .. 8 lane+7
// (sub-block lane / 4): every lane of the warp calls it together.
// st = max(|x|, 1e-6) / 127 over the sub-block; avg = the in-order sum of the
// 8 st / 8; ssub / blk = the truncated fp16 of st / avg and of avg; rep =
// 1 / st; all divisions correctly rounded, as the reference's scalar C.
struct HpScales { float st, rep; uint16_t ssub, blk; };
__device__ __forceinline__ HpScales hp_scales(const float (&e)[8]) {
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(e[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    amax = fmaxf(amax, 1e-6f);
    HpScales r;
    r.st = __fdiv_rn(amax, 127.0f);
    float avg = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) avg = __fadd_rn(avg, __shfl_sync(0xffffffffu, r.st, 4 * kk));
    avg = __fdiv_rn(avg, 8.0f);
    const float fac = avg != 0.f ? __fdiv_rn(1.0f, avg) : 0.f;
    r.rep = r.st != 0.f ? __fdiv_rn(1.0f, r.st) : 0.f;
    r.ssub = f32_to_f16_trunc(__fmul_rn(r.st, fac));
    r.blk = f32_to_f16_trunc(avg);
    return r;
}
// q = lrint(x * rep) clamped to int8 (round to nearest even)
__device__ __forceinline__ int hp_quant(float x, float rep) {
    return max(-128, min(127, __float2int_rn(__fmul_rn(x, rep))));
}

// pack_A_hp into XB blocks (the int4 "HP" engine's activations, used with
// Q4_0 weights): one warp per 256-element record of a row, 8 elements per
// lane.  Each 32-element block holds q and the effective scale the HP
// numerics give it, fp16(sub-scale) * fp16(average) (one fp32 product).
// K must be a multiple of 256.
template <class RowPtr, class XBT>
__device__ __forceinline__ void xprep_rows_hp8(RowPtr row, int K, int nrows, const XBT &xb) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int nsb = K / 256, total = nrows * nsb, u4 = lane & 3;
    for (int u = warp; u < total; u += nwarps) {   // warp-uniform
        const int c = nrows == 1 ? 0 : u / nsb, sb = u - c * nsb;
        const float4 *a = reinterpret_cast<const float4 *>(row(c) + sb * 256 + lane * 8);
        const float4 p0 = __ldcg(a), p1 = __ldcg(a + 1);
        const float e[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const HpScales hs = hp_scales(e);
        const float eff = __fmul_rn(__half2float(__ushort_as_half(hs.ssub)), __half2float(__ushort_as_half(hs.blk)));
        uint32_t w0 = 0, w1 = 0;
        int s8 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = hp_quant(e[k], hs.rep);
            (k < 4 ? w0 : w1) |= (uint32_t)(q & 0xFF) << (8 * (k & 3));
            s8 += q;
        }
        const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);   // lanes 4j, 4j+1: elements 0-15 of block j
        const int s16b = __shfl_xor_sync(0xffffffffu, s16, 2);       // lanes 4j+2, 4j+3: elements 16-31
        XB *o = xb.block(c, sb * 8 + (lane >> 2));
        uint32_t *h = reinterpret_cast<uint32_t *>(&o->h0), *l = reinterpret_cast<uint32_t *>(&o->l0);
        h[2 * u4] = w0;
        h[2 * u4 + 1] = w1;
        l[2 * u4] = 0u;
        l[2 * u4 + 1] = 0u;
        if (u4 == 0) o->f = make_float4(eff * (1.0f / 256.0f), eff * (float)(s16 + s16b), eff * (float)s16,
                                        eff * (float)s16b);
    }
}

// The whole CTA prepares `nrows` activation rows row(c)[0 .. K) into xb as
// tokens 0 .. nrows-1 (blocks past K, up to the slice boundary, are zero).
// A warp converts 4 blocks at a time; each pass first issues up to PF (kXPF
// by default) such groups of 16-byte loads per warp and only then converts
// them, so a pass costs one memory round trip.  Groups past the end are skipped whole (the
// test is warp-uniform, which keeps the shuffles legal).  The loads go
// through L2: the rows may have been written by other CTAs of the grid.
//
// RMS-norm folding: with `nw` set, the values prepared are x[k] * nw[k], and
// each 8-lane group adds the sum of squares of the raw x of its blocks into
// ss[(warp * 4 + group) * kSsTok + token] (kSsTok tokens per slot; one writer
// per slot, so no atomics).  The caller sums the slots in a fixed order into
// s = 1 / sqrt(mean(x^2) + eps) and scales its dot products by s, which gives
// W . rmsnorm(x) = s * (W . (x * nw)) without a second pass over x.
constexpr int kXPF = 4;
constexpr int kSsTok = 16;
template <int PF = kXPF, bool I8 = false, class RowPtr, class XBT>
__device__ __forceinline__ void xprep_rows(RowPtr row, int K, int nrows, const XBT &xb,
                                           const float *__restrict__ nw = nullptr, float *ss = nullptr) {
    const int nxb = xb.ns * 8, kb = K / 32;
    const int total = nrows * nxb;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 3, t = lane & 7;
    if (nw && t == 0)
        for (int c = 0; c < nrows; ++c) ss[(warp * 4 + g) * kSsTok + c] = 0.f;
    for (int base = 0; base < total; base += nwarps * 4 * PF) {
        float4 v[PF];
#pragma unroll
        for (int i = 0; i < PF; ++i) {
            const int blk = base + (i * nwarps + warp) * 4 + g;
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (blk < total) {
                const int c = nrows == 1 ? 0 : blk / nxb, j = blk - c * nxb;
                if (j < kb) v[i] = __ldcg(reinterpret_cast<const float4 *>(row(c) + j * 32) + t);
            }
        }
#pragma unroll
        for (int i = 0; i < PF; ++i) {
            const int blk0 = base + (i * nwarps + warp) * 4;
            if (blk0 < total) {
                const int blk = blk0 + g;
                const bool active = blk < total;
                const int c = !active || nrows == 1 ? 0 : blk / nxb, j = active ? blk - c * nxb : 0;
                float4 x = v[i];
                if (nw) {
                    float q = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
                    q += __shfl_xor_sync(0xffffffffu, q, 1);
                    q += __shfl_xor_sync(0xffffffffu, q, 2);
                    q += __shfl_xor_sync(0xffffffffu, q, 4);
                    if (active && t == 0) ss[(warp * 4 + g) * kSsTok + c] += q;
                    if (active && j < kb) {
                        const float4 w4 = __ldg(reinterpret_cast<const float4 *>(nw + j * 32) + t);
                        x = make_float4(x.x * w4.x, x.y * w4.y, x.z * w4.z, x.w * w4.w);
                    }
                }
                if constexpr (I8) xprep_vals_i8(x, xb.block(c, j), t, active);
                else xprep_vals(x, xb.block(c, j), t, active);
            }
        }
    }
}

// Activation preparation of a GEMV: a8 = 0 the exact 16-bit split
// (xprep_rows), 1 pack_A_i8 per 32 values, 2 pack_A_q3k per 256 values,
// 3 pack_A_hp per 256 values (no RMS-norm folding in the A8 forms).
template <class RowPtr, class XBT>
__device__ __forceinline__ void xprep_gemv(int a8, RowPtr row, int K, int nrows, const XBT &xb, const float *nw,
                                           float *ss) {
    if (a8 == 3) xprep_rows_hp8(row, K, nrows, xb);
    else if (a8 == 2) xprep_rows_q3k8(row, K, nrows, xb);
    else if (a8 == 1) xprep_rows<kXPF, true>(row, K, nrows, xb);
    else xprep_rows(row, K, nrows, xb, nw, ss);
}

// 1 / sqrt(mean of squares + eps) of token c from the slots xprep_rows filled
// (nslots = 4 * warps of the CTA), summed in slot order.
__device__ __forceinline__ float rms_scale(const float *ss, int nslots, int c, int K, float eps) {
    float s = 0.f;
    for (int i = 0; i < nslots; ++i) s += ss[i * kSsTok + c];
    return 1.0f / sqrtf(s / (float)K + eps);
}

// ---- programmatic dependent launch -------------------------------------------------
// Kernels launched with the programmatic-serialization attribute may start
// while the previous kernel of the stream is still running.  They first issue
// loads that do not depend on it (weights), then allow their own dependents
// to launch, and wait for the previous grid (its writes become visible)
// before reading its outputs.  Without the attribute both calls are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- staging rows in shared memory -------------------------------------------------------
// One thread: copy `bytes` (a multiple of 16) from global `src` to shared
// `dst` (both 16-byte aligned) in bulk copies of at most kBulkChunk bytes,
// completing as transaction bytes on `bar`.  The caller announces the bytes.
constexpr uint32_t kBulkChunk = 65536;
__device__ __forceinline__ void stage_bytes(uint8_t *dst, const uint8_t *src, uint32_t bytes, uint64_t *bar) {
    for (uint32_t o = 0; o < bytes; o += kBulkChunk) {
        const uint32_t n = bytes - o < kBulkChunk ? bytes - o : kBulkChunk;
        bulk_load(dst + o, src + o, n, bar);
    }
}

}  // namespace q
}  // namespace x100
