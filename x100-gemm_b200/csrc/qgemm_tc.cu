// qgemm_tc.cu -- many-token quantised linear layers on the 5th-generation
// tensor cores: Y[t][n] = sum_k W[n][k] X[t][k] with W block-quantised (Q4_0,
// Q8_0, Q4_K, Q3_K) and many tokens t sharing each weight row -- the linear
// layers of a prefill chunk (the reference's prefill_chunk4 and the vendor
// backend's grouped MUL_MAT_ID, qwen_moe_hp.c:1748-1858,
// reference/spacemit-backend/ime.cpp:543-700), where one weight stream serves
// up to 128 tokens.
//
// Work items: (group g, weight row tile of 128 rows, token tile of up to 128
// tokens).  A dense layer is one group; the experts of a MoE layer are one
// group each, their tokens a contiguous run of the activation rows (the
// routing sorted them by expert).  One CTA per SM walks items round-robin.
//
// Per item the K dimension is walked one 256-weight slice at a time:
//   warp 0    TMA producer: the 128 rows' raw slice bytes (one 2-D box of the
//             weight matrix, no swizzle) into a raw stage, and per 64-element
//             piece the token tile's activation planes X_hi / X_lo (2-D boxes
//             of 64 fp16 x tokens, 128-byte swizzle) into an A/B stage.
//   warps 2-9 dequantise: each thread owns one weight row and one half of
//             every 64-element piece; it decodes its 32 weights from the raw
//             stage in fp32 exactly as the scalar decoders do
//             (qwen_moe.c:162-165, qwen_moe_q3k.c:534-577, repack.cpp:222-283)
//             and writes W_hi = fp16(w) and W_lo = fp16(w - W_hi) into the A
//             planes in the 128-byte-swizzled K-major layout the MMA reads.
//   warp 1    MMA issuer: per 16 elements of K, two tcgen05.mma kind::f16
//             (fp32 accumulate in TMEM): W_hi against [X_hi | X_lo] (the two
//             planes sit one after the other, so one instruction with N =
//             64 + n tokens forms both products in separate column ranges),
//             then W_lo against X_hi into the first range; the epilogue adds
//             the ranges.  Weights and activations each carried to ~22 bits,
//             the products agree with the fp32 dequant-GEMV to ~1e-6 relative
//             (the dropped W_lo.X_lo term is ~2^-22 of a product).
//   warps 2-9 epilogue, once the item's MMAs are done: TMEM -> registers ->
//             out (store, += residual, or scattered to the rows pair_at names).
// Every wait is bounded; on a timeout the kernel records X100_E_TIMEOUT,
// drains its copies and MMAs in flight, frees TMEM and returns.
#include <cuda_fp16.h>

#include <algorithm>

#include "../../include/x100_gemm.h"
#include "ptx.cuh"
#include "qgemm.h"

namespace x100 {
namespace q {

constexpr int QG_ROWS = 128;                    // weight rows per item = TMEM lanes
constexpr int QG_NT = 64;                       // tokens per item (MMA N, at most)
constexpr int QG_NT_SMALL = 32;                 // box of the small token tiles
constexpr int QG_A_STAGES = 2;                  // dequantised weight planes
constexpr int QG_RAW_STAGES = 2;                // raw weight slices
constexpr int QG_DQ_WARPS = 16;
constexpr int QG_THREADS = 64 + 32 * QG_DQ_WARPS;
constexpr int QG_PLANE_A = QG_ROWS * 128;       // 128 rows x 64 fp16
constexpr int QG_PLANE_B = QG_NT * 128;         // 64 tokens x 64 fp16
constexpr int QG_A_BYTES = 2 * QG_PLANE_A;
constexpr int QG_B_BYTES = 2 * QG_PLANE_B;
constexpr int QG_MAX_GROUPS = 256;
constexpr uint32_t QG_TMEM_COLS = 2 * QG_NT;   // [W.X_hi | W_hi.X_lo]
constexpr unsigned long long kQgDrainNs = 100000000ull;
constexpr int QG_SMEM_CAP = 227 * 1024;

// Shared-memory plan of one weight format: the activation ring is as deep as
// the budget allows after the dequantised-weight and raw-slice rings.
struct QgLayout {
    int sb, raw_bytes, b_stages, a_off, b_off, raw_off, bar_off, pfx_off, smem;
};
__host__ __device__ constexpr QgLayout qg_layout(int qt) {
    QgLayout L{};
    L.sb = slice_bytes(qt);
    L.raw_bytes = (QG_ROWS * L.sb + 1023) / 1024 * 1024;
    const int fixed = QG_A_STAGES * QG_A_BYTES + QG_RAW_STAGES * L.raw_bytes + 4096 + 1024;
    L.b_stages = (QG_SMEM_CAP - fixed) / QG_B_BYTES;
    L.b_stages = L.b_stages > 8 ? 8 : L.b_stages;
    L.a_off = 0;
    L.b_off = QG_A_STAGES * QG_A_BYTES;
    L.raw_off = L.b_off + L.b_stages * QG_B_BYTES;
    L.bar_off = L.raw_off + QG_RAW_STAGES * L.raw_bytes;
    L.pfx_off = L.bar_off + 64 * 8;
    L.smem = L.pfx_off + 2 * (QG_MAX_GROUPS + 1) * 4 + 1024;
    return L;
}

struct QgParams {
    int nmat, n_rows, ns, ngroups, T, mode;
    const int *cnt;
    float *out;
    long ldo;
    const int *pair_at;
    int *status;
};

// ---- one item -------------------------------------------------------------------------
struct QgItem {
    int g, mat, rtile, tok0, nt;
};
// Item i of the list the prefix arrays describe: tiles[g] items before group
// g, tok[g] token rows before it; within a group, token tiles vary fastest
// (consecutive items share weight rows, so a second CTA reads them from L2).
__device__ __forceinline__ QgItem qg_item(int i, const int *tiles, const int *tok, int ngroups, int rt_per_mat,
                                          const int *cnt, int T) {
    int lo = 0, hi = ngroups - 1;
    while (lo < hi) {   // last group whose first item is <= i
        const int mid = (lo + hi + 1) >> 1;
        if (tiles[mid] <= i) lo = mid;
        else hi = mid - 1;
    }
    QgItem it;
    it.g = lo;
    const int c = cnt ? __ldcg(cnt + lo) : T;
    const int tt_n = (c + QG_NT - 1) / QG_NT;
    const int local = i - tiles[lo];
    const int rt = local / tt_n, tt = local - rt * tt_n;
    it.mat = rt / rt_per_mat;
    it.rtile = rt - it.mat * rt_per_mat;
    it.tok0 = tok[lo] + tt * QG_NT;
    it.nt = min(QG_NT, c - tt * QG_NT);
    return it;
}

// ---- dequantisation: 16 weights (elements 16 q16 .. 16 q16 + 15 of 32-element
// block b of a slice) as 8 fp16 pairs hi / lo, element order ---------------------------
__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ __half2 u2h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }
__device__ __forceinline__ uint32_t h22u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(unsigned short b) { return u2h2((uint32_t)b | ((uint32_t)b << 16)); }

// Bytes 0-1 (sel 0) or 2-3 (sel 1) of a word of unsigned bytes v (< 256) as
// the fp16 pair {1024 + v0, 1024 + v1}: the byte becomes the mantissa of a
// half with exponent 10, exact.
__device__ __forceinline__ __half2 bytes_h2(uint32_t w, int sel) {
    return u2h2(__byte_perm(w, 0x64646464u, sel ? 0x4342u : 0x4140u));
}
// hi = fp16(s * q), lo = fp16(s * q - hi) for two weights q (small integers,
// exact in fp16) under an fp16 scale s: the product has at most 19
// significant bits, the fma returns its exact remainder, so hi + lo = s * q.
__device__ __forceinline__ void split_h2(__half2 s, __half2 q, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __hmul2(s, q);
    hi = h22u(h);
    lo = h22u(__hfma2(s, q, __hneg2(h)));
}

// A thread's raw bytes of one slice, loaded once per slice (the bytes its 16
// weights of each of the slice's four 64-element pieces come from).  Thread
// quarter q4 owns elements 16 q4 .. 16 q4 + 15 of every piece, i.e. half
// q4 & 1 of 32-element block 2 j + (q4 >> 1) of piece j.
template <int QT> struct SliceRegs;
template <> struct SliceRegs<Q8_0> { uint4 hd; };                 // the 8 block scales
template <> struct SliceRegs<Q4_0> { uint4 hd; };
template <> struct SliceRegs<Q4_K> { uint4 hdr; };                // d, dmin, scales / mins
template <> struct SliceRegs<Q3_K> { uint32_t sc; float d; };   // the thread's scale byte of each piece, d

template <int QT> __device__ __forceinline__ void load_slice(const uint8_t *sl, int q4, SliceRegs<QT> &R);
template <> __device__ __forceinline__ void load_slice<Q8_0>(const uint8_t *sl, int, SliceRegs<Q8_0> &R) { R.hd = ld16(sl); }
template <> __device__ __forceinline__ void load_slice<Q4_0>(const uint8_t *sl, int, SliceRegs<Q4_0> &R) { R.hd = ld16(sl); }
template <> __device__ __forceinline__ void load_slice<Q4_K>(const uint8_t *sl, int, SliceRegs<Q4_K> &R) { R.hdr = ld16(sl); }
template <> __device__ __forceinline__ void load_slice<Q3_K>(const uint8_t *sl, int q4, SliceRegs<Q3_K> &R) {
    const uint4 hdr = ld16(sl + 96);
    // piece j's sub-block for quarter q4 is 4 j + q4: byte q4 of scale word j
    R.sc = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        R.sc |= ((q3k_scale_word(j >> 1, j & 1, hdr.x, hdr.y, hdr.z) >> (8 * q4)) & 0xFFu) << (8 * j);
    R.d = h2f_lo(hdr.w);
}

// The thread's 16 weights of piece j as 8 fp16 pairs hi / lo, element order.
template <int QT>
__device__ __forceinline__ void dq16(const SliceRegs<QT> &R, const uint8_t *sl, int j, int q4, uint32_t (&hv)[8],
                                     uint32_t (&lv)[8]);
// Q8_0 slice: [8 fp16 d][8 x 32 int8]; w = d * q (qwen_moe.c:162-163)
template <>
__device__ __forceinline__ void dq16<Q8_0>(const SliceRegs<Q8_0> &R, const uint8_t *sl, int j, int q4, uint32_t (&hv)[8],
                                           uint32_t (&lv)[8]) {
    const int b = 2 * j + (q4 >> 1), q16 = q4 & 1;
    const uint32_t dw = word_of(R.hd, b >> 1);
    const __half2 d2 = bits_h2((unsigned short)((b & 1) ? dw >> 16 : dw & 0xFFFF));
    const uint4 q = ld16(sl + 16 + 32 * b + 16 * q16);
    const __half2 off = __float2half2_rn(1152.0f);   // 1024 + 128: the bytes carry q + 128
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t u = word_of(q, wi) ^ 0x80808080u;
#pragma unroll
        for (int sel = 0; sel < 2; ++sel) split_h2(d2, __hsub2(bytes_h2(u, sel), off), hv[2 * wi + sel], lv[2 * wi + sel]);
    }
}
// Q4_0 slice: [8 fp16 d][8 x 16 B nibbles]; element i < 16 the low nibble of
// byte i, i >= 16 the high nibble of byte i - 16; w = (nib - 8) * d
// (qwen_moe.c:164-165)
template <>
__device__ __forceinline__ void dq16<Q4_0>(const SliceRegs<Q4_0> &R, const uint8_t *sl, int j, int q4, uint32_t (&hv)[8],
                                           uint32_t (&lv)[8]) {
    const int b = 2 * j + (q4 >> 1), q16 = q4 & 1;
    const uint32_t dw = word_of(R.hd, b >> 1);
    const __half2 d2 = bits_h2((unsigned short)((b & 1) ? dw >> 16 : dw & 0xFFFF));
    const uint4 q = ld16(sl + 16 + 16 * b);
    const __half2 off = __float2half2_rn(1032.0f);   // 1024 + 8: nib - 8
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t w = word_of(q, wi);
        const uint32_t nib = q16 ? (w >> 4) & 0x0F0F0F0Fu : w & 0x0F0F0F0Fu;
#pragma unroll
        for (int sel = 0; sel < 2; ++sel) split_h2(d2, __hsub2(bytes_h2(nib, sel), off), hv[2 * wi + sel], lv[2 * wi + sel]);
    }
}
// Q3_K slice: [8 x 12 B values][scales 12][d 2][pad 2]; block b's values v =
// q + 4 in the three words at 12 b (q3k_groups), sub-block 2 b + q16 with
// scale sc - 32; w = d * (sc - 32) * q (qwen_moe_q3k.c:557-577).  The scale
// (17 bits, exact in fp32) is carried as an fp16 pair dh + dl: hi = fp16(dh
// q), lo = fp16((dh q - hi) + dl q), so hi + lo = w to ~2^-22 relative.
template <>
__device__ __forceinline__ void dq16<Q3_K>(const SliceRegs<Q3_K> &R, const uint8_t *sl, int j, int q4, uint32_t (&hv)[8],
                                           uint32_t (&lv)[8]) {
    const int b = 2 * j + (q4 >> 1), q16 = q4 & 1;
    const uint32_t *wp = reinterpret_cast<const uint32_t *>(sl + 12 * b);
    uint4 ga, gb;
    q3k_groups(wp[0], wp[1], wp[2], ga, gb);
    const uint4 g = q16 ? gb : ga;
    const float dlf = R.d * (float)((int)((R.sc >> (8 * j)) & 0xFFu) - 32);
    const __half dh = __float2half_rn(dlf);
    const __half dlo = __float2half_rn(dlf - __half2float(dh));
    const __half2 dh2 = __halves2half2(dh, dh), dl2 = __halves2half2(dlo, dlo);
    const __half2 off = __float2half2_rn(1028.0f);   // 1024 + 4: v - 4
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t v = word_of(g, wi);
#pragma unroll
        for (int sel = 0; sel < 2; ++sel) {
            const __half2 q2 = __hsub2(bytes_h2(v, sel), off);
            const __half2 h = __hmul2(dh2, q2);
            const __half2 r = __hfma2(dh2, q2, __hneg2(h));
            hv[2 * wi + sel] = h22u(h);
            lv[2 * wi + sel] = h22u(__hfma2(dl2, q2, r));
        }
    }
}
// Q4_K superblock: fp16 d, fp16 dmin, 12 B scales/mins, qs[128]; elements
// 64c .. 64c+31 are the low nibbles of qs[32c .. 32c+31] (sub-block 2c),
// 64c+32 .. 64c+63 their high nibbles (sub-block 2c+1); w = d*sc*q - dmin*m
// (repack.cpp:222-283, the Q5_K decoder of qwen_moe_q3k.c:541-552 without the
// fifth bit), formed in fp32 and split by conversion.
template <>
__device__ __forceinline__ void dq16<Q4_K>(const SliceRegs<Q4_K> &R, const uint8_t *sl, int j, int q4, uint32_t (&hv)[8],
                                           uint32_t (&lv)[8]) {
    const int b = 2 * j + (q4 >> 1), q16 = q4 & 1;
    int sc, m;
    kq_scale_min(b, R.hdr.y, R.hdr.z, R.hdr.w, sc, m);
    const float d1 = h2f_lo(R.hdr.x) * (float)sc, m1 = h2f_hi(R.hdr.x) * (float)m;
    const uint4 q = ld16(sl + 16 + 32 * (b >> 1) + 16 * q16);
    const int sh = (b & 1) ? 4 : 0;
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t w = word_of(q, wi);
#pragma unroll
        for (int sel = 0; sel < 2; ++sel) {
            const float x0 = d1 * (float)((w >> (16 * sel + sh)) & 15) - m1;
            const float x1 = d1 * (float)((w >> (16 * sel + 8 + sh)) & 15) - m1;
            const __half2 h = __float22half2_rn(make_float2(x0, x1));
            const float2 f = __half22float2(h);
            hv[2 * wi + sel] = h22u(h);
            lv[2 * wi + sel] = h22u(__float22half2_rn(make_float2(x0 - f.x, x1 - f.y)));
        }
    }
}

// Roles (one CTA per SM, QG_THREADS threads):
//   warp 0 lane 0  raw weight slices (TMA, ring of QG_RAW_STAGES)
//   warp 0 lane 1  activation tiles (TMA, ring of b_stages)
//   warp 1 lane 0  MMA issuer; warp 1 allocates TMEM
//   warps 2..17    dequantise (thread: weight row r, 16 weights of every
//                  64-element piece), then the item's epilogue
template <int QT>
__global__ void __launch_bounds__(QG_THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                 const __grid_constant__ CUtensorMap tmXh, const __grid_constant__ CUtensorMap tmXl,
                 const __grid_constant__ CUtensorMap tmXhs, const __grid_constant__ CUtensorMap tmXls,
                 const QgParams p) {
    constexpr QgLayout LY = qg_layout(QT);
    constexpr int SB = LY.sb, BST = LY.b_stages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + LY.bar_off);
    uint64_t *a_full = bars;                          // [A]: dequant warps arrive
    uint64_t *a_empty = a_full + QG_A_STAGES;         // [A]: MMA commit
    uint64_t *raw_full = a_empty + QG_A_STAGES;       // [RAW]: TMA bytes
    uint64_t *raw_empty = raw_full + QG_RAW_STAGES;   // [RAW]: dequant warps arrive
    uint64_t *b_full = raw_empty + QG_RAW_STAGES;     // [B]: TMA bytes
    uint64_t *b_empty = b_full + BST;                 // [B]: MMA commit
    uint64_t *tfull = b_empty + BST;                  // MMA commit: accumulator complete
    uint64_t *tempty = tfull + 1;                     // dequant warps: accumulator read
    uint64_t *drain = tempty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *tiles = reinterpret_cast<int *>(smem + LY.pfx_off);   // [ngroups + 1]
    int *tok = tiles + QG_MAX_GROUPS + 1;                        // [ngroups + 1]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt_per_mat = (p.n_rows + QG_ROWS - 1) / QG_ROWS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < QG_A_STAGES; ++s) {
            mbar_init(&a_full[s], QG_DQ_WARPS);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < QG_RAW_STAGES; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], QG_DQ_WARPS);
        }
        for (int s = 0; s < BST; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, QG_DQ_WARPS);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmW0);
        tma_prefetch_desc(&tmXh);
        tma_prefetch_desc(&tmXl);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, QG_TMEM_COLS);
        tmem_relinquish();
    }
    pdl_wait();                                   // X planes and counts come from earlier kernels
    pdl_launch_dependents();
    // item list: per-group item and token prefixes (warp 0, groups spread over the lanes)
    if (warp == 0) {
        const int per = (p.ngroups + 31) / 32;
        int ts = 0, ks = 0;
        for (int k = 0; k < per; ++k) {
            const int g = lane * per + k;
            if (g < p.ngroups) {
                const int c = p.cnt ? __ldcg(p.cnt + g) : p.T;
                ts += p.nmat * rt_per_mat * ((c + QG_NT - 1) / QG_NT);
                ks += c;
            }
        }
        int ti = ts, ki = ks;   // inclusive scans over lanes
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, ti, off), b2 = __shfl_up_sync(0xffffffffu, ki, off);
            if (lane >= off) {
                ti += a;
                ki += b2;
            }
        }
        int tr = ti - ts, kr = ki - ks;   // exclusive starts of this lane's run
        for (int k = 0; k < per; ++k) {
            const int g = lane * per + k;
            if (g < p.ngroups) {
                tiles[g] = tr;
                tok[g] = kr;
                const int c = p.cnt ? __ldcg(p.cnt + g) : p.T;
                tr += p.nmat * rt_per_mat * ((c + QG_NT - 1) / QG_NT);
                kr += c;
            }
        }
        if (lane == 31) {
            tiles[p.ngroups] = ti;
            tok[p.ngroups] = ki;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total = tiles[p.ngroups];

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- raw weight slices ----------------
            uint32_t rs = 0, rph = 0, issued[QG_RAW_STAGES] = {0, 0};
            bool ok = true;
            for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
                const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.cnt, p.T);
                const CUtensorMap *tw = it.mat ? &tmW1 : &tmW0;
                const int wrow = it.g * p.n_rows + it.rtile * QG_ROWS;
                for (int s = 0; s < p.ns; ++s) {
                    if (!mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(QG_ROWS * SB));
                    tma_load_2d(smem + LY.raw_off + rs * LY.raw_bytes, tw, s * (SB / 2), wrow, &raw_full[rs]);
                    issued[rs]++;
                    if (++rs == QG_RAW_STAGES) {
                        rs = 0;
                        rph ^= 1u;
                    }
                }
            }
            if (!ok)   // copies still in flight after a timeout
                for (int k = 0; k < QG_RAW_STAGES; ++k)
                    if (issued[k]) mbar_wait_drain(&raw_full[k], (issued[k] - 1u) & 1u, kQgDrainNs);
        } else if (lane == 1) {
            // ---------------- activation tiles ----------------
            uint32_t sb = 0, bph = 0, issued[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            bool ok = true;
            for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
                const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.cnt, p.T);
                const bool small = it.nt <= QG_NT_SMALL;
                const CUtensorMap *th = small ? &tmXhs : &tmXh, *tl = small ? &tmXls : &tmXl;
                const uint32_t bbytes = 2u * (small ? QG_NT_SMALL : QG_NT) * 128u;
                for (int kk = 0; kk < 4 * p.ns; ++kk) {
                    if (!mbar_wait(&b_empty[sb], bph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst = smem + LY.b_off + sb * QG_B_BYTES;
                    mbar_arrive_expect_tx(&b_full[sb], bbytes);
                    tma_load_2d(dst, th, 64 * kk, it.tok0, &b_full[sb]);
                    tma_load_2d(dst + QG_PLANE_B, tl, 64 * kk, it.tok0, &b_full[sb]);
                    issued[sb]++;
                    if (++sb == (uint32_t)BST) {
                        sb = 0;
                        bph ^= 1u;
                    }
                }
            }
            if (!ok)
                for (int k = 0; k < BST; ++k)
                    if (issued[k]) mbar_wait_drain(&b_full[k], (issued[k] - 1u) & 1u, kQgDrainNs);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t sa = 0, aph = 0, sb = 0, bph = 0, tph = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
                const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.cnt, p.T);
                // MMA 1: A = W_hi against the X_hi plane (64 rows) and the X_lo
                // plane right after it, N = 64 + n: columns [0, 64) get
                // W_hi.X_hi, [64, 64 + n) W_hi.X_lo.  MMA 2: A = W_lo against
                // X_hi, N = n, adds W_lo.X_hi into columns [0, n).
                const uint32_t N = (uint32_t)max(16, (it.nt + 15) & ~15);
                const uint32_t idesc1 = idesc_make(1, 0, 0, QG_ROWS, QG_NT + N);
                const uint32_t idesc2 = idesc_make(1, 0, 0, QG_ROWS, N);
                if (!mbar_wait(tempty, tph ^ 1u, abort_flag, p.status)) break;   // previous item read out
                tph ^= 1u;
                tc_fence_after();
                for (int kk = 0; kk < 4 * p.ns; ++kk) {
                    if (!mbar_wait(&a_full[sa], aph, abort_flag, p.status) ||
                        !mbar_wait(&b_full[sb], bph, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(smem + LY.a_off + sa * QG_A_BYTES), a_lo = a_hi + QG_PLANE_A;
                    const uint32_t b_hi = smem_u32(smem + LY.b_off + sb * QG_B_BYTES), b_lo = b_hi + QG_PLANE_B;
                    (void)b_lo;   // the X_lo plane follows X_hi: one B operand of 64 + n rows
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t dah = smem_desc_sw128(a_hi + 32 * k, 16, 1024);
                        const uint64_t dal = smem_desc_sw128(a_lo + 32 * k, 16, 1024);
                        const uint64_t dbh = smem_desc_sw128(b_hi + 32 * k, 16, 1024);
                        umma_f16(tmem_base, dah, dbh, idesc1, (kk | k) ? 1u : 0u);
                        umma_f16(tmem_base, dal, dbh, idesc2, 1u);
                    }
                    umma_commit(&a_empty[sa]);
                    umma_commit(&b_empty[sb]);
                    if (++sa == QG_A_STAGES) {
                        sa = 0;
                        aph ^= 1u;
                    }
                    if (++sb == (uint32_t)BST) {
                        sb = 0;
                        bph ^= 1u;
                    }
                }
                if (ok) umma_commit(tfull);
            }
            umma_commit(drain);   // every MMA of this thread completes before TMEM is freed
            mbar_wait_drain(drain, 0, kQgDrainNs);
        }
    } else {
        // ---------------- dequantise, then epilogue ----------------
        const int dq = threadIdx.x - 64;
        const int r = dq & (QG_ROWS - 1), q4 = dq >> 7;   // weight row of the tile, 16-weight quarter of each piece
        const int qd = warp & 3;                          // TMEM lane quadrant this warp may read
        const int cpart = (warp - 2) >> 2;                // which 32 of the token columns (0..3; 0-1 used)
        uint32_t sa = 0, aph = 0, rs = 0, rph = 0, tph = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
            const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.cnt, p.T);
            for (int s = 0; s < p.ns && ok; ++s) {
                if (!mbar_wait(&raw_full[rs], rph, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                const uint8_t *sl = smem + LY.raw_off + rs * LY.raw_bytes + r * SB;
                SliceRegs<QT> R;
                load_slice<QT>(sl, q4, R);
                for (int j = 0; j < 4; ++j) {
                    uint32_t hv[8], lv[8];
                    dq16<QT>(R, sl, j, q4, hv, lv);
                    if (!mbar_wait(&a_empty[sa], aph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *ahi = smem + LY.a_off + sa * QG_A_BYTES + r * 128, *alo = ahi + QG_PLANE_A;
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int off = ((2 * q4 + cc) ^ (r & 7)) << 4;
                        *reinterpret_cast<uint4 *>(ahi + off) =
                            make_uint4(hv[4 * cc], hv[4 * cc + 1], hv[4 * cc + 2], hv[4 * cc + 3]);
                        *reinterpret_cast<uint4 *>(alo + off) =
                            make_uint4(lv[4 * cc], lv[4 * cc + 1], lv[4 * cc + 2], lv[4 * cc + 3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[sa]);
                    if (++sa == QG_A_STAGES) {
                        sa = 0;
                        aph ^= 1u;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                if (++rs == QG_RAW_STAGES) {
                    rs = 0;
                    rph ^= 1u;
                }
            }
            if (!ok) break;
            // epilogue of this item
            if (!mbar_wait(tfull, tph, abort_flag, p.status)) break;
            tph ^= 1u;
            tc_fence_after();
            const int row = it.rtile * QG_ROWS + qd * 32 + lane;
            const long col = (long)it.mat * p.n_rows + row;
            const int c0 = 32 * cpart;
            for (int c1 = c0; c1 < c0 + 32 && c1 < it.nt; c1 += 16) {   // warp-uniform
                uint32_t v[16], w[16];
                tmem_ld16(tmem_base + c1 + (static_cast<uint32_t>(qd * 32) << 16), v);
                tmem_ld16(tmem_base + QG_NT + c1 + (static_cast<uint32_t>(qd * 32) << 16), w);
                tmem_wait_ld();
                if (row < p.n_rows) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int c = c1 + k;
                        if (c < it.nt) {
                            const int t = it.tok0 + c;
                            const float val = __uint_as_float(v[k]) + __uint_as_float(w[k]);
                            if (p.mode == QG_SCATTER) {
                                p.out[(long)__ldg(p.pair_at + t) * p.ldo + col] = val;
                            } else {
                                float *o = p.out + (long)t * p.ldo + col;
                                *o = p.mode == QG_ADD ? *o + val : val;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, QG_TMEM_COLS);
    }
}

// ---- activation preparation ---------------------------------------------------------------
__device__ __forceinline__ void split_store(float x, __half &hi, __half &lo) {
    hi = __float2half_rn(x);
    lo = __float2half_rn(x - __half2float(hi));
}

// One CTA per row: optional RMS norm, then the fp16 hi / lo planes.
__global__ void __launch_bounds__(256) split_rows_kernel(const float *__restrict__ src, long lds, int K, int kp,
                                                         const float *__restrict__ nw, float eps,
                                                         __half *__restrict__ hi, __half *__restrict__ lo,
                                                         float *__restrict__ f32_out) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x;
    const float *x = src + (long)row * lds;
    __shared__ float red[8];
    float sc = 1.f;
    if (nw) {
        float s = 0.f;
        for (int k = threadIdx.x; k < K; k += blockDim.x) s += x[k] * x[k];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
        __syncthreads();
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        sc = 1.0f / sqrtf(t / (float)K + eps);
    }
    for (int k = threadIdx.x; k < kp; k += blockDim.x) {
        float v = 0.f;
        if (k < K) {
            v = nw ? x[k] * sc * nw[k] : x[k];
            if (f32_out) f32_out[(long)row * K + k] = v;
        }
        __half a, b;
        split_store(v, a, b);
        hi[(long)row * kp + k] = a;
        lo[(long)row * kp + k] = b;
    }
}

// h = silu(g) * u per row of gu [rows][2 ffn], into fp16 planes [rows][kp].
__global__ void __launch_bounds__(256) swiglu_split_kernel(const float *__restrict__ gu, int ffn, int kp,
                                                           __half *__restrict__ hi, __half *__restrict__ lo) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.x;
    for (int k = threadIdx.x; k < kp; k += blockDim.x) {
        float v = 0.f;
        if (k < ffn) {
            const float g = gu[(long)row * 2 * ffn + k], u = gu[(long)row * 2 * ffn + ffn + k];
            v = (g / (1.0f + expf(-g))) * u;   // qwen_moe.c:309
        }
        __half a, b;
        split_store(v, a, b);
        hi[(long)row * kp + k] = a;
        lo[(long)row * kp + k] = b;
    }
}

}  // namespace q

using namespace q;

int launch_split_rows(const float *src, long lds, int K, int kp, int rows, const float *nw, float eps, __half *hi,
                      __half *lo, float *f32_out, cudaStream_t s) {
    if (rows <= 0) return X100_OK;
    return launch_pdl(split_rows_kernel, dim3(rows), dim3(256), 0, s, src, lds, K, kp, nw, eps, hi, lo, f32_out);
}

int launch_swiglu_split(const float *gu, int ffn, int kp, int rows, __half *hi, __half *lo, cudaStream_t s) {
    if (rows <= 0) return X100_OK;
    return launch_pdl(swiglu_split_kernel, dim3(rows), dim3(256), 0, s, gu, ffn, kp, hi, lo);
}

template <int QT>
static int launch_qgemm_qt(DevCtx *c, const QgLaunch &L, const CUtensorMap *tw, const CUtensorMap *tx,
                           const QgParams &p, cudaStream_t s) {
    constexpr QgLayout LY = qg_layout(QT);
    static_assert(LY.smem <= QG_SMEM_CAP && LY.b_stages >= 2, "shared-memory plan");
    static bool attr[64];
    if (!attr[c->device]) {
        cudaFuncSetAttribute(qgemm_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, LY.smem);
        attr[c->device] = true;
    }
    const int grid = c->sm_count;
    return launch_pdl(qgemm_kernel<QT>, dim3(grid), dim3(QG_THREADS), (size_t)LY.smem, s, tw[0], tw[1], tx[0], tx[1],
                      tx[2], tx[3], p);
}

int launch_qgemm(DevCtx *c, const QgLaunch &L, cudaStream_t s) {
    const QMat &m0 = *L.mats[0];
    const int SB = slice_bytes(m0.qtype);
    if (!SB || L.nmat < 1 || L.nmat > 2 || L.ngroups < 1 || L.ngroups > QG_MAX_GROUPS || L.n_rows <= 0 ||
        (L.nmat == 2 && (!L.mats[1] || L.mats[1]->qtype != m0.qtype || L.mats[1]->K != m0.K)) ||
        (L.mode == QG_SCATTER && !L.pair_at) || !L.out || !L.xh || !L.xl || L.x_rows <= 0) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    CUtensorMap tw[2], tx[4];
    const int kp = m0.ns * 256;
    for (int i = 0; i < 2; ++i) {
        const QMat &m = *L.mats[i < L.nmat ? i : 0];
        if (!make_tmap_2d_sw(&tw[i], m.w, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)m.row_bytes / 2, (uint64_t)m.N,
                             (uint64_t)m.row_bytes, (uint32_t)(SB / 2), QG_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE)) {
            set_error(X100_E_UNSUPPORTED);
            return X100_E_UNSUPPORTED;
        }
    }
    const uint32_t boxes[2] = {QG_NT, QG_NT_SMALL};
    for (int b = 0; b < 2; ++b) {
        if (!make_tmap_2d(&tx[2 * b], L.xh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)kp, (uint64_t)L.x_rows,
                          (uint64_t)kp * 2, 64, boxes[b]) ||
            !make_tmap_2d(&tx[2 * b + 1], L.xl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (uint64_t)kp, (uint64_t)L.x_rows,
                          (uint64_t)kp * 2, 64, boxes[b])) {
            set_error(X100_E_UNSUPPORTED);
            return X100_E_UNSUPPORTED;
        }
    }
    QgParams p;
    p.nmat = L.nmat;
    p.n_rows = L.n_rows;
    p.ns = m0.ns;
    p.ngroups = L.ngroups;
    p.T = L.T;
    p.mode = L.mode;
    p.cnt = L.cnt;
    p.out = L.out;
    p.ldo = L.ldo;
    p.pair_at = L.pair_at;
    p.status = c->d_status;
    switch (m0.qtype) {
    case Q4_0: return launch_qgemm_qt<Q4_0>(c, L, tw, tx, p, s);
    case Q8_0: return launch_qgemm_qt<Q8_0>(c, L, tw, tx, p, s);
    case Q4_K: return launch_qgemm_qt<Q4_K>(c, L, tw, tx, p, s);
    case Q3_K: return launch_qgemm_qt<Q3_K>(c, L, tw, tx, p, s);
    default: set_error(X100_E_UNSUPPORTED); return X100_E_UNSUPPORTED;
    }
}

}  // namespace x100
