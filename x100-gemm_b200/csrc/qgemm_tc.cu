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
//   warp 1    MMA issuer: per 16 elements of K, three tcgen05.mma kind::f16
//             (fp32 accumulate in TMEM): W_hi.X_hi + W_hi.X_lo + W_lo.X_hi --
//             weights and activations each carried to ~22 bits, so the
//             products agree with the fp32 dequant-GEMV to ~1e-6 relative
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
constexpr int QG_NT = 128;                      // tokens per item (MMA N, at most)
constexpr int QG_NT_SMALL = 32;                 // box of the small token tiles
constexpr int QG_AB_STAGES = 2;
constexpr int QG_RAW_STAGES = 2;
constexpr int QG_DQ_WARPS = 8;
constexpr int QG_THREADS = 64 + 32 * QG_DQ_WARPS;
constexpr int QG_PLANE_A = QG_ROWS * 128;       // 128 rows x 64 fp16
constexpr int QG_PLANE_B = QG_NT * 128;         // 128 tokens x 64 fp16
constexpr int QG_AB_BYTES = 2 * QG_PLANE_A + 2 * QG_PLANE_B;
constexpr int QG_RAW_BYTES = QG_ROWS * 272;     // 128 rows of the largest slice (Q8_0)
constexpr int QG_MAX_GROUPS = 256;
constexpr int QG_RAW_OFF = QG_AB_STAGES * QG_AB_BYTES;
constexpr int QG_BAR_OFF = QG_RAW_OFF + QG_RAW_STAGES * QG_RAW_BYTES;
constexpr int QG_NBARS = 4 * QG_AB_STAGES + 2 * QG_RAW_STAGES + 3;   // a_full b_full ab_empty x2 ... raw, t
constexpr int QG_PFX_OFF = QG_BAR_OFF + QG_NBARS * 8 + 16;
constexpr int QG_SMEM = QG_PFX_OFF + 2 * (QG_MAX_GROUPS + 1) * 4 + 1024;
constexpr uint32_t QG_TMEM_COLS = QG_NT;
constexpr unsigned long long kQgDrainNs = 100000000ull;

struct QgParams {
    int nmat, n_rows, ns, ngroups, T, mode, sb;   // sb: slice bytes of the weight format
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
                                          int nmat, const int *cnt, int T) {
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

// ---- dequantisation of 32 weights (elements 32 b .. 32 b + 31 of a slice) -------------
__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ int byte_of(const uint4 &v, int i) { return (word_of(v, i >> 2) >> (8 * (i & 3))) & 0xFF; }

template <int QT> __device__ __forceinline__ void dq32(const uint8_t *sl, int b, float (&w)[32]);
// Q8_0 slice: [8 fp16 d][8 x 32 int8]; w = d * q (qwen_moe.c:162-163)
template <> __device__ __forceinline__ void dq32<Q8_0>(const uint8_t *sl, int b, float (&w)[32]) {
    const uint4 hd = ld16(sl);
    const uint32_t dw = word_of(hd, b >> 1);
    const float d = (b & 1) ? h2f_hi(dw) : h2f_lo(dw);
    const uint4 q0 = ld16(sl + 16 + 32 * b), q1 = ld16(sl + 32 + 32 * b);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        w[i] = d * (float)(int8_t)byte_of(q0, i);
        w[16 + i] = d * (float)(int8_t)byte_of(q1, i);
    }
}
// Q4_0 slice: [8 fp16 d][8 x 16 B nibbles]; element i < 16 the low nibble of
// byte i, i >= 16 the high nibble of byte i - 16; w = (nib - 8) * d
// (qwen_moe.c:164-165)
template <> __device__ __forceinline__ void dq32<Q4_0>(const uint8_t *sl, int b, float (&w)[32]) {
    const uint4 hd = ld16(sl);
    const uint32_t dw = word_of(hd, b >> 1);
    const float d = (b & 1) ? h2f_hi(dw) : h2f_lo(dw);
    const uint4 q = ld16(sl + 16 + 16 * b);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int v = byte_of(q, i);
        w[i] = (float)((v & 15) - 8) * d;
        w[16 + i] = (float)((v >> 4) - 8) * d;
    }
}
// Q4_K superblock: fp16 d, fp16 dmin, 12 B scales/mins, qs[128]; elements
// 64c .. 64c+31 are the low nibbles of qs[32c .. 32c+31] (sub-block 2c),
// 64c+32 .. 64c+63 their high nibbles (sub-block 2c+1); w = d*sc*q - dmin*m
// (repack.cpp:222-283, the Q5_K decoder of qwen_moe_q3k.c:541-552 without the
// fifth bit)
template <> __device__ __forceinline__ void dq32<Q4_K>(const uint8_t *sl, int b, float (&w)[32]) {
    const uint4 hdr = ld16(sl);
    const float d = h2f_lo(hdr.x), dmin = h2f_hi(hdr.x);
    int sc, m;
    kq_scale_min(b, hdr.y, hdr.z, hdr.w, sc, m);
    const float d1 = d * (float)sc, m1 = dmin * (float)m;
    const uint4 q0 = ld16(sl + 16 + 32 * (b >> 1)), q1 = ld16(sl + 32 + 32 * (b >> 1));
    const int sh = (b & 1) ? 4 : 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        w[i] = d1 * (float)((byte_of(q0, i) >> sh) & 15) - m1;
        w[16 + i] = d1 * (float)((byte_of(q1, i) >> sh) & 15) - m1;
    }
}
// Q3_K slice: [qs 64][hmask 32][scales 12][d 2][pad 2]; element e = 32 b + l:
// half hh = b / 4, shift 2t with t = b % 4, q = ((qs[32hh + l] >> 2t) & 3) -
// (hmask bit 4hh + t of byte l ? 0 : 4), sub-block scale 8hh + 2t + l/16;
// w = d * (sc - 32) * q (qwen_moe_q3k.c:557-577)
template <> __device__ __forceinline__ void dq32<Q3_K>(const uint8_t *sl, int b, float (&w)[32]) {
    const int hh = b >> 2, t = b & 3;
    const uint4 q0 = ld16(sl + 32 * hh), q1 = ld16(sl + 32 * hh + 16);
    const uint4 m0 = ld16(sl + 64), m1 = ld16(sl + 80);
    const uint4 hdr = ld16(sl + 96);
    const float d = h2f_lo(hdr.w);
    const float dl0 = d * (float)q3k_scale(8 * hh + 2 * t, hdr.x, hdr.y, hdr.z);
    const float dl1 = d * (float)q3k_scale(8 * hh + 2 * t + 1, hdr.x, hdr.y, hdr.z);
    const int hb = 4 * hh + t;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int a = ((byte_of(q0, i) >> (2 * t)) & 3) - (((byte_of(m0, i) >> hb) & 1) ? 0 : 4);
        const int c = ((byte_of(q1, i) >> (2 * t)) & 3) - (((byte_of(m1, i) >> hb) & 1) ? 0 : 4);
        w[i] = dl0 * (float)a;
        w[16 + i] = dl1 * (float)c;
    }
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

template <int QT>
__global__ void __launch_bounds__(QG_THREADS, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                 const __grid_constant__ CUtensorMap tmXh, const __grid_constant__ CUtensorMap tmXl,
                 const __grid_constant__ CUtensorMap tmXhs, const __grid_constant__ CUtensorMap tmXls,
                 const QgParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + QG_BAR_OFF);
    uint64_t *a_full = bars;                          // [AB]: 8 dequant warps arrive
    uint64_t *b_full = bars + QG_AB_STAGES;           // [AB]: producer + TMA bytes
    uint64_t *ab_empty = bars + 2 * QG_AB_STAGES;     // [AB]: MMA commit
    uint64_t *raw_full = bars + 3 * QG_AB_STAGES;     // [RAW]: producer + TMA bytes
    uint64_t *raw_empty = raw_full + QG_RAW_STAGES;   // [RAW]: 8 dequant warps arrive
    uint64_t *tfull = raw_empty + QG_RAW_STAGES;      // MMA commit: accumulator complete
    uint64_t *tempty = tfull + 1;                     // 8 epilogue warps: accumulator read
    uint64_t *drain = tempty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + QG_NBARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    int *tiles = reinterpret_cast<int *>(smem + QG_PFX_OFF);   // [ngroups + 1]
    int *tok = tiles + QG_MAX_GROUPS + 1;                        // [ngroups + 1]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rt_per_mat = (p.n_rows + QG_ROWS - 1) / QG_ROWS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < QG_AB_STAGES; ++s) {
            mbar_init(&a_full[s], QG_DQ_WARPS);
            mbar_init(&b_full[s], 1);
            mbar_init(&ab_empty[s], 1);
        }
        for (int s = 0; s < QG_RAW_STAGES; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], QG_DQ_WARPS);
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
    // item list: per-group item and token prefixes (warp 0, the groups 8 per lane at most)
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
    const int SB = p.sb;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t st = 0, ph = 0, rs = 0, rph = 0;
            uint32_t ab_issued[QG_AB_STAGES] = {0, 0}, raw_issued[QG_RAW_STAGES] = {0, 0};
            bool ok = true;
            for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
                const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.nmat, p.cnt, p.T);
                const CUtensorMap *tw = it.mat ? &tmW1 : &tmW0;
                const bool small = it.nt <= QG_NT_SMALL;
                const CUtensorMap *th = small ? &tmXhs : &tmXh, *tl = small ? &tmXls : &tmXl;
                const uint32_t bbytes = 2u * (small ? QG_NT_SMALL : QG_NT) * 128u;
                const int wrow = it.g * p.n_rows + it.rtile * QG_ROWS;
                for (int s = 0; s < p.ns && ok; ++s) {
                    if (!mbar_wait(&raw_empty[rs], rph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *raw = smem + QG_RAW_OFF + rs * QG_RAW_BYTES;
                    mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(QG_ROWS * SB));
                    tma_load_2d(raw, tw, s * (SB / 2), wrow, &raw_full[rs]);
                    raw_issued[rs]++;
                    if (++rs == QG_RAW_STAGES) {
                        rs = 0;
                        rph ^= 1u;
                    }
                    for (int j = 0; j < 4; ++j) {
                        if (!mbar_wait(&ab_empty[st], ph ^ 1u, abort_flag, p.status)) {
                            ok = false;
                            break;
                        }
                        uint8_t *stg = smem + st * QG_AB_BYTES;
                        mbar_arrive_expect_tx(&b_full[st], bbytes);
                        tma_load_2d(stg + 2 * QG_PLANE_A, th, s * 256 + 64 * j, it.tok0, &b_full[st]);
                        tma_load_2d(stg + 2 * QG_PLANE_A + QG_PLANE_B, tl, s * 256 + 64 * j, it.tok0, &b_full[st]);
                        ab_issued[st]++;
                        if (++st == QG_AB_STAGES) {
                            st = 0;
                            ph ^= 1u;
                        }
                    }
                }
            }
            if (!ok) {   // copies still in flight after a timeout
                for (int k = 0; k < QG_RAW_STAGES; ++k)
                    if (raw_issued[k]) mbar_wait_drain(&raw_full[k], (raw_issued[k] - 1u) & 1u, kQgDrainNs);
                for (int k = 0; k < QG_AB_STAGES; ++k)
                    if (ab_issued[k]) mbar_wait_drain(&b_full[k], (ab_issued[k] - 1u) & 1u, kQgDrainNs);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t st = 0, ph = 0, tph = 0;
            bool ok = true;
            for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
                const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.nmat, p.cnt, p.T);
                const uint32_t N = (uint32_t)max(16, (it.nt + 15) & ~15);
                const uint32_t idesc = idesc_make(1, 0, 0, QG_ROWS, N);
                if (!mbar_wait(tempty, tph ^ 1u, abort_flag, p.status)) break;   // previous item read out
                tph ^= 1u;
                tc_fence_after();
                for (int s = 0; s < p.ns && ok; ++s) {
                    for (int j = 0; j < 4; ++j) {
                        if (!mbar_wait(&a_full[st], ph, abort_flag, p.status) ||
                            !mbar_wait(&b_full[st], ph, abort_flag, p.status)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_hi = smem_u32(smem + st * QG_AB_BYTES), a_lo = a_hi + QG_PLANE_A;
                        const uint32_t b_hi = a_hi + 2 * QG_PLANE_A, b_lo = b_hi + QG_PLANE_B;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint64_t dah = smem_desc_sw128(a_hi + 32 * k, 16, 1024);
                            const uint64_t dal = smem_desc_sw128(a_lo + 32 * k, 16, 1024);
                            const uint64_t dbh = smem_desc_sw128(b_hi + 32 * k, 16, 1024);
                            const uint64_t dbl = smem_desc_sw128(b_lo + 32 * k, 16, 1024);
                            umma_f16(tmem_base, dah, dbh, idesc, (s | j | k) ? 1u : 0u);
                            umma_f16(tmem_base, dah, dbl, idesc, 1u);
                            umma_f16(tmem_base, dal, dbh, idesc, 1u);
                        }
                        umma_commit(&ab_empty[st]);
                        if (++st == QG_AB_STAGES) {
                            st = 0;
                            ph ^= 1u;
                        }
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
        const int r = dq & (QG_ROWS - 1), hf = dq >> 7;   // weight row of the tile, half of each piece
        const int q = warp & 3;                           // TMEM lane quadrant this warp may read
        const int cpart = (warp - 2) >> 2;                // which 64 of the 128 token columns
        uint32_t st = 0, ph = 0, rs = 0, rph = 0, tph = 0;
        bool ok = true;
        for (int i = blockIdx.x; i < total && ok; i += gridDim.x) {
            const QgItem it = qg_item(i, tiles, tok, p.ngroups, rt_per_mat, p.nmat, p.cnt, p.T);
            for (int s = 0; s < p.ns && ok; ++s) {
                if (!mbar_wait(&raw_full[rs], rph, abort_flag, p.status)) {
                    ok = false;
                    break;
                }
                const uint8_t *sl = smem + QG_RAW_OFF + rs * QG_RAW_BYTES + r * SB;
                for (int j = 0; j < 4; ++j) {
                    float w[32];
                    dq32<QT>(sl, 2 * j + hf, w);
                    if (!mbar_wait(&ab_empty[st], ph ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    uint8_t *ahi = smem + st * QG_AB_BYTES + r * 128, *alo = ahi + QG_PLANE_A;
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t hv[4], lv[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float x0 = w[8 * cc + 2 * e], x1 = w[8 * cc + 2 * e + 1];
                            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
                            hv[e] = pack_h2(h0, h1);
                            lv[e] = pack_h2(__float2half_rn(x0 - __half2float(h0)), __float2half_rn(x1 - __half2float(h1)));
                        }
                        const int off = ((4 * hf + cc) ^ (r & 7)) << 4;
                        *reinterpret_cast<uint4 *>(ahi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                        *reinterpret_cast<uint4 *>(alo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[st]);
                    if (++st == QG_AB_STAGES) {
                        st = 0;
                        ph ^= 1u;
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
            const int row = it.rtile * QG_ROWS + q * 32 + lane;
            const long col = (long)it.mat * p.n_rows + row;
            for (int c0 = 64 * cpart; c0 < 64 * cpart + 64 && c0 < it.nt; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem_base + c0 + (static_cast<uint32_t>(q * 32) << 16), v);
                tmem_wait_ld();
                if (row < p.n_rows) {
#pragma unroll 4
                    for (int k = 0; k < 32; ++k) {
                        const int c = c0 + k;
                        if (c < it.nt) {
                            const int t = it.tok0 + c;
                            const float val = __uint_as_float(v[k]);
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
    static bool attr[64];
    if (!attr[c->device]) {
        cudaFuncSetAttribute(qgemm_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, QG_SMEM);
        attr[c->device] = true;
    }
    const int grid = c->sm_count;
    return launch_pdl(qgemm_kernel<QT>, dim3(grid), dim3(QG_THREADS), (size_t)QG_SMEM, s, tw[0], tw[1], tx[0], tx[1],
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
    p.sb = SB;
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
