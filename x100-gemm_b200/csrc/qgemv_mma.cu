// qgemv_mma.cu -- dequant-GEMV of several tokens (2..16) on the tensor cores,
// for the Q4_0 and Q8_0 slice layouts.
//
// The single-token kernel (qgemv.cu) forms each block's integer dot with
// dp4a; with several tokens that work grows with the batch and bounds the
// call long before HBM does.  Here one m16n8k32 integer MMA computes a whole
// block (32 weights) for 16 rows x 8 tokens: A = the 16 rows' int8 weights
// (Q4_0: unsigned nibbles, the -8 folded in as -8 * sum(x) as the dp4a path
// does; Q8_0: signed bytes), B = the tokens' h or l activation plane
// (qformats.cuh: x ~= s (256 h + l)), so 256 * MMA(h) + MMA(l) is exactly the
// integer block dot of the dp4a path, and each half-slice (4 blocks) is
// scaled and summed in the same order.
//
// Persistent kernel, one CTA per SM, in three steps:
//  1. before the dependency wait, every thread starts 16-byte asynchronous
//     copies (cp.async) of the first weight items into a ring of shared-
//     memory stages; an item is a K-chunk of CK slices of a 16-row tile
//     (tile = blockIdx.x + i * gridDim.x), rows an odd multiple of 16 bytes
//     apart so the 8 rows of a fragment load hit distinct banks;
//  2. the CTA prepares every token's activations (block-major, see XBufBM)
//     with xprep_rows (a grid-wide preparation into device scratch behind a
//     grid barrier, and a deeper load prefetch, both measured slower);
//  3. the CTA walks its items through the ring: a warp takes one half-slice
//     of the chunk at a time; after a tile's last chunk its partials are
//     summed per row in slice order (first halves, then second halves) as in
//     the single-token kernel, so results do not depend on the chunking.
#include <cuda_fp16.h>

#include <algorithm>

#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace q {

constexpr int kMmaThreads = 512;
constexpr int kMmaRows = 16;       // rows per tile (the MMA's M)
constexpr int kMmaMaxStages = 4;
constexpr size_t kMmaSmemMax = 220 * 1024;

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Wait until at most n (0..3) of this thread's committed groups are pending.
__device__ __forceinline__ void cp_async_wait(int n) {
    switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    }
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D = A (16 x 32, row) . B (32 x 8, col) over int8, int32 accumulate from 0.
template <bool AU>
__device__ __forceinline__ void mma_i8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    if constexpr (AU)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %10, %10, %10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
            "{%10, %10, %10, %10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Row stride of a stage holding ck slices per row: an odd multiple of 16.
__host__ __device__ constexpr int mma_row_stride(int qt, int ck) {
    return ck * slice_bytes(qt) + (((ck * slice_bytes(qt)) / 16) % 2 ? 32 : 16);
}

struct MmaPlan {
    int nt = 0, ck = 0, stages = 0;
    size_t smem = 0;
};
// Shared memory: the block-major activations of 8 nt tokens, the
// per-half-slice partials [8 nt][16 rows][2 ns], and stages x 16 rows x ck
// slices.  Prefer 16 tokens per launch when at least 64 KB of weights can be
// in flight per SM; otherwise 8 tokens with the most bytes in flight.
static size_t mma_fixed(int K, int nt) {
    const int ns = slices_per_row(K);
    return (size_t)ns * 8 * 8 * nt * 80 + ((size_t)8 * nt * (kMmaRows * (2 * ns + 1) + 4) * 4 + 15) / 16 * 16;
}
static MmaPlan mma_plan(int qt, int K, int batch) {
    const int ns = slices_per_row(K);
    MmaPlan best;
    for (int nt = batch > 8 ? 2 : 1; nt >= 1; --nt) {
        const size_t fixed = mma_fixed(K, nt);
        if (fixed >= kMmaSmemMax) continue;
        // chunk sizes that divide the row first (no ragged last item, whose
        // per-item overhead buys few bytes), if one keeps >= 48 KB in flight
        MmaPlan p;
        size_t inflight = 0;
        for (int pass = 0; pass < 2 && inflight < 48 * 1024; ++pass) {
            p = MmaPlan();
            inflight = 0;
            for (int ck = ns; ck >= 1; --ck) {
                if (pass == 0 && ns % ck) continue;
                const size_t stage = (size_t)kMmaRows * mma_row_stride(qt, ck);
                const int st = (int)std::min<size_t>(kMmaMaxStages, (kMmaSmemMax - fixed) / stage);
                if (st >= 2 && st * stage > inflight) {
                    inflight = st * stage;
                    p.nt = nt;
                    p.ck = ck;
                    p.stages = st;
                    p.smem = fixed + st * stage;
                }
            }
        }
        if (p.stages && (nt == 1 || inflight >= 64 * 1024)) return p;
        if (p.stages && !best.stages) best = p;
    }
    return best;
}

// ---- activations prepared once per call (GemvOpts::prep) ----------------------------
// Layout of the scratch for `batch` tokens of a K-long row (nxb = 8 ns
// blocks): the prepared blocks, block-major in groups of ntok tokens (group
// g's block j of token t at ((g nxb + j) ntok + t % ntok) 80 bytes -- the
// XBufBM image of the CTA's shared memory for tokens g ntok .. g ntok + ntok
// - 1), then the blocks' sums of squares qs[token][nxb] (fp32).
static size_t prep_xbm_bytes(int K) { return (size_t)16 * slices_per_row(K) * 8 * 80; }
// Grid (ceil(nxb / 8), batch), 64 threads: each 8 threads convert one
// 32-element block of token blockIdx.y (x, times nw when given) with
// xprep_vals and record the block's sum of squares of x.
__global__ void __launch_bounds__(64) prep_bm_kernel(const float *__restrict__ x, int K, const float *__restrict__ nw,
                                                     int ntok, uint8_t *__restrict__ xbm, float *__restrict__ qs) {
    pdl_wait();                                   // x comes from the previous kernel
    pdl_launch_dependents();
    const int nxb = slices_per_row(K) * 8, kb = K / 32;
    const int t = threadIdx.x & 7, j = blockIdx.x * 8 + (threadIdx.x >> 3), c = blockIdx.y;
    const bool active = j < nxb;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < kb) v = __ldcg(reinterpret_cast<const float4 *>(x + (long)c * K + j * 32) + t);
    float q = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    q += __shfl_xor_sync(0xffffffffu, q, 1);
    q += __shfl_xor_sync(0xffffffffu, q, 2);
    q += __shfl_xor_sync(0xffffffffu, q, 4);
    if (active && t == 0) qs[(long)c * nxb + j] = q;
    if (nw && j < kb) {
        const float4 w4 = __ldg(reinterpret_cast<const float4 *>(nw + j * 32) + t);
        v = make_float4(v.x * w4.x, v.y * w4.y, v.z * w4.z, v.w * w4.w);
    }
    XB *o = reinterpret_cast<XB *>(xbm + (((long)(c / ntok) * nxb + (active ? j : 0)) * ntok + c % ntok) * 80);
    xprep_vals(v, o, t, active);
}

template <int QT, int NT>
__global__ void __launch_bounds__(kMmaThreads, 1)
    qgemv_mma_kernel(const uint8_t *__restrict__ W, int N, int K, int ck, int stages, const float *__restrict__ x,
                     float *__restrict__ y, int batch, const float *__restrict__ nw, float eps, int accum,
                     int a8, const uint8_t *__restrict__ xbm, const float *__restrict__ qs, long rbw, int *status) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float ssq[(kMmaThreads / 32) * 4][kSsTok];   // RMS-norm sums of squares per 8-lane group
    __shared__ float scale[16];
    __shared__ uint64_t xbar;
    __shared__ int abort_flag;
    constexpr int SB = slice_bytes(QT);
    constexpr int NTOK = 8 * NT;
    const int ns = slices_per_row(K), nb = ns * 8;
    const long rb = rbw ? rbw : (long)ns * SB;   // bytes per weight row (rbw: a piece of a longer row)
    const int rsp = mma_row_stride(QT, ck);
    // partials [tok][row][half-slice]: row stride RS odd and token stride TS =
    // 8 mod 32 words per two tokens, so the 32 lanes' writes hit distinct banks
    const int RS = 2 * ns + 1, TS = kMmaRows * RS + 4;
    const int ntiles = (N + kMmaRows - 1) / kMmaRows;
    const int nchunks = (ns + ck - 1) / ck;
    const int mytiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nitems = mytiles * nchunks;
    uint8_t *xbase = smem;
    float *red = reinterpret_cast<float *>(xbase + (size_t)nb * NTOK * 80);
    uint8_t *stage_base = xbase + (size_t)nb * NTOK * 80 + ((size_t)NTOK * TS * 4 + 15) / 16 * 16;
    const XBufBM xb{xbase, ns, NTOK};
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;

    // every thread copies its 16-byte chunks of item it into stage it % stages
    // and commits one group (empty past the last item, so counting stays uniform)
    auto issue = [&](int it) {
        if (it < nitems) {
            const int tile = blockIdx.x + (it / nchunks) * gridDim.x, chunk = it % nchunks;
            const int r0 = tile * kMmaRows, rows = min(kMmaRows, N - r0);
            const int c0 = chunk * ck, cb = min(ck, ns - c0) * SB / 16;
            uint8_t *dst = stage_base + (size_t)(it % stages) * kMmaRows * rsp;
            const uint8_t *src = W + (long)r0 * rb + (long)c0 * SB;
            for (int r = warp; r < rows; r += nwarps)   // a warp per row, no index division
                for (int c = lane; c < cb; c += 32) cp_async16(dst + (size_t)r * rsp + 16 * c, src + (long)r * rb + 16 * c);
        }
        cp_async_commit();
    };
    for (int s = 0; s < stages - 1; ++s) issue(s);
    pdl_launch_dependents();
    pdl_wait();   // x may come from the previous kernel; the previous call on this matrix is complete

    // ---- 2. activations ----
    if (xbm) {   // prepared by prep_bm_kernel: one bulk copy of this launch's group
        if (threadIdx.x == 0) {
            abort_flag = 0;
            mbar_init(&xbar, 1);
            fence_barrier_init();
            const uint32_t bytes = (uint32_t)nb * NTOK * 80;
            mbar_arrive_expect_tx(&xbar, bytes);
            stage_bytes(xbase, xbm, bytes, &xbar);
        }
        if (warp < batch) {   // a warp per token: its block sums of squares, lane-strided, then a fixed shuffle tree
            float q = 0.f;
            if (nw)
                for (int j = lane; j < nb; j += 32) q += __ldcg(qs + (long)warp * nb + j);
#pragma unroll
            for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
            if (lane == 0) scale[warp] = nw ? 1.0f / sqrtf(q / (float)K + eps) : 1.0f;
        }
        __syncthreads();   // the barrier is initialised
        mbar_wait(&xbar, 0, &abort_flag, status);   // bounded; on a timeout the status records it
        __syncthreads();
    } else {
        xprep_gemv(a8, [x, K](int c) { return x + (long)c * K; }, K, batch, xb, nw, &ssq[0][0]);
        __syncthreads();
        if (threadIdx.x < batch) scale[threadIdx.x] = nw ? rms_scale(&ssq[0][0], blockDim.x / 8, threadIdx.x, K, eps) : 1.0f;
        __syncthreads();
    }
    const uint32_t xs_addr = smem_u32(xbase);

    // ---- 3. the items ----
    for (int it = 0; it < nitems; ++it) {
        issue(it + stages - 1);   // into the stage item it - 1 used
        cp_async_wait(stages - 1);
        __syncthreads();
        const int st = it % stages;
        const int tile = blockIdx.x + (it / nchunks) * gridDim.x, chunk = it % nchunks;
        const int r0 = tile * kMmaRows, rows = min(kMmaRows, N - r0);
        const int c0 = chunk * ck, cs = min(ck, ns - c0);
        const uint8_t *tw = stage_base + (size_t)st * kMmaRows * rsp;
        for (int u = warp; u < 2 * cs; u += nwarps) {
            const int sll = u >> 1, h = u & 1, sl = c0 + sll;
            float acc[NT][4];
#pragma unroll
            for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
            const uint8_t *pg = tw + (size_t)g * rsp + (size_t)sll * SB, *pg8 = pg + (size_t)8 * rsp;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int bb = 4 * h + b, j = sl * 8 + bb;
                uint32_t a0, a1, a2, a3;
                if constexpr (QT == Q4_0) {
                    const uint32_t w0 = *reinterpret_cast<const uint32_t *>(pg + 16 + 16 * bb + 4 * t);
                    const uint32_t w1 = *reinterpret_cast<const uint32_t *>(pg8 + 16 + 16 * bb + 4 * t);
                    a0 = w0 & 0x0F0F0F0Fu;
                    a2 = (w0 >> 4) & 0x0F0F0F0Fu;
                    a1 = w1 & 0x0F0F0F0Fu;
                    a3 = (w1 >> 4) & 0x0F0F0F0Fu;
                } else {
                    a0 = *reinterpret_cast<const uint32_t *>(pg + 16 + 32 * bb + 4 * t);
                    a2 = *reinterpret_cast<const uint32_t *>(pg + 16 + 32 * bb + 16 + 4 * t);
                    a1 = *reinterpret_cast<const uint32_t *>(pg8 + 16 + 32 * bb + 4 * t);
                    a3 = *reinterpret_cast<const uint32_t *>(pg8 + 16 + 32 * bb + 16 + 4 * t);
                }
                const float d0 = __half2float(*reinterpret_cast<const __half *>(pg + 2 * bb));
                const float d1 = __half2float(*reinterpret_cast<const __half *>(pg8 + 2 * bb));
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    // lanes 8m .. 8m+7 address matrix m (h0, h1, l0, l1) of tokens 8n .. 8n+7
                    uint32_t h0, h1, l0, l1;
                    ldsm_x4(xs_addr + (uint32_t)(((long)j * NTOK + 8 * n + (lane & 7)) * 80 + (lane >> 3) * 16), h0,
                            h1, l0, l1);
                    int ch[4], cl[4];
                    mma_i8<QT == Q4_0>(ch, a0, a1, a2, a3, h0, h1);
                    mma_i8<QT == Q4_0>(cl, a0, a1, a2, a3, l0, l1);
                    const XB *x0 = xb.block(8 * n + 2 * t, j), *x1 = xb.block(8 * n + 2 * t + 1, j);
                    const float2 f0 = *reinterpret_cast<const float2 *>(&x0->f);
                    const float2 f1 = *reinterpret_cast<const float2 *>(&x1->f);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = (i & 1) ? f1 : f0;
                        const float d = i < 2 ? d0 : d1;
                        const int dot = ch[i] * 256 + cl[i];
                        if constexpr (QT == Q4_0)
                            acc[n][i] += d * (f.x * (float)dot - 8.0f * f.y);   // (nib - 8) * d
                        else
                            acc[n][i] += d * (f.x * (float)dot);                // q * d
                    }
                }
            }
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tok = 8 * n + 2 * t + (i & 1), row = g + (i < 2 ? 0 : 8);
                    red[(size_t)tok * TS + row * RS + 2 * sl + h] = acc[n][i];
                }
        }
        __syncthreads();   // the stage is consumed, this chunk's partials written
        if (chunk == nchunks - 1) {   // the next item's partials are written after the next barrier
            for (int p = threadIdx.x; p < rows * batch; p += blockDim.x) {
                const int b = p / rows, r = p - b * rows;
                const float *pr = red + (size_t)b * TS + r * RS;
                float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
                for (int sl = 0; sl < ns; ++sl) {
                    s0 += pr[2 * sl];
                    s1 += pr[2 * sl + 1];
                }
                float *o = y + (long)b * N + r0 + r;
                const float v = (s0 + s1) * scale[b];
                *o = accum ? *o + v : v;
            }
        }
    }
    cp_async_wait(0);   // no copy outlives the CTA
}

template <int QT, int NT>
static int launch_mma_nt(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const MmaPlan &p,
                         const GemvOpts &o, cudaStream_t s, const uint8_t *xbm, const float *qs, long rbw = 0) {
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_mma_kernel<QT, NT>, (int)kMmaSmemMax);
        attr[c->device] = true;
    }
    const int ntiles = (m.N + kMmaRows - 1) / kMmaRows;
    const int grid = std::min(ntiles, c->sm_count);
    return launch_k(qgemv_mma_kernel<QT, NT>, dim3(grid), dim3(kMmaThreads), p.smem, s, o.pdl, (const uint8_t *)m.w,
                    m.N, m.K, p.ck, p.stages, x, y, batch, o.norm_w, o.eps, o.accum ? 1 : 0, o.a8, xbm, qs, rbw,
                    c->d_status);
}

// Launches of 8 nt tokens each (nt from the plan).
// The launch plan of a call: the per-launch plan, K pieces, and whether the
// activations are prepared once in o.prep.
struct CallPlan {
    MmaPlan p;
    int kpieces = 1;
    bool prep = false;
};
static CallPlan call_plan(int qt, const QMat &m, int batch, const GemvOpts &o) {
    CallPlan cp;
    cp.p = mma_plan(qt, m.K, batch);
    if (!cp.p.stages) return cp;
    // activations prepared once for all the call's launches (not for the
    // reference's A8 packings, and not for independent calls, whose point is
    // to prepare before the dependency wait)
    cp.prep = o.prep && batch > 1 && o.a8 == 0 && !o.indep && m.K % 32 == 0;
    // K in pieces: when the tokens' activations over the whole row leave no
    // room for a 16-token launch but do over a piece of the row, the call is
    // one 16-token launch per piece, each adding its piece's dots into y, so
    // the weights stream once instead of once per 8-token group (Wo at 16
    // tokens).  Not with a folded RMS norm, whose scale needs the whole row.
    const int ns = slices_per_row(m.K);
    if (cp.prep && batch > 8 && cp.p.nt == 1 && !o.norm_w && m.K % 256 == 0)
        for (int k = 2; k <= 4 && cp.kpieces == 1; ++k)
            if (ns % k == 0) {
                const MmaPlan q = mma_plan(qt, m.K / k, batch);
                if (q.stages && q.nt == 2) {
                    cp.kpieces = k;
                    cp.p = q;
                }
            }
    return cp;
}

template <int QT>
static int launch_mma_qt(DevCtx *c, const QMat &m, const float *x, float *y, int batch, GemvOpts o,
                         cudaStream_t s) {
    const CallPlan cp = call_plan(QT, m, batch, o);
    const MmaPlan &p = cp.p;
    if (!p.stages) return X100_E_UNSUPPORTED;
    const bool prep = cp.prep;
    const int kpieces = cp.kpieces;
    const int ns = slices_per_row(m.K);
    const int per = 8 * p.nt;
    const int nxb = ns * 8;
    uint8_t *xbm = o.prep;
    float *qs = reinterpret_cast<float *>(o.prep + prep_xbm_bytes(m.K));
    if (prep && !o.prepared) {   // o.prepared: the producer of x prepared it, nothing to launch
        static bool attr[64];
        if (!attr[c->device]) {
            set_qkernel_attrs(prep_bm_kernel);
            attr[c->device] = true;
        }
        const int st = launch_k(prep_bm_kernel, dim3((nxb + 7) / 8, batch), dim3(64), 0, s, o.pdl, x, m.K, o.norm_w,
                                per, xbm, qs);
        if (st) return st;
        o.pdl = true;
    }
    if (kpieces > 1) {   // one group of `per` tokens, block-major: a piece's blocks are contiguous
        const int nsp = ns / kpieces;
        for (int i = 0; i < kpieces; ++i) {
            QMat mp = m;
            mp.w = m.w + (size_t)i * nsp * slice_bytes(QT);
            mp.K = nsp * 256;
            GemvOpts oi = o;
            oi.accum = i ? true : o.accum;
            const int st = launch_mma_nt<QT, 2>(c, mp, x, y, batch, p, oi, s, xbm + (size_t)i * nsp * 8 * per * 80,
                                                nullptr, m.row_bytes);
            if (st) return st;
            o.pdl = true;
        }
        return X100_OK;
    }
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int nb = std::min(per, batch - b0);
        const float *xb = x + (long)b0 * m.K;
        float *yb = y + (long)b0 * m.N;
        const uint8_t *gx = prep ? xbm + (size_t)(b0 / per) * nxb * per * 80 : nullptr;
        const float *gq = prep ? qs + (size_t)b0 * nxb : nullptr;
        const int st = p.nt == 2 ? launch_mma_nt<QT, 2>(c, m, xb, yb, nb, p, o, s, gx, gq)
                                 : launch_mma_nt<QT, 1>(c, m, xb, yb, nb, p, o, s, gx, gq);
        if (st) return st;
        o.pdl = true;
    }
    return X100_OK;
}

}  // namespace q

size_t qgemv_prep_bytes(int batch, int K) {
    return q::prep_xbm_bytes(K) + (size_t)batch * q::slices_per_row(K) * 8 * 4;
}

float *qgemv_prep_qs(uint8_t *prep, int K) { return reinterpret_cast<float *>(prep + q::prep_xbm_bytes(K)); }

int qgemv_mma_prep_group(const QMat &m, int batch, const GemvOpts &o) {
    const q::CallPlan cp = q::call_plan(m.qtype, m, batch, o);
    return cp.p.stages && cp.prep ? 8 * cp.p.nt : 0;
}

bool qgemv_mma_ok(int qt, int K) {
    return (qt == q::Q4_0 || qt == q::Q8_0) && q::mma_plan(qt, K, 8).stages > 0;
}

int launch_qgemv_mma(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const GemvOpts &o,
                     cudaStream_t s) {
    if (m.qtype == q::Q4_0) return q::launch_mma_qt<q::Q4_0>(c, m, x, y, batch, o, s);
    if (m.qtype == q::Q8_0) return q::launch_mma_qt<q::Q8_0>(c, m, x, y, batch, o, s);
    return X100_E_UNSUPPORTED;
}

}  // namespace x100
