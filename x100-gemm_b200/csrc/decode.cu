// decode.cu -- one decode step of a Qwen3-MoE-shaped model: the reference's
// forward() (qwen_moe_q3k.c:1842-1983) as a chain of sm_100a kernels, and the
// x100q_model_* entry points of include/x100q.h.
//
// Per layer and step (B tokens; token b uses sequence slot b, or slot[b]
// when a slot array is given -- several tokens of one sequence, e.g. a
// prefill chunk, then share a slot at different positions):
//   1. qkv  = Wqkv . rmsnorm(h; attn_norm)        qgemv (norm folded in), Q8_0
//   2. attention                                   attn_decode_kernel
//        q/k per-head rmsnorm (q_norm / k_norm) + NEOX RoPE, k and v of the
//        step written to the fp16 cache at pos (with a slot array: by
//        kv_write_kernel first, so every token of a shared slot sees the
//        others' earlier positions), softmax(q.K^T / sqrt(hd)) . V
//        over positions 0..pos (GQA: q head hh reads kv head hh / (nh/nkv))
//   3. h   += Wo . att                             qgemv (accumulate)
//   4. h   += MoE(rmsnorm(h; ffn_norm))            router (norm folded in) +
//                                                  expert kernels (accumulate)
// then logits = Wlm . rmsnorm(h; out_norm).  Every kernel is launched with
// programmatic dependent launch: it stages its weights, then waits for the
// previous kernel, so the chain of ~5 launches per layer streams weights
// back to back.
//
// KV cache: fp16, [layer][slot][kv_head][ctx][head_dim] for K and for V, so
// the positions a CTA attends over are one contiguous byte range per head
// (the reference's head-major layout, qwen_moe_q3k.c:1868-1880, in fp16).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../../include/x100q.h"
#include "moe.h"
#include "qgemm.h"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace dec {

using namespace q;

constexpr int kHD = 128;            // head_dim served by the attention kernel
constexpr int kAttnThreads = 256;   // 8 warps: one query head of the group each
constexpr int kPartStride = 132;    // floats per partial: o[128], m, l, pad

struct AttnArgs {
    const float *qkv;   // [B][qkv_n]: q heads, then k heads, then v heads
    int qkv_n;
    const float *q_norm, *k_norm;   // [hd]
    const int *pos;     // [B]: position of the step's token, < ctx
    int nh, nkv, ctx, nsplit, chunk;
    int cps;            // chunks of kChunk positions per split (1..8; above 1 a two-stage ring)
    float eps, rope_base, scale;
    const float2 *rope; // [ctx][hd / 2]: (cos, sin) of pos * base^(-2i / hd) (rope_table_kernel)
    __half *kc, *vc;    // this layer's cache, [B][nkv][ctx][hd]
    long row_base;      // cache row (of the tensor maps) of this layer's first row
    float *part;        // [B][nh][nsplit][kPartStride]
    int kv_early;       // stage K/V before waiting on the previous kernel (see the kernel)
    const int *slot;    // [B] sequence slot of each token, or null: token b uses slot b
    int nslots;         // slots of the cache (max_batch); a slot outside [0, nslots) is an error
    int prewritten;     // the step's k and v are already in the cache (kv_write_kernel)
    float *att;         // [B][nh * hd]
    int *status;
};

// The RoPE table: rope[pos][i] = (cos a, sin a), a = pos * base^(-2i/hd),
// i < hd / 2, with the reference's float expressions (rope_table,
// qwen_moe_q3k.c:1170-1172).  Built once per model: the angles depend only on
// the position, so every head, layer and attention split reads the same row.
__global__ void rope_table_kernel(float2 *__restrict__ rope, int ctx, float base) {
    for (long t = blockIdx.x * (long)blockDim.x + threadIdx.x; t < (long)ctx * (kHD / 2);
         t += (long)gridDim.x * blockDim.x) {
        const int pos = (int)(t / (kHD / 2)), i = (int)(t % (kHD / 2));
        const float fr = powf(base, -2.0f * (float)i / (float)kHD), a = (float)pos * fr;
        rope[t] = make_float2(cosf(a), sinf(a));
    }
}

// RMS norm (qwen_moe_q3k.c:1166) and NEOX RoPE (rope_apply,
// qwen_moe_q3k.c:1173-1175) of one 128-wide head held by a warp as 4
// consecutive elements per lane (lane l: elements 4l..4l+3).  The rotation
// pairs element i with i + 64, held by lane l ^ 16; rope_row = the table's
// row of the position.
__device__ __forceinline__ float4 norm_rope_head(float4 v, const float *__restrict__ nw, float eps,
                                                const float2 *__restrict__ rope_row) {
    const int lane = threadIdx.x & 31;
    float q = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
    const float s = 1.0f / sqrtf(q / (float)kHD + eps);
    const float4 w = __ldg(reinterpret_cast<const float4 *>(nw) + lane);
    v = make_float4(v.x * s * w.x, v.y * s * w.y, v.z * s * w.z, v.w * s * w.w);
    const float4 *rp = reinterpret_cast<const float4 *>(rope_row + ((4 * lane) & (kHD / 2 - 1)));
    const float4 r0 = __ldg(rp), r1 = __ldg(rp + 1);   // (cos, sin) of elements 4l .. 4l+3 mod 64
    const float cs[4] = {r0.x, r0.z, r1.x, r1.z}, sn[4] = {r0.y, r0.w, r1.y, r1.w};
    float e[4] = {v.x, v.y, v.z, v.w};
    float o[4];
    const bool first = lane < 16;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float other = __shfl_xor_sync(0xffffffffu, e[k], 16);
        o[k] = first ? e[k] * cs[k] - other * sn[k] : other * sn[k] + e[k] * cs[k];
    }
    return make_float4(o[0], o[1], o[2], o[3]);
}

// ---- tensor-core fragments (mma.sync m16n8k16, fp16 in, fp32 accumulate) ----
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    // A rows 8..15 are zero (a1 = a3 = 0): the 8 query heads of a kv head
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

constexpr int kChunk = 64;   // positions per CTA

// Byte offset of (row, dim) in a staged K or V tile: two sub-tiles of
// kChunk rows x 64 dims (128 B per row), 16-byte chunks XOR-swizzled by
// row % 8 -- the layout a 128-byte-swizzled TMA box writes.
__device__ __forceinline__ uint32_t kv_off(int row, int dim) {
    const int sub = dim >> 6, chunk = (dim & 63) >> 3;
    return (uint32_t)(sub * kChunk * 128 + row * 128 + ((chunk ^ (row & 7)) << 4) + (dim & 7) * 2);
}

// The step's k (normed, rotated) and v of every token into the cache at
// its slot and position, rounded to fp16 exactly as attn_decode_kernel's own
// write does.  Used when tokens may share a slot (a prefill chunk): the
// attention kernel then reads every position, the step's included, through
// the cache, so no token can miss another's earlier position.  grid (nkv, B),
// one warp; a position or slot out of range writes nothing (the attention
// kernel reports it).
__global__ void __launch_bounds__(32) kv_write_kernel(const AttnArgs a) {
    const int kvh = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();   // qkv comes from the previous kernel
    const int pos = a.pos[b], sb = a.slot ? a.slot[b] : b;
    if (pos < 0 || pos >= a.ctx || sb < 0 || sb >= a.nslots) return;
    const long head_row = ((long)sb * a.nkv + kvh) * a.ctx;
    const float *qrow = a.qkv + (long)b * a.qkv_n;
    float4 k = __ldcg(reinterpret_cast<const float4 *>(qrow + (a.nh + kvh) * kHD) + lane);
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(qrow + (a.nh + a.nkv + kvh) * kHD) + lane);
    k = norm_rope_head(k, a.k_norm, a.eps, a.rope + (long)pos * (kHD / 2));
    uint2 kk, vv;
    kk.x = h2u(__floats2half2_rn(k.x, k.y));
    kk.y = h2u(__floats2half2_rn(k.z, k.w));
    vv.x = h2u(__floats2half2_rn(v.x, v.y));
    vv.y = h2u(__floats2half2_rn(v.z, v.w));
    reinterpret_cast<uint2 *>(a.kc + (head_row + pos) * kHD)[lane] = kk;
    reinterpret_cast<uint2 *>(a.vc + (head_row + pos) * kHD)[lane] = vv;
}

// Grid (nsplit, nkv, B).  CTA (sp, kvh, b) attends the query heads of kv head
// kvh over positions [sp*64*cps, min((sp+1)*64*cps, pos+1)), cps chunks of 64
// positions (a.cps; above one they stream through a two-stage ring).  A
// chunk's K and V rows arrive by TMA (two 64-dim boxes each, 128-byte
// swizzle); the queries of the group (warp h: head kvh*gpr + h) are normed,
// rotated and held as the rows of an m16n8k16 A operand (rows gpr..15 zero).
// Warp w < 4 computes the scores S = Q.K^T of positions [16w, 16w+16) of the
// chunk on the tensor cores; the CTA-wide row max and sum go through shared
// memory and update the running max, sum and output of each head (online
// softmax); P = e^(S-M) is stored as fp16 and warp w accumulates
// O[:, 16w..16w+16) += P.V.  The chunk holding pos first gets the step's k
// and v (norm + RoPE on k), stored to the cache in fp16 and into the staged
// tile.  Output: a partial (o, m, l) per head, merged by attn_merge_kernel (or
// att itself when there is one split).
// With kv_early the step began behind a full barrier (every earlier step is
// complete), so positions < pos of the cache are final and the CTA reads pos
// and stages its K/V rows before waiting on the previous kernel.
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                   const __grid_constant__ CUtensorMap tmV,
                                                                   const AttnArgs a) {
    constexpr int C = kChunk, PS = C + 8;   // P row stride (halfs): conflict-free fragment loads
    constexpr uint32_t kStageBytes = 4u * C * 128;   // K and V of one chunk
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int cps = a.cps, nst = cps > 1 ? 2 : 1;            // chunks of this split, ring stages
    float *sQ = reinterpret_cast<float *>(base + nst * kStageBytes);   // [8][hd]
    __half *sP = reinterpret_cast<__half *>(sQ + 8 * kHD);        // [8][PS]
    float *sMax = reinterpret_cast<float *>(sP + 8 * PS);         // [8 warps][8 heads]
    float *sSum = sMax + 64;
    __shared__ uint64_t bar[2];
    __shared__ int abort_flag;
    const int sp = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gpr = a.nh / a.nkv;
    const int hq = lane >> 2, q4 = lane & 3;   // fragment row (head) and column pair
    const int j0s = sp * cps * C;               // first position of this split
    int sb = a.slot ? __ldg(a.slot + b) : b;                  // written before the step began
    const bool bad_slot = sb < 0 || sb >= a.nslots;
    if (bad_slot) sb = 0;                                     // nothing is staged or read for it
    const long head_row = ((long)sb * a.nkv + kvh) * a.ctx;  // cache row of position 0 in this layer
    int pos = 0, nch = 0;                                     // chunks holding positions <= pos
    auto chunks = [&]() {
        pos = bad_slot ? -1 : a.pos[b];
        nch = (pos < 0 || pos >= a.ctx) ? 0 : min(cps, (pos - j0s) / C + 1);
        if (pos < j0s) nch = 0;
    };
    auto stage = [&](int c) {   // thread 0: the four TMA boxes of chunk c into stage c % nst
        const int st = c % nst;
        uint8_t *sK = base + st * kStageBytes, *sV = sK + 2 * C * 128;
        mbar_arrive_expect_tx(&bar[st], kStageBytes);
        const int row = (int)(a.row_base + head_row + j0s + c * C);
        tma_load_2d(sK, &tmK, 0, row, &bar[st]);
        tma_load_2d(sK + C * 128, &tmK, 64, row, &bar[st]);
        tma_load_2d(sV, &tmV, 0, row, &bar[st]);
        tma_load_2d(sV + C * 128, &tmV, 64, row, &bar[st]);
    };
    int issued = 0;                              // thread 0: chunks whose copies were started
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int st = 0; st < nst; ++st) mbar_init(&bar[st], 1);
        fence_barrier_init();
    }
    bool staged = false;
    if (a.kv_early) {
        chunks();
        if (threadIdx.x == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            for (; issued < min(nst, nch); ++issued) stage(issued);
        }
        staged = true;
    }
    pdl_launch_dependents();
    pdl_wait();                                   // qkv comes from the previous kernel
    if (!staged) {
        chunks();
        if (threadIdx.x == 0)
            for (; issued < min(nst, nch); ++issued) stage(issued);
    }
    if (pos < 0 || pos >= a.ctx) {   // KV overflow (the reference aborts, qwen_moe_q3k.c:1865-1868)
        if (threadIdx.x == 0 && sp == 0 && kvh == 0) atomicCAS(a.status, 0, X100_E_ARG);
        return;
    }
    const float *qrow = a.qkv + (long)b * a.qkv_n;
    if (warp < gpr && nch > 0) {
        const int hh = kvh * gpr + warp;
        float4 v = __ldcg(reinterpret_cast<const float4 *>(qrow + hh * kHD) + lane);
        v = norm_rope_head(v, a.q_norm, a.eps, a.rope + (long)pos * (kHD / 2));
        reinterpret_cast<float4 *>(sQ + warp * kHD)[lane] = v;
    }
    __syncthreads();                              // barriers initialised, queries ready
    // running softmax state of head hq (the same in every warp) and this
    // warp's 16 output dims of it
    float m_run = -INFINITY, l_run = 0.f;
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    bool ok = nch > 0;
    int done = 0;
    for (int c = 0; c < nch; ++c) {
        const int st = c % nst, j0 = j0s + c * C, n = min(C, pos + 1 - j0);
        uint8_t *sK = base + st * kStageBytes, *sV = sK + 2 * C * 128;
        mbar_wait(&bar[st], (uint32_t)((c / nst) & 1), &abort_flag, a.status);   // raises abort_flag on timeout
        done = c + 1;
        if (pos < j0 + C && warp == 0 && !a.prewritten && abort_flag == 0) {
            // the step's own k (normed, rotated) and v, rounded to the cache's fp16
            float4 k = __ldcg(reinterpret_cast<const float4 *>(qrow + (a.nh + kvh) * kHD) + lane);
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(qrow + (a.nh + a.nkv + kvh) * kHD) + lane);
            k = norm_rope_head(k, a.k_norm, a.eps, a.rope + (long)pos * (kHD / 2));
            uint2 kk, vv;
            kk.x = h2u(__floats2half2_rn(k.x, k.y));
            kk.y = h2u(__floats2half2_rn(k.z, k.w));
            vv.x = h2u(__floats2half2_rn(v.x, v.y));
            vv.y = h2u(__floats2half2_rn(v.z, v.w));
            reinterpret_cast<uint2 *>(a.kc + (head_row + pos) * kHD)[lane] = kk;
            reinterpret_cast<uint2 *>(a.vc + (head_row + pos) * kHD)[lane] = vv;
            *reinterpret_cast<uint2 *>(sK + kv_off(pos - j0, 4 * lane)) = kk;
            *reinterpret_cast<uint2 *>(sV + kv_off(pos - j0, 4 * lane)) = vv;
        }
        __syncthreads();
        ok = abort_flag == 0;                     // uniform over the CTA
        if (!ok) break;
        // ---- S = Q . K^T for positions [16 warp, 16 warp + 16) of the chunk ----
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int pw = 16 * warp;
        const bool sw = pw < C;                   // warps holding score columns
        if (sw && pw < n) {
            const uint32_t kbase = smem_u32(sK);
            const int m = lane >> 3, r = lane & 7;
            const int prow = pw + (m >> 1) * 8 + r;
#pragma unroll
            for (int kk = 0; kk < kHD / 16; ++kk) {
                const float *qr = sQ + hq * kHD + 16 * kk + 2 * q4;
                const bool live = hq < gpr;
                const uint32_t a0 = live ? h2u(__floats2half2_rn(qr[0], qr[1])) : 0u;
                const uint32_t a2 = live ? h2u(__floats2half2_rn(qr[8], qr[9])) : 0u;
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbase + kv_off(prow, 16 * kk + (m & 1) * 8), b0, b1, b2, b3);
                mma16816(acc[0], a0, a2, b0, b1);
                mma16816(acc[1], a0, a2, b2, b3);
            }
        }
        // scores of head hq at positions pw + 8 nt + 2 q4 + {0, 1}; masked past n
        float sc[4];
        float mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int jj = pw + 8 * (t >> 1) + 2 * q4 + (t & 1);
            sc[t] = jj < n ? acc[t >> 1][t & 1] * a.scale : -INFINITY;
            mx = fmaxf(mx, sc[t]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (q4 == 0) sMax[warp * 8 + hq] = mx;
        __syncthreads();
        float M = m_run;
#pragma unroll
        for (int w = 0; w < 8; ++w) M = fmaxf(M, sMax[w * 8 + hq]);
        const float alpha = expf(m_run - M);      // 0 for the first chunk (m_run = -inf)
        float ps[4], lsum = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            ps[t] = sc[t] == -INFINITY ? 0.f : expf(sc[t] - M);
            lsum += ps[t];
        }
        if (sw) {
            *reinterpret_cast<__half2 *>(sP + hq * PS + pw + 2 * q4) = __floats2half2_rn(ps[0], ps[1]);
            *reinterpret_cast<__half2 *>(sP + hq * PS + pw + 8 + 2 * q4) = __floats2half2_rn(ps[2], ps[3]);
        }
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 1);
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 2);
        if (q4 == 0) sSum[warp * 8 + hq] = lsum;
        __syncthreads();
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) L += sSum[w * 8 + hq];
        l_run = l_run * alpha + L;
        m_run = M;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) o[nt][i] *= alpha;
        // ---- O[:, 16 warp .. +16) += P . V ----
        const int d0 = 16 * warp;
        {
            const uint32_t vbase = smem_u32(sV);
            const int m = lane >> 3, r = lane & 7;
#pragma unroll
            for (int kk = 0; kk < C / 16; ++kk) {
                if (16 * kk < n) {
                    const uint32_t a0 = *reinterpret_cast<const uint32_t *>(sP + hq * PS + 16 * kk + 2 * q4);
                    const uint32_t a2 = *reinterpret_cast<const uint32_t *>(sP + hq * PS + 16 * kk + 8 + 2 * q4);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(vbase + kv_off(16 * kk + (m & 1) * 8 + r, d0 + (m >> 1) * 8), b0, b1, b2, b3);
                    mma16816(o[0], a0, a2, b0, b1);
                    mma16816(o[1], a0, a2, b2, b3);
                }
            }
        }
        __syncthreads();                          // stage st and sP are free again
        if (threadIdx.x == 0 && issued < nch) stage(issued++);
    }
    // o[nt][0..1]: head hq, dims 16 warp + 8 nt + 2 q4 + {0, 1}
    const bool live = hq < gpr;
    const int hh = kvh * gpr + hq, d0 = 16 * warp;
    if (live && nch > 0) {
        if (a.nsplit == 1) {
            const float inv = ok && l_run > 0.f ? 1.0f / l_run : 0.f;
            float *out = a.att + (long)b * a.nh * kHD + hh * kHD + d0 + 2 * q4;
            *reinterpret_cast<float2 *>(out) = make_float2(o[0][0] * inv, o[0][1] * inv);
            *reinterpret_cast<float2 *>(out + 8) = make_float2(o[1][0] * inv, o[1][1] * inv);
        } else {
            float *pr = a.part + (((long)b * a.nh + hh) * a.nsplit + sp) * kPartStride;
            *reinterpret_cast<float2 *>(pr + d0 + 2 * q4) = make_float2(o[0][0], o[0][1]);
            *reinterpret_cast<float2 *>(pr + d0 + 8 + 2 * q4) = make_float2(o[1][0], o[1][1]);
            if (warp == 0 && q4 == 0) {
                pr[kHD] = ok ? m_run : -INFINITY;
                pr[kHD + 1] = ok ? l_run : 0.f;
            }
        }
    } else if (live && a.nsplit > 1) {            // a split past pos: an empty partial
        float *pr = a.part + (((long)b * a.nh + hh) * a.nsplit + sp) * kPartStride;
        *reinterpret_cast<float2 *>(pr + d0 + 2 * q4) = make_float2(0.f, 0.f);
        *reinterpret_cast<float2 *>(pr + d0 + 8 + 2 * q4) = make_float2(0.f, 0.f);
        if (warp == 0 && q4 == 0) {
            pr[kHD] = -INFINITY;
            pr[kHD + 1] = 0.f;
        }
    }
    if (threadIdx.x == 0 && !ok)                  // copies still in flight after a timeout
        for (int c = done; c < issued; ++c) mbar_wait_drain(&bar[c % nst], (uint32_t)((c / nst) & 1), 100000000ull);
}

// Grid (nh, B), 128 threads: att[b][head] = sum_s e^(m_s-M) o_s / sum_s
// e^(m_s-M) l_s over the splits of attn_decode_kernel.  Warp w sums the
// splits of its quarter (16 loads in flight per lane), the quarters are added
// in order, so the result does not depend on timing.  PREP: it also writes
// the head's four 32-element blocks prepared for the Wo GEMV into xbm
// (xprep_vals, the preparation kernel's layout: groups of ntok tokens, nxb
// blocks a token), so that call launches no preparation of its own (a
// separate instantiation: the code changes the main loop's register use,
// which cost the one-token step 4 us a layer).
template <bool PREP>
__global__ void __launch_bounds__(128) attn_merge_kernel(const float *__restrict__ part, int nh, int nsplit,
                                                         float *__restrict__ att, uint8_t *__restrict__ xbm,
                                                         int ntok, int nxb) {
    extern __shared__ float msm[];
    // sO [4][hd] starts on a 16-byte boundary (float4 accesses)
    float *sW = msm, *sL = msm + nsplit, *sO = msm + ((2 * nsplit + 3) & ~3);
    const int hh = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch_dependents();
    pdl_wait();                                   // the partials come from the attention kernel
    const float *pr = part + ((long)b * nh + hh) * nsplit * kPartStride;
    for (int s2 = threadIdx.x; s2 < nsplit; s2 += blockDim.x) {
        sW[s2] = __ldcg(pr + s2 * kPartStride + kHD);
        sL[s2] = __ldcg(pr + s2 * kPartStride + kHD + 1);
    }
    __syncthreads();
    if (warp == 0) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < nsplit; s2 += 32) M = fmaxf(M, sW[s2]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        for (int s2 = lane; s2 < nsplit; s2 += 32) {
            const float ms = sW[s2];
            sW[s2] = ms == -INFINITY ? 0.f : expf(ms - M);   // splits past pos weigh 0
        }
    }
    __syncthreads();
    const int q = (nsplit + 3) / 4, s_lo = warp * q, s_hi = min(nsplit, s_lo + q);
    const float4 *po = reinterpret_cast<const float4 *>(pr) + lane;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = s_lo; s0 < s_hi; s0 += 16) {
        float4 t[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
            if (s0 + u < s_hi) t[u] = __ldcg(po + (s0 + u) * (kPartStride / 4));
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            if (s0 + u < s_hi) {
                const float wgt = sW[s0 + u];
                O.x = fmaf(wgt, t[u].x, O.x);
                O.y = fmaf(wgt, t[u].y, O.y);
                O.z = fmaf(wgt, t[u].z, O.z);
                O.w = fmaf(wgt, t[u].w, O.w);
            }
        }
    }
    reinterpret_cast<float4 *>(sO + warp * kHD)[lane] = O;
    __syncthreads();
    if (warp == 0) {
        float Ls = 0.f;
        for (int s2 = 0; s2 < nsplit; ++s2) Ls = fmaf(sW[s2], sL[s2], Ls);
        float4 T = reinterpret_cast<const float4 *>(sO)[lane];
#pragma unroll
        for (int w = 1; w < 4; ++w) {
            const float4 u = reinterpret_cast<const float4 *>(sO + w * kHD)[lane];
            T = make_float4(T.x + u.x, T.y + u.y, T.z + u.z, T.w + u.w);
        }
        const float inv = Ls > 0.f ? 1.0f / Ls : 0.f;
        const float4 v = make_float4(T.x * inv, T.y * inv, T.z * inv, T.w * inv);
        reinterpret_cast<float4 *>(att + (long)b * nh * kHD + hh * kHD)[lane] = v;
        if constexpr (PREP) {   // lanes 8i .. 8i+7 hold block i of the head: the preparation's own grouping
            const int j = hh * (kHD / 32) + (lane >> 3);
            xprep_vals(v, reinterpret_cast<XB *>(xbm + (((long)(b / ntok) * nxb + j) * ntok + b % ntok) * 80),
                       lane & 7, true);
        }
    }
}

// h[b][:] = tok_embd[tok[b]][:] (the reference's memcpy of the embedding row,
// qwen_moe_q3k.c:1845).  Token ids outside [0, vocab) leave h untouched and
// raise X100_E_ARG in the status word.
__global__ void __launch_bounds__(256) embed_kernel(const float *__restrict__ emb, int vocab, int d,
                                                    const int *__restrict__ tok, float *__restrict__ h,
                                                    int *status) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.y;
    const int t = tok[b];
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicCAS(status, 0, X100_E_ARG);
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d / 4; i += gridDim.x * blockDim.x)
        reinterpret_cast<float4 *>(h + (long)b * d)[i] = __ldg(reinterpret_cast<const float4 *>(emb + (long)t * d) + i);
}

static size_t attn_smem(int cps = 1) {
    return 1024 + (size_t)(cps > 1 ? 2 : 1) * 4 * kChunk * 128 + 8 * kHD * 4 + 8 * (kChunk + 8) * 2 + 128 * 4;
}
// Chunks per attention split (cps) for a decode step of `batch` tokens over
// ctx positions.  A CTA streams its cps chunks through the TMA ring, so a wave
// of the grid lasts about cps chunk times: the choice minimises waves x cps,
// a wave being the SM count x the CTAs resident on an SM, and on a tie takes
// more chunks per CTA (fewer splits to merge, less setup per chunk).  At
// context 4096 this picks 1 at batch 1, 2 at batch 2, 3 at batch 4 and 5 at
// batch 16, the best of the measured settings (batch 16: 1948 tokens/s with
// 5, 1916 with 4, 1926 with 6; batch 4: 901 with 3, 892 with 4, 864 with 1).
// X100_ATTN_CPS (1..8) overrides the choice.
static int attn_cps(int batch, int nkv, int ctx, int device, int sm_count) {
    static const int forced = [] {
        const char *e = getenv("X100_ATTN_CPS");
        const int v = e ? atoi(e) : 0;
        return v >= 1 && v <= 8 ? v : 0;
    }();
    if (forced) return forced;
    static int occ[64][9];   // resident CTAs per SM for each cps (its shared memory)
    int best = 1;
    long best_cost = -1;
    for (int cps = 1; cps <= 8; ++cps) {
        int &r = occ[device & 63][cps];
        if (!r) {
            int n = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_decode_kernel, kAttnThreads, attn_smem(cps));
            r = n > 0 ? n : 1;
        }
        const long ctas = (long)((ctx + kChunk * cps - 1) / (kChunk * cps)) * nkv * batch;
        const long slots = (long)sm_count * r, cost = (ctas + slots - 1) / slots * cps;
        if (best_cost < 0 || cost <= best_cost) {
            best_cost = cost;
            best = cps;
        }
    }
    return best;
}
static size_t merge_smem(int nsplit) { return (size_t)(((2 * nsplit + 3) & ~3) + 4 * kHD) * 4; }

}  // namespace dec
}  // namespace x100

using namespace x100;
using namespace x100::dec;

struct ModelLayer {
    QMat qkv, o;
    float *norms = nullptr;   // attn_norm[d], ffn_norm[d], q_norm[hd], k_norm[hd]
    MoeLayer moe;
    bool set = false;
};

// Per-bucket step timing (x100q_model_timing): a CUDA event at each bucket
// boundary of a forward call; the interval from event i to event i + 1 is
// charged to bucket[i] (-1: not charged, the gap between calls).
struct StepTimer {
    bool on = false;
    std::vector<cudaEvent_t> ev;
    std::vector<int> bucket;
    int used = 0;
    double ms[X100Q_NBUCKETS] = {};
    long steps = 0;
};
static void timer_flush(StepTimer &t) {
    if (t.used >= 2 && cudaEventSynchronize(t.ev[t.used - 1]) == cudaSuccess)
        for (int i = 0; i + 1 < t.used; ++i) {
            float ms = 0.f;
            if (t.bucket[i] >= 0 && cudaEventElapsedTime(&ms, t.ev[i], t.ev[i + 1]) == cudaSuccess)
                t.ms[t.bucket[i]] += ms;
        }
    cudaGetLastError();
    t.used = 0;
}
// Start bucket b (-1: end of a call) on stream s.
static void timer_mark(StepTimer &t, int b, cudaStream_t s) {
    if (!t.on) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return;
    }
    if (t.used >= 4096) {   // keep the pool bounded: settle what is recorded, keep the open interval
        const int last = t.bucket[t.used - 1];
        timer_flush(t);
        if (last >= 0) timer_mark(t, last, s);
    }
    if (t.used == (int)t.ev.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        t.ev.push_back(e);
        t.bucket.push_back(-1);
    }
    if (cudaEventRecord(t.ev[t.used], s) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    t.bucket[t.used++] = b;
}
static void timer_mark_cb(void *ctx, int b, cudaStream_t s) { timer_mark(*static_cast<StepTimer *>(ctx), b, s); }

struct x100q_model {
    int device = 0;
    StepTimer timer;
    x100q_model_cfg cfg;
    std::vector<ModelLayer> layers;
    float *tok_embd = nullptr, *out_norm = nullptr;
    QMat lm;
    __half *kc = nullptr, *vc = nullptr;   // [layer][slot][nkv][ctx][hd]
    size_t layer_kv = 0;                   // halfs per layer
    CUtensorMap tmK, tmV;                  // the caches as rows of 128 fp16, boxes of 64 x 128
    // scratch
    void *scratch = nullptr;
    float *qkv = nullptr, *att = nullptr, *hn = nullptr, *part = nullptr;
    float2 *rope = nullptr;   // [ctx][64] RoPE table
    uint8_t *prep = nullptr;  // prepared activations of the batched GEMVs (GemvOpts::prep)
    void *moe_scratch = nullptr;
    MoeScratch S;
    int nsplit_max = 0;
    // many-token prefill (chunks of up to pf_tmax tokens on the tensor-core
    // GEMMs), allocated on first use
    void *pf_base = nullptr;
    int pf_tmax = 0;
    float *pf_qkv = nullptr, *pf_att = nullptr;   // [tmax][qkv rows], [tmax][n_heads * hd]
    __half *pf_xh = nullptr, *pf_xl = nullptr;    // [tmax][kp] fp16 planes of a linear's input
    int pf_kp = 0;
    MoeBigScratch pf_moe;
};

static bool cfg_ok(const x100q_model_cfg *c) {
    if (!c) return false;
    const bool qt_ok = (c->attn_qtype == X100Q_Q8_0 || c->attn_qtype == X100Q_Q4_0 || c->attn_qtype == X100Q_Q4_K ||
                        c->attn_qtype == X100Q_Q3_K) &&
                       (c->lm_qtype == X100Q_Q8_0 || c->lm_qtype == X100Q_Q4_0 || c->lm_qtype == X100Q_Q4_K ||
                        c->lm_qtype == X100Q_Q3_K);
    return qt_ok && c->n_layers > 0 && c->head_dim == kHD && c->n_kv_heads > 0 && c->n_heads % c->n_kv_heads == 0 &&
           c->n_heads / c->n_kv_heads <= 8 && c->vocab > 0 && c->ctx > 0 && c->ctx <= 131072 && c->max_batch >= 1 &&
           c->max_batch <= 16 && c->expert_lo >= 0 && c->expert_hi <= c->n_exp && c->expert_lo < c->expert_hi &&
           c->d % 256 == 0 && (c->n_heads * c->head_dim) % 256 == 0 &&
           moe_shapes_ok(c->d, c->n_exp, c->n_act, c->moe_ffn, c->expert_qtype) && c->eps > 0.f;
}

static int qkv_rows(const x100q_model_cfg &c) { return (c.n_heads + 2 * c.n_kv_heads) * c.head_dim; }

extern "C" {

x100q_model *x100q_model_create(const x100q_model_cfg *cfg) {
    set_error(X100_OK);
    if (!cfg_ok(cfg)) {
        set_error(X100_E_ARG);
        return nullptr;
    }
    DevCtx *c = ctx();
    if (!c) return nullptr;
    if (fault_injected("alloc")) return nullptr;
    x100q_model *m = new x100q_model();
    m->device = c->device;
    m->cfg = *cfg;
    m->layers.resize(cfg->n_layers);
    const x100q_model_cfg &g = *cfg;
    m->layer_kv = (size_t)g.max_batch * g.n_kv_heads * g.ctx * g.head_dim;
    const size_t kvb = (size_t)g.n_layers * m->layer_kv * 2;
    m->nsplit_max = (g.ctx + kChunk - 1) / kChunk;
    const size_t qkvb = (size_t)g.max_batch * qkv_rows(g) * 4, attb = (size_t)g.max_batch * g.n_heads * kHD * 4,
                 hnb = (size_t)g.max_batch * g.d * 4,
                 partb = (size_t)g.max_batch * g.n_heads * m->nsplit_max * kPartStride * 4,
                 ropeb = (size_t)g.ctx * (kHD / 2) * sizeof(float2),
                 prepb = qgemv_prep_bytes(16, std::max(g.d, g.n_heads * kHD));
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t sb = up(qkvb) + up(attb) + up(hnb) + up(partb) + up(ropeb) + up(prepb);
    const size_t msb = moe_scratch_bytes(g.d, g.n_exp, g.n_act, g.moe_ffn);
    bool ok = cudaMalloc(&m->kc, kvb) == cudaSuccess && cudaMalloc(&m->vc, kvb) == cudaSuccess &&
              cudaMalloc(&m->scratch, sb) == cudaSuccess && cudaMalloc(&m->moe_scratch, msb) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        x100q_model_destroy(m);
        return nullptr;
    }
    cudaMemset(m->kc, 0, kvb);
    cudaMemset(m->vc, 0, kvb);
    const uint64_t rows = (uint64_t)g.n_layers * g.max_batch * g.n_kv_heads * g.ctx;
    if (!make_tmap_2d(&m->tmK, m->kc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHD, rows, kHD * 2, 64, kChunk) ||
        !make_tmap_2d(&m->tmV, m->vc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kHD, rows, kHD * 2, 64, kChunk)) {
        set_error(X100_E_UNSUPPORTED);
        x100q_model_destroy(m);
        return nullptr;
    }
    cudaMemset(m->scratch, 0, sb);
    cudaMemset(m->moe_scratch, 0, msb);
    uint8_t *p = static_cast<uint8_t *>(m->scratch);
    m->qkv = reinterpret_cast<float *>(p);
    p += up(qkvb);
    m->att = reinterpret_cast<float *>(p);
    p += up(attb);
    m->hn = reinterpret_cast<float *>(p);
    p += up(hnb);
    m->part = reinterpret_cast<float *>(p);
    p += up(partb);
    m->rope = reinterpret_cast<float2 *>(p);
    p += up(ropeb);
    m->prep = p;
    rope_table_kernel<<<256, 256>>>(m->rope, g.ctx, g.rope_base);
    m->S = moe_scratch_carve(m->moe_scratch, g.d, g.n_exp, g.n_act, g.moe_ffn);
    if (check_cuda(cudaDeviceSynchronize(), X100_E_ALLOC)) {
        x100q_model_destroy(m);
        return nullptr;
    }
    return m;
}

void x100q_model_destroy(x100q_model *m) {
    if (!m) return;
    DeviceGuard dg(m->device);
    for (ModelLayer &L : m->layers) {
        cudaFree(L.qkv.w);
        cudaFree(L.o.w);
        cudaFree(L.norms);
        moe_layer_free(L.moe);
    }
    cudaFree(m->tok_embd);
    cudaFree(m->out_norm);
    cudaFree(m->lm.w);
    cudaFree(m->kc);
    cudaFree(m->vc);
    cudaFree(m->scratch);
    cudaFree(m->moe_scratch);
    cudaFree(m->pf_base);
    for (cudaEvent_t e : m->timer.ev) cudaEventDestroy(e);
    delete m;
}

int x100q_model_set_layer(x100q_model *m, int layer, const float *attn_norm, const void *wq, const void *wk,
                          const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                          const float *ffn_norm, const float *router, const void *gate_exps, const void *up_exps,
                          const void *down_exps) {
    set_error(X100_OK);
    if (!m || layer < 0 || layer >= m->cfg.n_layers || !attn_norm || !wq || !wk || !wv || !q_norm || !k_norm ||
        !wo || !ffn_norm || !router || !gate_exps || !up_exps || !down_exps) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const x100q_model_cfg &g = m->cfg;
    ModelLayer &L = m->layers[layer];
    if (L.set) {   // replace: free the old weights first
        cudaFree(L.qkv.w);
        cudaFree(L.o.w);
        cudaFree(L.norms);
        moe_layer_free(L.moe);
        L = ModelLayer();
    }
    const int qd = g.n_heads * g.head_dim, kvd = g.n_kv_heads * g.head_dim;
    const size_t rb = x100q_row_bytes(g.attn_qtype, g.d);
    // q, k, v rows concatenated into one matrix (one GEMV per step)
    void *cat = nullptr;
    bool ok = cudaMalloc(&cat, (size_t)qkv_rows(g) * rb) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        return X100_E_ALLOC;
    }
    uint8_t *cp = static_cast<uint8_t *>(cat);
    ok = check_cuda(cudaMemcpy(cp, wq, (size_t)qd * rb, cudaMemcpyDefault), X100_E_COPY) == 0 &&
         check_cuda(cudaMemcpy(cp + (size_t)qd * rb, wk, (size_t)kvd * rb, cudaMemcpyDefault), X100_E_COPY) == 0 &&
         check_cuda(cudaMemcpy(cp + (size_t)(qd + kvd) * rb, wv, (size_t)kvd * rb, cudaMemcpyDefault),
                    X100_E_COPY) == 0;
    ok = ok && qmat_upload(c, g.attn_qtype, qkv_rows(g), g.d, cat, L.qkv, c->stream);
    cudaFree(cat);
    ok = ok && qmat_upload(c, g.attn_qtype, g.d, qd, wo, L.o, c->stream);
    if (ok) {
        const size_t nb = (size_t)(2 * g.d + 2 * g.head_dim) * 4;
        if (cudaMalloc(&L.norms, nb) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            ok = false;
        } else {
            ok = check_cuda(cudaMemcpy(L.norms, attn_norm, (size_t)g.d * 4, cudaMemcpyDefault), X100_E_COPY) == 0 &&
                 check_cuda(cudaMemcpy(L.norms + g.d, ffn_norm, (size_t)g.d * 4, cudaMemcpyDefault), X100_E_COPY) ==
                     0 &&
                 check_cuda(cudaMemcpy(L.norms + 2 * g.d, q_norm, (size_t)g.head_dim * 4, cudaMemcpyDefault),
                            X100_E_COPY) == 0 &&
                 check_cuda(cudaMemcpy(L.norms + 2 * g.d + g.head_dim, k_norm, (size_t)g.head_dim * 4,
                                       cudaMemcpyDefault),
                            X100_E_COPY) == 0;
        }
    }
    ok = ok && moe_layer_upload(c, L.moe, g.d, g.n_exp, g.n_act, g.moe_ffn, g.expert_qtype, router, gate_exps,
                                up_exps, down_exps, g.expert_lo, g.expert_hi);
    if (!ok) {
        cudaFree(L.qkv.w);
        cudaFree(L.o.w);
        cudaFree(L.norms);
        L = ModelLayer();
        return get_error() ? get_error() : X100_E_COPY;
    }
    L.set = true;
    return X100_OK;
}

int x100q_model_set_output(x100q_model *m, const float *tok_embd, const float *out_norm, const void *lm) {
    set_error(X100_OK);
    if (!m || !out_norm) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const x100q_model_cfg &g = m->cfg;
    cudaFree(m->tok_embd);
    cudaFree(m->out_norm);
    cudaFree(m->lm.w);
    m->tok_embd = nullptr;
    m->out_norm = nullptr;
    m->lm = QMat();
    bool ok = cudaMalloc(&m->out_norm, (size_t)g.d * 4) == cudaSuccess;
    if (ok && tok_embd) ok = cudaMalloc(&m->tok_embd, (size_t)g.vocab * g.d * 4) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        return X100_E_ALLOC;
    }
    ok = check_cuda(cudaMemcpy(m->out_norm, out_norm, (size_t)g.d * 4, cudaMemcpyDefault), X100_E_COPY) == 0;
    if (ok && tok_embd)
        ok = check_cuda(cudaMemcpy(m->tok_embd, tok_embd, (size_t)g.vocab * g.d * 4, cudaMemcpyDefault),
                        X100_E_COPY) == 0;
    if (ok && lm) ok = qmat_upload(c, g.lm_qtype, g.vocab, g.d, lm, m->lm, c->stream);
    return ok ? X100_OK : get_error();
}

int x100q_model_kv_copy(x100q_model *m, int layer, int slot, int pos0, int npos, void *k, void *v, int to_cache) {
    set_error(X100_OK);
    const x100q_model_cfg *g = m ? &m->cfg : nullptr;
    if (!m || layer < 0 || layer >= g->n_layers || slot < 0 || slot >= g->max_batch || pos0 < 0 || npos < 0 ||
        pos0 + npos > g->ctx || !k || !v) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    const size_t row = (size_t)g->head_dim * 2, span = (size_t)npos * row;
    for (int h = 0; h < g->n_kv_heads; ++h) {
        const size_t off = (size_t)layer * m->layer_kv + (((size_t)slot * g->n_kv_heads + h) * g->ctx + pos0) * g->head_dim;
        uint8_t *hk = static_cast<uint8_t *>(k) + h * span, *hv = static_cast<uint8_t *>(v) + h * span;
        cudaError_t e1, e2;
        if (to_cache) {
            e1 = cudaMemcpy(m->kc + off, hk, span, cudaMemcpyDefault);
            e2 = cudaMemcpy(m->vc + off, hv, span, cudaMemcpyDefault);
        } else {
            e1 = cudaMemcpy(hk, m->kc + off, span, cudaMemcpyDefault);
            e2 = cudaMemcpy(hv, m->vc + off, span, cudaMemcpyDefault);
        }
        if (check_cuda(e1, X100_E_COPY) || check_cuda(e2, X100_E_COPY)) return X100_E_COPY;
    }
    return X100_OK;
}

int x100q_model_embed_dev(x100q_model *m, const int *tokens, float *h, int batch, void *stream) {
    set_error(X100_OK);
    if (!m || !tokens || !h || batch < 1 || batch > m->cfg.max_batch || !m->tok_embd) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(embed_kernel);
        attr[c->device] = true;
    }
    // an ordinary launch: the step starts behind a full barrier, which lets the
    // attention kernels of the step stage cache rows early (AttnArgs::kv_early)
    const int st = launch_k(embed_kernel, dim3(2, batch), dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                            (const float *)m->tok_embd, m->cfg.vocab, m->cfg.d, tokens, h, c->d_status);
    if (st) set_error(st);
    return st;
}

}  // extern "C"

// One layer, steps 1-4 of the file comment.  kv_early: the step began behind
// a full barrier (see attn_decode_kernel); barrier: launch the first kernel
// behind one.  slot: per-token cache slots (null: token b uses slot b); with
// it the step's k and v go to the cache in a kernel of their own first.
// next_m / next_nw: the GEMV that reads h after this layer (the next layer's
// q/k/v, or the lm_head) and its RMS norm, for the MoE combine to prepare its
// activations (*next_prepared says whether it does); qkv_prepared: this
// layer's q/k/v activations were prepared that way by the previous layer.
static int layer_launch(x100q_model *m, DevCtx *c, int layer, float *h, const int *pos, int batch, float *eout,
                        cudaStream_t s, bool kv_early, bool barrier, const int *slot = nullptr,
                        const QMat *next_m = nullptr, const float *next_nw = nullptr, bool qkv_prepared = false,
                        bool *next_prepared = nullptr) {
    if (next_prepared) *next_prepared = false;
    const x100q_model_cfg &g = m->cfg;
    ModelLayer &L = m->layers[layer];
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(attn_decode_kernel);
        set_qkernel_attrs(attn_merge_kernel<false>);
        set_qkernel_attrs(attn_merge_kernel<true>);
        attr[c->device] = true;
    }
    // 1. qkv = Wqkv . rmsnorm(h)
    timer_mark(m->timer, X100Q_T_QKV, s);
    GemvOpts o1;
    o1.norm_w = L.norms;
    o1.eps = g.eps;
    o1.pdl = !barrier;
    o1.prep = m->prep;
    o1.prepared = qkv_prepared;
    int st = launch_qgemv_ex(c, L.qkv, h, m->qkv, batch, o1, s);
    if (st) return st;
    // 2. attention (+ merge of the splits)
    AttnArgs a;
    a.qkv = m->qkv;
    a.qkv_n = qkv_rows(g);
    a.q_norm = L.norms + 2 * g.d;
    a.k_norm = L.norms + 2 * g.d + g.head_dim;
    a.pos = pos;
    a.nh = g.n_heads;
    a.nkv = g.n_kv_heads;
    a.ctx = g.ctx;
    a.chunk = kChunk;
    a.cps = attn_cps(batch, g.n_kv_heads, g.ctx, c->device, c->sm_count);
    a.nsplit = (g.ctx + kChunk * a.cps - 1) / (kChunk * a.cps);
    a.eps = g.eps;
    a.rope_base = g.rope_base;
    a.rope = m->rope;
    a.scale = 1.0f / sqrtf((float)g.head_dim);
    a.kc = m->kc + (size_t)layer * m->layer_kv;
    a.vc = m->vc + (size_t)layer * m->layer_kv;
    a.row_base = (long)layer * g.max_batch * g.n_kv_heads * g.ctx;
    a.part = m->part;
    a.kv_early = (kv_early && !slot) ? 1 : 0;
    a.slot = slot;
    a.nslots = g.max_batch;
    a.prewritten = slot ? 1 : 0;
    a.att = m->att;
    a.status = c->d_status;
    timer_mark(m->timer, X100Q_T_ATTN, s);
    if (slot) {
        st = launch_pdl(kv_write_kernel, dim3(g.n_kv_heads, batch), dim3(32), 0, s, a);
        if (st) return st;
    }
    st = launch_pdl(attn_decode_kernel, dim3(a.nsplit, g.n_kv_heads, batch), dim3(kAttnThreads), attn_smem(a.cps), s,
                    m->tmK, m->tmV, a);
    if (st) return st;
    GemvOpts o3;   // the Wo call: its activations prepared by the merge when it prepares them once
    o3.accum = true;
    o3.prep = m->prep;
    if (a.nsplit > 1) {
        const int grp = qgemv_prep_group(L.o, batch, o3);
        st = launch_pdl(grp ? attn_merge_kernel<true> : attn_merge_kernel<false>, dim3(g.n_heads, batch), dim3(128),
                        merge_smem(a.nsplit), s, (const float *)m->part, g.n_heads, a.nsplit, m->att,
                        grp ? m->prep : nullptr, grp, slices_per_row(g.n_heads * kHD) * 8);
        if (st) return st;
        o3.prepared = grp > 0;
    }
    // 3. h += Wo . att
    timer_mark(m->timer, X100Q_T_O, s);
    st = launch_qgemv_ex(c, L.o, m->att, h, batch, o3, s);
    if (st) return st;
    // 4. h += MoE(rmsnorm(h))  (or eout = this process's experts' share)
    MoeOpts o4;
    o4.norm_w = L.norms + g.d;
    o4.eps = g.eps;
    o4.hn_out = m->hn;
    o4.accum = eout == nullptr;
    o4.mark = timer_mark_cb;
    o4.mark_ctx = &m->timer;
    if (next_m && !eout) {   // h is complete after the combine: it prepares the next GEMV's activations
        GemvOpts on;
        on.norm_w = next_nw;
        on.eps = g.eps;
        on.prep = m->prep;
        const int grp = qgemv_prep_group(*next_m, batch, on);
        if (grp) {
            o4.next_xbm = m->prep;
            o4.next_qs = qgemv_prep_qs(m->prep, next_m->K);
            o4.next_nw = next_nw;
            o4.next_ntok = grp;
            o4.next_nxb = slices_per_row(next_m->K) * 8;
            if (next_prepared) *next_prepared = true;
        }
    }
    return launch_moe_ex(c, L.moe, m->S, h, eout ? eout : h, batch, o4, s);
}

static int forward_impl(x100q_model *m, const int *tokens, float *h, const int *pos, const int *slot, float *logits,
                        int batch, void *stream);
static int prefill_tc(x100q_model *m, int slot, const int *tokens, int n, int pos0, float *logits);

extern "C" {

int x100q_model_layer_dev(x100q_model *m, int layer, float *h, const int *pos, int batch, float *eout,
                          int *sel_out, float *w_out, void *stream) {
    set_error(X100_OK);
    if (!m || layer < 0 || layer >= m->cfg.n_layers || !h || !pos || batch < 1 || batch > m->cfg.max_batch ||
        !m->layers[layer].set) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    const bool full = m->cfg.expert_lo == 0 && m->cfg.expert_hi == m->cfg.n_exp;
    if (!eout && !full) {   // a partial expert range cannot add into h alone
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = layer_launch(m, c, layer, h, pos, batch, eout, s, false, false);
    if (m->timer.on) {
        timer_mark(m->timer, -1, s);
        ++m->timer.steps;
    }
    if (st) return st;
    if (sel_out || w_out) {
        const size_t nb = (size_t)batch * m->cfg.n_act * 4;
        if (sel_out && check_cuda(cudaMemcpyAsync(sel_out, m->S.sel, nb, cudaMemcpyDefault, s), X100_E_COPY))
            return X100_E_COPY;
        if (w_out && check_cuda(cudaMemcpyAsync(w_out, m->S.w, nb, cudaMemcpyDefault, s), X100_E_COPY))
            return X100_E_COPY;
    }
    return X100_OK;
}

// logits = lm_head . rmsnorm(h, out_norm); prepared: the last layer's combine
// prepared the activations
static int head_launch(x100q_model *m, DevCtx *c, const float *h, float *logits, int batch, cudaStream_t s,
                       bool prepared) {
    GemvOpts o;
    o.norm_w = m->out_norm;
    o.eps = m->cfg.eps;
    o.prep = m->prep;
    o.prepared = prepared;
    return launch_qgemv_ex(c, m->lm, h, logits, batch, o, s);
}

int x100q_model_head_dev(x100q_model *m, const float *h, float *logits, int batch, void *stream) {
    set_error(X100_OK);
    if (!m || !h || !logits || batch < 1 || batch > m->cfg.max_batch || !m->out_norm || !m->lm.w) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    return head_launch(m, c, h, logits, batch, static_cast<cudaStream_t>(stream), false);
}

int x100q_model_forward_dev(x100q_model *m, const int *tokens, float *h, const int *pos, float *logits, int batch,
                            void *stream) {
    return forward_impl(m, tokens, h, pos, nullptr, logits, batch, stream);
}

int x100q_model_forward_slots_dev(x100q_model *m, const int *tokens, float *h, const int *pos, const int *slot,
                                  float *logits, int batch, void *stream) {
    if (!slot) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    return forward_impl(m, tokens, h, pos, slot, logits, batch, stream);
}

}  // extern "C"

static int forward_impl(x100q_model *m, const int *tokens, float *h, const int *pos, const int *slot, float *logits,
                        int batch, void *stream) {
    set_error(X100_OK);
    if (!m || !h || !pos) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (batch < 1 || batch > m->cfg.max_batch || m->cfg.expert_lo != 0 || m->cfg.expert_hi != m->cfg.n_exp) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    for (int l = 0; l < m->cfg.n_layers; ++l)
        if (!m->layers[l].set) {
            set_error(X100_E_ARG);
            return X100_E_ARG;
        }
    DevCtx *c = ctx();
    if (!c) return get_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the step starts behind a full barrier (embed, or layer 0's first
    // kernel), so every attention kernel of the step may stage early
    int st = X100_OK;
    if (tokens) {
        timer_mark(m->timer, X100Q_T_EMBED, s);
        st = x100q_model_embed_dev(m, tokens, h, batch, stream);
    }
    // each layer's combine prepares the activations of the GEMV after it (the
    // next layer's q/k/v, the lm_head) when that call prepares them once
    const bool head_ok = logits && m->out_norm && m->lm.w;
    bool prepared = false;
    for (int l = 0; st == X100_OK && l < m->cfg.n_layers; ++l) {
        const bool last = l + 1 == m->cfg.n_layers;
        const QMat *nm = !last ? &m->layers[l + 1].qkv : (head_ok ? &m->lm : nullptr);
        const float *nnw = !last ? m->layers[l + 1].norms : m->out_norm;
        bool np = false;
        st = layer_launch(m, c, l, h, pos, batch, nullptr, s, true, l == 0 && !tokens, slot, nm, nnw, prepared, &np);
        prepared = np;
    }
    if (st == X100_OK && logits) {
        timer_mark(m->timer, X100Q_T_LM, s);
        st = head_ok ? head_launch(m, c, h, logits, batch, s, prepared) : x100q_model_head_dev(m, h, logits, batch, stream);
    }
    if (m->timer.on) {
        timer_mark(m->timer, -1, s);
        ++m->timer.steps;
    }
    if (st) set_error(st);
    return st;
}

// ---- many-token prefill on the tensor-core GEMMs -------------------------------------------
// Tokens per chunk of the tensor-core path: a chunk streams every weight once,
// so longer chunks reuse each weight over more tokens (the experts see
// ~chunk * top-k / n_exp tokens each) at the cost of scratch memory (about
// 0.28 MB per token of chunk at the config-5 shape).  X100_PREFILL_CHUNK
// overrides the default (32 .. 4096), read when a model first prefills.
constexpr int kPrefillChunk = 1024;

static bool prefill_alloc(x100q_model *m) {
    if (m->pf_base) return true;
    const x100q_model_cfg &g = m->cfg;
    int T = kPrefillChunk;
    if (const char *e = getenv("X100_PREFILL_CHUNK")) {
        const int v = atoi(e);
        if (v >= 32 && v <= 4096) T = v;
    }
    const int kpd = slices_per_row(g.d) * 256, kpq = slices_per_row(g.n_heads * g.head_dim) * 256;
    m->pf_kp = kpd > kpq ? kpd : kpq;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    const size_t qb = up((size_t)T * qkv_rows(g) * 4), ab = up((size_t)T * g.n_heads * g.head_dim * 4),
                 xb = up((size_t)T * m->pf_kp * 2),
                 mb = moe_big_scratch_bytes(g.d, g.n_exp, g.n_act, g.moe_ffn, T);
    if (cudaMalloc(&m->pf_base, qb + ab + 2 * xb + mb + 256) != cudaSuccess) {
        cudaGetLastError();
        m->pf_base = nullptr;
        set_error(X100_E_ALLOC);
        return false;
    }
    uint8_t *p = static_cast<uint8_t *>(m->pf_base);
    m->pf_qkv = reinterpret_cast<float *>(p);
    m->pf_att = reinterpret_cast<float *>(p + qb);
    m->pf_xh = reinterpret_cast<__half *>(p + qb + ab);
    m->pf_xl = reinterpret_cast<__half *>(p + qb + ab + xb);
    m->pf_moe = moe_big_scratch_carve(p + qb + ab + 2 * xb, g.d, g.n_exp, g.n_act, g.moe_ffn, T);
    m->pf_tmax = T;
    return true;
}

// One dense linear of a chunk: y (=, or += with add) W . x for T token rows
// of x [T][K] (fp32, row pitch K), through the fp16 planes of x.
static int prefill_linear(x100q_model *m, DevCtx *c, const QMat &W, const float *x, int K, int T,
                          const float *norm_w, float *y, long ldy, bool add, cudaStream_t s) {
    const int kp = W.ns * 256;
    int st = launch_split_rows(x, K, K, kp, T, norm_w, m->cfg.eps, m->pf_xh, m->pf_xl, nullptr, s);
    if (st) return st;
    QgLaunch L;
    L.mats[0] = &W;
    L.n_rows = W.N;
    L.T = T;
    L.xh = m->pf_xh;
    L.xl = m->pf_xl;
    L.x_rows = T;
    L.mode = add ? QG_ADD : QG_STORE;
    L.out = y;
    L.ldo = ldy;
    return launch_qgemm(c, L, s);
}

// forward() over T consecutive tokens of one sequence (the reference's
// prefill, qwen_moe_hp.c:1748-1858): per layer the q/k/v, Wo and expert
// linears run as tensor-core GEMMs over all T tokens (each weight row
// streamed once per 128 tokens), every token's k and v go to the cache
// before any token attends, and the attention runs per token over its
// positions 0 .. pos (causal) in groups of max_batch tokens.
// position of token i of a chunk whose first token sits at pos0 (the
// positions of a prefill chunk are consecutive)
static inline int hpos_last(int pos0, int i) { return pos0 + i; }

static int prefill_chunk_tc(x100q_model *m, DevCtx *c, const int *tok, float *h, const int *pos, const int *slot,
                            int hpos0, float *logits, int T, cudaStream_t s) {
    const x100q_model_cfg &g = m->cfg;
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(embed_kernel);
        set_qkernel_attrs(attn_decode_kernel);
        set_qkernel_attrs(attn_merge_kernel<false>);
        set_qkernel_attrs(attn_merge_kernel<true>);
        attr[c->device] = true;
    }
    const int qd = g.n_heads * g.head_dim, qn = qkv_rows(g);
    int st = launch_k(embed_kernel, dim3(2, T), dim3(256), 0, s, false, (const float *)m->tok_embd, g.vocab, g.d,
                      tok, h, c->d_status);
    for (int l = 0; st == X100_OK && l < g.n_layers; ++l) {
        ModelLayer &L = m->layers[l];
        // 1. qkv = Wqkv . rmsnorm(h, attn_norm)
        st = prefill_linear(m, c, L.qkv, h, g.d, T, L.norms, m->pf_qkv, qn, false, s);
        if (st) break;
        // 2. every token's k, v into the cache, then attention per token
        AttnArgs a;
        a.qkv = m->pf_qkv;
        a.qkv_n = qn;
        a.q_norm = L.norms + 2 * g.d;
        a.k_norm = L.norms + 2 * g.d + g.head_dim;
        a.pos = pos;
        a.nh = g.n_heads;
        a.nkv = g.n_kv_heads;
        a.ctx = g.ctx;
        a.chunk = kChunk;
        a.cps = 1;
        a.nsplit = (g.ctx + kChunk - 1) / kChunk;
        a.eps = g.eps;
        a.rope_base = g.rope_base;
        a.rope = m->rope;
        a.scale = 1.0f / sqrtf((float)g.head_dim);
        a.kc = m->kc + (size_t)l * m->layer_kv;
        a.vc = m->vc + (size_t)l * m->layer_kv;
        a.row_base = (long)l * g.max_batch * g.n_kv_heads * g.ctx;
        a.part = m->part;
        a.kv_early = 0;
        a.slot = slot;
        a.nslots = g.max_batch;
        a.prewritten = 1;
        a.att = m->pf_att;
        a.status = c->d_status;
        st = launch_pdl(kv_write_kernel, dim3(g.n_kv_heads, T), dim3(32), 0, s, a);
        // groups of tokens whose (token, split) partials fit the decode step's
        // buffer (max_batch x nsplit_max of them); the group's splits cover
        // its largest position only (the chunk's positions are consecutive:
        // hpos[g0 + gb - 1] is the group's largest), so early chunks need few
        const int cap = g.max_batch * m->nsplit_max;
        for (int g0 = 0; st == X100_OK && g0 < T;) {
            int gb = T - g0;
            int nsp = (hpos_last(hpos0, g0 + gb - 1) + kChunk) / kChunk;
            while (gb > 1 && gb * nsp > cap) {
                gb = cap / nsp < gb ? cap / nsp : gb - 1;
                if (gb < 1) gb = 1;
                nsp = (hpos_last(hpos0, g0 + gb - 1) + kChunk) / kChunk;
            }
            AttnArgs ag = a;
            ag.qkv = m->pf_qkv + (size_t)g0 * qn;
            ag.pos = pos + g0;
            ag.slot = slot + g0;
            ag.att = m->pf_att + (size_t)g0 * qd;
            ag.nsplit = nsp;
            st = launch_pdl(attn_decode_kernel, dim3(ag.nsplit, g.n_kv_heads, gb), dim3(kAttnThreads), attn_smem(), s,
                            m->tmK, m->tmV, ag);
            if (!st && ag.nsplit > 1)
                st = launch_pdl(attn_merge_kernel<false>, dim3(g.n_heads, gb), dim3(128), merge_smem(ag.nsplit), s,
                                (const float *)m->part, g.n_heads, ag.nsplit, ag.att, (uint8_t *)nullptr, 0, 0);
            g0 += gb;
        }
        if (st) break;
        // 3. h += Wo . att
        st = prefill_linear(m, c, L.o, m->pf_att, qd, T, nullptr, h, g.d, true, s);
        if (st) break;
        // 4. h += MoE(rmsnorm(h, ffn_norm))
        st = launch_moe_prefill(c, L.moe, m->pf_moe, h, T, L.norms + g.d, g.eps, s);
    }
    // logits = Wlm . rmsnorm(h, out_norm)
    if (st == X100_OK && logits) st = prefill_linear(m, c, m->lm, h, g.d, T, m->out_norm, logits, g.vocab, false, s);
    return st;
}

extern "C" {

int x100q_model_timing(x100q_model *m, int on) {
    set_error(X100_OK);
    if (!m) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    StepTimer &t = m->timer;
    if (on) {
        timer_flush(t);
        for (double &v : t.ms) v = 0.0;
        t.steps = 0;
    }
    t.on = on != 0;
    return X100_OK;
}

int x100q_model_timing_read(x100q_model *m, double *ms, long *steps) {
    set_error(X100_OK);
    if (!m) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    StepTimer &t = m->timer;
    timer_flush(t);   // every call ends with its closing mark, so nothing is left open
    if (ms)
        for (int i = 0; i < X100Q_NBUCKETS; ++i) ms[i] = t.ms[i];
    if (steps) *steps = t.steps;
    return X100_OK;
}

const char *x100q_timing_bucket_name(int bucket) {
    static const char *names[X100Q_NBUCKETS] = {"embed", "qkv", "attention", "o", "router", "expert", "combine", "lm"};
    return bucket >= 0 && bucket < X100Q_NBUCKETS ? names[bucket] : nullptr;
}

int x100q_model_forward(x100q_model *m, const int *tokens, const int *pos, float *logits, int batch) {
    set_error(X100_OK);
    if (!m || !tokens || !pos || !logits || batch < 1 || batch > m->cfg.max_batch || !m->tok_embd) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DeviceGuard dg(m->device);
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const x100q_model_cfg &g = m->cfg;
    // staging: tokens, pos, h, logits
    const size_t tb = 256, hb = (size_t)batch * g.d * 4, lb = (size_t)batch * g.vocab * 4;
    uint8_t *buf = static_cast<uint8_t *>(stage_buf(c, 0, 2 * tb + hb));
    if (!buf) return get_error();
    int *dtok = reinterpret_cast<int *>(buf), *dpos = reinterpret_cast<int *>(buf + tb);
    float *dh = reinterpret_cast<float *>(buf + 2 * tb);
    float *dl = static_cast<float *>(stage_buf(c, 1, lb));
    if (!dl) return get_error();
    int st = check_cuda(cudaMemcpyAsync(dtok, tokens, batch * 4, cudaMemcpyDefault, c->stream), X100_E_COPY);
    if (!st) st = check_cuda(cudaMemcpyAsync(dpos, pos, batch * 4, cudaMemcpyDefault, c->stream), X100_E_COPY);
    if (!st) st = x100q_model_forward_dev(m, dtok, dh, dpos, dl, batch, c->stream);
    if (!st) st = check_cuda(cudaMemcpyAsync(logits, dl, lb, cudaMemcpyDefault, c->stream), X100_E_COPY);
    const int st2 = sync_and_status(c, c->stream);
    if (st == X100_OK) st = st2;
    if (st) set_error(st);
    return st;
}

int x100q_model_prefill(x100q_model *m, int slot, const int *tokens, int n, int pos0, float *logits) {
    set_error(X100_OK);
    if (!m || !tokens || n < 1 || slot < 0 || slot >= m->cfg.max_batch || pos0 < 0 || pos0 + n > m->cfg.ctx ||
        !m->tok_embd || (logits && (!m->out_norm || !m->lm.w))) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (n > m->cfg.max_batch) return prefill_tc(m, slot, tokens, n, pos0, logits);
    DeviceGuard dg(m->device);
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const x100q_model_cfg &g = m->cfg;
    // staging: tokens, positions, slots, h, logits
    const size_t tb = 256, hb = (size_t)n * g.d * 4, lb = (size_t)n * g.vocab * 4;
    uint8_t *buf = static_cast<uint8_t *>(stage_buf(c, 0, 3 * tb + hb));
    if (!buf) return get_error();
    int *dtok = reinterpret_cast<int *>(buf), *dpos = reinterpret_cast<int *>(buf + tb),
        *dslot = reinterpret_cast<int *>(buf + 2 * tb);
    float *dh = reinterpret_cast<float *>(buf + 3 * tb);
    float *dl = nullptr;
    if (logits && !(dl = static_cast<float *>(stage_buf(c, 1, lb)))) return get_error();
    std::vector<int> hp(n), hs(n, slot);
    for (int i = 0; i < n; ++i) hp[i] = pos0 + i;
    int st = check_cuda(cudaMemcpyAsync(dtok, tokens, n * 4, cudaMemcpyDefault, c->stream), X100_E_COPY);
    if (!st) st = check_cuda(cudaMemcpyAsync(dpos, hp.data(), n * 4, cudaMemcpyHostToDevice, c->stream), X100_E_COPY);
    if (!st) st = check_cuda(cudaMemcpyAsync(dslot, hs.data(), n * 4, cudaMemcpyHostToDevice, c->stream), X100_E_COPY);
    if (!st) st = forward_impl(m, dtok, dh, dpos, dslot, dl, n, c->stream);
    if (!st && logits)
        st = check_cuda(cudaMemcpyAsync(logits, dl, lb, cudaMemcpyDefault, c->stream), X100_E_COPY);
    const int st2 = sync_and_status(c, c->stream);   // the host vectors outlive the copies
    if (st == X100_OK) st = st2;
    if (st) set_error(st);
    return st;
}

}  // extern "C"

// x100q_model_prefill for n > max_batch: chunks of up to pf_tmax tokens,
// each through prefill_chunk_tc, in order (a chunk attends over the cache the
// earlier chunks wrote).  Synchronous; host or device tokens / logits.
static int prefill_tc(x100q_model *m, int slot, const int *tokens, int n, int pos0, float *logits) {
    for (int l = 0; l < m->cfg.n_layers; ++l)
        if (!m->layers[l].set || m->cfg.expert_lo != 0 || m->cfg.expert_hi != m->cfg.n_exp) {
            set_error(X100_E_ARG);
            return X100_E_ARG;
        }
    DeviceGuard dg(m->device);
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    if (!prefill_alloc(m)) return get_error();
    const x100q_model_cfg &g = m->cfg;
    const int T = m->pf_tmax;
    const size_t tb = 4 * (size_t)T, hb = (size_t)T * g.d * 4, lb = (size_t)T * g.vocab * 4;
    uint8_t *buf = static_cast<uint8_t *>(stage_buf(c, 0, 3 * tb + hb + 1024));
    if (!buf) return get_error();
    int *dtok = reinterpret_cast<int *>(buf), *dpos = reinterpret_cast<int *>(buf + tb),
        *dslot = reinterpret_cast<int *>(buf + 2 * tb);
    float *dh = reinterpret_cast<float *>(buf + ((3 * tb + 255) & ~size_t(255)));
    float *dl = nullptr;
    if (logits && !(dl = static_cast<float *>(stage_buf(c, 1, lb)))) return get_error();
    std::vector<int> hp(T), hs(T, slot);
    int st = X100_OK;
    for (int c0 = 0; st == X100_OK && c0 < n; c0 += T) {
        const int cn = n - c0 < T ? n - c0 : T;
        for (int i = 0; i < cn; ++i) hp[i] = pos0 + c0 + i;
        st = check_cuda(cudaMemcpyAsync(dtok, tokens + c0, cn * 4, cudaMemcpyDefault, c->stream), X100_E_COPY);
        if (!st) st = check_cuda(cudaMemcpyAsync(dpos, hp.data(), cn * 4, cudaMemcpyHostToDevice, c->stream), X100_E_COPY);
        if (!st) st = check_cuda(cudaMemcpyAsync(dslot, hs.data(), cn * 4, cudaMemcpyHostToDevice, c->stream), X100_E_COPY);
        if (!st) st = prefill_chunk_tc(m, c, dtok, dh, dpos, dslot, pos0 + c0, dl, cn, c->stream);
        if (!st && logits)
            st = check_cuda(cudaMemcpyAsync(logits + (size_t)c0 * g.vocab, dl, (size_t)cn * g.vocab * 4, cudaMemcpyDefault,
                                            c->stream), X100_E_COPY);
        const int st2 = sync_and_status(c, c->stream);   // the host vectors are reused by the next chunk
        if (st == X100_OK) st = st2;
    }
    if (st) set_error(st);
    return st;
}
