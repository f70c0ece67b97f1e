// moe.cu -- the top-k SwiGLU mixture-of-experts FFN of the decode step and the
// x100q_moe_* entry points of include/x100q.h.
//
// Replaces the MoE block of the reference's forward() (qwen_moe.c:295-311;
// qwen_moe_q3k.c:1916-1978 with router mode 0 = fp32 and SwiGLU mode 0 =
// exact): router GEMV -> softmax -> greedy top-k -> renormalise -> for each
// selected expert gate/up GEMV, silu(g)*u, down GEMV, weighted sum.
//
// Three kernels per call (captured into one CUDA graph by callers that loop):
//   router_topk   one warp per expert row: fp32 logits for every token; the
//                 last CTA to finish (atomic ticket, no waiting) does the
//                 softmax, the greedy top-k (strict >, lowest index wins)
//                 and the renormalisation, writing sel / w.
//   gate_up       grid (ffn rows, token x slot): each warp streams gate row i
//                 and up row i of the selected expert once and writes
//                 h[token][slot][i] = silu(g) * u (SwiGLU fused).
//   down_combine  grid (d rows, token): each warp streams row n of the down
//                 matrix of every selected expert and writes
//                 eout[token][n] = sum_a w_a * (down_a[n] . h_a), summed in
//                 slot order a = 0..k-1 like the reference (no atomics).
// Experts outside [expert_lo, expert_hi) contribute nothing (expert
// parallelism: the caller sums eout over processes, e.g. NCCL all-reduce).
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>

#include "../../include/x100q.h"
#include "moe.h"
#include "qgemv.h"

namespace x100 {
namespace q {

constexpr int kMaxBatch = 16;
constexpr int kMaxAct = 16;
constexpr int kMaxExp = 256;

// ---- router + softmax + top-k ------------------------------------------------------
__global__ void __launch_bounds__(256) router_topk_kernel(const float *__restrict__ router,
                                                          const float *__restrict__ hn, int d, int n_exp, int n_act,
                                                          int batch, float *__restrict__ logits, int *__restrict__ sel,
                                                          float *__restrict__ wsel, unsigned *__restrict__ ticket) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int e = blockIdx.x * nwarps + warp;
    // the router row (independent of the previous kernel) is loaded before
    // waiting on it: up to 16 float4 per lane held in registers (d <= 2048),
    // the rest of a longer row is streamed afterwards
    constexpr int RV = 16;
    const int nv = d / 128;
    const float4 *rw = reinterpret_cast<const float4 *>(router + (long)(e < n_exp ? e : 0) * d);
    float4 r[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i)
        if (e < n_exp && i < nv) r[i] = __ldg(rw + lane + 32 * i);
    pdl_launch_dependents();
    pdl_wait();
    if (e < n_exp) {
        for (int b = 0; b < batch; ++b) {
            const float4 *x = reinterpret_cast<const float4 *>(hn + (long)b * d);
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < RV; ++i) {
                if (i < nv) {
                    const float4 v = __ldg(x + lane + 32 * i);
                    s = fmaf(r[i].x, v.x, s);
                    s = fmaf(r[i].y, v.y, s);
                    s = fmaf(r[i].z, v.z, s);
                    s = fmaf(r[i].w, v.w, s);
                }
            }
            for (int i = lane + 32 * RV; i < d / 4; i += 32) {
                const float4 rr = __ldg(rw + i), v = __ldg(x + i);
                s = fmaf(rr.x, v.x, s);
                s = fmaf(rr.y, v.y, s);
                s = fmaf(rr.z, v.z, s);
                s = fmaf(rr.w, v.w, s);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (lane == 0) logits[b * n_exp + e] = s;
        }
    }
    // last CTA to arrive finishes the routing (threadFenceReduction pattern)
    __shared__ unsigned s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int b = warp; b < batch; b += nwarps) {
        const volatile float *lg = logits + b * n_exp;
        float p[kMaxExp / 32];
        float m = -1e30f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            p[i] = ee < n_exp ? lg[ee] : -1e30f;
            m = fmaxf(m, p[i]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            p[i] = ee < n_exp ? expf(p[i] - m) : 0.f;
            s += p[i];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        const float inv = 1.0f / s;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) p[i] *= inv;
        unsigned used = 0;   // bit i: this lane's entry i is taken
        float sw[kMaxAct];
        int si[kMaxAct];
        for (int a = 0; a < n_act; ++a) {
            float bv = -1e30f;
            int bi = 0x7fffffff;
#pragma unroll
            for (int i = 0; i < kMaxExp / 32; ++i) {
                const int ee = lane + 32 * i;
                if (ee < n_exp && !(used & (1u << i)) && p[i] > bv) {
                    bv = p[i];
                    bi = ee;
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if ((bi & 31) == lane) used |= 1u << (bi >> 5);
            sw[a] = bv;
            si[a] = bi;
        }
        if (lane == 0) {
            float ssum = 0.f;
            for (int a = 0; a < n_act; ++a) ssum += sw[a];
            for (int a = 0; a < n_act; ++a) {
                sel[b * n_act + a] = si[a];
                wsel[b * n_act + a] = sw[a] / ssum;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) *ticket = 0;   // ready for the next call
}

// ---- router logits only + per-CTA routing --------------------------------------------
// router_logits: one warp per expert row (loaded before waiting on the
// previous kernel); writes logits[b][e].  The consumers (gate/up and down
// kernels) each finish the routing themselves with route_cta, so no kernel
// waits on a last-arriving CTA.
__global__ void __launch_bounds__(64) router_logits_kernel(const float *__restrict__ router,
                                                           const float *__restrict__ hn, int d, int n_exp,
                                                           int batch, float *__restrict__ logits) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int e = blockIdx.x * nwarps + warp;
    constexpr int RV = 16;
    const int nv = d / 128;
    const float4 *rw = reinterpret_cast<const float4 *>(router + (long)(e < n_exp ? e : 0) * d);
    float4 r[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i)
        if (e < n_exp && i < nv) r[i] = __ldg(rw + lane + 32 * i);
    pdl_launch_dependents();
    pdl_wait();
    if (e >= n_exp) return;
    for (int b = 0; b < batch; ++b) {
        const float4 *x = reinterpret_cast<const float4 *>(hn + (long)b * d);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < RV; ++i) {
            if (i < nv) {
                const float4 v = __ldg(x + lane + 32 * i);
                s = fmaf(r[i].x, v.x, s);
                s = fmaf(r[i].y, v.y, s);
                s = fmaf(r[i].z, v.z, s);
                s = fmaf(r[i].w, v.w, s);
            }
        }
        for (int i = lane + 32 * RV; i < d / 4; i += 32) {
            const float4 rr = __ldg(rw + i), v = __ldg(x + i);
            s = fmaf(rr.x, v.x, s);
            s = fmaf(rr.y, v.y, s);
            s = fmaf(rr.z, v.z, s);
            s = fmaf(rr.w, v.w, s);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) logits[b * n_exp + e] = s;
    }
}

// Softmax over one token's logits, greedy top-k (strict >, lowest index wins)
// and renormalisation, by a whole CTA: warp 0 forms the probabilities exactly
// as router_topk_kernel does; every thread then ranks its experts (rank =
// number of experts with a larger probability, or an equal one at a lower
// index), which reproduces the greedy selection order.  Results in shared
// memory: s_sel[a], s_w[a] for a < n_act.  All threads must call it.
__device__ __forceinline__ void route_cta(const float *lg, int n_exp, int n_act, float *s_p, int *s_sel, float *s_w) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp == 0) {
        float p[kMaxExp / 32];
        float m = -1e30f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            p[i] = ee < n_exp ? __ldcg(lg + ee) : -1e30f;   // L2: written by an earlier grid
            m = fmaxf(m, p[i]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            p[i] = ee < n_exp ? expf(p[i] - m) : 0.f;
            s += p[i];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        const float inv = 1.0f / s;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            if (ee < n_exp) s_p[ee] = p[i] * inv;
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_exp; e += blockDim.x) {
        const float pe = s_p[e];
        int rank = 0;
        for (int f = 0; f < n_exp; ++f) {
            const float pf = s_p[f];
            rank += (pf > pe) || (pf == pe && f < e);
        }
        if (rank < n_act) {
            s_sel[rank] = e;
            s_w[rank] = pe;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float ssum = 0.f;
        for (int a = 0; a < n_act; ++a) ssum += s_w[a];
        for (int a = 0; a < n_act; ++a) s_w[a] = s_w[a] / ssum;
    }
    __syncthreads();
}

// ---- gate / up + SwiGLU ------------------------------------------------------------------
template <int QT>
__global__ void __launch_bounds__(256) gate_up_kernel(QView G, QView U, int ffn, int d, int n_act, int lo, int hi,
                                                      const float *__restrict__ hn, const int *__restrict__ sel,
                                                      float *__restrict__ h) {
    __shared__ XBlk xq[kMaxDXB];
    __shared__ XF xf[kMaxDXB];
    const int pair = blockIdx.y;                 // token * n_act + slot
    const int tok = pair / n_act;
    const int e = sel[pair];
    if (e < lo || e >= hi) return;               // expert held by another process
    xprep_all(hn + (long)tok * d, d, 1, xq, xf);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * (blockDim.x >> 5) + warp;
    if (i >= ffn) return;
    const int row = (e - lo) * ffn + i;
    const int units = units_per_row(QT, d);
    float g = 0.f, u = 0.f;
    for (int k = lane; k < units; k += 32) {
        const WUnit<QT> wg = load_unit<QT>(G, row, k);
        const WUnit<QT> wu = load_unit<QT>(U, row, k);
        g += dot_unit<QT>(wg, xq, xf, k);
        u += dot_unit<QT>(wu, xq, xf, k);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        g += __shfl_xor_sync(0xffffffffu, g, off);
        u += __shfl_xor_sync(0xffffffffu, u, off);
    }
    if (lane == 0) h[(long)pair * ffn + i] = (g / (1.0f + expf(-g))) * u;   // silu(g) * u, qwen_moe.c:309
}

// ---- down projection + weighted combine -------------------------------------------------------
template <int QT>
__global__ void __launch_bounds__(256) down_combine_kernel(QView D, int ffn, int d, int n_act, int lo, int hi,
                                                           const float *__restrict__ h, const int *__restrict__ sel,
                                                           const float *__restrict__ wsel, float *__restrict__ eout,
                                                           int lpr) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nxb = ffn / 32;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * n_act * nxb);
    const int tok = blockIdx.y;
    // activation planes of every slot's h (slots of remote experts are unused)
    xprep_all(h + (long)tok * n_act * ffn, ffn, n_act, xq, xf);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n = blockIdx.x * (blockDim.x >> 5) + warp;
    if (n >= d) return;
    const int groups = 32 / lpr, grp = lane / lpr, sig = lane % lpr;
    const int units = units_per_row(QT, ffn);
    float total = 0.f;
    for (int a0 = 0; a0 < n_act; a0 += groups) {
        const int a = a0 + grp;
        float acc = 0.f;
        int e = -1;
        if (a < n_act) {
            e = sel[tok * n_act + a];
            if (e >= lo && e < hi) {
                const int row = (e - lo) * d + n;
                for (int k = sig; k < units; k += lpr) {
                    const WUnit<QT> wd = load_unit<QT>(D, row, k);
                    acc += dot_unit<QT>(wd, xq + a * nxb, xf + a * nxb, k);
                }
            }
        }
        for (int off = lpr >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        // lane 0 folds the groups' results in slot order
        for (int gi = 0; gi < groups; ++gi) {
            const float v = __shfl_sync(0xffffffffu, acc, gi * lpr);
            const int ag = a0 + gi;
            if (lane == 0 && ag < n_act) {
                const int eg = sel[tok * n_act + ag];
                if (eg >= lo && eg < hi) total += wsel[tok * n_act + ag] * v;
            }
        }
    }
    if (lane == 0) eout[(long)tok * d + n] = total;
}

// ---- slice versions (d a multiple of 256 up to 2048, ffn a multiple of 256 up to 4096) ----------
// gate/up: CTA = 32 consecutive rows of one selected expert for one
// (token, slot); warp w owns slice w of both the gate and the up row of its
// lane; partial sums are added in slice order, then h = silu(g) * u.
template <int QT>
__global__ void __launch_bounds__(256) gate_up_slice_kernel(QView G, QView U, int ffn, int d, int n_act, int lo,
                                                            int hi, const float *__restrict__ hn,
                                                            const int *__restrict__ sel, float *__restrict__ h) {
    __shared__ XBlk xq[kMaxDXB];
    __shared__ XF xf[kMaxDXB];
    __shared__ float red[2][8][32];
    const int pair = blockIdx.y;
    const int tok = pair / n_act;
    pdl_wait();                                  // sel comes from the router kernel
    pdl_launch_dependents();
    const int e = sel[pair];
    if (e < lo || e >= hi) return;
    const int lane = threadIdx.x & 31, sl = threadIdx.x >> 5, ns = d / 256;
    const int i = blockIdx.x * 32 + lane;
    const int row = (e - lo) * ffn + i;
    WSlice<QT> wg, wu;
    if (i < ffn) {
        load_slice<QT>(G, row, sl, wg);
        load_slice<QT>(U, row, sl, wu);
    }
    xprep_all(hn + (long)tok * d, d, 1, xq, xf);
    __syncthreads();
    float g = 0.f, u = 0.f;
    if (i < ffn) {
        g = dot_slice<QT>(wg, xq + sl * 8, xf + sl * 8);
        u = dot_slice<QT>(wu, xq + sl * 8, xf + sl * 8);
    }
    red[0][sl][lane] = g;
    red[1][sl][lane] = u;
    __syncthreads();
    if (threadIdx.x < 32 && i < ffn) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < ns; ++k) {
            gs += red[0][k][lane];
            us += red[1][k][lane];
        }
        h[(long)pair * ffn + i] = (gs / (1.0f + expf(-gs))) * us;   // silu(g) * u, qwen_moe.c:309
    }
}

// down + combine: CTA = 32 consecutive output rows n of one token; warp w
// owns (slot w / ns, slice w % ns), looping over slots when there are more
// than fit in 32 warps; the weighted sum over slots runs in slot order.
template <int QT>
__global__ void __launch_bounds__(1024) down_slice_kernel(QView D, int ffn, int d, int n_act, int lo, int hi,
                                                          const float *__restrict__ h, const int *__restrict__ sel,
                                                          const float *__restrict__ wsel, float *__restrict__ eout) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nxb = ffn / 32, ns = ffn / 256;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * n_act * nxb);
    float *red = reinterpret_cast<float *>(xf + n_act * nxb);      // [slot][slice][lane]
    const int tok = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int n = blockIdx.x * 32 + lane;
    const int slots_per_pass = nwarps / ns;
    // The routing was finished by the kernel before the previous one (the
    // gate/up kernel lets this grid launch only after it has waited for the
    // router), so the first pass's weights are loaded before waiting for h.
    const int sl = warp % ns;
    const bool active = warp < slots_per_pass * ns;
    WSlice<QT> w0;
    bool have0 = false;
    {
        const int a = warp / ns;
        if (active && a < n_act) {
            const int e = sel[tok * n_act + a];
            if (e >= lo && e < hi && n < d) {
                load_slice<QT>(D, (e - lo) * d + n, sl, w0);
                have0 = true;
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();                                  // h comes from the gate/up kernel
    xprep_all(h + (long)tok * n_act * ffn, ffn, n_act, xq, xf);
    __syncthreads();
    for (int a0 = 0; a0 < n_act; a0 += slots_per_pass) {
        const int a = a0 + warp / ns;
        if (active && a < n_act) {
            float v = 0.f;
            if (a0 == 0) {
                if (have0) v = dot_slice<QT>(w0, xq + a * nxb + sl * 8, xf + a * nxb + sl * 8);
            } else {
                const int e = sel[tok * n_act + a];
                if (e >= lo && e < hi && n < d) {
                    WSlice<QT> w;
                    load_slice<QT>(D, (e - lo) * d + n, sl, w);
                    v = dot_slice<QT>(w, xq + a * nxb + sl * 8, xf + a * nxb + sl * 8);
                }
            }
            red[(a * ns + sl) * 32 + lane] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x < 32 && n < d) {
        float total = 0.f;
        for (int a = 0; a < n_act; ++a) {
            const int e = sel[tok * n_act + a];
            if (e < lo || e >= hi) continue;
            float v = 0.f;
            for (int k = 0; k < ns; ++k) v += red[(a * ns + k) * 32 + lane];
            total += wsel[tok * n_act + a] * v;
        }
        eout[(long)tok * d + n] = total;
    }
}

// ---- bulk-copy versions --------------------------------------------------------------------
// gate/up: CTA = 32 consecutive rows (lane = row) of the gate and the up
// matrix of one selected expert for one (token, slot); warp 0 stages both
// 32-row tiles in shared memory with per-row bulk copies while the CTA
// prepares the activation planes; warp w dots slices w, w+nw, ...
template <int QT>
__global__ void __launch_bounds__(256, 2) gate_up_bulk_kernel(QView G, QView U, int ffn, int d, int n_exp, int n_act,
                                                           int lo, int hi, const float *__restrict__ hn,
                                                           const float *__restrict__ logits, int *__restrict__ sel_out,
                                                           float *__restrict__ w_out, float *__restrict__ h,
                                                           int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ float red[2][8][32];
    __shared__ float s_p[kMaxExp];
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct];
    const int pair = blockIdx.y;
    const int tok = pair / n_act, slot = pair % n_act;
    pdl_wait();                                  // logits come from the router kernel
    pdl_launch_dependents();
    route_cta(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_sel, s_w);
    if (blockIdx.x == 0 && slot == 0 && threadIdx.x < n_act) {   // routing result for the API
        sel_out[tok * n_act + threadIdx.x] = s_sel[threadIdx.x];
        w_out[tok * n_act + threadIdx.x] = s_w[threadIdx.x];
    }
    const int e = s_sel[slot];
    if (e < lo || e >= hi) return;               // expert held by another process
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, ns = d / 256;
    const int i0 = blockIdx.x * 32;
    const int rows = min(32, ffn - i0);
    const int tb = tile_bytes(QT, d, 32);
    uint8_t *tg = smem, *tu = smem + tb;
    XBlk *xq = reinterpret_cast<XBlk *>(smem + 2 * tb);
    XF *xf = reinterpret_cast<XF *>(xq + d / 32);
    tile_cp_async(G, (long)(e - lo) * ffn + i0, rows, tg, 32);
    tile_cp_async(U, (long)(e - lo) * ffn + i0, rows, tu, 32);
    cp_async_commit();
    xprep_all(hn + (long)tok * d, d, 1, xq, xf);
    cp_async_wait_all();
    __syncthreads();
    const bool ok = true;
    float g = 0.f, u = 0.f;
    if (ok && lane < rows) {
        const QView TG = tile_view(QT, d, tg, 32), TU = tile_view(QT, d, tu, 32);
        for (int sl = warp; sl < ns; sl += nw) {
            WSlice<QT> w;
            load_slice<QT, false>(TG, lane, sl, w);
            g += dot_slice<QT>(w, xq + sl * 8, xf + sl * 8);
            load_slice<QT, false>(TU, lane, sl, w);
            u += dot_slice<QT>(w, xq + sl * 8, xf + sl * 8);
        }
    }
    red[0][warp][lane] = g;
    red[1][warp][lane] = u;
    __syncthreads();
    if (threadIdx.x < 32 && lane < rows) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < nw; ++k) {
            gs += red[0][k][lane];
            us += red[1][k][lane];
        }
        h[(long)pair * ffn + i0 + lane] = (gs / (1.0f + expf(-gs))) * us;   // silu(g) * u, qwen_moe.c:309
    }
}

// down + combine: CTA = 32 consecutive output rows n of one token; warp 0
// stages the 32 rows of the down matrix of every locally held selected expert
// (per-row bulk copies, issued before waiting for h); warp w handles
// (slot w / ns, slice w % ns) pairs; the weighted sum runs in slot order.
template <int QT>
__global__ void __launch_bounds__(1024) down_bulk_kernel(QView D, int ffn, int d, int n_exp, int n_act, int lo,
                                                         int hi, const float *__restrict__ h,
                                                         const float *__restrict__ logits, float *__restrict__ eout,
                                                         int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct];
    __shared__ float s_p[kMaxExp];
    const int nxb = ffn / 32, ns = ffn / 256;
    const int tok = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int n0 = blockIdx.x * 32;
    const int rows = min(32, d - n0);
    const int tb = tile_bytes(QT, ffn, 32);
    XBlk *xq = reinterpret_cast<XBlk *>(smem + n_act * tb);
    XF *xf = reinterpret_cast<XF *>(xq + n_act * nxb);
    float *red = reinterpret_cast<float *>(xf + n_act * nxb);   // [slot][slice][lane]
    // The router kernel finished before the gate/up kernel let this grid
    // launch, so the logits may be read before waiting for h.
    route_cta(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_sel, s_w);
    for (int a = 0; a < n_act; ++a) {
        const int e = s_sel[a];
        if (e >= lo && e < hi) tile_cp_async(D, (long)(e - lo) * d + n0, rows, smem + a * tb, 32);
    }
    cp_async_commit();
    pdl_launch_dependents();
    pdl_wait();                                  // h comes from the gate/up kernel
    xprep_all(h + (long)tok * n_act * ffn, ffn, n_act, xq, xf);
    cp_async_wait_all();
    __syncthreads();
    const bool ok = true;
    for (int p = warp; p < n_act * ns; p += nwarps) {
        const int a = p / ns, sl = p % ns;
        const int e = s_sel[a];
        float v = 0.f;
        if (ok && e >= lo && e < hi && lane < rows) {
            const QView T = tile_view(QT, ffn, smem + a * tb, 32);
            WSlice<QT> w;
            load_slice<QT, false>(T, lane, sl, w);
            v = dot_slice<QT>(w, xq + a * nxb + sl * 8, xf + a * nxb + sl * 8);
        }
        red[p * 32 + lane] = v;
    }
    __syncthreads();
    if (threadIdx.x < 32 && lane < rows) {
        float total = 0.f;
        for (int a = 0; a < n_act; ++a) {
            const int e = s_sel[a];
            if (e < lo || e >= hi) continue;
            float v = 0.f;
            for (int k = 0; k < ns; ++k) v += red[(a * ns + k) * 32 + lane];
            total += s_w[a] * v;
        }
        eout[(long)tok * d + n0 + lane] = total;
    }
}

// ---- TMA-staged versions ---------------------------------------------------------------------
// Same work split as the bulk kernels; the 32-row tiles arrive as 2-D TMA
// boxes (32 rows x 128 bytes, 128-byte swizzle) issued by one thread.
template <int QT>
__global__ void __launch_bounds__(256, 2) gate_up_tma_kernel(
    const __grid_constant__ CUtensorMap tgw, const __grid_constant__ CUtensorMap tgd,
    const __grid_constant__ CUtensorMap tuw, const __grid_constant__ CUtensorMap tud, int ffn, int d, int n_exp,
    int n_act, int lo, int hi, const float *__restrict__ hn, const float *__restrict__ logits,
    int *__restrict__ sel_out, float *__restrict__ w_out, float *__restrict__ h, int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    __shared__ float red[2][8][32];
    __shared__ float s_p[kMaxExp];
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct];
    const int pair = blockIdx.y;
    const int tok = pair / n_act, slot = pair % n_act;
    pdl_wait();                                  // logits come from the router kernel
    pdl_launch_dependents();
    route_cta(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_sel, s_w);
    if (blockIdx.x == 0 && slot == 0 && threadIdx.x < n_act) {   // routing result for the API
        sel_out[tok * n_act + threadIdx.x] = s_sel[threadIdx.x];
        w_out[tok * n_act + threadIdx.x] = s_w[threadIdx.x];
    }
    const int e = s_sel[slot];
    if (e < lo || e >= hi) return;               // expert held by another process
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5, ns = d / 256;
    const int i0 = blockIdx.x * 32;
    const int rows = min(32, ffn - i0);
    const int tb = tma_tile_bytes(QT, d);
    uint8_t *tg = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
    uint8_t *tu = tg + tb;
    XBlk *xq = reinterpret_cast<XBlk *>(tu + tb);
    XF *xf = reinterpret_cast<XF *>(xq + d / 32);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, 2u * (uint32_t)tb);
        const int row0 = (e - lo) * ffn + i0;
        tma_issue_tile(&tgw, &tgd, QT, d, row0, tg, &bar);
        tma_issue_tile(&tuw, &tud, QT, d, row0, tu, &bar);
    }
    xprep_all(hn + (long)tok * d, d, 1, xq, xf);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status);
    float g = 0.f, u = 0.f;
    if (ok && lane < rows) {
        const int nwb = tma_wboxes(QT, d);
        for (int sl = warp; sl < ns; sl += nw) {
            WSlice<QT> w;
            load_slice_swz<QT>(tg, nwb, lane, sl, w);
            g += dot_slice<QT>(w, xq + sl * 8, xf + sl * 8);
            load_slice_swz<QT>(tu, nwb, lane, sl, w);
            u += dot_slice<QT>(w, xq + sl * 8, xf + sl * 8);
        }
    }
    red[0][warp][lane] = g;
    red[1][warp][lane] = u;
    __syncthreads();
    if (abort_flag) {
        if (threadIdx.x == 0) mbar_wait_drain(&bar, 0, 100000000ull);
        return;
    }
    if (threadIdx.x < 32 && lane < rows) {
        float gs = 0.f, us = 0.f;
        for (int k = 0; k < nw; ++k) {
            gs += red[0][k][lane];
            us += red[1][k][lane];
        }
        h[(long)pair * ffn + i0 + lane] = (gs / (1.0f + expf(-gs))) * us;   // silu(g) * u, qwen_moe.c:309
    }
}

template <int QT>
__global__ void __launch_bounds__(1024) down_tma_kernel(const __grid_constant__ CUtensorMap tdw,
                                                        const __grid_constant__ CUtensorMap tdd, int ffn, int d,
                                                        int n_exp, int n_act, int lo, int hi,
                                                        const float *__restrict__ h, const float *__restrict__ logits,
                                                        float *__restrict__ eout, int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct];
    __shared__ float s_p[kMaxExp];
    const int nxb = ffn / 32, ns = ffn / 256;
    const int tok = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int n0 = blockIdx.x * 32;
    const int rows = min(32, d - n0);
    const int tb = tma_tile_bytes(QT, ffn);
    uint8_t *tiles = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
    XBlk *xq = reinterpret_cast<XBlk *>(tiles + n_act * tb);
    XF *xf = reinterpret_cast<XF *>(xq + n_act * nxb);
    float *red = reinterpret_cast<float *>(xf + n_act * nxb);   // [slot][slice][lane]
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    // The router kernel finished before the gate/up kernel let this grid
    // launch, so the logits may be read before waiting for h.
    route_cta(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_sel, s_w);
    if (threadIdx.x == 0) {
        int nloc = 0;
        for (int a = 0; a < n_act; ++a) nloc += (s_sel[a] >= lo && s_sel[a] < hi);
        mbar_arrive_expect_tx(&bar, (uint32_t)(nloc * tb));
        for (int a = 0; a < n_act; ++a) {
            const int e = s_sel[a];
            if (e >= lo && e < hi) tma_issue_tile(&tdw, &tdd, QT, ffn, (e - lo) * d + n0, tiles + a * tb, &bar);
        }
    }
    pdl_launch_dependents();
    pdl_wait();                                  // h comes from the gate/up kernel
    xprep_all(h + (long)tok * n_act * ffn, ffn, n_act, xq, xf);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status);
    const int nwb = tma_wboxes(QT, ffn);
    for (int p = warp; p < n_act * ns; p += nwarps) {
        const int a = p / ns, sl = p % ns;
        const int e = s_sel[a];
        float v = 0.f;
        if (ok && e >= lo && e < hi && lane < rows) {
            WSlice<QT> w;
            load_slice_swz<QT>(tiles + a * tb, nwb, lane, sl, w);
            v = dot_slice<QT>(w, xq + a * nxb + sl * 8, xf + a * nxb + sl * 8);
        }
        red[p * 32 + lane] = v;
    }
    __syncthreads();
    if (abort_flag) {
        if (threadIdx.x == 0) mbar_wait_drain(&bar, 0, 100000000ull);
        return;
    }
    if (threadIdx.x < 32 && lane < rows) {
        float total = 0.f;
        for (int a = 0; a < n_act; ++a) {
            const int e = s_sel[a];
            if (e < lo || e >= hi) continue;
            float v = 0.f;
            for (int k = 0; k < ns; ++k) v += red[(a * ns + k) * 32 + lane];
            total += s_w[a] * v;
        }
        eout[(long)tok * d + n0 + lane] = total;
    }
}

}  // namespace q

using namespace q;

bool moe_shapes_ok(int d, int n_exp, int n_act, int ffn, int qtype) {
    const int be = (int)qtype_block_elems(qtype);
    return be && d > 0 && ffn > 0 && d % be == 0 && ffn % be == 0 && d % 32 == 0 && ffn % 32 == 0 &&
           d / 32 <= kMaxDXB && n_exp > 0 && n_exp <= kMaxExp && n_act > 0 && n_act <= kMaxAct &&
           n_act <= n_exp && (size_t)n_act * (ffn / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)n_act * (ffn / 256 + 1) * 128 <= 200 * 1024;
}

template <int QT>
static int launch_moe_qt(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *hn, float *eout, int batch,
                         cudaStream_t s) {
    const QView G = qmat_view(L.gate, 0), U = qmat_view(L.up, 0), D = qmat_view(L.down, 0);
    static const bool regs_only = getenv("X100_GEMV_KERNEL") && atoi(getenv("X100_GEMV_KERNEL")) >= 2;
    const size_t up_smem = 2 * (size_t)tile_bytes(QT, L.d, 32) + (size_t)(L.d / 32) * (sizeof(XBlk) + sizeof(XF));
    const size_t dn_smem = (size_t)L.n_act * tile_bytes(QT, L.ffn, 32) +
                           (size_t)L.n_act * (L.ffn / 32) * (sizeof(XBlk) + sizeof(XF)) +
                           (size_t)L.n_act * (L.ffn / 256) * 32 * 4;
    static bool attr_r[64];
    if (!attr_r[c->device]) {
        set_qkernel_attrs(router_logits_kernel);
        set_qkernel_attrs(router_topk_kernel);
        attr_r[c->device] = true;
    }
    const bool bulk_path = !regs_only && L.d % 256 == 0 && L.d <= 2048 && L.ffn % 256 == 0 &&
                           up_smem <= 200 * 1024 && dn_smem <= 200 * 1024;
    int st = bulk_path ? launch_pdl(router_logits_kernel, dim3((L.n_exp + 1) / 2), dim3(64), 0, s,
                                    (const float *)L.router, hn, L.d, L.n_exp, batch, S.logits)
                       : launch_pdl(router_topk_kernel, dim3((L.n_exp + 1) / 2), dim3(64), 0, s,
                                    (const float *)L.router, hn, L.d, L.n_exp, L.n_act, batch, S.logits, S.sel, S.w,
                                    S.ticket);
    if (st) return st;
    const bool tma_path = bulk_path && L.gate.tma_ok && L.up.tma_ok && L.down.tma_ok && !getenv("X100_MOE_NO_TMA");
    if (tma_path) {
        const size_t up_t = 1024 + 2 * (size_t)tma_tile_bytes(QT, L.d) + (size_t)(L.d / 32) * (sizeof(XBlk) + sizeof(XF));
        const size_t dn_t = 1024 + (size_t)L.n_act * tma_tile_bytes(QT, L.ffn) +
                            (size_t)L.n_act * (L.ffn / 32) * (sizeof(XBlk) + sizeof(XF)) +
                            (size_t)L.n_act * (L.ffn / 256) * 32 * 4;
        if (up_t <= 200 * 1024 && dn_t <= 200 * 1024) {
            static bool attr4[64];
            if (!attr4[c->device]) {
                set_qkernel_attrs(gate_up_tma_kernel<QT>);
                set_qkernel_attrs(down_tma_kernel<QT>);
                attr4[c->device] = true;
            }
            dim3 g1((L.ffn + 31) / 32, batch * L.n_act);
            st = launch_pdl(gate_up_tma_kernel<QT>, g1, dim3(32 * std::min(L.d / 256, 8)), up_t, s, L.gate.tmw,
                            L.gate.tmd, L.up.tmw, L.up.tmd, L.ffn, L.d, L.n_exp, L.n_act, L.lo, L.hi, hn,
                            (const float *)S.logits, S.sel, S.w, S.h, c->d_status);
            if (st) return st;
            const int pairs = L.n_act * (L.ffn / 256);
            dim3 g2((L.d + 31) / 32, batch);
            return launch_pdl(down_tma_kernel<QT>, g2, dim3(32 * std::min(pairs, 32)), dn_t, s, L.down.tmw, L.down.tmd,
                              L.ffn, L.d, L.n_exp, L.n_act, L.lo, L.hi, (const float *)S.h, (const float *)S.logits,
                              eout, c->d_status);
        }
    }
    if (bulk_path) {
        static bool attr3[64];
        if (!attr3[c->device]) {
            set_qkernel_attrs(gate_up_bulk_kernel<QT>);
            set_qkernel_attrs(down_bulk_kernel<QT>);
            attr3[c->device] = true;
        }
        dim3 g1((L.ffn + 31) / 32, batch * L.n_act);
        st = launch_pdl(gate_up_bulk_kernel<QT>, g1, dim3(32 * std::min(L.d / 256, 8)), up_smem, s, G, U, L.ffn,
                        L.d, L.n_exp, L.n_act, L.lo, L.hi, hn, (const float *)S.logits, S.sel, S.w, S.h,
                        c->d_status);
        if (st) return st;
        const int pairs = L.n_act * (L.ffn / 256);
        dim3 g2((L.d + 31) / 32, batch);
        return launch_pdl(down_bulk_kernel<QT>, g2, dim3(32 * std::min(pairs, 32)), dn_smem, s, D, L.ffn, L.d,
                          L.n_exp, L.n_act, L.lo, L.hi, (const float *)S.h, (const float *)S.logits, eout,
                          c->d_status);
    }
    if (L.d % 256 == 0 && L.d <= 2048 && L.ffn % 256 == 0 && L.ffn <= 4096) {
        dim3 g1((L.ffn + 31) / 32, batch * L.n_act);
        st = launch_pdl(gate_up_slice_kernel<QT>, g1, dim3(32 * (L.d / 256)), 0, s, G, U, L.ffn, L.d, L.n_act, L.lo,
                        L.hi, hn, (const int *)S.sel, S.h);
        if (st) return st;
        const int ns = L.ffn / 256;
        const int warps = std::min(32, L.n_act * ns) / ns * ns;
        const size_t smem = (size_t)L.n_act * (L.ffn / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)L.n_act * ns * 32 * 4;
        static bool attr2[64];
        if (!attr2[c->device]) {
            set_qkernel_attrs(down_slice_kernel<QT>);
            attr2[c->device] = true;
        }
        dim3 g2((L.d + 31) / 32, batch);
        return launch_pdl(down_slice_kernel<QT>, g2, dim3(32 * warps), smem, s, D, L.ffn, L.d, L.n_act, L.lo, L.hi,
                          (const float *)S.h, (const int *)S.sel, (const float *)S.w, eout);
    }
    dim3 g1((L.ffn + 7) / 8, batch * L.n_act);
    gate_up_kernel<QT><<<g1, 256, 0, s>>>(G, U, L.ffn, L.d, L.n_act, L.lo, L.hi, hn, S.sel, S.h);
    const int lpr = lanes_per_row(units_per_row(QT, L.ffn));
    const size_t smem = (size_t)L.n_act * (L.ffn / 32) * (sizeof(XBlk) + sizeof(XF));
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(down_combine_kernel<QT>);
        attr[c->device] = true;
    }
    dim3 g2((L.d + 7) / 8, batch);
    down_combine_kernel<QT><<<g2, 256, smem, s>>>(D, L.ffn, L.d, L.n_act, L.lo, L.hi, S.h, S.sel, S.w, eout, lpr);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_moe(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *hn, float *eout, int batch,
               cudaStream_t s) {
    if (batch < 1 || batch > kMaxBatch) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    switch (L.qtype) {
    case Q4_0: return launch_moe_qt<Q4_0>(c, L, S, hn, eout, batch, s);
    case Q8_0: return launch_moe_qt<Q8_0>(c, L, S, hn, eout, batch, s);
    case Q4_K: return launch_moe_qt<Q4_K>(c, L, S, hn, eout, batch, s);
    case Q3_K: return launch_moe_qt<Q3_K>(c, L, S, hn, eout, batch, s);
    default: set_error(X100_E_UNSUPPORTED); return X100_E_UNSUPPORTED;
    }
}

size_t moe_scratch_bytes(int n_exp, int n_act, int ffn) {
    size_t b = 0;
    b += (size_t)kMaxBatch * n_exp * 4;           // logits
    b += (size_t)kMaxBatch * n_act * 4 * 2;       // sel, w
    b += (size_t)kMaxBatch * n_act * ffn * 4;     // h
    b += 256 * 5;                                 // alignment + ticket
    return b;
}

// Carve the scratch regions out of one buffer of moe_scratch_bytes().
MoeScratch moe_scratch_carve(void *base, int n_exp, int n_act, int ffn) {
    MoeScratch S;
    uintptr_t p = (reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255);
    auto take = [&](size_t bytes) {
        void *r = reinterpret_cast<void *>(p);
        p = (p + bytes + 255) & ~uintptr_t(255);
        return r;
    };
    S.ticket = static_cast<unsigned *>(take(256));
    S.logits = static_cast<float *>(take((size_t)kMaxBatch * n_exp * 4));
    S.sel = static_cast<int *>(take((size_t)kMaxBatch * n_act * 4));
    S.w = static_cast<float *>(take((size_t)kMaxBatch * n_act * 4));
    S.h = static_cast<float *>(take((size_t)kMaxBatch * n_act * ffn * 4));
    return S;
}

}  // namespace x100

using namespace x100;

struct x100q_moe {
    int device;
    MoeLayer L;
    void *scratch = nullptr;
    MoeScratch S;
};

extern "C" {

x100q_moe *x100q_moe_create(int d, int n_exp, int n_act, int ffn, int qtype, const float *router,
                            const void *gate_exps, const void *up_exps, const void *down_exps, int expert_lo,
                            int expert_hi) {
    set_error(X100_OK);
    if (!moe_shapes_ok(d, n_exp, n_act, ffn, qtype) || !router || !gate_exps || !up_exps || !down_exps ||
        expert_lo < 0 || expert_hi > n_exp || expert_lo >= expert_hi) {
        set_error(X100_E_ARG);
        return nullptr;
    }
    DevCtx *c = ctx();
    if (!c) return nullptr;
    std::lock_guard<std::mutex> lk(c->mu);
    x100q_moe *m = new x100q_moe();
    m->device = c->device;
    MoeLayer &L = m->L;
    L.d = d;
    L.n_exp = n_exp;
    L.n_act = n_act;
    L.ffn = ffn;
    L.qtype = qtype;
    L.lo = expert_lo;
    L.hi = expert_hi;
    const int ne = expert_hi - expert_lo;
    const size_t rb_d = x100q_row_bytes(qtype, d), rb_f = x100q_row_bytes(qtype, ffn);
    const uint8_t *g = static_cast<const uint8_t *>(gate_exps) + (size_t)expert_lo * ffn * rb_d;
    const uint8_t *u = static_cast<const uint8_t *>(up_exps) + (size_t)expert_lo * ffn * rb_d;
    const uint8_t *dn = static_cast<const uint8_t *>(down_exps) + (size_t)expert_lo * d * rb_f;
    bool ok = cudaMalloc(&L.router, (size_t)n_exp * d * 4) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
    }
    ok = ok && check_cuda(cudaMemcpy(L.router, router, (size_t)n_exp * d * 4, cudaMemcpyHostToDevice), X100_E_COPY) == 0;
    ok = ok && qmat_upload(c, qtype, ne * ffn, d, g, L.gate, c->stream);
    ok = ok && qmat_upload(c, qtype, ne * ffn, d, u, L.up, c->stream);
    ok = ok && qmat_upload(c, qtype, ne * d, ffn, dn, L.down, c->stream);
    if (ok) {
        const size_t sb = moe_scratch_bytes(n_exp, n_act, ffn);
        if (fault_injected("alloc") || cudaMalloc(&m->scratch, sb) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            ok = false;
        } else {
            cudaMemset(m->scratch, 0, sb);
            m->S = moe_scratch_carve(m->scratch, n_exp, n_act, ffn);
        }
    }
    if (!ok) {
        cudaFree(L.router);
        cudaFree(L.gate.w);
        cudaFree(L.up.w);
        cudaFree(L.down.w);
        cudaFree(m->scratch);
        delete m;
        return nullptr;
    }
    return m;
}

void x100q_moe_destroy(x100q_moe *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaFree(m->L.router);
    cudaFree(m->L.gate.w);
    cudaFree(m->L.up.w);
    cudaFree(m->L.down.w);
    cudaFree(m->scratch);
    delete m;
}

int x100q_moe_ffn_dev(const x100q_moe *m, const float *hn, float *eout, int batch, int *sel_out, float *w_out,
                      void *stream) {
    set_error(X100_OK);
    if (!m || !hn || !eout || (reinterpret_cast<uintptr_t>(hn) & 15) != 0) {   // 16-byte loads of hn
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = launch_moe(c, m->L, m->S, hn, eout, batch, s);
    const size_t rb = (size_t)batch * m->L.n_act * 4;
    if (st == X100_OK && sel_out)
        st = check_cuda(cudaMemcpyAsync(sel_out, m->S.sel, rb, cudaMemcpyDeviceToDevice, s), X100_E_COPY);
    if (st == X100_OK && w_out)
        st = check_cuda(cudaMemcpyAsync(w_out, m->S.w, rb, cudaMemcpyDeviceToDevice, s), X100_E_COPY);
    if (st) set_error(st);
    return st;
}

int x100q_moe_ffn(const x100q_moe *m, const float *hn, float *eout, int batch, int *sel_out, float *w_out) {
    set_error(X100_OK);
    if (!m || !hn || !eout || batch < 1 || batch > kMaxBatch) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const size_t xb = (size_t)batch * m->L.d * 4;
    const float *hd = hn;
    float *ed = eout;
    const bool hdev = is_device_ptr(hn), edev = is_device_ptr(eout);
    if (!hdev) {
        void *b = stage_buf(c, 0, xb);
        if (!b) return get_error();
        if (fault_injected("copy") || check_cuda(cudaMemcpyAsync(b, hn, xb, cudaMemcpyHostToDevice, c->stream), X100_E_COPY))
            return get_error();
        hd = static_cast<const float *>(b);
    }
    if (!edev) {
        void *b = stage_buf(c, 1, xb);
        if (!b) return get_error();
        ed = static_cast<float *>(b);
    }
    int st = launch_moe(c, m->L, m->S, hd, ed, batch, c->stream);
    const size_t rb = (size_t)batch * m->L.n_act * 4;
    if (st == X100_OK && !edev)
        st = check_cuda(cudaMemcpyAsync(eout, ed, xb, cudaMemcpyDeviceToHost, c->stream), X100_E_COPY);
    if (st == X100_OK && sel_out)
        st = check_cuda(cudaMemcpyAsync(sel_out, m->S.sel, rb, cudaMemcpyDefault, c->stream), X100_E_COPY);
    if (st == X100_OK && w_out)
        st = check_cuda(cudaMemcpyAsync(w_out, m->S.w, rb, cudaMemcpyDefault, c->stream), X100_E_COPY);
    const int st2 = sync_and_status(c, c->stream);
    if (st == X100_OK) st = st2;
    if (st) set_error(st);
    return st;
}

}  // extern "C"

// ---- routing without allocation ----------------------------------------------------------
// Scratch of x100q_router_topk_noalloc: the completion ticket (first 256
// bytes) and up to kNoAllocLogits routing logits.  One copy per device,
// created when the library's module loads, shared by every call.
namespace {
constexpr int kNoAllocLogits = 2048;
static __device__ __align__(256) unsigned char g_router_scratch[256 + kNoAllocLogits * 4];
std::mutex g_noalloc_mu;
void *g_noalloc_addr[64];   // device address of g_router_scratch, per device
}  // namespace

extern "C" int x100q_router_topk_noalloc(const float *router, const float *hn, int d, int n_exp, int n_act,
                                         int batch, int *sel_out, float *w_out, void *stream) {
    set_error(X100_OK);
    if (!router || !hn || !sel_out || !w_out || d <= 0 || d % 4 || n_exp < 1 || n_exp > kMaxExp || n_act < 1 ||
        n_act > kMaxAct || n_act > n_exp || batch < 1 || batch > kMaxBatch ||
        (reinterpret_cast<uintptr_t>(router) & 15) || (reinterpret_cast<uintptr_t>(hn) & 15)) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (batch * n_exp > kNoAllocLogits) {
        set_error(X100_E_TOO_LARGE);
        return X100_E_TOO_LARGE;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        set_error(X100_E_NODEV);
        return X100_E_NODEV;
    }
    void *base;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_addr[dev]) {   // once per device, with that device current
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
            if (e != cudaSuccess || !p) return check_cuda(e != cudaSuccess ? e : cudaErrorUnknown, X100_E_LAUNCH);
            g_noalloc_addr[dev] = p;
        }
        base = g_noalloc_addr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned *ticket = static_cast<unsigned *>(base);
    float *logits = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + 256);
    // the ticket must start at zero; the logits are fully written before use
    if (check_cuda(cudaMemsetAsync(ticket, 0, sizeof(unsigned), s), X100_E_LAUNCH)) return get_error();
    q::router_topk_kernel<<<(n_exp + 7) / 8, 256, 0, s>>>(router, hn, d, n_exp, n_act, batch, logits, sel_out,
                                                          w_out, ticket);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

