// moe.cu -- the top-k SwiGLU mixture-of-experts FFN of the decode step and the
// x100q_moe_* entry points of include/x100q.h.
//
// Replaces the MoE block of the reference's forward() (qwen_moe.c:295-311;
// qwen_moe_q3k.c:1916-1978 with router mode 0 = fp32 and SwiGLU mode 0 =
// exact): router GEMV -> softmax -> greedy top-k -> renormalise -> for each
// selected expert gate/up GEMV, silu(g)*u, down GEMV, weighted sum.
//
// Kernels per call (each launched with programmatic dependent launch, so the
// next one starts staging weights while the previous one finishes):
//   router_logits  one warp per expert row (row held in registers before the
//                  wait): fp32 logits of every token.
//   batch 1 -- moe_fused: one CTA per SM; each CTA routes the token itself
//                  (softmax, greedy top-k with strict > and lowest index
//                  first, renormalisation), stages every gate/up and down
//                  row it owns at once, writes h = silu(g) * u for its
//                  gate/up rows, and -- once a grid-wide counter shows all h
//                  written -- sums the down rows of the selected experts in
//                  slot order a = 0..k-1 like the reference (no atomics).
//   batch > 1 -- gate_up (grid: row tile x token x slot) writes
//                  h[token][slot][rows]; down (grid: row tile x token) stages
//                  the rows of every selected expert and writes
//                  eout[token][rows] = sum_a w_a * (down_a . h_a) in slot order.
// router_topk (router logits + the routing in the last CTA to finish) serves
// x100q_router_topk_noalloc.
// Experts outside [expert_lo, expert_hi) contribute nothing (expert
// parallelism: the caller sums eout over processes, e.g. NCCL all-reduce).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../../include/x100q.h"
#include "moe.h"
#include "qgemv.h"
#include "qgemm.h"

namespace x100 {
namespace q {

constexpr int kMaxBatch = 16;
constexpr int kMaxAct = 16;
constexpr int kMaxExp = 256;

// ---- router + softmax + top-k ------------------------------------------------------
// When `zero` is set, CTA 0 also clears zero[0 .. nzero) (the completion
// counter of the fused expert kernel that follows) once the previous kernel
// on the stream is done with it.
__global__ void __launch_bounds__(256) router_topk_kernel(const float *__restrict__ router,
                                                          const float *__restrict__ hn, int d, int n_exp, int n_act,
                                                          int batch, float *__restrict__ logits, int *__restrict__ sel,
                                                          float *__restrict__ wsel, unsigned *__restrict__ ticket,
                                                          int *__restrict__ zero, int nzero) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int e = blockIdx.x * nwarps + warp;
    // the router row (independent of the previous kernel) is loaded before
    // waiting on it: the first nv * 128 floats (at most 2048) held in
    // registers, 16 bytes per lane per step; the rest of the row -- a longer
    // row, or a d that is not a multiple of 128 -- is streamed afterwards,
    // starting at float4 32 * nv
    constexpr int RV = 16;
    const int nv = min(d / 128, RV);
    const float4 *rw = reinterpret_cast<const float4 *>(router + (long)(e < n_exp ? e : 0) * d);
    float4 r[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i)
        if (e < n_exp && i < nv) r[i] = __ldg(rw + lane + 32 * i);
    pdl_launch_dependents();
    pdl_wait();
    if (zero && blockIdx.x == 0)
        for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
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
            for (int i = lane + 32 * nv; i < d / 4; i += 32) {
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
// router_logits: grid (experts / 2, batch); one warp per (expert row, token),
// the row and (with a norm) the norm weights loaded into registers before
// waiting on the previous kernel, then the token's 16-byte loads all issued
// before any arithmetic, so a CTA costs one memory round trip after the
// wait.  Writes logits[b][e].  The consumers (the expert kernels) finish the
// routing themselves, so no kernel waits on a last-arriving CTA.
// When `zero` is set, CTA (0, 0) also clears zero[0 .. nzero) -- the
// completion counters of the expert kernels that follow -- after the previous
// kernel on the stream has finished with them.
// With `nw` set the input is the residual stream: each warp applies the RMS
// norm of qwen_moe_q3k.c:1166 (x * s * nw, s = 1/sqrt(mean(x^2) + eps)) to
// its token, and warp 0 of CTA (0, b) writes the normed token b to hn_out for
// the expert kernels.
__global__ void __launch_bounds__(64) router_logits_kernel(const float *__restrict__ router,
                                                           const float *__restrict__ hn, int d, int n_exp,
                                                           int batch, float *__restrict__ logits,
                                                           int *__restrict__ zero, int nzero,
                                                           const float *__restrict__ nw, float eps,
                                                           float *__restrict__ hn_out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int e = blockIdx.x * nwarps + warp, b = blockIdx.y;
    constexpr int RV = 16;
    const int nv = min(d / 128, RV);
    const float4 *rw = reinterpret_cast<const float4 *>(router + (long)(e < n_exp ? e : 0) * d);
    const float4 *nw4 = reinterpret_cast<const float4 *>(nw);
    float4 r[RV], w[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i) {
        if (e < n_exp && i < nv) r[i] = __ldg(rw + lane + 32 * i);
        if (nw && i < nv) w[i] = __ldg(nw4 + lane + 32 * i);
    }
    pdl_launch_dependents();
    pdl_wait();
    if (zero && blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
    if (e >= n_exp || b >= batch) return;
    const float4 *x = reinterpret_cast<const float4 *>(hn + (long)b * d);
    float4 v[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i)
        if (i < nv) v[i] = __ldcg(x + lane + 32 * i);
    float sc = 1.f;
    if (nw) {
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < RV; ++i)
            if (i < nv) q += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        for (int i = lane + 32 * nv; i < d / 4; i += 32) {   // past the registers' share
            const float4 t = __ldcg(x + i);
            q += t.x * t.x + t.y * t.y + t.z * t.z + t.w * t.w;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
        sc = 1.0f / sqrtf(q / (float)d + eps);
#pragma unroll
        for (int i = 0; i < RV; ++i)
            if (i < nv)
                v[i] = make_float4(v[i].x * sc * w[i].x, v[i].y * sc * w[i].y, v[i].z * sc * w[i].z,
                                   v[i].w * sc * w[i].w);
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < RV; ++i) {
        if (i < nv) {
            s = fmaf(r[i].x, v[i].x, s);
            s = fmaf(r[i].y, v[i].y, s);
            s = fmaf(r[i].z, v[i].z, s);
            s = fmaf(r[i].w, v[i].w, s);
        }
    }
    const bool write_hn = nw && hn_out && blockIdx.x == 0 && warp == 0;
    for (int i = lane + 32 * nv; i < d / 4; i += 32) {
        const float4 rr = __ldg(rw + i);
        float4 t = __ldcg(x + i);
        if (nw) {
            const float4 ww = __ldg(nw4 + i);
            t = make_float4(t.x * sc * ww.x, t.y * sc * ww.y, t.z * sc * ww.z, t.w * sc * ww.w);
            if (write_hn) reinterpret_cast<float4 *>(hn_out + (long)b * d)[i] = t;
        }
        s = fmaf(rr.x, t.x, s);
        s = fmaf(rr.y, t.y, s);
        s = fmaf(rr.z, t.z, s);
        s = fmaf(rr.w, t.w, s);
    }
    if (write_hn) {
#pragma unroll
        for (int i = 0; i < RV; ++i)
            if (i < nv) reinterpret_cast<float4 *>(hn_out + (long)b * d)[lane + 32 * i] = v[i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) logits[b * n_exp + e] = s;
}

// Softmax over one token's logits, greedy top-k (strict >, lowest index wins)
// and renormalisation, by a whole CTA (qwen_moe.c:296-301).  Warp 0 forms the
// probabilities exactly as router_topk_kernel does; the rank of expert e is
// the number of experts with a larger probability, or an equal one at a lower
// index, which reproduces the greedy selection order.  A thread ranks one
// expert against one quarter of the experts (read four at a time) and the
// four counts are added.  Results in shared memory: s_sel[a], s_w[a] for
// a < n_act.  s_p holds kMaxExp + 16 floats, s_rk 4 * kMaxExp ints; s_wr is
// scratch of kMaxAct floats.  blockDim.x must be >= 64 and >= n_act.
//
// Warp 0 (lane l) loads logits l, l+32, ... of one token into pre[].
__device__ __forceinline__ void route_load(const float *lg, int n_exp, float (&pre)[kMaxExp / 32]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < kMaxExp / 32; ++i) {
        const int ee = lane + 32 * i;
        pre[i] = ee < n_exp ? __ldcg(lg + ee) : -1e30f;
    }
}
// Routing from logits already loaded by warp 0 (route_load).
__device__ __forceinline__ void route_from(const float (&pre)[kMaxExp / 32], int n_exp, int n_act, float *s_p,
                                           int *s_rk, int *s_sel, float *s_w, float *s_wr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ql = ((n_exp + 15) / 16) * 4;   // experts per quarter, a multiple of 4
    if (warp == 0) {
        float p[kMaxExp / 32];
        float m = -1e30f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            p[i] = pre[i];
            m = fmaxf(m, p[i]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            p[i] = ee < n_exp ? expf(p[i] - m) : 0.f;
            sum += p[i];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        const float inv = 1.0f / sum;
#pragma unroll
        for (int i = 0; i < kMaxExp / 32; ++i) {
            const int ee = lane + 32 * i;
            if (ee < n_exp) s_p[ee] = p[i] * inv;
            else if (ee < 4 * ql) s_p[ee] = -1.0f;   // padding never outranks a probability
        }
        if (lane < 16 && kMaxExp + lane < 4 * ql) s_p[kMaxExp + lane] = -1.0f;
    }
    __syncthreads();
    // rank of expert e = experts with a larger probability, or an equal one at
    // a lower index; thread task (e, quarter) counts one quarter of the experts
    for (int idx = threadIdx.x; idx < 4 * n_exp; idx += blockDim.x) {
        const int qq = idx / n_exp, e = idx - qq * n_exp;
        const float pe = s_p[e];
        const float4 *qv = reinterpret_cast<const float4 *>(s_p + qq * ql);
        int rank = 0;
#pragma unroll 4
        for (int i = 0; i < ql / 4; ++i) {
            const float4 v = qv[i];
            const int f = qq * ql + 4 * i;
            rank += (v.x > pe) || (v.x == pe && f < e);
            rank += (v.y > pe) || (v.y == pe && f + 1 < e);
            rank += (v.z > pe) || (v.z == pe && f + 2 < e);
            rank += (v.w > pe) || (v.w == pe && f + 3 < e);
        }
        s_rk[qq * kMaxExp + e] = rank;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_exp; e += blockDim.x) {
        const int rank = s_rk[e] + s_rk[kMaxExp + e] + s_rk[2 * kMaxExp + e] + s_rk[3 * kMaxExp + e];
        if (rank < n_act) {
            s_sel[rank] = e;
            s_wr[rank] = s_p[e];
        }
    }
    __syncthreads();
    if (threadIdx.x < n_act) {
        float ssum = 0.f;
        for (int a = 0; a < n_act; ++a) ssum += s_wr[a];
        s_w[threadIdx.x] = s_wr[threadIdx.x] / ssum;
    }
    __syncthreads();
}

__device__ __forceinline__ void route_fast(const float *lg, int n_exp, int n_act, float *s_p, int *s_rk, int *s_sel,
                                           float *s_w, float *s_wr) {
    float pre[kMaxExp / 32];
    if ((threadIdx.x >> 5) == 0) route_load(lg, n_exp, pre);
    route_from(pre, n_exp, n_act, s_p, s_rk, s_sel, s_w, s_wr);
}

// ---- expert kernels ---------------------------------------------------------------------
// Weights are in the slice layout of qformats.cuh: the rows of one expert are
// contiguous, so a run of rows is one bulk copy into shared memory, and a
// thread dots half a slice (half p of a staged run is half p % 2 of slice
// p / 2, which is row (p/2) / ns, slice (p/2) % ns).  red[] holds the sums
// row by row, [matrix or expert][row][slice][half] with an odd row stride
// 2 ns + 1, so the writes (consecutive threads, consecutive words) and the
// per-row sums (consecutive threads, rows an odd stride apart) are free of
// bank conflicts.
__host__ __device__ constexpr int red_stride(int ns) { return 2 * ns + 1; }
__host__ __device__ constexpr int gu_red_floats(int R, int ns) { return 2 * R * red_stride(ns); }
__host__ __device__ constexpr int dn_red_floats(int R, int ns, int n_act) { return n_act * R * (red_stride(ns) + 1); }

// silu(g) * u of one row (qwen_moe.c:309)
__device__ __forceinline__ float swiglu(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// sum of a row's 2 ns half-slice terms: the first halves, then the second halves
__device__ __forceinline__ float row_sum(const float *pr, int ns) {
    float a = 0.f, b = 0.f;
#pragma unroll 4
    for (int j = 0; j < ns; ++j) {
        a += pr[2 * j];
        b += pr[2 * j + 1];
    }
    return a + b;
}

// Down rows [0, rows) of nl local experts staged at dt + li * R * rb, dotted
// with token li of xb (h of that expert's slot); thread t < rows gets the
// weighted sum over li in order (slot order), weight s_w[s_loc[li]].  The
// per-expert row sums are formed by nl * rows threads at once.
template <int QT>
__device__ __forceinline__ float down_rows(const uint8_t *dt, int nl, int rows, int R, int ns, long rb, const XBuf &xb,
                                           float *red, int n_act, bool ok, const int *s_loc, const float *s_w) {
    constexpr int SB = slice_bytes(QT);
    const int S = red_stride(ns);
    float *yv = red + n_act * R * S;   // [expert][row]
    const int per = rows * ns * 2;     // halves per expert
    for (int p = threadIdx.x; p < nl * per; p += blockDim.x) {
        const int li = p / per, q = p - li * per;
        const int sp = q >> 1, hf = q & 1;
        const int r = sp / ns, sl = sp - r * ns;
        float v = 0.f;
        if (ok) {
            WHalf<QT> w;
            load_half<QT>(dt + li * R * rb + (long)sp * SB, hf, w);
            v = dot_half<QT>(w, hf, xb.half(li, sl, hf));
        }
        red[(li * R + r) * S + 2 * sl + hf] = v;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < nl * rows; t += blockDim.x) {
        const int li = t / rows, r = t - li * rows;
        yv[li * R + r] = row_sum(red + (li * R + r) * S, ns);
    }
    __syncthreads();
    float tot = 0.f;
    if (threadIdx.x < rows)
        for (int li = 0; li < nl; ++li) tot += s_w[s_loc[li]] * yv[li * R + threadIdx.x];   // eout += w_a * y_a in slot order (qwen_moe.c:310)
    return tot;
}

// ---- batched path (batch > 1): tokens grouped by expert ---------------------------------
// Group layout in S.grp: cnt[le] tokens of local expert le (le < n_exp),
// [n_exp] the number of active experts, [n_exp + 1 + k] the k-th active
// expert, then pairs[le][16] = token * n_act + slot.  The order of experts
// and pairs follows the atomics, but every (token, slot) is computed by one
// CTA and the combine adds the slots in order, so results do not vary.
constexpr int kMoeThreads = 512;
__host__ __device__ inline int grp_active(int n_exp) { return n_exp; }
__host__ __device__ inline int grp_list(int n_exp) { return n_exp + 1; }
__host__ __device__ inline int grp_pairs(int n_exp, int le) { return 2 * n_exp + 1 + le * kMaxBatch; }

// route_group: one CTA per token routes it, appends its local (token, slot)
// pairs to their experts' lists, and writes its prepared activations to
// xq (token tok at tok * xbuf_bytes(ns, 1)) once for all experts.
__global__ void __launch_bounds__(kMoeThreads, 1)
    route_group_kernel(int d, int n_exp, int n_act, int lo, int hi, const float *__restrict__ hn,
                       const float *__restrict__ logits, int *__restrict__ sel_out, float *__restrict__ w_out,
                       int *__restrict__ grp, uint8_t *__restrict__ xq, int *__restrict__ work) {
    __shared__ __align__(16) float s_p[kMaxExp + 16];
    __shared__ int s_rk[4 * kMaxExp];
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct], s_wr[kMaxAct];
    const int tok = blockIdx.x;
    const int ns = slices_per_row(d);
    pdl_wait();                                  // logits and the cleared groups come from the router kernel
    pdl_launch_dependents();
    if (tok == 0 && threadIdx.x < 2) work[threadIdx.x] = 0;   // work counters of the expert kernels
    route_fast(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_rk, s_sel, s_w, s_wr);
    if (threadIdx.x < n_act) {
        const int a = threadIdx.x, e = s_sel[a];
        sel_out[tok * n_act + a] = e;
        w_out[tok * n_act + a] = s_w[a];
        if (e >= lo && e < hi) {
            const int le = e - lo;
            const int pos = atomicAdd(&grp[le], 1);
            grp[grp_pairs(n_exp, le) + pos] = tok * n_act + a;
            if (pos == 0) grp[grp_list(n_exp) + atomicAdd(&grp[grp_active(n_exp)], 1)] = le;
        }
    }
    xprep_rows([hn, tok, d](int) { return hn + (long)tok * d; }, d, 1,
               xbuf_at(xq + (size_t)tok * xbuf_bytes(ns, 1), ns));
}

// ---- persistent pipelined expert kernels (batch > 1) ------------------------------
// The work is a list of items (active expert k, row tile t), expert-major.
// Thread 0 of each CTA claims chunks of kGrab consecutive items from a
// per-call counter (so CTAs stay balanced whatever the tokens per expert),
// and keeps kStages
// claimed items in flight as bulk copies (one mbarrier per stage, use u of a
// stage waits parity u & 1) while the CTA computes the oldest.  A stage is
// refilled only after the barrier that ends the item last held in it.  The
// routing metadata (active list, counts, pairs) is read into shared memory
// once per CTA.
constexpr int kStages = 4;
// Items per claim: one.  With ~13 items per CTA at batch 16, claims of 4
// left CTAs finishing up to a claim (~5 us) apart; one item per claim:
// decode batch 16 2057 -> 2277 tokens/s, MoE batch 16 150.8 K -> 165.6 K
// (2: 2199 / 160.3 K).
constexpr int kGrab = 1;

struct PipeMeta {            // shared-memory copy of the groups
    int n_active;
    int list[kMaxExp];       // active local experts
    int cnt[kMaxExp];        // pairs per active expert (by list index)
    int start[kMaxExp];      // exclusive prefix of cnt: the expert's first slot
    uint8_t pairs[kMaxExp][kMaxBatch];   // token * n_act + slot (< kMaxBatch * kMaxAct = 256)
    uint8_t tok[kMaxExp][kMaxBatch];     // the pair's token
};
static_assert(kMaxBatch * kMaxAct <= 256, "pairs are stored as bytes");

__device__ __forceinline__ void load_meta(const int *__restrict__ grp, int n_exp, int n_act, PipeMeta &M) {
    if (threadIdx.x == 0) M.n_active = __ldcg(grp + grp_active(n_exp));
    __syncthreads();
    const int na = M.n_active;
    for (int k = threadIdx.x; k < na; k += blockDim.x) {
        const int le = __ldcg(grp + grp_list(n_exp) + k);
        M.list[k] = le;
        M.cnt[k] = __ldcg(grp + le);
    }
    __syncthreads();
    if (threadIdx.x < 32) {   // slot starts: warp 0 scans cnt, kMaxExp / 32 entries per lane
        constexpr int E = kMaxExp / 32;
        const int l = threadIdx.x;
        int c[E], run = 0;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            c[i] = E * l + i < na ? M.cnt[E * l + i] : 0;
            run += c[i];
        }
        int incl = run;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (l >= o) incl += v;
        }
        int base = incl - run;
#pragma unroll
        for (int i = 0; i < E; ++i) {
            if (E * l + i < na) M.start[E * l + i] = base;
            base += c[i];
        }
    }
    for (int t = threadIdx.x; t < na * kMaxBatch; t += blockDim.x) {
        const int k = t / kMaxBatch, j = t - k * kMaxBatch;
        if (j < M.cnt[k]) {
            const int pr = __ldcg(grp + grp_pairs(n_exp, M.list[k]) + j);
            M.pairs[k][j] = (uint8_t)pr;
            M.tok[k][j] = (uint8_t)(pr / n_act);
        }
    }
    __syncthreads();
}

// gate_up_pipe: items (k, t) with t over ffn / TRg tiles; an item stages TRg
// gate rows and TRg up rows of expert list[k], dots every half-slice with
// each of the expert's tokens and writes h[pair][rows] = silu(g) * u.  The
// prepared activations of the expert's first kXsTok tokens are copied into
// shared memory once per run of items of the same expert (the dot products
// then read them at shared-memory latency); further tokens are read from xq
// through L2.
constexpr int kXsTok = 8;
template <int QT>
__global__ void __launch_bounds__(kMoeThreads, 1)
    gate_up_pipe_kernel(const uint8_t *__restrict__ gw, const uint8_t *__restrict__ uw, int ffn, int d, int n_exp,
                        int n_act, int TRg, const int *__restrict__ grp, const uint8_t *__restrict__ xq,
                        float *__restrict__ h, int *__restrict__ work, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t full[kStages];
    __shared__ int abort_flag;
    __shared__ int s_item[kStages];
    __shared__ PipeMeta M;
    constexpr int SB = slice_bytes(QT);
    const int ns = slices_per_row(d), xb1 = xbuf_bytes(ns, 1), S = red_stride(ns);
    const long rb = row_bytes_dev(QT, d);
    const int stage_bytes_ = (int)(2 * TRg * rb);
    uint8_t *xs = smem + kStages * stage_bytes_;                               // [kXsTok] staged activations
    float *red = reinterpret_cast<float *>(xs + kXsTok * xb1);                 // [pair][matrix][row][slice][half]
    if (threadIdx.x == 0) {
        for (int st = 0; st < kStages; ++st) mbar_init(&full[st], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    pdl_wait();                                  // groups and activations come from the routing kernel
    pdl_launch_dependents();
    load_meta(grp, n_exp, n_act, M);
    const int tiles = (ffn + TRg - 1) / TRg;
    const int W = M.n_active * tiles;
    int g_next = 0, g_end = 0;                   // thread 0: the claimed chunk not yet issued
    auto issue = [&](int i) {                    // thread 0: the next claimed item into stage i % kStages
        if (g_next == g_end) {
            g_next = atomicAdd(work, kGrab);
            g_end = min(g_next + kGrab, W);
        }
        const int it = g_next < W ? g_next++ : -1;
        s_item[i % kStages] = it;
        if (it < 0) return;
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TRg, ffn - t * TRg);
        uint8_t *dst = smem + (i % kStages) * stage_bytes_;
        const long r0 = (long)M.list[k] * ffn + (long)t * TRg;
        mbar_arrive_expect_tx(&full[i % kStages], (uint32_t)(2 * rows * rb));
        stage_bytes(dst, gw + r0 * rb, (uint32_t)(rows * rb), &full[i % kStages]);
        stage_bytes(dst + TRg * rb, uw + r0 * rb, (uint32_t)(rows * rb), &full[i % kStages]);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < kStages - 1; ++i) issue(i);
    __syncthreads();
    int done = 0, kprep = -1;
    for (int i = 0;; ++i) {
        const int it = s_item[i % kStages];      // claimed items form a prefix: -1 ends the loop
        if (it < 0) break;
        __syncthreads();                         // everyone has read the slot before it is refilled
        if (threadIdx.x == 0) issue(i + kStages - 1);
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TRg, ffn - t * TRg), np = M.cnt[k];
        if (k != kprep) {                        // uniform: every thread sees the same item
            const int nst = min(np, kXsTok), nv = xb1 / 16;
            for (int v = threadIdx.x; v < nst * nv; v += blockDim.x) {
                const int j = v / nv, o = v - j * nv;
                reinterpret_cast<uint4 *>(xs + (size_t)j * xb1)[o] =
                    __ldcg(reinterpret_cast<const uint4 *>(xq + (size_t)(M.pairs[k][j] / n_act) * xb1) + o);
            }
            __syncthreads();
            kprep = k;
        }
        const uint8_t *tg = smem + (i % kStages) * stage_bytes_, *tu = tg + TRg * rb;
        const bool ok = mbar_wait(&full[i % kStages], (uint32_t)((i / kStages) & 1), &abort_flag, status);
        done = i + 1;
        const int per = rows * ns * 2;   // halves per matrix
        for (int p = threadIdx.x; p < 2 * per; p += blockDim.x) {
            const int mat = p >= per, q = p - mat * per;
            const int sp = q >> 1, hf = q & 1;
            const int r = sp / ns, sl = sp - r * ns;
            WHalf<QT> w;
            if (ok) load_half<QT>((mat ? tu : tg) + (long)sp * SB, hf, w);
            for (int j = 0; j < np; ++j) {
                const XBuf xj = j < kXsTok ? xbuf_at(xs + (size_t)j * xb1, ns)
                                           : xbuf_at(const_cast<uint8_t *>(xq) + (size_t)(M.pairs[k][j] / n_act) * xb1, ns);
                red[((j * 2 + mat) * TRg + r) * S + 2 * sl + hf] = ok ? dot_half<QT>(w, hf, xj.half(0, sl, hf)) : 0.f;
            }
        }
        __syncthreads();
        for (int u = threadIdx.x; u < np * rows; u += blockDim.x) {
            const int j = u / rows, r = u - j * rows;
            h[(long)M.pairs[k][j] * ffn + t * TRg + r] =
                swiglu(row_sum(red + ((2 * j) * TRg + r) * S, ns), row_sum(red + ((2 * j + 1) * TRg + r) * S, ns));
        }
        if (__syncthreads_or(abort_flag)) break;   // the same decision in every thread
    }
    if (threadIdx.x == 0 && abort_flag) {        // copies still in flight after a timeout
        for (int i = done; i < done + kStages - 1; ++i)
            if (s_item[i % kStages] >= 0)
                mbar_wait_drain(&full[i % kStages], (uint32_t)((i / kStages) & 1), 100000000ull);
        if (done > 0) mbar_wait_drain(&full[(done - 1) % kStages], (uint32_t)(((done - 1) / kStages) & 1), 100000000ull);
    }
}

// down_pipe: items (k, t) with t over d / TRd tiles; an item stages TRd down
// rows of expert list[k] and writes the unweighted part[pair][rows] =
// down . h[pair] for each of the expert's pairs.  The expert's h rows are
// prepared (xprep_rows) once per run of items of the same expert.
template <int QT>
__global__ void __launch_bounds__(kMoeThreads, 1)
    down_pipe_kernel(const uint8_t *__restrict__ dw, int ffn, int d, int n_exp, int TRd, int nb,
                     const int *__restrict__ grp, const float *__restrict__ h, float *__restrict__ part,
                     int *__restrict__ work, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t full[kStages];
    __shared__ int abort_flag;
    __shared__ int s_item[kStages];
    __shared__ PipeMeta M;
    constexpr int SB = slice_bytes(QT);
    const int ns = slices_per_row(ffn), S = red_stride(ns);
    const long rb = row_bytes_dev(QT, ffn);
    const int stage_bytes_ = (int)(TRd * rb);
    const XBuf xb = xbuf_at(smem + kStages * stage_bytes_, ns);   // [pair] prepared h of the current expert
    float *red = reinterpret_cast<float *>(smem + kStages * stage_bytes_ + xbuf_bytes(ns, nb));
    if (threadIdx.x == 0) {
        for (int st = 0; st < kStages; ++st) mbar_init(&full[st], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    // The routing kernel finished before the gate/up kernel let this grid
    // launch, so the groups may be read, and weights staged, before waiting
    // for h.
    load_meta(grp, n_exp, 1, M);
    const int tiles = (d + TRd - 1) / TRd;
    const int W = M.n_active * tiles;
    int g_next = 0, g_end = 0;
    auto issue = [&](int i) {
        if (g_next == g_end) {
            g_next = atomicAdd(work, kGrab);
            g_end = min(g_next + kGrab, W);
        }
        const int it = g_next < W ? g_next++ : -1;
        s_item[i % kStages] = it;
        if (it < 0) return;
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TRd, d - t * TRd);
        mbar_arrive_expect_tx(&full[i % kStages], (uint32_t)(rows * rb));
        stage_bytes(smem + (i % kStages) * stage_bytes_, dw + ((long)M.list[k] * d + (long)t * TRd) * rb,
                    (uint32_t)(rows * rb), &full[i % kStages]);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < kStages - 1; ++i) issue(i);
    pdl_launch_dependents();
    pdl_wait();                                  // h comes from the gate/up kernel
    __syncthreads();
    int done = 0, kprep = -1;
    for (int i = 0;; ++i) {
        const int it = s_item[i % kStages];
        if (it < 0) break;
        __syncthreads();
        if (threadIdx.x == 0) issue(i + kStages - 1);
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TRd, d - t * TRd), np = M.cnt[k];
        if (k != kprep) {                        // uniform: every thread sees the same item
            const uint8_t *pr = M.pairs[k];
            xprep_rows([h, pr, ffn](int j) { return h + (long)pr[j] * ffn; }, ffn, np, xb);
            __syncthreads();
            kprep = k;
        }
        const uint8_t *dt = smem + (i % kStages) * stage_bytes_;
        const bool ok = mbar_wait(&full[i % kStages], (uint32_t)((i / kStages) & 1), &abort_flag, status);
        done = i + 1;
        const int per = rows * ns * 2;
        for (int p = threadIdx.x; p < per; p += blockDim.x) {
            const int sp = p >> 1, hf = p & 1;
            const int r = sp / ns, sl = sp - r * ns;
            WHalf<QT> w;
            if (ok) load_half<QT>(dt + (long)sp * SB, hf, w);
            for (int j = 0; j < np; ++j)
                red[(j * TRd + r) * S + 2 * sl + hf] = ok ? dot_half<QT>(w, hf, xb.half(j, sl, hf)) : 0.f;
        }
        __syncthreads();
        for (int u = threadIdx.x; u < np * rows; u += blockDim.x) {
            const int j = u / rows, r = u - j * rows;
            part[(long)M.pairs[k][j] * d + t * TRd + r] = row_sum(red + (j * TRd + r) * S, ns);
        }
        if (__syncthreads_or(abort_flag)) break;   // the same decision in every thread
    }
    if (threadIdx.x == 0 && abort_flag) {        // copies still in flight after a timeout
        for (int i = done; i < done + kStages - 1; ++i)
            if (s_item[i % kStages] >= 0)
                mbar_wait_drain(&full[i % kStages], (uint32_t)((i / kStages) & 1), 100000000ull);
        if (done > 0) mbar_wait_drain(&full[(done - 1) % kStages], (uint32_t)(((done - 1) / kStages) & 1), 100000000ull);
    }
}

// ---- warp-specialised expert kernels (batch > 1) ----------------------------------
// A producer warp streams the items (active expert k, row tile) into a ring
// of nst shared-memory stages with bulk copies (full[s] completes on the
// copied bytes; empty[s] takes one arrival per consumer warp once it has read
// the stage) and NW consumer warps compute them; warps wait for one
// another only through the ring.  A consumer lane owns one half slice of a
// row (or several, seg apart), unpacks it once (unpack_half) and dots it with
// every token of the expert; the seg lanes of a row then sum their terms with
// shuffles.  Expert k's tokens are its slots start[k] .. start[k] + cnt[k] - 1
// of the grouped h / hq buffers.
// Consumer warps per kernel, with the producer 16 (4 on each of the SM's
// four schedulers, whose register files then cap a thread at 128 registers)
// when the ring of the wider item still has two stages in the shared memory
// left by the batch's activations, else 12 (3 per scheduler, 168 registers).
// A 17th warp would put 5 warps on one scheduler and cap every thread at 96.
constexpr int kWsWide = 15;
constexpr int kWsNarrow = 11;
// Q4_K's two unpacked half slices do not fit 128 registers (ptxas spills)
constexpr bool ws_wide_fits(int qt) { return qt != Q4_K; }
constexpr int kWsMaxSt = 4;
constexpr int kWsTok = 2;                    // tokens dotted per pass over a lane's half slices (more need more registers)
constexpr size_t kWsSmem = 215 * 1024;       // dynamic shared memory (PipeMeta and the barriers are static)
template <int N> struct IntC { static constexpr int value = N; };   // a token count as a type
// f(IntC<n>{}) for a run-time n in 1 .. N
template <int N, typename F> __device__ __forceinline__ void with_count(int n, F &&f) {
    if constexpr (N > 1) {
        if (n < N) {
            with_count<N - 1>(n, f);
            return;
        }
    }
    f(IntC<N>{});
}

// lanes per row: the row's 2 ns half slices, at most cap lanes (then a lane
// takes half slices ls, ls + cap, ...)
__host__ __device__ inline int ws_seg(int hsr, int cap) { return hsr < cap ? hsr : cap; }
// top = the largest power of two below seg (0 for seg = 1)
__host__ __device__ inline int ws_top(int seg) {
    int top = 1;
    while (2 * top < seg) top <<= 1;
    return seg > 1 ? top : 0;
}
// sum over the seg lanes of each segment (lanes rr * seg .. rr * seg + seg - 1
// of the warp); the first lane of a segment receives it.  top = ws_top(seg).
__device__ __forceinline__ float seg_sum(float v, int ls, int seg, int top) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        if (off <= top) {
            const float o = __shfl_down_sync(0xffffffffu, v, off);
            if (ls + off < seg) v += o;
        }
    return v;
}

// The producer lane's loop, shared by both kernels: claim items in chunks of
// kGrab from *work, and for each stage wait until the consumers released it,
// record the item (-1 ends the consumers' loop) and start its copies
// (fill(stage, item) announces and issues them).  On a timeout it waits for
// its copies still in flight before returning.
template <typename Fill>
__device__ __forceinline__ void ws_produce(int nst, int W, int *work, uint64_t *full, uint64_t *empty, int *s_item,
                                           volatile int *abort_flag, int *status, Fill fill) {
    int g_next = 0, g_end = 0, i = 0;
    for (;; ++i) {
        const int st = i % nst;
        if (i >= nst && !mbar_wait(&empty[st], (uint32_t)(((i / nst) - 1) & 1), abort_flag, status)) break;
        if (g_next == g_end) {
            g_next = atomicAdd(work, kGrab);
            g_end = min(g_next + kGrab, W);
        }
        const int it = g_next < W ? g_next++ : -1;
        s_item[st] = it;
        if (it < 0) {
            mbar_arrive(&full[st]);
            return;
        }
        fill(st, it);
    }
    for (int u = max(0, i - nst); u < i; ++u)   // copies issued but perhaps not landed
        mbar_wait_drain(&full[u % nst], (uint32_t)((u / nst) & 1), 100000000ull);
}

// gate / up: an item is (k, TR = NW * rpw rows of gate and the same
// rows of up); a warp holds rpw rows of seg lanes, and a lane the same half
// slice of the row in both matrices, so each activation load serves both
// dots.  The prepared activations of the batch's nb tokens (xq, token after
// token) are copied into shared memory once per CTA.  Writes h[slot][row] =
// silu(gate . x) * (up . x) (qwen_moe.c:304-309).
template <int QT, int NW>
__global__ void __launch_bounds__(32 * (NW + 1), 1)
    gate_up_ws_kernel(const uint8_t *__restrict__ gw, const uint8_t *__restrict__ uw, int ffn, int d, int n_exp,
                      int n_act, int nb, int nst, const int *__restrict__ grp, const uint8_t *__restrict__ xq,
                      float *__restrict__ h, int *__restrict__ work, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t full[kWsMaxSt], empty[kWsMaxSt], xbar;
    __shared__ int s_item[kWsMaxSt];
    __shared__ int abort_flag;
    __shared__ PipeMeta M;
    constexpr int SB = slice_bytes(QT);
    const int ns = slices_per_row(d), xb1 = xbuf_bytes(ns, 1), hsr = 2 * ns;
    const long rb = row_bytes_dev(QT, d);
    const int seg = ws_seg(hsr, 32), rpw = 32 / seg, TR = NW * rpw;
    const int stage_b = (int)(2 * TR * rb);
    uint8_t *xa = smem + (size_t)nst * stage_b;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int st = 0; st < nst; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], NW);
        }
        mbar_init(&xbar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    pdl_wait();                                  // groups and activations come from the routing kernel
    pdl_launch_dependents();
    load_meta(grp, n_exp, n_act, M);
    const int tiles = (ffn + TR - 1) / TR, W = M.n_active * tiles;
    if (warp == NW) {                      // producer
        if (lane == 0) {
            mbar_arrive_expect_tx(&xbar, (uint32_t)(nb * xb1));
            stage_bytes(xa, xq, (uint32_t)(nb * xb1), &xbar);
            ws_produce(nst, W, work, full, empty, s_item, &abort_flag, status, [&](int st, int it) {
                const int k = it / tiles, t = it - k * tiles;
                const int rows = min(TR, ffn - t * TR);
                const long r0 = (long)M.list[k] * ffn + (long)t * TR;
                uint8_t *dst = smem + (size_t)st * stage_b;
                mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * rows * rb));
                stage_bytes(dst, gw + r0 * rb, (uint32_t)(rows * rb), &full[st]);
                stage_bytes(dst + TR * rb, uw + r0 * rb, (uint32_t)(rows * rb), &full[st]);
            });
            mbar_wait_drain(&xbar, 0, 100000000ull);
        }
        return;
    }
    if (!mbar_wait(&xbar, 0, &abort_flag, status)) return;
    const int rr = lane / seg, ls = lane - rr * seg, top = ws_top(seg);
    const int rin = warp * rpw + rr;             // row within the item
    for (int i = 0;; ++i) {
        const int st = i % nst;
        if (!mbar_wait(&full[st], (uint32_t)((i / nst) & 1), &abort_flag, status)) break;
        const int it = *(volatile int *)&s_item[st];
        if (it < 0) break;
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TR, ffn - t * TR), np = M.cnt[k];
        const bool live = rr < rpw && rin < rows;
        const uint8_t *wg = smem + (size_t)st * stage_b + (long)rin * rb, *wu = wg + TR * rb;
        // one pass over the lane's half slices for NT tokens j0 .. j0 + NT - 1;
        // NT is a compile-time constant, so no dot is issued for an empty token slot
        auto pass = [&](int j0, auto ntc) {
            constexpr int NT = decltype(ntc)::value;
            float ag[NT] = {}, au[NT] = {};
            const uint8_t *xt[NT];
#pragma unroll
            for (int jj = 0; jj < NT; ++jj) xt[jj] = xa + (size_t)M.tok[k][j0 + jj] * xb1;
            for (int hq = ls; live && hq < hsr; hq += seg) {
                UHalf<QT> ug, uu;
                {
                    WHalf<QT> w;
                    load_half<QT>(wg + (long)(hq >> 1) * SB, hq & 1, w);
                    unpack_half<QT>(w, hq & 1, ug);
                    load_half<QT>(wu + (long)(hq >> 1) * SB, hq & 1, w);
                    unpack_half<QT>(w, hq & 1, uu);
                }
                const int xo = (hq >> 1) * kXSlice + (hq & 1) * kXHalf;
#pragma unroll
                for (int jj = 0; jj < NT; ++jj) {
                    const XB *x = reinterpret_cast<const XB *>(xt[jj] + xo);
                    ag[jj] += dot_uhalf<QT>(ug, x);
                    au[jj] += dot_uhalf<QT>(uu, x);
                }
            }
            if (j0 + NT >= np) {                 // the last read of this stage
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
#pragma unroll
            for (int jj = 0; jj < NT; ++jj) {
                const float g = seg_sum(ag[jj], ls, seg, top), u = seg_sum(au[jj], ls, seg, top);
                if (ls == 0 && live) h[(long)(M.start[k] + j0 + jj) * ffn + t * TR + rin] = swiglu(g, u);
            }
        };
        for (int j0 = 0; j0 < np; j0 += kWsTok) {   // passes of up to kWsTok tokens (one for most experts)
            with_count<kWsTok>(min(np - j0, kWsTok), [&](auto c) { pass(j0, c); });
        }
    }
}

// h of every slot -> the prepared form (xprep_rows) the down kernel dots.
__global__ void __launch_bounds__(256) prep_slots_kernel(const float *__restrict__ h, int ffn, uint8_t *__restrict__ hq) {
    pdl_wait();                                  // h comes from the gate / up kernel
    pdl_launch_dependents();
    const int p = blockIdx.x, ns = slices_per_row(ffn);
    xprep_rows([h, p, ffn](int) { return h + (long)p * ffn; }, ffn, 1, xbuf_at(hq + (size_t)p * xbuf_bytes(ns, 1), ns));
}

// down: an item is (k, TR = 2 NW rpw rows of down); a warp holds rpw
// pairs of rows of seg lanes, a lane the same half slice of row r and row r
// + TR / 2 (one activation load, two dots); a stage holds the rows and the
// expert's prepared h (its slots, contiguous in hq).  Writes
// the unweighted part[pair][row] for the combine.  The weights of the first
// stages are requested before the dependency wait (the groups are final once
// this kernel runs: the gate / up kernel read them behind its own wait).
template <int QT, int NW>
__global__ void __launch_bounds__(32 * (NW + 1), 1)
    down_ws_kernel(const uint8_t *__restrict__ dw, int ffn, int d, int n_exp, int nb, int nst,
                   const int *__restrict__ grp, const uint8_t *__restrict__ hq, float *__restrict__ part,
                   int *__restrict__ work, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t full[kWsMaxSt], empty[kWsMaxSt];
    __shared__ int s_item[kWsMaxSt];
    __shared__ int abort_flag;
    __shared__ PipeMeta M;
    constexpr int SB = slice_bytes(QT);
    const int ns = slices_per_row(ffn), xb1 = xbuf_bytes(ns, 1), hsr = 2 * ns;
    const long rb = row_bytes_dev(QT, ffn);
    const int seg = ws_seg(hsr, 32), rpw = 32 / seg, TRh = NW * rpw, TR = 2 * TRh;
    const int wbytes = (int)(TR * rb), stage_b = wbytes + nb * xb1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int st = 0; st < nst; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], NW);
        }
        abort_flag = 0;
        fence_barrier_init();
    }
    load_meta(grp, n_exp, 1, M);
    const int tiles = (d + TR - 1) / TR, W = M.n_active * tiles;
    if (warp == NW) {                      // producer
        if (lane == 0) {
            int nfill = 0;                       // stages whose h copies wait for the dependency
            int pend_st[kWsMaxSt], pend_k[kWsMaxSt];
            ws_produce(nst, W, work, full, empty, s_item, &abort_flag, status, [&](int st, int it) {
                const int k = it / tiles, t = it - k * tiles;
                const int rows = min(TR, d - t * TR);
                uint8_t *dst = smem + (size_t)st * stage_b;
                mbar_arrive_expect_tx(&full[st], (uint32_t)(rows * rb + M.cnt[k] * xb1));
                stage_bytes(dst, dw + ((long)M.list[k] * d + (long)t * TR) * rb, (uint32_t)(rows * rb), &full[st]);
                if (nfill >= 0 && nfill < nst) {  // still before the dependency wait
                    pend_st[nfill] = st;
                    pend_k[nfill] = k;
                    if (++nfill == nst) {
                        pdl_wait();              // hq comes from the preparation kernel
                        for (int f = 0; f < nst; ++f)
                            stage_bytes(smem + (size_t)pend_st[f] * stage_b + wbytes,
                                        hq + (size_t)M.start[pend_k[f]] * xb1, (uint32_t)(M.cnt[pend_k[f]] * xb1),
                                        &full[pend_st[f]]);
                        nfill = -1;
                    }
                    return;
                }
                stage_bytes(dst + wbytes, hq + (size_t)M.start[k] * xb1, (uint32_t)(M.cnt[k] * xb1), &full[st]);
            });
            if (nfill > 0) {                     // fewer items than stages
                pdl_wait();
                for (int f = 0; f < nfill; ++f)
                    stage_bytes(smem + (size_t)pend_st[f] * stage_b + wbytes, hq + (size_t)M.start[pend_k[f]] * xb1,
                                (uint32_t)(M.cnt[pend_k[f]] * xb1), &full[pend_st[f]]);
            }
            if (nfill != -1) pdl_wait();
        }
        pdl_launch_dependents();
        return;
    }
    pdl_launch_dependents();
    const int rr = lane / seg, ls = lane - rr * seg, top = ws_top(seg);
    const int rin = warp * rpw + rr;             // rows rin and rin + TRh of the item
    for (int i = 0;; ++i) {
        const int st = i % nst;
        if (!mbar_wait(&full[st], (uint32_t)((i / nst) & 1), &abort_flag, status)) break;
        const int it = *(volatile int *)&s_item[st];
        if (it < 0) break;
        const int k = it / tiles, t = it - k * tiles;
        const int rows = min(TR, d - t * TR), np = M.cnt[k];
        const bool live0 = rr < rpw && rin < rows, live1 = rr < rpw && rin + TRh < rows;
        const uint8_t *w0 = smem + (size_t)st * stage_b + (long)rin * rb, *w1 = w0 + (long)TRh * rb;
        const uint8_t *xh = smem + (size_t)st * stage_b + wbytes;   // the expert's slots, xb1 apart
        auto pass = [&](int j0, auto ntc) {      // NT tokens from j0, NT known at compile time
            constexpr int NT = decltype(ntc)::value;
            float a0[NT] = {}, a1[NT] = {};
            for (int hq2 = ls; live0 && hq2 < hsr; hq2 += seg) {
                UHalf<QT> u0, u1;
                {
                    WHalf<QT> w;
                    load_half<QT>(w0 + (long)(hq2 >> 1) * SB, hq2 & 1, w);
                    unpack_half<QT>(w, hq2 & 1, u0);
                    if (live1) load_half<QT>(w1 + (long)(hq2 >> 1) * SB, hq2 & 1, w);
                    unpack_half<QT>(w, hq2 & 1, u1);   // a copy of row 0 when row 1 is past the matrix
                }
                const uint8_t *xo = xh + (size_t)j0 * xb1 + (hq2 >> 1) * kXSlice + (hq2 & 1) * kXHalf;
#pragma unroll
                for (int jj = 0; jj < NT; ++jj) {
                    const XB *x = reinterpret_cast<const XB *>(xo + (size_t)jj * xb1);
                    a0[jj] += dot_uhalf<QT>(u0, x);
                    a1[jj] += dot_uhalf<QT>(u1, x);
                }
            }
            if (j0 + NT >= np) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
#pragma unroll
            for (int jj = 0; jj < NT; ++jj) {
                const float v0 = seg_sum(a0[jj], ls, seg, top), v1 = seg_sum(a1[jj], ls, seg, top);
                float *o = part + (long)M.pairs[k][j0 + jj] * d + t * TR + rin;
                if (ls == 0 && live0) o[0] = v0;
                if (ls == 0 && live1) o[TRh] = v1;
            }
        };
        for (int j0 = 0; j0 < np; j0 += kWsTok) {
            with_count<kWsTok>(min(np - j0, kWsTok), [&](auto c) { pass(j0, c); });
        }
    }
}

// Launch shape of the warp-specialised kernels: stages and staged tokens.
struct WsPlan {
    int nst = 0, nw = 0;
    size_t smem = 0;
};
static WsPlan ws_plan_gate_up(int qt, int d, int batch, int nw) {
    const int ns = slices_per_row(d), seg = ws_seg(2 * ns, 32), TR = nw * (32 / seg);
    const size_t stage = 2 * (size_t)TR * row_bytes_dev(qt, d), xb1 = xbuf_bytes(ns, 1);
    WsPlan p;   // the deepest ring that leaves room for every token (none: the pipelined kernels)
    const size_t xs = (size_t)batch * xb1;
    if (xs < kWsSmem) p.nst = (int)std::min<size_t>(kWsMaxSt, (kWsSmem - xs) / stage);
    if (p.nst < 2) p.nst = 0;
    if (p.nst) p.smem = p.nst * stage + xs;
    p.nw = nw;
    return p;
}
static WsPlan ws_plan_down(int qt, int ffn, int batch, int nw) {
    const int ns = slices_per_row(ffn), seg = ws_seg(2 * ns, 32), TR = 2 * nw * (32 / seg);
    const size_t stage = (size_t)TR * row_bytes_dev(qt, ffn) + (size_t)batch * xbuf_bytes(ns, 1);
    WsPlan p;
    p.nst = (int)std::min<size_t>(kWsMaxSt, kWsSmem / stage);
    if (p.nst < 2) p.nst = 0;
    if (p.nst) p.smem = p.nst * stage;
    p.nw = nw;
    return p;
}
// the wide kernel when its ring fits, else the narrow one (nst = 0: neither)
static WsPlan ws_plan(WsPlan (*plan)(int, int, int, int), int qt, int n, int batch) {
    const WsPlan w = ws_wide_fits(qt) ? plan(qt, n, batch, kWsWide) : WsPlan{};
    return w.nst ? w : plan(qt, n, batch, kWsNarrow);
}

// combine: eout[token][n] = sum over the token's local slots, in slot order,
// of w * part[token][slot][n] (qwen_moe.c:310); zero if none is local.  With
// xbm set (d a multiple of 32: a warp holds one 32-element block of the row)
// each warp also writes its block prepared for the next GEMV: lanes 0-7
// gather four consecutive values each and form the block's sum of squares
// and its xprep_vals form of row * nw, the operations of the preparation
// kernel on the same values.
__global__ void __launch_bounds__(256) combine_kernel(int d, int n_act, int lo, int hi, const int *__restrict__ sel,
                                                      const float *__restrict__ w, const float *__restrict__ part,
                                                      float *__restrict__ eout, int accum, uint8_t *__restrict__ xbm,
                                                      float *__restrict__ qs, const float *__restrict__ nw, int ntok,
                                                      int nxb) {
    const int tok = blockIdx.y, n = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();                                  // part comes from the down kernel
    pdl_launch_dependents();
    if (n >= d) return;
    float tot = 0.f;
    for (int a = 0; a < n_act; ++a) {
        const int e = __ldcg(sel + tok * n_act + a);
        if (e >= lo && e < hi) tot += __ldcg(w + tok * n_act + a) * __ldcg(part + ((long)tok * n_act + a) * d + n);
    }
    float *o = eout + (long)tok * d + n;
    const float val = accum ? *o + tot : tot;
    *o = val;
    if (xbm) {
        const int lane = threadIdx.x & 31, t = lane & 7, j = n >> 5;
        float4 v;
        v.x = __shfl_sync(0xffffffffu, val, 4 * t);
        v.y = __shfl_sync(0xffffffffu, val, 4 * t + 1);
        v.z = __shfl_sync(0xffffffffu, val, 4 * t + 2);
        v.w = __shfl_sync(0xffffffffu, val, 4 * t + 3);
        float q = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        q += __shfl_xor_sync(0xffffffffu, q, 1);
        q += __shfl_xor_sync(0xffffffffu, q, 2);
        q += __shfl_xor_sync(0xffffffffu, q, 4);
        if (lane == 0) qs[(long)tok * nxb + j] = q;
        if (nw) {
            const float4 w4 = __ldg(reinterpret_cast<const float4 *>(nw + j * 32) + t);
            v = make_float4(v.x * w4.x, v.y * w4.y, v.z * w4.z, v.w * w4.w);
        }
        xprep_vals(v, reinterpret_cast<XB *>(xbm + (((long)(tok / ntok) * nxb + j) * ntok + tok % ntok) * 80), t,
                   lane < 8);
    }
}

// ---- many-token (prefill) path: pairs sorted by expert ------------------------------------
// router_many: logits[t][e] = router[e] . hn[t] (fp32, qwen_moe.c:296) for
// many tokens: one warp per (expert, group of 32 tokens) holds the expert's
// row in registers (d <= 2048: 16 float4 per lane; the rest streamed) and
// walks its tokens two at a time, all of a token's 16-byte loads issued
// before its arithmetic.  Grid (n_exp, ceil(T / 32)).  CTA (0, 0) also
// clears zero[0, nzero) (the counters of the kernels that follow).
constexpr int kRmTok = 32;
__global__ void __launch_bounds__(32) router_many_kernel(const float *__restrict__ router,
                                                         const float *__restrict__ hn, int d, int n_exp, int T,
                                                         float *__restrict__ logits, int *__restrict__ zero,
                                                         int nzero) {
    constexpr int RV = 16;
    const int lane = threadIdx.x, e = blockIdx.x, t0 = blockIdx.y * kRmTok;
    const int nv = min(d / 128, RV);
    const float4 *rw = reinterpret_cast<const float4 *>(router + (long)e * d);
    float4 r[RV];
#pragma unroll
    for (int i = 0; i < RV; ++i)
        if (i < nv) r[i] = __ldg(rw + lane + 32 * i);
    pdl_wait();
    pdl_launch_dependents();
    if (zero && blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = lane; i < nzero; i += 32) zero[i] = 0;
    const int tend = min(T, t0 + kRmTok);
    for (int t = t0; t < tend; t += 2) {
        const bool two = t + 1 < tend;
        const float4 *x0 = reinterpret_cast<const float4 *>(hn + (long)t * d);
        const float4 *x1 = reinterpret_cast<const float4 *>(hn + (long)(two ? t + 1 : t) * d);
        float4 v0[RV], v1[RV];
#pragma unroll
        for (int i = 0; i < RV; ++i)
            if (i < nv) {
                v0[i] = __ldcg(x0 + lane + 32 * i);
                v1[i] = __ldcg(x1 + lane + 32 * i);
            }
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < RV; ++i)
            if (i < nv) {
                s0 = fmaf(r[i].x, v0[i].x, s0);
                s0 = fmaf(r[i].y, v0[i].y, s0);
                s0 = fmaf(r[i].z, v0[i].z, s0);
                s0 = fmaf(r[i].w, v0[i].w, s0);
                s1 = fmaf(r[i].x, v1[i].x, s1);
                s1 = fmaf(r[i].y, v1[i].y, s1);
                s1 = fmaf(r[i].z, v1[i].z, s1);
                s1 = fmaf(r[i].w, v1[i].w, s1);
            }
        for (int i = lane + 32 * nv; i < d / 4; i += 32) {   // past the registers' share
            const float4 rr = __ldg(rw + i), a0 = __ldcg(x0 + i), a1 = __ldcg(x1 + i);
            s0 = fmaf(rr.x, a0.x, s0);
            s0 = fmaf(rr.y, a0.y, s0);
            s0 = fmaf(rr.z, a0.z, s0);
            s0 = fmaf(rr.w, a0.w, s0);
            s1 = fmaf(rr.x, a1.x, s1);
            s1 = fmaf(rr.y, a1.y, s1);
            s1 = fmaf(rr.z, a1.z, s1);
            s1 = fmaf(rr.w, a1.w, s1);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            s0 += __shfl_xor_sync(0xffffffffu, s0, off);
            s1 += __shfl_xor_sync(0xffffffffu, s1, off);
        }
        if (lane == 0) {
            logits[(long)t * n_exp + e] = s0;
            if (two) logits[(long)(t + 1) * n_exp + e] = s1;
        }
    }
}

// route_count: one CTA per token routes it (route_fast: softmax, greedy top-k,
// renormalise), writes sel / w, and counts its pairs per local expert.
__global__ void __launch_bounds__(128) route_count_kernel(int n_exp, int n_act, int lo, int hi,
                                                          const float *__restrict__ logits, int *__restrict__ sel,
                                                          float *__restrict__ wsel, int *__restrict__ cnt) {
    __shared__ __align__(16) float s_p[kMaxExp + 16];
    __shared__ int s_rk[4 * kMaxExp];
    __shared__ int s_sel[kMaxAct];
    __shared__ float s_w[kMaxAct], s_wr[kMaxAct];
    const int tok = blockIdx.x;
    pdl_wait();                                   // logits and the cleared counters come from the router kernel
    pdl_launch_dependents();
    route_fast(logits + (long)tok * n_exp, n_exp, n_act, s_p, s_rk, s_sel, s_w, s_wr);
    if (threadIdx.x < n_act) {
        const int a = threadIdx.x, e = s_sel[a];
        sel[tok * n_act + a] = e;
        wsel[tok * n_act + a] = s_w[a];
        if (e >= lo && e < hi) atomicAdd(&cnt[e - lo], 1);
    }
}

// scatter: one CTA per token places each of its local pairs at the next free
// position of its expert's run (runs in expert order: start = exclusive
// prefix of the counts) and copies the token's activation planes there.  The
// order of pairs inside a run does not change any result: every pair is its
// own GEMM column.
__global__ void __launch_bounds__(256) pair_scatter_kernel(int n_act, int lo, int hi, int kp,
                                                           const int *__restrict__ sel, int *__restrict__ cnt,
                                                           int *__restrict__ pair_at, const __half *__restrict__ xt_hi,
                                                           const __half *__restrict__ xt_lo, __half *__restrict__ xg_hi,
                                                           __half *__restrict__ xg_lo) {
    __shared__ int s_start[kMaxExp + 1];
    __shared__ int s_pos[kMaxAct];
    const int tok = blockIdx.x, nl = hi - lo;
    pdl_wait();                                   // counts complete: the routing kernel has finished
    pdl_launch_dependents();
    if (threadIdx.x < 32) {                       // exclusive prefix of the counts, one warp
        const int per = (nl + 31) / 32, lane = threadIdx.x;
        int sum = 0;
        for (int k = 0; k < per; ++k) {
            const int g = lane * per + k;
            if (g < nl) sum += __ldcg(cnt + g);
        }
        int inc = sum;
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += v;
        }
        int run = inc - sum;
        for (int k = 0; k < per; ++k) {
            const int g = lane * per + k;
            if (g < nl) {
                s_start[g] = run;
                run += __ldcg(cnt + g);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x < n_act) {
        const int a = threadIdx.x, e = __ldcg(sel + tok * n_act + a);
        int pos = -1;
        if (e >= lo && e < hi) {
            pos = s_start[e - lo] + atomicAdd(&cnt[nl + e - lo], 1);
            pair_at[pos] = tok * n_act + a;
        }
        s_pos[a] = pos;
    }
    __syncthreads();
    const int nv = kp / 8;                        // 16-byte vectors per plane row
    for (int a = 0; a < n_act; ++a) {
        const int pos = s_pos[a];
        if (pos < 0) continue;
        for (int v = threadIdx.x; v < nv; v += blockDim.x) {
            reinterpret_cast<uint4 *>(xg_hi + (long)pos * kp)[v] = __ldcg(reinterpret_cast<const uint4 *>(xt_hi + (long)tok * kp) + v);
            reinterpret_cast<uint4 *>(xg_lo + (long)pos * kp)[v] = __ldcg(reinterpret_cast<const uint4 *>(xt_lo + (long)tok * kp) + v);
        }
    }
}

// ---- fused expert kernel (one token) ----------------------------------------------------
// One CTA per SM.  After routing (route_fast on the router kernel's logits)
// every CTA stages, at once, all the weight rows it owns: gate/up items (kFR
// rows of one local expert's gate and up matrices) and down units (kFR output
// rows: those rows of every local expert's down matrix).  A gate/up item
// writes h = silu(g) * u for its rows and counts itself on a global counter;
// a CTA's down units start once the counter shows every item of the token
// done, and sum their experts in slot order, so the result does not depend on
// timing.  The grid is the SM count with one CTA per SM, so every CTA is
// resident while others wait for it; the waits are bounded.
constexpr int kFusedMaxItems = 12;
constexpr int kFR = 16;   // rows per item / unit

struct FusedArgs {
    const uint8_t *gw, *uw, *dw;
    int ffn, d, n_exp, n_act, lo, hi;
    int tile_region;   // bytes of shared memory for staged rows
    const float *hn, *logits;
    float *h;
    int *cnt;
    int *sel_out;         // routing result (CTA 0 writes it)
    float *w_out;
    float *eout;
    int accum;            // eout += (residual) instead of eout =
    int *status;
};

// Work split of the fused kernel, shared by the host planner and the kernel:
// down unit u goes to CTA u % G; the CTAs left with one unit fewer first take
// up to kfill gate/up items each, and the remaining items go round-robin over
// all CTAs.
struct FusedSplit {
    int dn_n, rA, fill, gu_a, gu_b;
    __host__ __device__ FusedSplit(int c, int G, int n_gu, int n_dn, int kfill) {
        dn_n = n_dn > c ? (n_dn - c + G - 1) / G : 0;
        rA = n_dn % G;
        fill = 0;
        if (rA > 0) fill = n_gu < (G - rA) * kfill ? n_gu : (G - rA) * kfill;
        gu_a = (rA > 0 && c >= rA && fill > c - rA) ? (fill - (c - rA) + (G - rA) - 1) / (G - rA) : 0;
        const int rest = n_gu - fill;
        gu_b = rest > c ? (rest - c + G - 1) / G : 0;
    }
    __host__ __device__ int gu_n() const { return gu_a + gu_b; }
    __host__ __device__ int gu_item(int c, int G, int k) const {
        return k < gu_a ? (c - rA) + k * (G - rA) : fill + c + (k - gu_a) * G;
    }
    __host__ __device__ int dn_unit(int c, int G, int k) const { return c + k * G; }
};
// gate/up items that balance one CTA's down unit (bytes, rounded)
__host__ __device__ inline int fused_kfill(int nl, int unit_tile_bytes, int item_bytes) {
    return (nl * unit_tile_bytes + item_bytes / 2) / item_bytes;
}

template <int QT>
__global__ void __launch_bounds__(kMoeThreads, 1) moe_fused_kernel(const FusedArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t bars[kFusedMaxItems];
    __shared__ int abort_flag;
    __shared__ __align__(16) float s_p[kMaxExp + 16];
    __shared__ int s_rk[4 * kMaxExp];
    __shared__ int s_sel[kMaxAct], s_loc[kMaxAct];
    __shared__ float s_w[kMaxAct], s_wr[kMaxAct];
    __shared__ int s_nl;
    const int G = gridDim.x, c = blockIdx.x;
    const int ffn = a.ffn, d = a.d;
    const int nsg = slices_per_row(d), nsd = slices_per_row(ffn);
    const long rbg = row_bytes_dev(QT, d), rbd = row_bytes_dev(QT, ffn);
    const int tbg = kFR * (int)rbg, tbd = kFR * (int)rbd;
    const int tpg = ffn / kFR;   // gate/up items per expert
    uint8_t *tiles = smem;
    uint8_t *xbase = smem + a.tile_region;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kFusedMaxItems; ++i) mbar_init(&bars[i], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    pdl_launch_dependents();
    pdl_wait();                                  // logits and the cleared counter come from the router kernel
    route_fast(a.logits, a.n_exp, a.n_act, s_p, s_rk, s_sel, s_w, s_wr);
    if (c == 0 && threadIdx.x < a.n_act) {       // routing result for the API
        a.sel_out[threadIdx.x] = s_sel[threadIdx.x];
        a.w_out[threadIdx.x] = s_w[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        int nl = 0;
        for (int s2 = 0; s2 < a.n_act; ++s2)
            if (s_sel[s2] >= a.lo && s_sel[s2] < a.hi) s_loc[nl++] = s2;
        s_nl = nl;
    }
    __syncthreads();
    const int nl = s_nl;
    const int n_gu = nl * tpg, n_dn = (d + kFR - 1) / kFR;
    const FusedSplit sp(c, G, n_gu, n_dn, fused_kfill(nl, tbd, 2 * tbg));
    const int gu_n = sp.gu_n();
    const int dn_n = nl > 0 ? sp.dn_n : 0;       // units with no local expert load nothing
    if (threadIdx.x < 16) {                      // lanes 0-15 issue the gate/up items
        for (int k = threadIdx.x; k < gu_n; k += 16) {
            const int i = sp.gu_item(c, G, k);
            const long r0 = (long)(s_sel[s_loc[i / tpg]] - a.lo) * ffn + (i % tpg) * kFR;
            uint8_t *t = tiles + k * 2 * tbg;
            mbar_arrive_expect_tx(&bars[k], 2u * (uint32_t)tbg);
            stage_bytes(t, a.gw + r0 * rbg, (uint32_t)tbg, &bars[k]);
            stage_bytes(t + tbg, a.uw + r0 * rbg, (uint32_t)tbg, &bars[k]);
        }
    } else if (threadIdx.x < 32) {               // lanes 16-31 the down units
        for (int k = threadIdx.x - 16; k < dn_n; k += 16) {
            const int u = sp.dn_unit(c, G, k);
            const int rows = min(kFR, d - u * kFR);
            uint8_t *t = tiles + gu_n * 2 * tbg + k * nl * tbd;
            mbar_arrive_expect_tx(&bars[gu_n + k], (uint32_t)(nl * rows * rbd));
            for (int li = 0; li < nl; ++li)
                stage_bytes(t + li * tbd, a.dw + ((long)(s_sel[s_loc[li]] - a.lo) * d + u * kFR) * rbd,
                            (uint32_t)(rows * rbd), &bars[gu_n + k]);
        }
    }
    // the hidden state is prepared while the copies are in flight
    {
        const float *hn = a.hn;
        xprep_rows([hn](int) { return hn; }, d, 1, xbuf_at(xbase, nsg));
        __syncthreads();
    }
    // gate / up items: h[li][rows] = silu(gate . hn) * (up . hn), all items of
    // this CTA in one pass (their copies were issued together)
    const XBuf xh = xbuf_at(xbase, nsg);
    float *red_g = reinterpret_cast<float *>(xbase + xbuf_bytes(nsg, 1));
    if (gu_n > 0) {
        bool ok = true;
        for (int k = 0; k < gu_n; ++k) ok = mbar_wait(&bars[k], 0, &abort_flag, a.status) && ok;
        constexpr int SB = slice_bytes(QT);
        const int S = red_stride(nsg), per = kFR * nsg * 2;   // halves per matrix of an item
        for (int p = threadIdx.x; p < gu_n * 2 * per; p += blockDim.x) {
            const int km = p / per, q = p - km * per;          // km = 2 * item + matrix
            const int sp = q >> 1, hf = q & 1;
            const int r = sp / nsg, sl = sp - r * nsg;
            float v = 0.f;
            if (ok) {
                WHalf<QT> w;
                load_half<QT>(tiles + km * tbg + (long)sp * SB, hf, w);
                v = dot_half<QT>(w, hf, xh.half(0, sl, hf));
            }
            red_g[(km * kFR + r) * S + 2 * sl + hf] = v;
        }
        __syncthreads();
        for (int t = threadIdx.x; t < gu_n * kFR; t += blockDim.x) {
            const int k = t / kFR, r = t - k * kFR;
            const float hv = swiglu(row_sum(red_g + ((2 * k) * kFR + r) * S, nsg),
                                    row_sum(red_g + ((2 * k + 1) * kFR + r) * S, nsg));
            const int i = sp.gu_item(c, G, k);
            a.h[(i / tpg) * ffn + (i % tpg) * kFR + r] = hv;
            __threadfence();
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(a.cnt, gu_n);
        }
    }
    // down units: eout[rows] = sum over local slots (slot order) of w * (down . h)
    if (sp.dn_n > 0) {
        const XBuf xd = xbuf_at(xbase, nsd);
        float *red_d = reinterpret_cast<float *>(xbase + xbuf_bytes(nsd, a.n_act));
        if (nl > 0) {
            if (threadIdx.x == 0) spin_until_geq(a.cnt, n_gu, &abort_flag, a.status);
            __syncthreads();
            const float *hs = a.h;
            xprep_rows([hs, ffn](int li) { return hs + (long)li * ffn; }, ffn, nl, xd);
            __syncthreads();
        }
        for (int k = 0; k < sp.dn_n; ++k) {
            const int u = sp.dn_unit(c, G, k);
            const int rows = min(kFR, d - u * kFR);
            const bool ok = nl > 0 && mbar_wait(&bars[gu_n + k], 0, &abort_flag, a.status);
            const float v = down_rows<QT>(tiles + gu_n * 2 * tbg + k * nl * tbd, nl, rows, kFR, nsd, rbd, xd, red_d,
                                          a.n_act, ok, s_loc, s_w);
            if (threadIdx.x < rows) {
                float *o = a.eout + u * kFR + threadIdx.x;
                *o = a.accum ? *o + v : v;
            }
            __syncthreads();
        }
    }
    if (threadIdx.x == 0 && abort_flag)          // copies still in flight after a timeout
        for (int k = 0; k < gu_n + dn_n; ++k) mbar_wait_drain(&bars[k], 0, 100000000ull);
}

}  // namespace q

using namespace q;

// Rows per item of the pipelined batched kernels: about one half-slice per
// thread (gate and up together for gate/up), with kStages stages, the
// reduction buffer and (down) the prepared activations within kPipeSmem
// bytes of dynamic shared memory.
constexpr size_t kPipeSmem = 200 * 1024;
static size_t gate_up_smem(int qt, int d, int TR, int nb) {
    const int ns = slices_per_row(d);
    return (size_t)kStages * 2 * TR * row_bytes_dev(qt, d) + (size_t)kXsTok * xbuf_bytes(ns, 1) +
           (size_t)nb * 2 * TR * red_stride(ns) * 4;
}
static size_t down_smem(int qt, int ffn, int TR, int nb) {
    const int ns = slices_per_row(ffn);
    return (size_t)kStages * TR * row_bytes_dev(qt, ffn) + xbuf_bytes(ns, nb) + (size_t)nb * TR * red_stride(ns) * 4;
}
static int gate_up_rows_per_cta(int qt, int d) {
    int tr = std::max(1, kMoeThreads / (4 * slices_per_row(d)));
    while (tr > 1 && gate_up_smem(qt, d, tr, kMaxBatch) > kPipeSmem) --tr;
    return tr;
}
static int down_rows_per_cta(int qt, int ffn) {
    int tr = std::max(1, kMoeThreads / (2 * slices_per_row(ffn)));
    while (tr > 1 && down_smem(qt, ffn, tr, kMaxBatch) > kPipeSmem) --tr;
    return tr;
}

bool moe_shapes_ok(int d, int n_exp, int n_act, int ffn, int qtype) {
    const int be = (int)qtype_block_elems(qtype);
    if (!be || d <= 0 || ffn <= 0 || d % be || ffn % be || d % 32 || ffn % 32 || d / 32 > kMaxDXB || n_exp <= 0 ||
        n_exp > kMaxExp || n_act <= 0 || n_act > kMaxAct || n_act > n_exp)
        return false;
    return gate_up_smem(qtype, d, gate_up_rows_per_cta(qtype, d), kMaxBatch) <= kPipeSmem &&
           down_smem(qtype, ffn, down_rows_per_cta(qtype, ffn), kMaxBatch) <= kPipeSmem;
}

static void fused_plan_impl(MoeLayer &L, int G) {
    L.fused_ok = false;
    if (G <= 0) return;
    const int qt = L.qtype;
    const int tbg = kFR * (int)row_bytes_dev(qt, L.d), tbd = kFR * (int)row_bytes_dev(qt, L.ffn);
    const int n_dn = (L.d + kFR - 1) / kFR;
    long maxb = 0;
    int maxi = 0, gu_max = 0;
    for (int nl = 0; nl <= L.n_act; ++nl) {
        const int n_gu = nl * (L.ffn / kFR);
        const int kf = fused_kfill(nl, tbd, 2 * tbg);
        for (int c = 0; c < G; ++c) {
            const FusedSplit sp(c, G, n_gu, n_dn, kf);
            const int dn = nl > 0 ? sp.dn_n : 0;
            maxb = std::max(maxb, (long)sp.gu_n() * 2 * tbg + (long)dn * nl * tbd);
            maxi = std::max(maxi, sp.gu_n() + dn);
            gu_max = std::max(gu_max, sp.gu_n());
        }
    }
    const int nsg = slices_per_row(L.d), nsd = slices_per_row(L.ffn);
    const size_t xg = (size_t)xbuf_bytes(nsg, 1) + (size_t)std::max(gu_max, 1) * gu_red_floats(kFR, nsg) * 4;
    const size_t xd = (size_t)xbuf_bytes(nsd, L.n_act) + (size_t)dn_red_floats(kFR, nsd, L.n_act) * 4;
    L.fused_grid = G;
    L.fused_tiles = (int)((maxb + 127) / 128 * 128);
    L.fused_smem = (size_t)L.fused_tiles + std::max(xg, xd);
    L.fused_ok = maxi <= kFusedMaxItems && L.fused_smem <= 220 * 1024 && L.ffn % kFR == 0;
}

template <int QT>
static int launch_moe_qt(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *x, float *eout, int batch,
                         const MoeOpts &o, cudaStream_t s) {
    // with a norm the router kernel writes the normed tokens for the experts
    const float *hn = o.norm_w ? o.hn_out : x;
    const int accum = o.accum ? 1 : 0;
    static const bool no_fused = getenv("X100_MOE_NO_FUSED") != nullptr;
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(router_logits_kernel);
        set_qkernel_attrs(router_topk_kernel);
        set_qkernel_attrs(route_group_kernel);
        set_qkernel_attrs(gate_up_pipe_kernel<QT>, (int)kPipeSmem);
        set_qkernel_attrs(down_pipe_kernel<QT>, (int)kPipeSmem);
        if constexpr (ws_wide_fits(QT)) {
            set_qkernel_attrs(gate_up_ws_kernel<QT, kWsWide>, (int)kWsSmem);
            set_qkernel_attrs(down_ws_kernel<QT, kWsWide>, (int)kWsSmem);
        }
        set_qkernel_attrs(gate_up_ws_kernel<QT, kWsNarrow>, (int)kWsSmem);
        set_qkernel_attrs(down_ws_kernel<QT, kWsNarrow>, (int)kWsSmem);
        set_qkernel_attrs(prep_slots_kernel);
        set_qkernel_attrs(combine_kernel);
        set_qkernel_attrs(moe_fused_kernel<QT>, 220 * 1024);
        attr[c->device] = true;
    }
    if (batch == 1 && L.fused_ok && !no_fused) {
        if (o.mark) o.mark(o.mark_ctx, X100Q_T_ROUTER, s);
        int st = launch_pdl(router_logits_kernel, dim3((L.n_exp + 1) / 2, 1), dim3(64), 0, s,
                            (const float *)L.router, x, L.d, L.n_exp, 1, S.logits, S.cnt, 1, o.norm_w, o.eps,
                            o.hn_out);
        if (st) return st;
        FusedArgs fa;
        fa.gw = L.gate.w;
        fa.uw = L.up.w;
        fa.dw = L.down.w;
        fa.ffn = L.ffn;
        fa.d = L.d;
        fa.n_exp = L.n_exp;
        fa.n_act = L.n_act;
        fa.lo = L.lo;
        fa.hi = L.hi;
        fa.tile_region = L.fused_tiles;
        fa.hn = hn;
        fa.logits = S.logits;
        fa.h = S.h;
        fa.cnt = S.cnt;
        fa.sel_out = S.sel;
        fa.w_out = S.w;
        fa.eout = eout;
        fa.accum = accum;
        fa.status = c->d_status;
        if (o.mark) o.mark(o.mark_ctx, X100Q_T_EXPERT, s);   // routing, experts and combine in one kernel
        return launch_pdl(moe_fused_kernel<QT>, dim3(L.fused_grid), dim3(kMoeThreads), L.fused_smem, s, fa);
    }
    // batch > 1: tokens grouped by expert
    if (o.mark) o.mark(o.mark_ctx, X100Q_T_ROUTER, s);
    int st = launch_pdl(router_logits_kernel, dim3((L.n_exp + 1) / 2, batch), dim3(64), 0, s,
                        (const float *)L.router, x, L.d, L.n_exp, batch, S.logits, S.grp, L.n_exp + 1, o.norm_w,
                        o.eps, o.hn_out);
    if (st) return st;
    st = launch_pdl(route_group_kernel, dim3(batch), dim3(kMoeThreads), 0, s, L.d, L.n_exp, L.n_act, L.lo, L.hi, hn,
                    (const float *)S.logits, S.sel, S.w, S.grp, S.xq, S.cnt + 1);
    if (st) return st;
    if (o.mark) o.mark(o.mark_ctx, X100Q_T_EXPERT, s);
    const int G = c->sm_count;   // persistent: one CTA per SM
    static const bool no_ws = getenv("X100_MOE_NO_WS") != nullptr;
    const WsPlan pg = ws_plan(ws_plan_gate_up, QT, L.d, batch), pd = ws_plan(ws_plan_down, QT, L.ffn, batch);
    if (pg.nst && pd.nst && !no_ws) {
        auto gate_up = [&](auto nwc) {
            constexpr int NW = decltype(nwc)::value;
            return launch_pdl(gate_up_ws_kernel<QT, NW>, dim3(G), dim3(32 * (NW + 1)), pg.smem, s,
                              (const uint8_t *)L.gate.w, (const uint8_t *)L.up.w, L.ffn, L.d, L.n_exp, L.n_act, batch,
                              pg.nst, (const int *)S.grp, (const uint8_t *)S.xq, S.h, S.cnt + 1, c->d_status);
        };
        auto down = [&](auto nwc) {
            constexpr int NW = decltype(nwc)::value;
            return launch_pdl(down_ws_kernel<QT, NW>, dim3(G), dim3(32 * (NW + 1)), pd.smem, s,
                              (const uint8_t *)L.down.w, L.ffn, L.d, L.n_exp, batch, pd.nst, (const int *)S.grp,
                              (const uint8_t *)S.hq, S.part, S.cnt + 2, c->d_status);
        };
        if constexpr (ws_wide_fits(QT))
            st = pg.nw == kWsWide ? gate_up(IntC<kWsWide>{}) : gate_up(IntC<kWsNarrow>{});
        else
            st = gate_up(IntC<kWsNarrow>{});
        if (st) return st;
        st = launch_pdl(prep_slots_kernel, dim3(batch * L.n_act), dim3(256), 0, s, (const float *)S.h, L.ffn, S.hq);
        if (st) return st;
        if constexpr (ws_wide_fits(QT))
            st = pd.nw == kWsWide ? down(IntC<kWsWide>{}) : down(IntC<kWsNarrow>{});
        else
            st = down(IntC<kWsNarrow>{});
        if (st) return st;
    } else {
        const int TRg = gate_up_rows_per_cta(QT, L.d), TRd = down_rows_per_cta(QT, L.ffn);
        st = launch_pdl(gate_up_pipe_kernel<QT>, dim3(G), dim3(kMoeThreads), gate_up_smem(QT, L.d, TRg, batch), s,
                        (const uint8_t *)L.gate.w, (const uint8_t *)L.up.w, L.ffn, L.d, L.n_exp, L.n_act, TRg,
                        (const int *)S.grp, (const uint8_t *)S.xq, S.h, S.cnt + 1, c->d_status);
        if (st) return st;
        st = launch_pdl(down_pipe_kernel<QT>, dim3(G), dim3(kMoeThreads), down_smem(QT, L.ffn, TRd, batch), s,
                        (const uint8_t *)L.down.w, L.ffn, L.d, L.n_exp, TRd, batch, (const int *)S.grp,
                        (const float *)S.h, S.part, S.cnt + 2, c->d_status);
        if (st) return st;
    }
    if (o.mark) o.mark(o.mark_ctx, X100Q_T_COMBINE, s);
    return launch_pdl(combine_kernel, dim3((L.d + 255) / 256, batch), dim3(256), 0, s, L.d, L.n_act, L.lo, L.hi,
                      (const int *)S.sel, (const float *)S.w, (const float *)S.part, eout, accum,
                      L.d % 32 == 0 ? o.next_xbm : nullptr, o.next_qs, o.next_nw, o.next_ntok, o.next_nxb);
}

int launch_moe(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *hn, float *eout, int batch,
               cudaStream_t s) {
    return launch_moe_ex(c, L, S, hn, eout, batch, MoeOpts(), s);
}

int launch_moe_ex(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *x, float *eout, int batch,
                  const MoeOpts &o, cudaStream_t s) {
    if (batch < 1 || batch > kMaxBatch || (o.norm_w && !o.hn_out)) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    switch (L.qtype) {
    case Q4_0: return launch_moe_qt<Q4_0>(c, L, S, x, eout, batch, o, s);
    case Q8_0: return launch_moe_qt<Q8_0>(c, L, S, x, eout, batch, o, s);
    case Q4_K: return launch_moe_qt<Q4_K>(c, L, S, x, eout, batch, o, s);
    case Q3_K: return launch_moe_qt<Q3_K>(c, L, S, x, eout, batch, o, s);
    default: set_error(X100_E_UNSUPPORTED); return X100_E_UNSUPPORTED;
    }
}

void moe_fused_plan(MoeLayer &L, int sm_count) { fused_plan_impl(L, sm_count); }

size_t moe_big_scratch_bytes(int d, int n_exp, int n_act, int ffn, int tmax) {
    const size_t kpd = (size_t)slices_per_row(d) * 256, kpf = (size_t)slices_per_row(ffn) * 256;
    const size_t P = (size_t)tmax * n_act;
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    return up((size_t)tmax * d * 4) + 2 * up((size_t)tmax * kpd * 2) + up((size_t)tmax * n_exp * 4) +
           2 * up(P * 4) + up((size_t)2 * n_exp * 4) + up(P * 4) + 2 * up(P * kpd * 2) + up(P * 2 * ffn * 4) +
           2 * up(P * kpf * 2) + up(P * d * 4) + 256;
}

MoeBigScratch moe_big_scratch_carve(void *base, int d, int n_exp, int n_act, int ffn, int tmax) {
    const size_t kpd = (size_t)slices_per_row(d) * 256, kpf = (size_t)slices_per_row(ffn) * 256;
    const size_t P = (size_t)tmax * n_act;
    uintptr_t p = (reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255);
    auto take = [&](size_t bytes) {
        void *r = reinterpret_cast<void *>(p);
        p = (p + bytes + 255) & ~uintptr_t(255);
        return r;
    };
    MoeBigScratch S;
    S.tmax = tmax;
    S.hn = static_cast<float *>(take((size_t)tmax * d * 4));
    S.xt_hi = static_cast<__half *>(take((size_t)tmax * kpd * 2));
    S.xt_lo = static_cast<__half *>(take((size_t)tmax * kpd * 2));
    S.logits = static_cast<float *>(take((size_t)tmax * n_exp * 4));
    S.sel = static_cast<int *>(take(P * 4));
    S.w = static_cast<float *>(take(P * 4));
    S.cnt = static_cast<int *>(take((size_t)2 * n_exp * 4));
    S.pair_at = static_cast<int *>(take(P * 4));
    S.xg_hi = static_cast<__half *>(take(P * kpd * 2));
    S.xg_lo = static_cast<__half *>(take(P * kpd * 2));
    S.gu = static_cast<float *>(take(P * 2 * ffn * 4));
    S.hh_hi = static_cast<__half *>(take(P * kpf * 2));
    S.hh_lo = static_cast<__half *>(take(P * kpf * 2));
    S.part = static_cast<float *>(take(P * d * 4));
    return S;
}

int launch_moe_prefill(DevCtx *c, const MoeLayer &L, const MoeBigScratch &S, float *h, int T, const float *norm_w,
                       float eps, cudaStream_t s) {
    const int nl = L.hi - L.lo;
    if (T < 1 || T > S.tmax || nl > kMaxExp || !norm_w) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    const int kpd = slices_per_row(L.d) * 256, kpf = slices_per_row(L.ffn) * 256;
    const int P = T * L.n_act;
    // 1. hn = rmsnorm(h, norm_w) (qwen_moe_q3k.c:1166), fp32 for the router
    //    and as fp16 hi / lo planes for the experts
    int st = launch_split_rows(h, L.d, L.d, kpd, T, norm_w, eps, S.xt_hi, S.xt_lo, S.hn, s);
    if (st) return st;
    // 2. router logits (qwen_moe.c:296); the counters cleared
    st = launch_pdl(router_many_kernel, dim3(L.n_exp, (T + kRmTok - 1) / kRmTok), dim3(32), 0, s,
                    (const float *)L.router, (const float *)S.hn, L.d, L.n_exp, T, S.logits, S.cnt, 2 * nl);
    if (st) return st;
    // 3. softmax, top-k, renormalise (qwen_moe.c:297-301); pairs per expert
    st = launch_pdl(route_count_kernel, dim3(T), dim3(128), 0, s, L.n_exp, L.n_act, L.lo, L.hi,
                    (const float *)S.logits, S.sel, S.w, S.cnt);
    if (st) return st;
    // 4. pairs sorted by expert, each with its token's planes
    st = launch_pdl(pair_scatter_kernel, dim3(T), dim3(256), 0, s, L.n_act, L.lo, L.hi, kpd, (const int *)S.sel,
                    S.cnt, S.pair_at, (const __half *)S.xt_hi, (const __half *)S.xt_lo, S.xg_hi, S.xg_lo);
    if (st) return st;
    // 5. gate and up of every pair's expert: gu[pos] = [gate . hn, up . hn]
    QgLaunch g;
    g.mats[0] = &L.gate;
    g.mats[1] = &L.up;
    g.nmat = 2;
    g.n_rows = L.ffn;
    g.ngroups = nl;
    g.cnt = S.cnt;
    g.xh = S.xg_hi;
    g.xl = S.xg_lo;
    g.x_rows = P;
    g.mode = QG_STORE;
    g.out = S.gu;
    g.ldo = 2L * L.ffn;
    st = launch_qgemm(c, g, s);
    if (st) return st;
    // 6. h = silu(g) * u (qwen_moe.c:309)
    st = launch_swiglu_split(S.gu, L.ffn, kpf, P, S.hh_hi, S.hh_lo, s);
    if (st) return st;
    // 7. down of every pair's expert, to the pair's row
    QgLaunch dn;
    dn.mats[0] = &L.down;
    dn.nmat = 1;
    dn.n_rows = L.d;
    dn.ngroups = nl;
    dn.cnt = S.cnt;
    dn.xh = S.hh_hi;
    dn.xl = S.hh_lo;
    dn.x_rows = P;
    dn.mode = QG_SCATTER;
    dn.out = S.part;
    dn.ldo = L.d;
    dn.pair_at = S.pair_at;
    st = launch_qgemm(c, dn, s);
    if (st) return st;
    // 8. h += sum over the token's local slots, in slot order, of w * part (qwen_moe.c:310)
    return launch_pdl(combine_kernel, dim3((L.d + 255) / 256, T), dim3(256), 0, s, L.d, L.n_act, L.lo, L.hi,
                      (const int *)S.sel, (const float *)S.w, (const float *)S.part, h, 1, (uint8_t *)nullptr,
                      (float *)nullptr, (const float *)nullptr, 0, 0);
}

bool moe_layer_upload(DevCtx *c, MoeLayer &L, int d, int n_exp, int n_act, int ffn, int qtype, const float *router,
                      const void *gate_exps, const void *up_exps, const void *down_exps, int lo, int hi) {
    L = MoeLayer();
    L.d = d;
    L.n_exp = n_exp;
    L.n_act = n_act;
    L.ffn = ffn;
    L.qtype = qtype;
    L.lo = lo;
    L.hi = hi;
    const int ne = hi - lo;
    const size_t rb_d = x100q_row_bytes(qtype, d), rb_f = x100q_row_bytes(qtype, ffn);
    const uint8_t *g = static_cast<const uint8_t *>(gate_exps) + (size_t)lo * ffn * rb_d;
    const uint8_t *u = static_cast<const uint8_t *>(up_exps) + (size_t)lo * ffn * rb_d;
    const uint8_t *dn = static_cast<const uint8_t *>(down_exps) + (size_t)lo * d * rb_f;
    bool ok = cudaMalloc(&L.router, (size_t)n_exp * d * 4) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        L.router = nullptr;
    }
    ok = ok && check_cuda(cudaMemcpy(L.router, router, (size_t)n_exp * d * 4, cudaMemcpyDefault), X100_E_COPY) == 0;
    ok = ok && qmat_upload(c, qtype, ne * ffn, d, g, L.gate, c->stream);
    ok = ok && qmat_upload(c, qtype, ne * ffn, d, u, L.up, c->stream);
    ok = ok && qmat_upload(c, qtype, ne * d, ffn, dn, L.down, c->stream);
    if (!ok) {
        moe_layer_free(L);
        return false;
    }
    moe_fused_plan(L, c->sm_count);
    return true;
}

void moe_layer_free(MoeLayer &L) {
    cudaFree(L.router);
    cudaFree(L.gate.w);
    cudaFree(L.up.w);
    cudaFree(L.down.w);
    L = MoeLayer();
}

size_t moe_scratch_bytes(int d, int n_exp, int n_act, int ffn) {
    size_t b = 0;
    b += (size_t)kMaxBatch * n_exp * 4;                               // logits
    b += (size_t)kMaxBatch * n_act * 4 * 2;                           // sel, w
    b += (size_t)kMaxBatch * n_act * ffn * 4;                         // h
    b += (size_t)(2 * n_exp + 1 + n_exp * kMaxBatch) * 4;             // groups
    b += (size_t)kMaxBatch * xbuf_bytes(slices_per_row(d), 1);        // prepared activations
    b += (size_t)kMaxBatch * n_act * d * 4;                           // partial outputs
    b += (size_t)kMaxBatch * n_act * xbuf_bytes(slices_per_row(ffn), 1);   // prepared h per slot
    b += 256 * 11;                                                    // alignment, ticket, counter
    return b;
}

// Carve the scratch regions out of one buffer of moe_scratch_bytes().
MoeScratch moe_scratch_carve(void *base, int d, int n_exp, int n_act, int ffn) {
    MoeScratch S;
    uintptr_t p = (reinterpret_cast<uintptr_t>(base) + 255) & ~uintptr_t(255);
    auto take = [&](size_t bytes) {
        void *r = reinterpret_cast<void *>(p);
        p = (p + bytes + 255) & ~uintptr_t(255);
        return r;
    };
    S.ticket = static_cast<unsigned *>(take(256));
    S.cnt = static_cast<int *>(take(256));
    S.logits = static_cast<float *>(take((size_t)kMaxBatch * n_exp * 4));
    S.sel = static_cast<int *>(take((size_t)kMaxBatch * n_act * 4));
    S.w = static_cast<float *>(take((size_t)kMaxBatch * n_act * 4));
    S.h = static_cast<float *>(take((size_t)kMaxBatch * n_act * ffn * 4));
    S.grp = static_cast<int *>(take((size_t)(2 * n_exp + 1 + n_exp * kMaxBatch) * 4));
    S.xq = static_cast<uint8_t *>(take((size_t)kMaxBatch * xbuf_bytes(slices_per_row(d), 1)));
    S.part = static_cast<float *>(take((size_t)kMaxBatch * n_act * d * 4));
    S.hq = static_cast<uint8_t *>(take((size_t)kMaxBatch * n_act * xbuf_bytes(slices_per_row(ffn), 1)));
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
    if (!moe_layer_upload(c, m->L, d, n_exp, n_act, ffn, qtype, router, gate_exps, up_exps, down_exps, expert_lo,
                          expert_hi)) {
        delete m;
        return nullptr;
    }
    const size_t sb = moe_scratch_bytes(d, n_exp, n_act, ffn);
    if (fault_injected("alloc") || cudaMalloc(&m->scratch, sb) != cudaSuccess) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        moe_layer_free(m->L);
        delete m;
        return nullptr;
    }
    cudaMemset(m->scratch, 0, sb);
    m->S = moe_scratch_carve(m->scratch, d, n_exp, n_act, ffn);
    return m;
}

void x100q_moe_destroy(x100q_moe *m) {
    if (!m) return;
    DeviceGuard dg(m->device);
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
void *g_noalloc_addr[64];                  // device address of g_router_scratch, per device
unsigned long long g_noalloc_ctx[64];      // unique id of the context that address belongs to

// Unique id of the calling thread's current CUDA context (cuCtxGetId: ids are
// never reused within a process), or 0 when there is none or the driver does
// not offer the call.  A device reset destroys the primary context and the
// module's static array moves with the new one, so the cached address is
// trusted only while this id is unchanged.
unsigned long long current_ctx_id() {
    typedef CUresult (*PFN_getCurrent)(CUcontext *);
    typedef CUresult (*PFN_getId)(CUcontext, unsigned long long *);
    static PFN_getCurrent get_current = nullptr;
    static PFN_getId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr, *q = nullptr;
        cudaDriverEntryPointQueryResult r1, r2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r1) == cudaSuccess &&
            cudaGetDriverEntryPoint("cuCtxGetId", &q, cudaEnableDefault, &r2) == cudaSuccess &&
            r1 == cudaDriverEntryPointSuccess && r2 == cudaDriverEntryPointSuccess) {
            get_current = reinterpret_cast<PFN_getCurrent>(p);
            get_id = reinterpret_cast<PFN_getId>(q);
        } else {
            cudaGetLastError();
        }
    });
    CUcontext cx = nullptr;
    unsigned long long id = 0;
    if (!get_current || get_current(&cx) != CUDA_SUCCESS || !cx || get_id(cx, &id) != CUDA_SUCCESS) return 0;
    return id;
}
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
        // once per device, with that device current; again only if the device
        // was reset since (a new context: the array lives at a new address)
        const unsigned long long id = current_ctx_id();
        if (!g_noalloc_addr[dev] || id != g_noalloc_ctx[dev]) {
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
            if (e != cudaSuccess || !p) return check_cuda(e != cudaSuccess ? e : cudaErrorUnknown, X100_E_LAUNCH);
            g_noalloc_addr[dev] = p;
            g_noalloc_ctx[dev] = current_ctx_id();   // the lookup made the context current if it was not
        }
        base = g_noalloc_addr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned *ticket = static_cast<unsigned *>(base);
    float *logits = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + 256);
    // the ticket must start at zero; the logits are fully written before use
    if (check_cuda(cudaMemsetAsync(ticket, 0, sizeof(unsigned), s), X100_E_LAUNCH)) return get_error();
    q::router_topk_kernel<<<(n_exp + 7) / 8, 256, 0, s>>>(router, hn, d, n_exp, n_act, batch, logits, sel_out,
                                                          w_out, ticket, (int *)nullptr, 0);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

