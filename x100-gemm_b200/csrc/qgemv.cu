// qgemv.cu -- block-quantised dequant-GEMV (Q4_0 / Q8_0 / Q4_K / Q3_K) and the
// x100q_lin_* entry points of include/x100q.h.
//
// Replaces the reference's per-linear decode path: lin_new_* (weight
// requant/repack, qwen_moe_q3k.c:843-909) + pack_act_* + lin_mm_*
// (qwen_moe_q3k.c:1029-1082, qwen_moe.c:90-107), whose hot loop streams each
// weight row once per token through the IME micro-kernels.
//
// Kernel: a CTA owns TR consecutive rows, a contiguous byte range in the
// slice layout of qformats.cuh that one thread stages into shared memory with
// bulk copies before waiting on the previous kernel (programmatic dependent
// launch), so the weight stream of call i+1 overlaps the tail of call i.  The
// CTA then prepares the activations (one memory round trip), and each thread
// dots half a slice -- half p of the tile is half p % 2 of slice p / 2, which
// is row (p/2) / ns, slice (p/2) % ns -- against every batch column (exact
// dp4a int32 sums, one fp32 scale per block), so each weight byte is read
// from HBM once per call whatever the batch.  Row sums add the first halves
// in slice order, then the second halves.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "../../include/x100q.h"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace q {

static bool pdl_enabled_impl() {
    static const bool on = [] {
        const char *e = getenv("X100_NO_PDL");
        return !(e && *e && *e != '0');
    }();
    return on;
}

constexpr int kGemvThreads = 512;

// With `nw` set the kernel computes y = W . rmsnorm(x; nw, eps) (RMS norm of
// each token folded into the activation preparation, see xprep_rows); with
// `accum` set it adds into y (y += W . x: a residual connection).  With
// `indep` the caller guarantees that no kernel still running touches x or y:
// the CTA prepares x without waiting on the previous kernel and waits only
// before it exits (so grids still complete in stream order), which lets a run
// of independent calls stream weights back to back.
template <int QT, int B>
__global__ void __launch_bounds__(kGemvThreads, 1)
    qgemv_kernel(const uint8_t *__restrict__ W, int N, int K, int TR, const float *__restrict__ x,
                 float *__restrict__ y, int batch, const float *__restrict__ nw, float eps, int accum,
                 int indep, int a8, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    __shared__ float ss[(kGemvThreads / 32) * 4 * kSsTok];
    __shared__ float scale[B];
    constexpr int SB = slice_bytes(QT);
    const int ns = slices_per_row(K);
    const int rb = ns * SB;
    const int row0 = blockIdx.x * TR;
    const int rows = min(TR, N - row0);
    uint8_t *tile = smem;
    const XBuf xb = xbuf_at(smem + TR * rb, ns);
    float *red = reinterpret_cast<float *>(smem + TR * rb + xbuf_bytes(ns, B));   // [b][row][slice][half], row stride 2ns+1
    const int S = 2 * ns + 1;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, (uint32_t)(rows * rb));
        stage_bytes(tile, W + (long)row0 * rb, (uint32_t)(rows * rb), &bar);
    }
    pdl_launch_dependents();
    if (!indep) pdl_wait();                       // x may come from the previous kernel
    xprep_gemv(a8, [x, K](int c) { return x + (long)c * K; }, K, batch, xb, nw, ss);
    __syncthreads();
    if (threadIdx.x < batch) scale[threadIdx.x] = nw ? rms_scale(ss, blockDim.x / 8, threadIdx.x, K, eps) : 1.0f;
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status);
    if constexpr (B == 1) {
        const int nh = rows * ns * 2;
        for (int p = threadIdx.x; p < nh; p += blockDim.x) {
            const int sp = p >> 1, h = p & 1;
            const int r = sp / ns, sl = sp - r * ns;
            WHalf<QT> w;
            load_half<QT>(tile + (long)sp * SB, h, w);
            red[r * S + 2 * sl + h] = ok ? dot_half<QT>(w, h, xb.half(0, sl, h)) : 0.f;
        }
    } else {
        // two rows per thread: each token's activation half is read from
        // shared memory once for both rows (the loads are shared by the two
        // dot products), halving the activation traffic that bounds batches
        const int hp = ns * 2, rp = (rows + 1) >> 1;
        for (int p = threadIdx.x; p < rp * hp; p += blockDim.x) {
            const int rr = p / hp, qh = p - rr * hp;
            const int sl = qh >> 1, h = qh & 1;
            const int r0 = 2 * rr, r1 = r0 + 1;
            const bool two = r1 < rows;
            WHalf<QT> w0, w1;
            load_half<QT>(tile + ((long)r0 * ns + sl) * SB, h, w0);
            load_half<QT>(tile + ((long)(two ? r1 : r0) * ns + sl) * SB, h, w1);
#pragma unroll
            for (int b = 0; b < B; ++b) {
                if (b < batch) {
                    const XB *xh = xb.half(b, sl, h);
                    const float d0 = dot_half<QT>(w0, h, xh);
                    const float d1 = dot_half<QT>(w1, h, xh);
                    red[(b * TR + r0) * S + 2 * sl + h] = ok ? d0 : 0.f;
                    if (two) red[(b * TR + r1) * S + 2 * sl + h] = ok ? d1 : 0.f;
                }
            }
        }
    }
    __syncthreads();
    if (abort_flag) {
        if (threadIdx.x == 0) {
            mbar_wait_drain(&bar, 0, 100000000ull);   // the copy may still be in flight
            if (indep) pdl_wait();
        }
        return;
    }
    for (int t = threadIdx.x; t < rows * batch; t += blockDim.x) {
        const int b = t / rows, r = t - b * rows;
        const float *pr = red + (b * TR + r) * S;
        float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
        for (int sl = 0; sl < ns; ++sl) {
            s0 += pr[2 * sl];
            s1 += pr[2 * sl + 1];
        }
        float *o = y + (long)b * N + row0 + r;
        const float v = (s0 + s1) * scale[b];
        *o = accum ? *o + v : v;
    }
    if (indep && threadIdx.x == 0) pdl_wait();   // complete only after the previous grid
}

// ---- device re-layout of GGUF-native blocks ------------------------------------
// One thread per output slice (row r, slice s) of an N x K matrix.
__global__ void repack_kernel(int qt, int N, int K, const uint8_t *__restrict__ src, uint8_t *__restrict__ w) {
    const int ns = slices_per_row(K), SB = slice_bytes(qt);
    const long total = (long)N * ns;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long r = i / ns;
        const int s = (int)(i - r * ns);
        uint8_t *o = w + i * SB;
        if (qt == Q4_0 || qt == Q8_0) {
            // block_q4_0 {fp16 d; qs[16]} / block_q8_0 {fp16 d; qs[32]} (qwen_moe.c:162-165)
            const int qb = qt == Q4_0 ? 16 : 32, bb = qb + 2, nb = K / 32;
            for (int j = 0; j < 8; ++j) {
                const int blk = 8 * s + j;
                const uint8_t *b = src + ((long)r * nb + blk) * bb;
                const bool in = blk < nb;
                o[2 * j] = in ? b[0] : 0;
                o[2 * j + 1] = in ? b[1] : 0;
                for (int k = 0; k < qb; ++k) o[16 + qb * j + k] = in ? b[2 + k] : 0;
            }
        } else if (qt == Q4_K) {
            const uint8_t *b = src + i * 144;   // block_q4_K: d, dmin, scales[12], qs[128]
            for (int k = 0; k < 144; ++k) o[k] = b[k];
        } else if (qt == Q3_K) {
            // block_q3_K (qwen_moe_q3k.c:531): hmask[32] @0, qs[64] @32,
            // scales[12] @96, d @108.  Element e's value v = q + 4 is the two
            // bits of qs[32 (e / 128) + e % 32] at shift 2 ((e % 128) / 32)
            // plus 4 x bit e / 32 of hmask[e % 32] (qwen_moe_q3k.c:568-577);
            // the values go to the 3-word blocks of q3k_groups, scales and d
            // to @96 / @108.
            const uint8_t *b = src + i * 110;
            for (int blk = 0; blk < 8; ++blk) {
                uint8_t wb[12] = {};
                for (int g = 0; g < 8; ++g)
                    for (int ii = 0; ii < 4; ++ii) {
                        const int e = 32 * blk + 4 * g + ii;
                        const int q2 = (b[32 + 32 * (e / 128) + e % 32] >> (2 * ((e % 128) / 32))) & 3;
                        const int v = q2 | (((b[e % 32] >> (e / 32)) & 1) << 2);
                        if (g < 6) {
                            wb[4 * (g / 2) + ii] |= (uint8_t)(v << (3 * (g % 2)));
                        } else {
                            wb[4 * (g - 6) + ii] |= (uint8_t)((v & 3) << 6);
                            wb[8 + ii] |= (uint8_t)((v >> 2) << (g == 6 ? 6 : 7));
                        }
                    }
                for (int k = 0; k < 12; ++k) o[12 * blk + k] = wb[k];
            }
            for (int k = 0; k < 14; ++k) o[96 + k] = b[96 + k];
            o[110] = 0;
            o[111] = 0;
        }
    }
}

// ---- the reference's activation records (pack_act_i8 / pack_act_q3k) ----------
__device__ __forceinline__ void st_bytes(uint8_t *p, const void *v, int n) {
    for (int i = 0; i < n; ++i) p[i] = static_cast<const uint8_t *>(v)[i];
}
// One warp per 32-value record of 38 bytes (qwen_moe_q3k.c:420-426); the
// arithmetic of xprep_vals_i8.
__global__ void pack_i8_kernel(const float *__restrict__ x, long nrec, uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < nrec;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const float v = x[32 * r + lane];
        float amax = fabsf(v);
        for (int m = 16; m; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        amax = fmaxf(amax, 1e-6f);
        const float scale = __fdiv_rn(amax, 127.0f);
        const float inv = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
        const int q = max(-128, min(127, __float2int_rn(__fmul_rn(v, inv))));
        int sum = q;
        for (int m = 16; m; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
        uint8_t *o = out + 38 * r;
        o[6 + lane] = (uint8_t)(int8_t)q;
        if (lane == 0) {
            const int16_t s16 = (int16_t)sum;
            st_bytes(o, &scale, 4);
            st_bytes(o + 4, &s16, 2);
        }
    }
}
// One warp per 256-value record of 292 bytes (qwen_moe_q3k.c:613-623); the
// arithmetic of xprep_rows_q3k8.
__global__ void pack_q3k_kernel(const float *__restrict__ x, long nrec, uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < nrec;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const float4 *a = reinterpret_cast<const float4 *>(x + 256 * r + 8 * lane);
        const float4 p0 = a[0], p1 = a[1];
        const float e[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float amax = 0.f;
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(e[k]));
        for (int m = 16; m; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
        const float scale = __fdiv_rn(amax, 127.0f);
        const float rep = scale != 0.f ? __fdiv_rn(1.0f, scale) : 0.f;
        uint8_t *o = out + 292 * r;
        int s8 = 0;
        for (int k = 0; k < 8; ++k) {
            const int q = max(-128, min(127, (int)roundf(__fmul_rn(e[k], rep))));
            o[36 + 8 * lane + k] = (uint8_t)(int8_t)q;
            s8 += q;
        }
        const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);   // sub-block lane / 2
        if (!(lane & 1)) {
            const int16_t neg = (int16_t)(-s16);
            st_bytes(o + 4 + 2 * (lane >> 1), &neg, 2);
        }
        if (lane == 0) st_bytes(o, &scale, 4);
    }
}

// One warp per 256-value record of 290 bytes (pack_A_hp, qwen_moe_hp.c:131-180);
// the arithmetic of xprep_rows_hp8.
__global__ void pack_hp_kernel(const float *__restrict__ x, long nrec, uint8_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < nrec;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const float4 *a = reinterpret_cast<const float4 *>(x + 256 * r + 8 * lane);
        const float4 p0 = a[0], p1 = a[1];
        const float e[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const HpScales hs = hp_scales(e);
        uint8_t *o = out + 290 * r;
        const int kk = lane >> 2;
        int s8 = 0;
        for (int k = 0; k < 8; ++k) {
            const int q = hp_quant(e[k], hs.rep);
            o[34 * kk + 2 + 8 * (lane & 3) + k] = (uint8_t)(int8_t)q;
            s8 += q;
        }
        int s32 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
        s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
        if ((lane & 3) == 0) {
            const uint16_t as = f32_to_f16_trunc(__fmul_rn(-(float)(int16_t)s32, 8.0f));
            st_bytes(o + 34 * kk, &hs.ssub, 2);
            st_bytes(o + 272 + 2 * kk, &as, 2);
        }
        if (lane == 0) st_bytes(o + 288, &hs.blk, 2);
    }
}

constexpr size_t kGemvSmemMax = 220 * 1024;

static size_t gemv_smem(int qt, int K, int TR, int B) {
    const int ns = slices_per_row(K);
    return (size_t)TR * row_bytes_dev(qt, K) + xbuf_bytes(ns, B) + (size_t)B * TR * (2 * ns + 1) * 4;
}
// Rows per CTA.  One token: about one half-slice per thread and at most 40 KB
// of weights, so the next call's CTAs fit beside this call's (the chain of
// single-token calls overlaps).  Several tokens: every CTA prepares all the
// tokens' activations, so the rows go to at most one CTA per SM (one wave)
// when shared memory allows.
static int gemv_rows(int qt, int N, int K, int B, int sm_count) {
    const int ns = slices_per_row(K);
    const long rb = row_bytes_dev(qt, K);
    long tr = std::max<long>(std::min<long>(kGemvThreads / (2 * ns), 40960 / rb), 1);
    if (B > 1 && sm_count > 0) {
        const long wave = (N + sm_count - 1) / sm_count;
        while (tr < wave && gemv_smem(qt, K, (int)tr + 1, B) <= kGemvSmemMax) ++tr;
    }
    return (int)tr;
}

template <int QT, int B>
static int launch_B(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const GemvOpts &o,
                    cudaStream_t s) {
    // independent calls overlap, so they keep the small single-token tiles
    // (several CTAs per SM) instead of one wave of large ones
    const int TR = o.indep ? gemv_rows(QT, m.N, m.K, 1, 0) : gemv_rows(QT, m.N, m.K, B, c->sm_count);
    const size_t smem = gemv_smem(QT, m.K, TR, B);
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_kernel<QT, B>, (int)kGemvSmemMax);
        attr[c->device] = true;
    }
    // independent calls: half-size CTAs, so more of them fit an SM and more
    // weight bytes are in flight while the calls overlap
    const int threads = o.indep ? kGemvThreads / 2 : kGemvThreads;
    return launch_k(qgemv_kernel<QT, B>, dim3((m.N + TR - 1) / TR), dim3(threads), smem, s, o.pdl,
                    (const uint8_t *)m.w, m.N, m.K, TR, x, y, batch, o.norm_w, o.eps, o.accum ? 1 : 0,
                    o.indep ? 1 : 0, o.a8, c->d_status);
}

template <int QT>
static int launch_qt(DevCtx *c, const QMat &m, const float *x, float *y, int batch, GemvOpts o, cudaStream_t s) {
    const int TR = gemv_rows(QT, m.N, m.K, 1, 0);
    // tokens per launch: the largest template whose shared memory fits
    int bmax = 16;
    while (bmax > 1 && gemv_smem(QT, m.K, TR, bmax) > kGemvSmemMax) bmax >>= 1;
    if (gemv_smem(QT, m.K, TR, bmax) > kGemvSmemMax) {
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    for (int b0 = 0; b0 < batch; b0 += bmax) {
        const int nb = std::min(bmax, batch - b0);
        const float *xb = x + (long)b0 * m.K;
        float *yb = y + (long)b0 * m.N;
        int st;
        if (nb <= 1) st = launch_B<QT, 1>(c, m, xb, yb, nb, o, s);
        else if (nb <= 2) st = launch_B<QT, 2>(c, m, xb, yb, nb, o, s);
        else if (nb <= 4) st = launch_B<QT, 4>(c, m, xb, yb, nb, o, s);
        else if (nb <= 8) st = launch_B<QT, 8>(c, m, xb, yb, nb, o, s);
        else st = launch_B<QT, 16>(c, m, xb, yb, nb, o, s);
        if (st) return st;
        o.pdl = true;
    }
    return X100_OK;
}

}  // namespace q

bool pdl_enabled() { return q::pdl_enabled_impl(); }

using namespace q;

size_t qtype_block_elems(int qt) { return qt == Q4_0 || qt == Q8_0 ? 32 : (qt == Q4_K || qt == Q3_K ? 256 : 0); }
size_t qtype_block_bytes(int qt) {
    return qt == Q4_0 ? 18 : qt == Q8_0 ? 34 : qt == Q4_K ? 144 : qt == Q3_K ? 110 : 0;
}

bool qmat_upload(DevCtx *c, int qt, int N, int K, const void *blocks, QMat &m, cudaStream_t s) {
    const size_t be = qtype_block_elems(qt), bb = qtype_block_bytes(qt);
    if (!be || N <= 0 || K <= 0 || K % (int)be || !blocks) {
        set_error(X100_E_ARG);
        return false;
    }
    if (fault_injected("alloc")) return false;
    const size_t native = (size_t)N * (K / be) * bb;
    m = QMat();
    m.qtype = qt;
    m.N = N;
    m.K = K;
    m.ns = slices_per_row(K);
    m.row_bytes = row_bytes_dev(qt, K);
    m.bytes = (size_t)N * m.row_bytes;
    void *tmp = nullptr;
    if (cudaMalloc(reinterpret_cast<void **>(&m.w), m.bytes + 256) != cudaSuccess) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        m.w = nullptr;
        return false;
    }
    if (qt == Q4_K) {   // the native superblocks are already the slices
        if (check_cuda(cudaMemcpyAsync(m.w, blocks, native, cudaMemcpyDefault, s), X100_E_COPY)) goto fail;
    } else {
        if (cudaMalloc(&tmp, native) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            goto fail;
        }
        if (check_cuda(cudaMemcpyAsync(tmp, blocks, native, cudaMemcpyDefault, s), X100_E_COPY)) goto fail;
        const long total = (long)N * m.ns;
        repack_kernel<<<(int)std::min<long>((total + 255) / 256, 65535), 256, 0, s>>>(
            qt, N, K, static_cast<const uint8_t *>(tmp), m.w);
        if (check_cuda(cudaGetLastError(), X100_E_LAUNCH)) goto fail;
    }
    if (check_cuda(cudaStreamSynchronize(s), X100_E_COPY)) goto fail;
    cudaFree(tmp);
    return true;
fail:
    cudaStreamSynchronize(s);
    cudaFree(tmp);
    cudaFree(m.w);
    m.w = nullptr;
    return false;
}

int launch_qgemv(DevCtx *c, const QMat &m, const float *x, float *y, int batch, cudaStream_t s) {
    return launch_qgemv_ex(c, m, x, y, batch, GemvOpts(), s);
}

// Whether the tensor-core kernel takes a call.  Independent calls of up to 4
// tokens stay on the dp4a kernel: its small CTAs let consecutive calls
// overlap, which the persistent tensor-core kernel (one CTA per SM) cannot
// (Q4_0 6144 x 2048, 4 tokens: 1187 vs 900 GB/s measured; from 8 tokens the
// tensor-core kernel is ahead).  One token on a very tall matrix (an
// lm_head): the persistent tensor-core kernel streams it faster than the
// single-token dp4a kernel's many waves of small CTAs (151936 x 2048 Q8_0:
// 118 vs 145 us).  X100_GEMV_DP4A=1 keeps every call on the dp4a kernel.
static bool takes_mma(const QMat &m, int batch, const GemvOpts &o) {
    static const bool dp4a_only = [] {
        const char *e = getenv("X100_GEMV_DP4A");
        return e && *e && *e != '0';
    }();
    const bool tall = batch == 1 && m.N >= 65536;
    return (batch > 1 || tall) && !dp4a_only && !(o.indep && batch <= 4) && qgemv_mma_ok(m.qtype, m.K);
}

int qgemv_prep_group(const QMat &m, int batch, const GemvOpts &o) {
    if (batch < 2 || batch > 16 || !takes_mma(m, batch, o)) return 0;
    return qgemv_mma_prep_group(m, batch, o);
}

int launch_qgemv_ex(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const GemvOpts &o,
                    cudaStream_t s) {
    if (batch < 1 || batch > 16) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    if (takes_mma(m, batch, o)) {
        const int st = launch_qgemv_mma(c, m, x, y, batch, o, s);
        if (st) set_error(st);
        return st;
    }
    switch (m.qtype) {
    case Q4_0: return launch_qt<Q4_0>(c, m, x, y, batch, o, s);
    case Q8_0: return launch_qt<Q8_0>(c, m, x, y, batch, o, s);
    case Q4_K: return launch_qt<Q4_K>(c, m, x, y, batch, o, s);
    case Q3_K: return launch_qt<Q3_K>(c, m, x, y, batch, o, s);
    default: set_error(X100_E_UNSUPPORTED); return X100_E_UNSUPPORTED;
    }
}

}  // namespace x100

using namespace x100;

struct x100q_lin {
    int device;
    QMat m;
};

extern "C" {

size_t x100q_row_bytes(int qtype, int K) {
    const size_t be = qtype_block_elems(qtype), bb = qtype_block_bytes(qtype);
    if (qtype == X100Q_F32) return K > 0 ? (size_t)K * 4 : 0;
    if (!be || K <= 0 || K % (int)be) return 0;
    return (size_t)(K / be) * bb;
}

x100q_lin *x100q_lin_create(int qtype, int N, int K, const void *blocks) {
    set_error(X100_OK);
    if (qtype != X100Q_Q4_0 && qtype != X100Q_Q8_0 && qtype != X100Q_Q4_K && qtype != X100Q_Q3_K) {
        set_error(X100_E_UNSUPPORTED);
        return nullptr;
    }
    DevCtx *c = ctx();
    if (!c) return nullptr;
    x100q_lin *l = new x100q_lin();
    l->device = c->device;
    std::lock_guard<std::mutex> lk(c->mu);
    if (!qmat_upload(c, qtype, N, K, blocks, l->m, c->stream)) {
        delete l;
        return nullptr;
    }
    return l;
}

void x100q_lin_destroy(x100q_lin *l) {
    if (!l) return;
    DeviceGuard dg(l->device);
    cudaFree(l->m.w);
    delete l;
}

int x100q_lin_info(const x100q_lin *l, int *qtype, int *N, int *K, size_t *device_bytes) {
    if (!l) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (qtype) *qtype = l->m.qtype;
    if (N) *N = l->m.N;
    if (K) *K = l->m.K;
    if (device_bytes) *device_bytes = l->m.bytes;
    return X100_OK;
}

int x100q_lin_gemv_dev(const x100q_lin *l, const float *x, float *y, int batch, void *stream) {
    return x100q_lin_gemv_dev_flags(l, x, y, batch, 0, stream);
}

int x100q_lin_gemv_dev_flags(const x100q_lin *l, const float *x, float *y, int batch, int flags, void *stream) {
    set_error(X100_OK);
    if (flags & ~(X100Q_GEMV_INDEPENDENT | X100Q_GEMV_A8)) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (!l || !x || !y) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) {   // the kernel reads x with 16-byte loads
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    GemvOpts o;
    o.indep = (flags & X100Q_GEMV_INDEPENDENT) != 0;
    if (flags & X100Q_GEMV_A8) {   // the reference's activation packing for the weight type
        if (l->m.qtype == Q8_0) o.a8 = 1;
        else if (l->m.qtype == Q3_K) o.a8 = 2;
        else if (l->m.qtype == Q4_0 && l->m.K % 256 == 0) o.a8 = 3;
        else {
            set_error(X100_E_UNSUPPORTED);
            return X100_E_UNSUPPORTED;
        }
    }
    int st = launch_qgemv_ex(c, l->m, x, y, batch, o, static_cast<cudaStream_t>(stream));
    if (st) set_error(st);
    return st;
}

int x100q_pack_act_dev(int mode, const float *x, int K, int batch, void *out, void *stream) {
    set_error(X100_OK);
    const int per = mode == X100Q_PACK_I8 ? 32 : 256;
    if ((mode != X100Q_PACK_I8 && mode != X100Q_PACK_Q3K && mode != X100Q_PACK_HP) || !x || !out || K <= 0 ||
        K % per || batch < 1 ||
        (reinterpret_cast<uintptr_t>(x) & 15)) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    const long nrec = (long)batch * (K / per);
    const int grid = (int)std::min<long>((nrec + 7) / 8, (long)c->sm_count * 16);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (mode == X100Q_PACK_I8) pack_i8_kernel<<<grid, 256, 0, s>>>(x, nrec, static_cast<uint8_t *>(out));
    else if (mode == X100Q_PACK_HP) pack_hp_kernel<<<grid, 256, 0, s>>>(x, nrec, static_cast<uint8_t *>(out));
    else pack_q3k_kernel<<<grid, 256, 0, s>>>(x, nrec, static_cast<uint8_t *>(out));
    const int st = check_cuda(cudaGetLastError(), X100_E_LAUNCH);
    if (st) set_error(st);
    return st;
}

int x100q_lin_gemv(const x100q_lin *l, const float *x, float *y, int batch) {
    set_error(X100_OK);
    if (!l || !x || !y || batch < 1 || batch > 16) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    DevCtx *c = ctx();
    if (!c) return get_error();
    std::lock_guard<std::mutex> lk(c->mu);
    const size_t xb = (size_t)batch * l->m.K * 4, yb = (size_t)batch * l->m.N * 4;
    const float *xd = x;
    float *yd = y;
    const bool xdev = is_device_ptr(x), ydev = is_device_ptr(y);
    if (!xdev) {
        void *b = stage_buf(c, 0, xb);
        if (!b) return get_error();
        if (fault_injected("copy") || check_cuda(cudaMemcpyAsync(b, x, xb, cudaMemcpyHostToDevice, c->stream), X100_E_COPY))
            return get_error();
        xd = static_cast<const float *>(b);
    } else if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (!ydev) {
        void *b = stage_buf(c, 1, yb);
        if (!b) return get_error();
        yd = static_cast<float *>(b);
    }
    int st = launch_qgemv(c, l->m, xd, yd, batch, c->stream);
    if (st == X100_OK && !ydev)
        st = check_cuda(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, c->stream), X100_E_COPY);
    int st2 = sync_and_status(c, c->stream);
    if (st == X100_OK) st = st2;
    if (st) set_error(st);
    return st;
}

}  // extern "C"
