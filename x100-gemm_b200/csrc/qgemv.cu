// qgemv.cu -- block-quantised dequant-GEMV (Q4_0 / Q8_0 / Q4_K / Q3_K) and the
// x100q_lin_* entry points of include/x100q.h.
//
// Replaces the reference's per-linear decode path: lin_new_* (weight
// requant/repack, qwen_moe_q3k.c:843-909) + pack_act_* + lin_mm_*
// (qwen_moe_q3k.c:1029-1082, qwen_moe.c:90-107), whose hot loop streams each
// weight row once per token through the IME micro-kernels.
//
// Kernel: each warp owns `RR` rows per lane group; its lanes split a row's
// 32-weight units (lanes-per-row LPR = 32, or fewer for short rows so a warp
// covers several rows).  A lane loads its unit of RR rows with 16-byte loads,
// then for every batch column dots it against the activation planes held in
// shared memory (exact dp4a int32 sums, one fp32 scale per block), so each
// weight byte is read from HBM once per call whatever the batch.  Partial sums
// are combined with warp shuffles.  The activation planes are prepared by the
// CTA itself from the fp32 x (qformats.cuh: xprep_block).
#include <cuda_fp16.h>

#include <cstring>

#include "../../include/x100q.h"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace q {

int lanes_per_row(int units) {
    int l = 32;
    while (l > 1 && l > units) l >>= 1;
    return l;
}

template <int QT, int B, int RR>
__global__ void __launch_bounds__(256) qgemv_kernel(QView W, const float *__restrict__ x, float *__restrict__ y,
                                                    int batch, int lpr) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int nxb = W.K / 32;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * B * nxb);
    // activation planes for all batch columns
    xprep_all(x, W.K, batch, xq, xf);
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int units = units_per_row(QT, W.K);
    const int slot = lane / lpr, sig = lane % lpr;
    const int rows_per_pass = (32 / lpr) * RR;
    for (long r0 = ((long)blockIdx.x * nwarps + warp) * rows_per_pass; r0 < W.N;
         r0 += (long)gridDim.x * nwarps * rows_per_pass) {
        const int rbase = (int)r0 + slot * RR;
        float acc[RR][B];
#pragma unroll
        for (int r = 0; r < RR; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
        for (int u = sig; u < units; u += lpr) {
            WUnit<QT> wu[RR];
#pragma unroll
            for (int r = 0; r < RR; ++r)
                if (rbase + r < W.N) wu[r] = load_unit<QT>(W, rbase + r, u);
#pragma unroll
            for (int b = 0; b < B; ++b) {
                if (b < batch) {
#pragma unroll
                    for (int r = 0; r < RR; ++r)
                        if (rbase + r < W.N) acc[r][b] += dot_unit<QT>(wu[r], xq + b * nxb, xf + b * nxb, u);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RR; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b)
                for (int off = lpr >> 1; off > 0; off >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], off);
        if (sig == 0) {
#pragma unroll
            for (int r = 0; r < RR; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b)
                    if (b < batch && rbase + r < W.N) y[(long)b * W.N + rbase + r] = acc[r][b];
        }
    }
}

// ---- device re-layout of GGUF-native blocks ------------------------------------
__global__ void repack_kernel(int qt, long nblocks, const uint8_t *__restrict__ src, uint8_t *__restrict__ w,
                              __half *__restrict__ d) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nblocks; i += (long)gridDim.x * blockDim.x) {
        if (qt == Q4_0) {
            const uint8_t *s = src + i * 18;
            d[i] = __ushort_as_half((unsigned short)(s[0] | (s[1] << 8)));
            for (int k = 0; k < 16; ++k) w[i * 16 + k] = s[2 + k];
        } else if (qt == Q8_0) {
            const uint8_t *s = src + i * 34;
            d[i] = __ushort_as_half((unsigned short)(s[0] | (s[1] << 8)));
            for (int k = 0; k < 32; ++k) w[i * 32 + k] = s[2 + k];
        } else if (qt == Q3_K) {
            // block_q3_K (qwen_moe_q3k.c:531): hmask[32] @0, qs[64] @32,
            // scales[12] @96, d @108  ->  qs @0, hmask @64, scales @96, d @108
            const uint8_t *s = src + i * 110;
            uint8_t *o = w + i * 112;
            for (int k = 0; k < 64; ++k) o[k] = s[32 + k];
            for (int k = 0; k < 32; ++k) o[64 + k] = s[k];
            for (int k = 0; k < 14; ++k) o[96 + k] = s[96 + k];
            o[110] = 0;
            o[111] = 0;
        }
    }
}

}  // namespace q

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
    const long nblk = (long)N * (K / (long)be);
    const size_t native = (size_t)nblk * bb;
    m = QMat();
    m.qtype = qt;
    m.N = N;
    m.K = K;
    const size_t wbytes = (size_t)N * row_bytes_dev(qt, K);
    const size_t dbytes = (qt == Q4_0 || qt == Q8_0) ? (size_t)nblk * 2 : 0;
    if (cudaMalloc(&m.w, wbytes + dbytes + 256) != cudaSuccess) {
        cudaGetLastError();
        set_error(X100_E_ALLOC);
        return false;
    }
    m.bytes = wbytes + dbytes;
    if (dbytes) m.d = reinterpret_cast<__half *>(static_cast<uint8_t *>(m.w) + ((wbytes + 255) / 256) * 256);
    if (qt == Q4_K) {
        if (check_cuda(cudaMemcpyAsync(m.w, blocks, native, cudaMemcpyHostToDevice, s), X100_E_COPY)) goto fail;
    } else {
        void *tmp = nullptr;
        if (cudaMalloc(&tmp, native) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            goto fail;
        }
        if (check_cuda(cudaMemcpyAsync(tmp, blocks, native, cudaMemcpyHostToDevice, s), X100_E_COPY)) {
            cudaFree(tmp);
            goto fail;
        }
        repack_kernel<<<(int)std::min<long>((nblk + 255) / 256, 65535), 256, 0, s>>>(
            qt, nblk, static_cast<const uint8_t *>(tmp), static_cast<uint8_t *>(m.w), m.d);
        cudaError_t e = cudaStreamSynchronize(s);
        cudaFree(tmp);
        if (check_cuda(e == cudaSuccess ? cudaGetLastError() : e, X100_E_LAUNCH)) goto fail;
    }
    if (check_cuda(cudaStreamSynchronize(s), X100_E_COPY)) goto fail;
    return true;
fail:
    cudaFree(m.w);
    m.w = nullptr;
    return false;
}

QView qmat_view(const QMat &m, long row0) {
    QView v;
    v.qt = m.qtype;
    v.wstride = row_bytes_dev(m.qtype, m.K);
    v.dstride = m.K / 32;
    v.w = static_cast<const uint8_t *>(m.w) + row0 * v.wstride;
    v.d = m.d ? m.d + row0 * v.dstride : nullptr;
    v.N = m.N - (int)row0;
    v.K = m.K;
    return v;
}

template <int QT, int B>
static int launch_B(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    constexpr int RR = B <= 2 ? 2 : 1;
    const int lpr = lanes_per_row(units_per_row(QT, v.K));
    const int rows_per_warp = (32 / lpr) * RR;
    const long passes = (v.N + rows_per_warp - 1) / rows_per_warp;
    const size_t smem = (size_t)B * (v.K / 32) * (sizeof(XBlk) + sizeof(XF));
    if (smem > 200 * 1024) {
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    static bool attr[64][2];
    if (smem > 48 * 1024 && !attr[c->device][0]) {
        cudaFuncSetAttribute(qgemv_kernel<QT, B, RR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr[c->device][0] = true;
    }
    long grid = (passes + 7) / 8;
    const long cap = (long)c->sm_count * 4;
    if (grid > cap) grid = cap;
    qgemv_kernel<QT, B, RR><<<(int)grid, 256, smem, s>>>(v, x, y, batch, lpr);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

template <int QT>
static int launch_qt(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    if (batch <= 1) return launch_B<QT, 1>(c, v, x, y, batch, s);
    if (batch <= 2) return launch_B<QT, 2>(c, v, x, y, batch, s);
    if (batch <= 4) return launch_B<QT, 4>(c, v, x, y, batch, s);
    if (batch <= 8) return launch_B<QT, 8>(c, v, x, y, batch, s);
    return launch_B<QT, 16>(c, v, x, y, batch, s);
}

int launch_qgemv(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    if (batch < 1 || batch > 16) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    switch (v.qt) {
    case Q4_0: return launch_qt<Q4_0>(c, v, x, y, batch, s);
    case Q8_0: return launch_qt<Q8_0>(c, v, x, y, batch, s);
    case Q4_K: return launch_qt<Q4_K>(c, v, x, y, batch, s);
    case Q3_K: return launch_qt<Q3_K>(c, v, x, y, batch, s);
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
    cudaSetDevice(l->device);
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
    set_error(X100_OK);
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
    int st = launch_qgemv(c, qmat_view(l->m, 0), x, y, batch, static_cast<cudaStream_t>(stream));
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
    }
    if (!ydev) {
        void *b = stage_buf(c, 1, yb);
        if (!b) return get_error();
        yd = static_cast<float *>(b);
    }
    int st = launch_qgemv(c, qmat_view(l->m, 0), xd, yd, batch, c->stream);
    if (st == X100_OK && !ydev)
        st = check_cuda(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, c->stream), X100_E_COPY);
    int st2 = sync_and_status(c, c->stream);
    if (st == X100_OK) st = st2;
    if (st) set_error(st);
    return st;
}

}  // extern "C"
