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

template <int QT, int B>
__global__ void __launch_bounds__(kGemvThreads, 1)
    qgemv_kernel(const uint8_t *__restrict__ W, int N, int K, int TR, const float *__restrict__ x,
                 float *__restrict__ y, int batch, int *status) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
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
    pdl_wait();                                   // x may come from the previous kernel
    xprep_rows([x, K](int c) { return x + (long)c * K; }, K, batch, xb);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status);
    const int nh = rows * ns * 2;
    for (int p = threadIdx.x; p < nh; p += blockDim.x) {
        const int sp = p >> 1, h = p & 1;
        const int r = sp / ns, sl = sp - r * ns;
        WHalf<QT> w;
        load_half<QT>(tile + (long)sp * SB, h, w);
#pragma unroll
        for (int b = 0; b < B; ++b)
            if (b < batch) red[(b * TR + r) * S + 2 * sl + h] = ok ? dot_half<QT>(w, h, xb.half(b, sl, h)) : 0.f;
    }
    __syncthreads();
    if (abort_flag) {
        if (threadIdx.x == 0) mbar_wait_drain(&bar, 0, 100000000ull);   // the copy may still be in flight
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
        y[(long)b * N + row0 + r] = s0 + s1;
    }
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
            // scales[12] @96, d @108  ->  qs @0, hmask @64, scales @96, d @108
            const uint8_t *b = src + i * 110;
            for (int k = 0; k < 64; ++k) o[k] = b[32 + k];
            for (int k = 0; k < 32; ++k) o[64 + k] = b[k];
            for (int k = 0; k < 14; ++k) o[96 + k] = b[96 + k];
            o[110] = 0;
            o[111] = 0;
        }
    }
}

// Rows per CTA: about one half-slice per thread, and at most 40 KB of weights
// so the next call's CTAs fit beside this call's.
static int gemv_rows(int qt, int K) {
    const int ns = slices_per_row(K);
    const long rb = row_bytes_dev(qt, K);
    long tr = std::min<long>(kGemvThreads / (2 * ns), 40960 / rb);
    return (int)std::max<long>(tr, 1);
}
static size_t gemv_smem(int qt, int K, int TR, int B) {
    const int ns = slices_per_row(K);
    return (size_t)TR * row_bytes_dev(qt, K) + xbuf_bytes(ns, B) + (size_t)B * TR * (2 * ns + 1) * 4;
}

template <int QT, int B>
static int launch_B(DevCtx *c, const QMat &m, const float *x, float *y, int batch, cudaStream_t s) {
    const int TR = gemv_rows(QT, m.K);
    const size_t smem = gemv_smem(QT, m.K, TR, B);
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_kernel<QT, B>);
        attr[c->device] = true;
    }
    return launch_pdl(qgemv_kernel<QT, B>, dim3((m.N + TR - 1) / TR), dim3(kGemvThreads), smem, s,
                      (const uint8_t *)m.w, m.N, m.K, TR, x, y, batch, c->d_status);
}

template <int QT>
static int launch_qt(DevCtx *c, const QMat &m, const float *x, float *y, int batch, cudaStream_t s) {
    const int TR = gemv_rows(QT, m.K);
    // tokens per launch: the largest template whose shared memory fits
    int bmax = 16;
    while (bmax > 1 && gemv_smem(QT, m.K, TR, bmax) > 200 * 1024) bmax >>= 1;
    if (gemv_smem(QT, m.K, TR, bmax) > 200 * 1024) {
        set_error(X100_E_UNSUPPORTED);
        return X100_E_UNSUPPORTED;
    }
    for (int b0 = 0; b0 < batch; b0 += bmax) {
        const int nb = std::min(bmax, batch - b0);
        const float *xb = x + (long)b0 * m.K;
        float *yb = y + (long)b0 * m.N;
        int st;
        if (nb <= 1) st = launch_B<QT, 1>(c, m, xb, yb, nb, s);
        else if (nb <= 2) st = launch_B<QT, 2>(c, m, xb, yb, nb, s);
        else if (nb <= 4) st = launch_B<QT, 4>(c, m, xb, yb, nb, s);
        else if (nb <= 8) st = launch_B<QT, 8>(c, m, xb, yb, nb, s);
        else st = launch_B<QT, 16>(c, m, xb, yb, nb, s);
        if (st) return st;
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
        if (check_cuda(cudaMemcpyAsync(m.w, blocks, native, cudaMemcpyHostToDevice, s), X100_E_COPY)) goto fail;
    } else {
        if (cudaMalloc(&tmp, native) != cudaSuccess) {
            cudaGetLastError();
            set_error(X100_E_ALLOC);
            goto fail;
        }
        if (check_cuda(cudaMemcpyAsync(tmp, blocks, native, cudaMemcpyHostToDevice, s), X100_E_COPY)) goto fail;
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
    if (batch < 1 || batch > 16) {
        set_error(X100_E_ARG);
        return X100_E_ARG;
    }
    if (fault_injected("launch")) return X100_E_INJECTED;
    switch (m.qtype) {
    case Q4_0: return launch_qt<Q4_0>(c, m, x, y, batch, s);
    case Q8_0: return launch_qt<Q8_0>(c, m, x, y, batch, s);
    case Q4_K: return launch_qt<Q4_K>(c, m, x, y, batch, s);
    case Q3_K: return launch_qt<Q3_K>(c, m, x, y, batch, s);
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
    int st = launch_qgemv(c, l->m, x, y, batch, static_cast<cudaStream_t>(stream));
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
