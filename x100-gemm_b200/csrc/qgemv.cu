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

#include <cstdlib>
#include <cstring>

#include "../../include/x100q.h"
#include "qgemv.h"
#include "runtime.h"

namespace x100 {
namespace q {

bool pdl_enabled_impl() {
    static const bool on = [] {
        const char *e = getenv("X100_NO_PDL");
        return !(e && *e && *e != '0');
    }();
    return on;
}

int lanes_per_row(int units) {
    int l = 32;
    while (l > 1 && l > units) l >>= 1;
    return l;
}

template <int QT, int B, int RR>
__global__ void __launch_bounds__(256) qgemv_kernel(QView W, const float *__restrict__ x, float *__restrict__ y,
                                                    int batch, int lpr) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nxb = W.K / 32;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * B * nxb);
    pdl_launch_dependents();
    pdl_wait();
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

// Slice kernel (K % 256 == 0, K <= 4096): warp w owns the 256-element slice
// w of 32 consecutive rows (lane = row).  Each lane issues its slice's
// 16-byte weight loads first, the CTA then prepares the activation planes in
// shared memory while those loads are in flight, every lane dots its slice
// against the same (broadcast) activation blocks, and the per-slice partial
// sums are added in slice order through shared memory.
template <int QT, int B>
__global__ void __launch_bounds__(512) qgemv_slice_kernel(QView W, const float *__restrict__ x,
                                                          float *__restrict__ y, int batch) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nxb = W.K / 32, ns = W.K / 256;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * B * nxb);
    float *red = reinterpret_cast<float *>(xf + B * nxb);   // [slice][b][lane]
    const int lane = threadIdx.x & 31, sl = threadIdx.x >> 5;
    const int row = blockIdx.x * 32 + lane;
    WSlice<QT> ws;
    if (row < W.N) load_slice<QT>(W, row, sl, ws);
    pdl_launch_dependents();
    pdl_wait();
    xprep_all(x, W.K, batch, xq, xf);
    __syncthreads();
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float a = 0.f;
        if (b < batch && row < W.N) a = dot_slice<QT>(ws, xq + b * nxb + sl * 8, xf + b * nxb + sl * 8);
        red[(sl * B + b) * 32 + lane] = a;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < 32 * B; t += blockDim.x) {
        const int l = t & 31, b = t >> 5;
        const int r = blockIdx.x * 32 + l;
        if (b < batch && r < W.N) {
            float acc = 0.f;
            for (int k = 0; k < ns; ++k) acc += red[(k * B + b) * 32 + l];
            y[(long)b * W.N + r] = acc;
        }
    }
}

// Half-slice kernel (K % 256 == 0, K <= 2048): warp w owns half w % 2 of
// slice w / 2 for 32 consecutive rows (lane = row), so a CTA of K/4 threads
// covers 32 full rows.  Weight loads are issued before waiting on the
// previous kernel of the stream (programmatic dependent launch), the
// activation planes are prepared once per CTA, every lane of a warp reads the
// same activation blocks (broadcast), and the per-half partial sums are added
// in K order through shared memory.
template <int QT, int B>
__global__ void __launch_bounds__(512) qgemv_half_kernel(QView W, const float *__restrict__ x,
                                                         float *__restrict__ y, int batch) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nxb = W.K / 32, nh = W.K / 128;
    XBlk *xq = reinterpret_cast<XBlk *>(smem);
    XF *xf = reinterpret_cast<XF *>(smem + sizeof(XBlk) * B * nxb);
    float *red = reinterpret_cast<float *>(xf + B * nxb);   // [half slice][b][lane]
    const int lane = threadIdx.x & 31, hs = threadIdx.x >> 5;
    const int row = blockIdx.x * 32 + lane;
    WHalf<QT> wh;
    if (row < W.N) load_half<QT>(W, row, hs >> 1, hs & 1, wh);
    pdl_launch_dependents();
    pdl_wait();
    xprep_all(x, W.K, batch, xq, xf);
    __syncthreads();
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float a = 0.f;
        if (b < batch && row < W.N) a = dot_half<QT>(wh, hs & 1, xq + b * nxb + hs * 4, xf + b * nxb + hs * 4);
        red[(hs * B + b) * 32 + lane] = a;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < 32 * B; t += blockDim.x) {
        const int l = t & 31, b = t >> 5;
        const int r = blockIdx.x * 32 + l;
        if (b < batch && r < W.N) {
            float acc = 0.f;
            for (int k = 0; k < nh; ++k) acc += red[(k * B + b) * 32 + l];
            y[(long)b * W.N + r] = acc;
        }
    }
}

// Staged kernel (K % 256 == 0): a CTA owns 32 consecutive rows.  All threads
// copy the 32 rows (and their scale rows) into padded shared memory with
// 16-byte cp.async requests -- issued before waiting on the previous kernel
// of the stream, with no registers tied up by loads in flight -- and then
// prepare the activation planes while the copies land.  Warp w dots slices
// w, w+nw, ... of every row (lane = row) against the broadcast activation
// blocks; the per-warp partial sums are added in warp order.
template <int QT, int B>
__global__ void __launch_bounds__(256, 2) qgemv_bulk_kernel(QView W, const float *__restrict__ x,
                                                         float *__restrict__ y, int batch, int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int K = W.K, nxb = K / 32, ns = K / 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row0 = blockIdx.x * 32;
    const int rows = min(32, W.N - row0);
    uint8_t *tile = smem;
    XBlk *xq = reinterpret_cast<XBlk *>(smem + tile_bytes(QT, K, 32));
    XF *xf = reinterpret_cast<XF *>(xq + B * nxb);
    float *red = reinterpret_cast<float *>(xf + B * nxb);   // [warp][b][lane]
    if (rows > 0) tile_cp_async(W, row0, rows, tile, 32);
    cp_async_commit();
    pdl_launch_dependents();
    pdl_wait();
    xprep_all(x, K, batch, xq, xf);
    cp_async_wait_all();
    __syncthreads();
    const bool ok = true;
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    if (ok && lane < rows) {
        const QView T = tile_view(QT, K, tile, 32);
        for (int sl = warp; sl < ns; sl += nw) {
            WSlice<QT> ws;
            load_slice<QT, false>(T, lane, sl, ws);
#pragma unroll
            for (int b = 0; b < B; ++b)
                if (b < batch) acc[b] += dot_slice<QT>(ws, xq + b * nxb + sl * 8, xf + b * nxb + sl * 8);
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) red[(warp * B + b) * 32 + lane] = acc[b];
    __syncthreads();
    for (int t = threadIdx.x; t < 32 * B; t += blockDim.x) {
        const int l = t & 31, b = t >> 5;
        if (b < batch && l < rows) {
            float sum = 0.f;
            for (int k = 0; k < nw; ++k) sum += red[(k * B + b) * 32 + l];
            y[(long)b * W.N + row0 + l] = sum;
        }
    }
}

// Warp-independent kernel (K % 256 == 0): a CTA owns 32 consecutive rows
// and warp w owns K-slices w, w+nw, ...  Each warp stages its own slices of
// the 32 rows (one 1-D bulk copy per row and slice, issued before waiting on
// the previous kernel of the stream) behind its own mbarrier, prepares the
// activation blocks of those slices, and computes as soon as its bytes have
// landed; the only CTA-wide synchronisation is the final reduction of the
// per-warp partial sums (added in warp order).
template <int QT> struct SliceBytes;
template <> struct SliceBytes<Q4_0> { static constexpr int w = 128, s = 16; };
template <> struct SliceBytes<Q8_0> { static constexpr int w = 256, s = 16; };
template <> struct SliceBytes<Q4_K> { static constexpr int w = 144, s = 0; };
template <> struct SliceBytes<Q3_K> { static constexpr int w = 112, s = 0; };
template <int QT> __host__ __device__ constexpr int ws_slice_stride() { return bulk_stride(SliceBytes<QT>::w); }
template <int QT> __host__ __device__ constexpr int ws_scale_stride() { return SliceBytes<QT>::s ? bulk_stride(SliceBytes<QT>::s) : 0; }
// shared bytes for one staged slice of 32 rows
template <int QT> __host__ __device__ constexpr int ws_slice_tile() { return 32 * (ws_slice_stride<QT>() + ws_scale_stride<QT>()); }

template <int QT, int B>
__global__ void __launch_bounds__(256, 2) qgemv_ws_kernel(QView W, const float *__restrict__ x,
                                                          float *__restrict__ y, int batch, int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bars[8];
    __shared__ int abort_flag;
    const int K = W.K, ns = K / 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int spw = (ns + nw - 1) / nw;                        // slices per warp (last warps may have fewer)
    const int row0 = blockIdx.x * 32;
    const int rows = min(32, W.N - row0);
    constexpr int TS = ws_slice_tile<QT>();
    uint8_t *tiles = smem + (size_t)warp * spw * TS;
    XBlk *xq = reinterpret_cast<XBlk *>(smem + (size_t)nw * spw * TS) + (size_t)warp * spw * 8 * B;
    XF *xf = reinterpret_cast<XF *>(reinterpret_cast<XBlk *>(smem + (size_t)nw * spw * TS) + (size_t)nw * spw * 8 * B) +
             (size_t)warp * spw * 8 * B;
    float *red = reinterpret_cast<float *>(reinterpret_cast<XF *>(reinterpret_cast<XBlk *>(smem + (size_t)nw * spw * TS) +
                                                                  (size_t)nw * spw * 8 * B) + (size_t)nw * spw * 8 * B);
    if (threadIdx.x == 0) {
        for (int i = 0; i < nw; ++i) mbar_init(&bars[i], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    int my_slices = 0;
    for (int k = 0; k < spw; ++k) my_slices += (warp + k * nw < ns);
    if (lane == 0)
        mbar_arrive_expect_tx(&bars[warp], (uint32_t)(my_slices * rows * (SliceBytes<QT>::w + SliceBytes<QT>::s)));
    __syncwarp();
    if (lane < rows) {
        const long grow = row0 + lane;
        for (int k = 0; k < my_slices; ++k) {
            const int sl = warp + k * nw;
            uint8_t *t = tiles + k * TS;
            bulk_load(t + lane * ws_slice_stride<QT>(), W.w + grow * W.wstride + (long)sl * SliceBytes<QT>::w,
                      SliceBytes<QT>::w, &bars[warp]);
            if (SliceBytes<QT>::s)
                bulk_load(t + 32 * ws_slice_stride<QT>() + lane * ws_scale_stride<QT>(),
                          reinterpret_cast<const uint8_t *>(W.d + grow * W.dstride) + sl * SliceBytes<QT>::s,
                          SliceBytes<QT>::s, &bars[warp]);
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    // this warp's activation blocks: batch b, slice k -> 8 blocks at xq[(k * B + b) * 8]
    {
        const int total = my_slices * batch * 8;
        for (int b0 = 0; b0 < total; b0 += 4) {
            const int blk = b0 + (lane >> 3);
            const bool act = blk < total;
            const int k = act ? blk / (batch * 8) : 0, rem = act ? blk % (batch * 8) : 0;
            const int b = rem / 8, j = rem % 8;
            const int sl = warp + k * nw;
            xprep_block(x + (long)b * K + sl * 256 + j * 32, &xq[(k * B + b) * 8 + j], &xf[(k * B + b) * 8 + j],
                        lane & 7, act);
        }
    }
    __syncwarp();
    const bool ok = mbar_wait(&bars[warp], 0, &abort_flag, status);
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    if (ok && lane < rows) {
        for (int k = 0; k < my_slices; ++k) {
            QView T;
            T.qt = QT;
            T.K = 256;
            T.N = 32;
            T.w = tiles + k * TS;
            T.wstride = ws_slice_stride<QT>();
            T.d = reinterpret_cast<const __half *>(tiles + k * TS + 32 * ws_slice_stride<QT>());
            T.dstride = ws_scale_stride<QT>() / 2;
            WSlice<QT> w;
            load_slice<QT, false>(T, lane, 0, w);
#pragma unroll
            for (int b = 0; b < B; ++b)
                if (b < batch) acc[b] += dot_slice<QT>(w, xq + (k * B + b) * 8, xf + (k * B + b) * 8);
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) red[(warp * B + b) * 32 + lane] = acc[b];
    __syncthreads();
    if (abort_flag) {
        if (lane == 0) mbar_wait_drain(&bars[warp], 0, 100000000ull);
        return;
    }
    for (int t = threadIdx.x; t < 32 * B; t += blockDim.x) {
        const int l = t & 31, b = t >> 5;
        if (b < batch && l < rows) {
            float sum = 0.f;
            for (int k = 0; k < nw; ++k) sum += red[(k * B + b) * 32 + l];
            y[(long)b * W.N + row0 + l] = sum;
        }
    }
}

// TMA kernel (K % 256 == 0): a CTA owns 32 consecutive rows; one thread
// stages them with 2-D TMA boxes (32 rows x 128 bytes, a handful of requests
// per CTA) issued before waiting on the previous kernel of the stream; the
// CTA prepares the activation planes while the boxes land; warp w then dots
// slices w, w+nw, ... of every row (lane = row) against the broadcast
// activation blocks; the per-warp partial sums are added in warp order.
template <int QT, int B>
__global__ void __launch_bounds__(256, 2) qgemv_tma_kernel(const __grid_constant__ CUtensorMap tmw,
                                                           const __grid_constant__ CUtensorMap tmd, QView W,
                                                           const float *__restrict__ x, float *__restrict__ y,
                                                           int batch, int *status) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    const int K = W.K, nxb = K / 32, ns = K / 256;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int row0 = blockIdx.x * 32;
    const int rows = min(32, W.N - row0);
    // TMA 128-byte swizzle needs 1024-byte aligned boxes
    uint8_t *tile = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
    XBlk *xq = reinterpret_cast<XBlk *>(tile + tma_tile_bytes(QT, K));
    XF *xf = reinterpret_cast<XF *>(xq + B * nxb);
    float *red = reinterpret_cast<float *>(xf + B * nxb);   // [warp][b][lane]
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
        mbar_arrive_expect_tx(&bar, (uint32_t)tma_tile_bytes(QT, K));
        tma_issue_tile(&tmw, &tmd, QT, K, row0, tile, &bar);
    }
    pdl_launch_dependents();
    pdl_wait();
    xprep_all(x, K, batch, xq, xf);
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, status);
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    if (ok && lane < rows) {
        const int nwb = tma_wboxes(QT, K);
        for (int sl = warp; sl < ns; sl += nw) {
            WSlice<QT> ws;
            load_slice_swz<QT>(tile, nwb, lane, sl, ws);
#pragma unroll
            for (int b = 0; b < B; ++b)
                if (b < batch) acc[b] += dot_slice<QT>(ws, xq + b * nxb + sl * 8, xf + b * nxb + sl * 8);
        }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) red[(warp * B + b) * 32 + lane] = acc[b];
    __syncthreads();
    if (abort_flag) {
        if (threadIdx.x == 0) mbar_wait_drain(&bar, 0, 100000000ull);   // boxes still in flight
        return;
    }
    for (int t = threadIdx.x; t < 32 * B; t += blockDim.x) {
        const int l = t & 31, b = t >> 5;
        if (b < batch && l < rows) {
            float sum = 0.f;
            for (int k = 0; k < nw; ++k) sum += red[(k * B + b) * 32 + l];
            y[(long)b * W.N + row0 + l] = sum;
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
    {
        const int wb = (int)row_bytes_dev(qt, K), sb = qscale_row_bytes(qt, K);
        m.tma_ok = make_tmap_2d(&m.tmw, m.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)wb, (uint64_t)N, (uint64_t)wb, 128,
                                32);
        if (m.tma_ok && sb)
            m.tma_ok = make_tmap_2d(&m.tmd, m.d, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)sb, (uint64_t)N, (uint64_t)sb,
                                    128, 32);
        if (!sb) m.tmd = m.tmw;
    }
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
static int launch_slice(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    const int ns = v.K / 256;
    const size_t smem = (size_t)B * (v.K / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)ns * B * 32 * 4;
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_slice_kernel<QT, B>);
        attr[c->device] = true;
    }
    return launch_pdl(qgemv_slice_kernel<QT, B>, dim3((v.N + 31) / 32), dim3(32 * ns), smem, s, v, x, y, batch);
}

// The slice kernel serves K % 256 == 0, K <= 4096 while its shared memory
// fits; other shapes take the unit kernel.
static bool slice_ok(int K, int B) {
    if (K % 256 || K > 4096) return false;
    const size_t smem = (size_t)B * (K / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)(K / 256) * B * 32 * 4;
    return smem <= 200 * 1024;
}

template <int QT, int B>
static int launch_half(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    const int nh = v.K / 128;
    const size_t smem = (size_t)B * (v.K / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)nh * B * 32 * 4;
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_half_kernel<QT, B>);
        attr[c->device] = true;
    }
    return launch_pdl(qgemv_half_kernel<QT, B>, dim3((v.N + 31) / 32), dim3(32 * nh), smem, s, v, x, y, batch);
}

static bool half_ok(int K, int B) {
    if (K % 256 || K > 2048) return false;
    const size_t smem = (size_t)B * (K / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)(K / 128) * B * 32 * 4;
    return smem <= 200 * 1024;
}

template <int QT, int B>
static size_t bulk_smem(int K) {
    const int nw = std::min(K / 256, 8);
    return (size_t)tile_bytes(QT, K, 32) + (size_t)B * (K / 32) * (sizeof(XBlk) + sizeof(XF)) + (size_t)nw * B * 32 * 4;
}

template <int QT, int B>
static int launch_bulk(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    const size_t smem = bulk_smem<QT, B>(v.K);
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_bulk_kernel<QT, B>);
        attr[c->device] = true;
    }
    const int nw = std::min(v.K / 256, 8);
    return launch_pdl(qgemv_bulk_kernel<QT, B>, dim3((v.N + 31) / 32), dim3(32 * nw), smem, s, v, x, y, batch,
                      c->d_status);
}

template <int QT, int B>
static size_t ws_smem(int K) {
    const int ns = K / 256, nw = std::min(ns, 8), spw = (ns + nw - 1) / nw;
    return (size_t)nw * spw * ws_slice_tile<QT>() + (size_t)nw * spw * 8 * B * (sizeof(XBlk) + sizeof(XF)) +
           (size_t)nw * B * 32 * 4;
}

template <int QT, int B>
static int launch_ws(DevCtx *c, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    const size_t smem = ws_smem<QT, B>(v.K);
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_ws_kernel<QT, B>);
        attr[c->device] = true;
    }
    const int nw = std::min(v.K / 256, 8);
    return launch_pdl(qgemv_ws_kernel<QT, B>, dim3((v.N + 31) / 32), dim3(32 * nw), smem, s, v, x, y, batch,
                      c->d_status);
}

template <int QT, int B>
static size_t tma_smem(int K) {
    const int nw = std::min(K / 256, 8);
    return 1024 + (size_t)tma_tile_bytes(QT, K) + (size_t)B * (K / 32) * (sizeof(XBlk) + sizeof(XF)) +
           (size_t)nw * B * 32 * 4;
}

template <int QT, int B>
static int launch_tma(DevCtx *c, const QMat &m, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    const size_t smem = tma_smem<QT, B>(v.K);
    static bool attr[64];
    if (!attr[c->device]) {
        set_qkernel_attrs(qgemv_tma_kernel<QT, B>);
        attr[c->device] = true;
    }
    const int nw = std::min(v.K / 256, 8);
    return launch_pdl(qgemv_tma_kernel<QT, B>, dim3((v.N + 31) / 32), dim3(32 * nw), smem, s, m.tmw, m.tmd, v, x, y,
                      batch, c->d_status);
}

template <int QT, int B>
static int launch_B(DevCtx *c, const QMat &m, const QView &v, const float *x, float *y, int batch, cudaStream_t s) {
    static const int mode = [] { const char *e = getenv("X100_GEMV_KERNEL"); return e ? atoi(e) : 0; }();
    if (mode == 0 && m.tma_ok && v.K % 256 == 0 && tma_smem<QT, B>(v.K) <= 200 * 1024)
        return launch_tma<QT, B>(c, m, v, x, y, batch, s);
    if (mode == 3 && v.K % 256 == 0 && ws_smem<QT, B>(v.K) <= 200 * 1024) return launch_ws<QT, B>(c, v, x, y, batch, s);
    if (mode <= 1 && v.K % 256 == 0 && bulk_smem<QT, B>(v.K) <= 200 * 1024)
        return launch_bulk<QT, B>(c, v, x, y, batch, s);
    if (half_ok(v.K, B)) return launch_half<QT, B>(c, v, x, y, batch, s);
    if (slice_ok(v.K, B)) return launch_slice<QT, B>(c, v, x, y, batch, s);
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
    if (!attr[c->device][0]) {
        set_qkernel_attrs(qgemv_kernel<QT, B, RR>);
        attr[c->device][0] = true;
    }
    long grid = (passes + 7) / 8;
    const long cap = (long)c->sm_count * 4;
    if (grid > cap) grid = cap;
    return launch_pdl(qgemv_kernel<QT, B, RR>, dim3((unsigned)grid), dim3(256), smem, s, v, x, y, batch, lpr);
}

template <int QT>
static int launch_qt(DevCtx *c, const QMat &m, const float *x, float *y, int batch, cudaStream_t s) {
    const QView v = qmat_view(m, 0);
    if (batch <= 1) return launch_B<QT, 1>(c, m, v, x, y, batch, s);
    if (batch <= 2) return launch_B<QT, 2>(c, m, v, x, y, batch, s);
    if (batch <= 4) return launch_B<QT, 4>(c, m, v, x, y, batch, s);
    if (batch <= 8) return launch_B<QT, 8>(c, m, v, x, y, batch, s);
    return launch_B<QT, 16>(c, m, v, x, y, batch, s);
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
