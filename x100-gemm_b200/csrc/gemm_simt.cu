// gemm_simt.cu -- CUDA-core GEMM kernels:
//   * exact int8 GEMM for operand layouts TMA cannot address (ragged
//     leading dimensions) and for gemm_ref_i8 (src/gemm_ref.c:17-26);
//   * reference-order fp32 GEMM for gemm_ref_f32 (src/gemm_ref.c:5-14):
//     per output, k ascending, separately rounded multiply and add, which is
//     bit-identical to the scalar loop compiled without FMA contraction;
//   * fast fp32 / fp16-operand GEMM (FFMA, 128 x 128 tiles, 8 x 8 outputs
//     per thread) for gemm_rvv_f32 (src/gemm_rvv_f32.c:15-63) and the fp16
//     fallback;
//   * unpacking of the IME-2 packed operands (src/gemm_ime2_i8.c:39-56).
#include <cuda_fp16.h>

#include "gemm_kernels.h"

namespace x100 {

// ---- exact int8 --------------------------------------------------------------
namespace {
constexpr int I8_BM = 64, I8_BN = 64, I8_BK = 32;

__global__ void __launch_bounds__(256) gemm_i8_simt_kernel(int M, int N, int K, const int8_t *__restrict__ A,
                                                           long lda, const int8_t *__restrict__ B, long ldb,
                                                           int32_t *__restrict__ C, long ldc) {
    __shared__ int32_t As[I8_BK][I8_BM + 4];
    __shared__ int32_t Bs[I8_BK][I8_BN + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * I8_BM, n0 = blockIdx.x * I8_BN;
    int32_t acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += I8_BK) {
        for (int e = threadIdx.x; e < I8_BM * I8_BK; e += 256) {
            int r = e / I8_BK, kk = e % I8_BK;
            int gm = m0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? (int32_t)A[(long)gm * lda + gk] : 0;
        }
        for (int e = threadIdx.x; e < I8_BK * I8_BN; e += 256) {
            int kk = e / I8_BN, cc = e % I8_BN;
            int gk = k0 + kk, gn = n0 + cc;
            Bs[kk][cc] = (gk < K && gn < N) ? (int32_t)B[(long)gk * ldb + gn] : 0;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < I8_BK; ++kk) {
            int32_t a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int gm = m0 + ty * 4 + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int gn = n0 + tx * 4 + j;
            if (gn < N) {
                uint32_t *p = reinterpret_cast<uint32_t *>(&C[(long)gm * ldc + gn]);
                *p = *p + static_cast<uint32_t>(acc[i][j]);
            }
        }
    }
}

// ---- reference-order fp32 --------------------------------------------------------
constexpr int R_T = 16;

__global__ void __launch_bounds__(256) gemm_f32_ref_kernel(int M, int N, int K, const float *__restrict__ A, long lda,
                                                           const float *__restrict__ B, long ldb,
                                                           float *__restrict__ C, long ldc) {
    __shared__ float As[R_T][R_T + 1];
    __shared__ float Bs[R_T][R_T + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i = blockIdx.y * R_T + ty, j = blockIdx.x * R_T + tx;
    float c = (i < M && j < N) ? C[(long)i * ldc + j] : 0.f;
    for (int k0 = 0; k0 < K; k0 += R_T) {
        As[ty][tx] = (i < M && k0 + tx < K) ? A[(long)i * lda + k0 + tx] : 0.f;
        Bs[ty][tx] = (k0 + ty < K && j < N) ? B[(long)(k0 + ty) * ldb + j] : 0.f;
        __syncthreads();
        const int kn = min(R_T, K - k0);
        for (int kk = 0; kk < kn; ++kk) c = __fadd_rn(c, __fmul_rn(As[ty][kk], Bs[kk][tx]));
        __syncthreads();
    }
    if (i < M && j < N) C[(long)i * ldc + j] = c;
}

// ---- fast fp32-accumulate GEMM (fp32 or fp16 operands) --------------------------
constexpr int F_BM = 128, F_BN = 128, F_BK = 8;

__device__ __forceinline__ float ld_f(const float *p) { return __ldg(p); }
__device__ __forceinline__ float ld_f(const __half *p) { return __half2float(p[0]); }
__device__ __forceinline__ void st_acc(float *p, float v) { *p = *p + v; }
__device__ __forceinline__ void st_acc(__half *p, float v) { *p = __float2half_rn(__half2float(*p) + v); }

template <typename TI, typename TC>
__global__ void __launch_bounds__(256) gemm_fast_kernel(int M, int N, int K, const TI *__restrict__ A, long lda,
                                                        const TI *__restrict__ B, long ldb, TC *__restrict__ C,
                                                        long ldc) {
    __shared__ float As[2][F_BK][F_BM + 4];
    __shared__ float Bs[2][F_BK][F_BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * F_BM, n0 = blockIdx.x * F_BN;
    // global-load mapping: A tile 128 x 8 (4 per thread), B tile 8 x 128 (4 per thread)
    const int a_r = tid >> 1, a_k = (tid & 1) * 4;
    const int b_k = tid >> 5, b_c = (tid & 31) * 4;
    float ra[4], rb[4];
    auto load = [&](int k0) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            int gm = m0 + a_r, gk = k0 + a_k + u;
            ra[u] = (gm < M && gk < K) ? ld_f(A + (long)gm * lda + gk) : 0.f;
            int gk2 = k0 + b_k, gn = n0 + b_c + u;
            rb[u] = (gk2 < K && gn < N) ? ld_f(B + (long)gk2 * ldb + gn) : 0.f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            As[buf][a_k + u][a_r] = ra[u];
            Bs[buf][b_k][b_c + u] = rb[u];
        }
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    load(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += F_BK) {
        const bool more = k0 + F_BK < K;
        if (more) load(k0 + F_BK);
#pragma unroll
        for (int kk = 0; kk < F_BK; ++kk) {
            float a[8], b[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[buf][kk][ty * 4 + i];
                a[i + 4] = As[buf][kk][64 + ty * 4 + i];
                b[i] = Bs[buf][kk][tx * 4 + i];
                b[i + 4] = Bs[buf][kk][64 + tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (more) {
            stash(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (gn < N) st_acc(C + (long)gm * ldc + gn, acc[i][j]);
        }
    }
}

// ---- IME-2 packed operands -----------------------------------------------------------
__global__ void ime2_unpack_a(int M, int K, const int8_t *__restrict__ pa, int8_t *__restrict__ A) {
    const long n = (long)M * K;
    const int Kb = K / 16;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < n; idx += (long)gridDim.x * blockDim.x) {
        long tile = idx >> 7;
        int w = (int)(idx & 127), r = w >> 4, cc = w & 15;
        long mb = tile / Kb, kb = tile % Kb;
        A[(mb * 8 + r) * K + kb * 16 + cc] = pa[idx];
    }
}
__global__ void ime2_unpack_b(int K, int N, const int8_t *__restrict__ pb, int8_t *__restrict__ B) {
    const long n = (long)K * N;
    const int Kb = K / 16;
    for (long idx = blockIdx.x * (long)blockDim.x + threadIdx.x; idx < n; idx += (long)gridDim.x * blockDim.x) {
        long t = idx >> 7;
        int w = (int)(idx & 127), nin = w >> 4, kin = w & 15;
        long g = t % 8, rest = t / 8, kb = rest % Kb, ng = rest / Kb;
        B[(kb * 16 + kin) * N + (ng * 8 + g) * 8 + nin] = pb[idx];
    }
}
}  // namespace

int launch_gemm_i8_simt(DevCtx *c, int M, int N, int K, const int8_t *A, long lda, const int8_t *B, long ldb,
                        int32_t *C, long ldc, cudaStream_t s) {
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    dim3 grid((N + I8_BN - 1) / I8_BN, (M + I8_BM - 1) / I8_BM);
    gemm_i8_simt_kernel<<<grid, 256, 0, s>>>(M, N, K, A, lda, B, ldb, C, ldc);
    (void)c;
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_gemm_f32_ref(DevCtx *c, int M, int N, int K, const float *A, long lda, const float *B, long ldb,
                        float *C, long ldc, cudaStream_t s) {
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    dim3 grid((N + R_T - 1) / R_T, (M + R_T - 1) / R_T);
    gemm_f32_ref_kernel<<<grid, 256, 0, s>>>(M, N, K, A, lda, B, ldb, C, ldc);
    (void)c;
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_gemm_f32_fast(DevCtx *c, int M, int N, int K, const float *A, long lda, const float *B, long ldb,
                         float *C, long ldc, cudaStream_t s) {
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    dim3 grid((N + F_BN - 1) / F_BN, (M + F_BM - 1) / F_BM);
    gemm_fast_kernel<float, float><<<grid, 256, 0, s>>>(M, N, K, A, lda, B, ldb, C, ldc);
    (void)c;
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_gemm_f16_simt(DevCtx *c, int M, int N, int K, const void *A, long lda, const void *B, long ldb, void *C,
                         long ldc, bool c_half, cudaStream_t s) {
    if (M <= 0 || N <= 0 || K <= 0) return X100_OK;
    if (fault_injected("launch")) return X100_E_INJECTED;
    dim3 grid((N + F_BN - 1) / F_BN, (M + F_BM - 1) / F_BM);
    const __half *a = static_cast<const __half *>(A), *b = static_cast<const __half *>(B);
    if (c_half)
        gemm_fast_kernel<__half, __half><<<grid, 256, 0, s>>>(M, N, K, a, lda, b, ldb, static_cast<__half *>(C), ldc);
    else
        gemm_fast_kernel<__half, float><<<grid, 256, 0, s>>>(M, N, K, a, lda, b, ldb, static_cast<float *>(C), ldc);
    (void)c;
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

int launch_ime2_unpack(DevCtx *c, int M, int N, int K, const int8_t *pa, const int8_t *pb, int8_t *A, int8_t *B,
                       cudaStream_t s) {
    if (fault_injected("launch")) return X100_E_INJECTED;
    const int blocks = c->sm_count * 8;
    ime2_unpack_a<<<blocks, 256, 0, s>>>(M, K, pa, A);
    ime2_unpack_b<<<blocks, 256, 0, s>>>(K, N, pb, B);
    return check_cuda(cudaGetLastError(), X100_E_LAUNCH);
}

}  // namespace x100
