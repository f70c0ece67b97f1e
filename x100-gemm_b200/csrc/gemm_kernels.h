// gemm_kernels.h -- launchers of the dense GEMM kernels (all C += A*B,
// row-major).  Each returns X100_OK or an X100_E* status (also recorded).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "runtime.h"

namespace x100 {

// tcgen05 tensor-core GEMM (gemm_tc.cu).  lda/ldb in elements; requirements:
// A, B 16-byte aligned, lda*es and ldb*es multiples of 16 bytes, device is
// sm_100.  kind 0: int8 x int8 -> int32 C; kind 1: fp16 -> fp32 C;
// kind 2: fp16 -> fp16 C (fp32 accumulate); kind 3: fp32 -> fp32 C as three
// tf32 products (returns X100_E_UNSUPPORTED where CTA pairs cannot run).
int launch_gemm_tc(DevCtx *c, int kind, int M, int N, int K, const void *A, long lda, const void *B, long ldb,
                   void *C, long ldc, cudaStream_t s);
// True when (A, lda, B, ldb) satisfy the tensor-map alignment rules above.
bool tc_operands_ok(int kind, const void *A, long lda, const void *B, long ldb);
// The pieces of kind 3, for callers that prepare an operand once for several
// products (row panels of one call):
// hi[i] = x[i] rounded to tf32, lo[i] = x[i] - hi[i], i < n;
int tf32_split(DevCtx *c, const float *x, long n, float *hi, float *lo, cudaStream_t s);
// bt[n][k] = hi(B[k][n]), btlo[n][k] = lo(B[k][n]) (row stride ldt >= K,
// ldt * 4 a multiple of 16 bytes);
int tf32_split_transpose(DevCtx *c, const float *B, long ldb, int K, int N, float *bt, float *btlo, long ldt,
                         cudaStream_t s);
// C += A_hi.B_hi + A_hi.B_lo + A_lo.B_hi from split operands (A parts row
// stride lda, B parts transposed with row stride ldt).
int launch_gemm_tf32x3(DevCtx *c, int M, int N, int K, const float *ahi, const float *alo, long lda, const float *bt,
                       const float *btlo, long ldt, float *C, long ldc, cudaStream_t s);

// CUDA-core kernels (gemm_simt.cu).
int launch_gemm_i8_simt(DevCtx *c, int M, int N, int K, const int8_t *A, long lda, const int8_t *B, long ldb,
                        int32_t *C, long ldc, cudaStream_t s);
// Reference-order fp32 GEMM: per output, k ascending, separately rounded
// multiply and add (bit-identical to the scalar reference).
int launch_gemm_f32_ref(DevCtx *c, int M, int N, int K, const float *A, long lda, const float *B, long ldb,
                        float *C, long ldc, cudaStream_t s);
// Fast fp32 GEMM (FFMA, fp32 accumulate).
int launch_gemm_f32_fast(DevCtx *c, int M, int N, int K, const float *A, long lda, const float *B, long ldb,
                         float *C, long ldc, cudaStream_t s);
// fp16 operands on CUDA cores (fallback for layouts TMA cannot address).
// c_half: C is fp16 (else fp32).
int launch_gemm_f16_simt(DevCtx *c, int M, int N, int K, const void *A, long lda, const void *B, long ldb,
                         void *C, long ldc, bool c_half, cudaStream_t s);
// Unpack the IME-2 packed operands of the reference's src/gemm_ime2_i8.c
// into row-major A (M x K) and B (K x N).
int launch_ime2_unpack(DevCtx *c, int M, int N, int K, const int8_t *pa, const int8_t *pb, int8_t *A, int8_t *B,
                       cudaStream_t s);

}  // namespace x100
