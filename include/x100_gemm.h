/*
 * x100_gemm.h -- drop-in C ABI of the x100-gemm GEMM library, served by
 * hand-written sm_100a (B200) CUDA kernels in libx100gemm_b200.so.
 *
 * Every symbol of the reference header keeps its name, argument list and
 * meaning (reference include/x100_gemm.h:30-61):
 *
 *   C[M x N] += A[M x K] * B[K x N]      (beta = 1: zero C first for C = A*B)
 *   row-major, contiguous, lda = K, ldb = N, ldc = N; int dimensions.
 *   Pointers may be host memory (pageable or pinned) or CUDA device memory;
 *   the library detects which.  Calls are synchronous: C is valid on return.
 *
 * The reference's functions return void and have no error channel.  They keep
 * that signature here; a failure leaves C untouched where possible and is
 * reported through x100_last_error() / x100_strerror(), never by aborting.
 *
 * Additions (new symbols; the reference ones are untouched):
 *   - gemm_rvv_f16 is exported on every host (the reference declares it only
 *     under __riscv_zvfh, include/x100_gemm.h:54-56);
 *   - gemm_f16_f32acc: fp16 inputs, fp32 accumulate and fp32 C;
 *   - *_dev variants: device pointers, caller-chosen cudaStream_t, no copies,
 *     asynchronous, int status return;
 *   - gemm_ime2_* : the packed-operand IME-2 driver of the reference's
 *     src/gemm_ime2_i8.c:40-147 (packed layouts accepted as-is);
 *   - error reporting and device selection.
 */
#ifndef X100_GEMM_H
#define X100_GEMM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* ---- capability detection ------------------------------------------------
 * Byte-identical layout to the reference struct (include/x100_gemm.h:30-39).
 * On a B200 the fields mean: vlen_bits / vlenb = 0 (no RVV), has_v = 0,
 * has_zvfh = 1 (fp16 GEMM available), has_zvbb = 0, has_ime = 1 when the
 * tcgen05 tensor-core path is usable (compute capability 10.x), mvendorid =
 * 0x10de (NVIDIA PCI vendor id), isa = "<gpu name> sm_XX <n> SMs ...".      */
typedef struct {
    int  vlen_bits;
    int  vlenb;
    int  has_v;
    int  has_zvfh;
    int  has_zvbb;
    int  has_ime;
    unsigned long mvendorid;
    char isa[1024];
} x100_caps_t;

/* replaces x100_detect (reference src/x100_caps.c:24-62) */
void x100_detect(x100_caps_t *caps);
/* replaces x100_caps_print (reference src/x100_caps.c:64-76) */
void x100_caps_print(const x100_caps_t *caps);

/* ---- GEMM backends (all C += A*B) ---------------------------------------- */

/* replaces gemm_ref_f32 (reference src/gemm_ref.c:5-14).  GPU kernel that
 * keeps the reference's summation order: for each (i,j), k ascending,
 * c = c + a*b with separately rounded multiply and add, so the result is
 * bit-identical to the scalar reference built without -ffast-math.        */
void gemm_ref_f32 (int M, int N, int K, const float *A, const float *B, float *C);
/* replaces gemm_rvv_f32 (reference src/gemm_rvv_f32.c:15-63).  Fast fp32
 * GEMM (fp32 operands, fp32 accumulate).                                    */
void gemm_rvv_f32 (int M, int N, int K, const float *A, const float *B, float *C);

/* replaces gemm_rvv_f16 (reference src/gemm_rvv_f16.c:15-57): fp16 A, B, C.
 * Products accumulate in fp32 on the tensor cores (tcgen05 kind::f16); the
 * fp16 C is read, added in fp32 and rounded once to fp16.                   */
void gemm_rvv_f16 (int M, int N, int K, const _Float16 *A, const _Float16 *B, _Float16 *C);
/* new: fp16 A, B; fp32 accumulate; fp32 C (C += A*B).                       */
void gemm_f16_f32acc(int M, int N, int K, const _Float16 *A, const _Float16 *B, float *C);

/* replaces gemm_ref_i8 (reference src/gemm_ref.c:17-26): exact int8 x int8
 * -> int32 on CUDA cores.                                                    */
void gemm_ref_i8  (int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C);
/* replaces gemm_ime_i8 (reference src/gemm_ime_i8.c:60-89): exact int8 x
 * int8 -> int32 on the tcgen05 tensor cores (kind::i8, TMEM accumulator).  */
void gemm_ime_i8  (int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C);

/* ---- packed-operand driver (reference src/gemm_ime2_i8.c) ----------------
 * Same packed layouts as the reference:
 *   pa[(mb*Kb+kb)*128 + r*16 + c]           = A[(mb*8+r)*K + kb*16 + c]
 *   pb[((ng*Kb+kb)*8+g)*128 + nin*16 + kin] = B[(kb*16+kin)*N + (ng*8+g)*8 + nin]
 * with M%8 == 0, N%64 == 0, K%16 == 0.  gemm_ime2_i8_st / _mt compute
 * C = A*B (they overwrite C, as reference src/gemm_ime2_i8.c:109,136-143 do
 * for the first K panel).  nthreads is accepted and ignored.               */
void gemm_ime2_pack_a(int Mt, int Kt, const int8_t *A, int8_t *pa);           /* :40 */
void gemm_ime2_pack_b(int Kt, int Nt, const int8_t *B, int8_t *pb);           /* :49 */
void gemm_ime2_i8_st(int Mt, int Nt, int Kt, const int8_t *pa, const int8_t *pb,
                     int32_t *C);                                            /* :102 */
void gemm_ime2_i8_mt(int Mt, int Nt, int Kt, const int8_t *pa, const int8_t *pb,
                     int32_t *C, int nthreads);                              /* :116 */

/* ---- device-pointer variants (new) ---------------------------------------
 * A, B, C are device pointers on the current device; the GEMM is enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream) and the call returns
 * without synchronising.  Return 0 or an X100_E* code.                      */
int gemm_ime_i8_dev   (int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, void *stream);
int gemm_ref_i8_dev   (int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, void *stream);
int gemm_f16_f32acc_dev(int M, int N, int K, const void *A, const void *B, float *C, void *stream);
int gemm_f16_dev      (int M, int N, int K, const void *A, const void *B, void *C, void *stream);
int gemm_f32_dev      (int M, int N, int K, const float *A, const float *B, float *C, void *stream);
int gemm_ref_f32_dev  (int M, int N, int K, const float *A, const float *B, float *C, void *stream);
/* int8 GEMM with explicit leading dimensions (elements); tensor cores when
 * A, B are 16-byte aligned and lda, ldb are multiples of 16, CUDA cores
 * otherwise.                                                                */
int gemm_ime_i8_dev_ld(int M, int N, int K, const int8_t *A, long lda, const int8_t *B, long ldb,
                       int32_t *C, long ldc, void *stream);
/* Synchronise `stream` and return the status the library's kernels left in
 * the device status word (0, or X100_E_TIMEOUT when a bounded device-side
 * wait gave up), clearing it.                                               */
int x100_sync(void *stream);

/* ---- errors and device selection (new) ---------------------------------- */
enum {
    X100_OK         = 0,
    X100_E_ARG      = 1,   /* bad dimension / NULL pointer                   */
    X100_E_NODEV    = 2,   /* no usable CUDA device                          */
    X100_E_ARCH     = 3,   /* device is not sm_100 (tcgen05 path needs it)   */
    X100_E_ALLOC    = 4,   /* device or pinned allocation failed             */
    X100_E_COPY     = 5,   /* host<->device copy failed                      */
    X100_E_LAUNCH   = 6,   /* kernel launch or execution failed              */
    X100_E_TIMEOUT  = 7,   /* a device-side wait hit its iteration limit     */
    X100_E_COMM     = 8,   /* collective / peer exchange failed              */
    X100_E_INJECTED = 9,   /* failure injected by X100_FAULT                 */
    X100_E_UNSUPPORTED = 10,
    X100_E_TOO_LARGE = 11, /* request exceeds a fixed-size scratch area      */
    X100_E_FORMAT   = 12   /* malformed file, or a tensor missing / of a type that cannot be used */
};
/* Last status recorded on the calling thread (0 when the last call worked). */
int         x100_last_error(void);
const char *x100_strerror(int code);
/* Select the CUDA device used by later calls on this thread (default: the  */
/* thread's current CUDA device, so one process per GPU needs no call).      */
int         x100_set_device(int device);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* X100_GEMM_H */
