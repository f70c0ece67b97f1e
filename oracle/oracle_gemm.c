/*
 * oracle_gemm.c -- CPU restatement of the reference's scalar GEMM oracles.
 * TEST INFRASTRUCTURE ONLY (checker for tests/, smoke() and bench.py's
 * cpu_baseline); never part of the product library.
 */
#include "x100_oracle.h"
#include <pthread.h>
#include <stdlib.h>

/* src/gemm_ref.c:17-26 -- i-k-j loop, int32 accumulate into C.  The int32
 * adds wrap modulo 2^32 (done in uint32 here to keep C's overflow defined). */
void orc_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C)
{
    for (int i = 0; i < M; i++) {
        uint32_t *c = (uint32_t *)&C[(size_t)i * N];
        for (int k = 0; k < K; k++) {
            const int32_t a = A[(size_t)i * K + k];
            const int8_t *b = &B[(size_t)k * N];
            for (int j = 0; j < N; j++) c[j] += (uint32_t)(a * (int32_t)b[j]);
        }
    }
}

/* src/gemm_ref.c:5-14 -- i-k-j loop; each step rounds the product and then
 * the sum (this file is built with -ffp-contract=off, no -ffast-math).     */
void orc_gemm_f32(int M, int N, int K, const float *A, const float *B, float *C)
{
    for (int i = 0; i < M; i++) {
        float *c = &C[(size_t)i * N];
        for (int k = 0; k < K; k++) {
            const float a = A[(size_t)i * K + k];
            const float *b = &B[(size_t)k * N];
            for (int j = 0; j < N; j++) c[j] += a * b[j];
        }
    }
}

typedef struct {
    int kind, M, N, K, r0, r1;
    const void *A, *B; void *C;
} gemm_job;

static void *gemm_worker(void *p)
{
    gemm_job *j = (gemm_job *)p;
    int rows = j->r1 - j->r0;
    if (rows <= 0) return NULL;
    if (j->kind == 0)
        orc_gemm_i8(rows, j->N, j->K, (const int8_t *)j->A + (size_t)j->r0 * j->K,
                    (const int8_t *)j->B, (int32_t *)j->C + (size_t)j->r0 * j->N);
    else
        orc_gemm_f32(rows, j->N, j->K, (const float *)j->A + (size_t)j->r0 * j->K,
                     (const float *)j->B, (float *)j->C + (size_t)j->r0 * j->N);
    return NULL;
}

static void gemm_mt(int kind, int M, int N, int K, const void *A, const void *B, void *C, int nt)
{
    if (nt < 1) nt = 1;
    if (nt > M) nt = M > 0 ? M : 1;
    pthread_t *th = (pthread_t *)calloc((size_t)nt, sizeof(pthread_t));
    gemm_job *jb = (gemm_job *)calloc((size_t)nt, sizeof(gemm_job));
    for (int t = 0; t < nt; t++) {
        jb[t] = (gemm_job){kind, M, N, K, (int)((long)M * t / nt), (int)((long)M * (t + 1) / nt), A, B, C};
        if (t) pthread_create(&th[t], NULL, gemm_worker, &jb[t]);
    }
    gemm_worker(&jb[0]);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
    free(th); free(jb);
}

void orc_gemm_i8_mt(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, int nt)
{ gemm_mt(0, M, N, K, A, B, C, nt); }
void orc_gemm_f32_mt(int M, int N, int K, const float *A, const float *B, float *C, int nt)
{ gemm_mt(1, M, N, K, A, B, C, nt); }

/* Packed layouts of src/gemm_ime2_i8.c:39-56: A as [mb][kb][8x16] tiles,
 * B as [ng][kb][g<8][16 K x 8 N transposed] tiles.                          */
void orc_ime2_pack_a(int M, int K, const int8_t *A, int8_t *pa)
{
    int Mb = M / 8, Kb = K / 16;
    for (int mb = 0; mb < Mb; mb++)
        for (int kb = 0; kb < Kb; kb++) {
            int8_t *d = pa + ((size_t)mb * Kb + kb) * 128;
            for (int r = 0; r < 8; r++)
                for (int c = 0; c < 16; c++) d[r * 16 + c] = A[(size_t)(mb * 8 + r) * K + kb * 16 + c];
        }
}

void orc_ime2_pack_b(int K, int N, const int8_t *B, int8_t *pb)
{
    int Kb = K / 16, Ng = N / 64;
    for (int ng = 0; ng < Ng; ng++)
        for (int kb = 0; kb < Kb; kb++)
            for (int g = 0; g < 8; g++) {
                int8_t *d = pb + (((size_t)ng * Kb + kb) * 8 + g) * 128;
                int nb = ng * 8 + g;
                for (int nin = 0; nin < 8; nin++)
                    for (int kin = 0; kin < 16; kin++)
                        d[nin * 16 + kin] = B[(size_t)(kb * 16 + kin) * N + nb * 8 + nin];
            }
}
