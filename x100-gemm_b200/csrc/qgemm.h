// qgemm.h -- many-token quantised linear layers on the tcgen05 tensor cores
// (the prefill path) and the activation preparation they take.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "qgemv.h"

namespace x100 {

// Output of one launch (per item's token rows t and weight rows n):
//   QG_STORE    out[t * ldo + col] = acc
//   QG_ADD      out[t * ldo + col] += acc   (the residual stream)
//   QG_SCATTER  out[pair_at[t] * ldo + col] = acc
// col = mat * n_rows + n: with two matrices per group (gate and up) their
// outputs sit side by side in one row.
enum { QG_STORE = 0, QG_ADD = 1, QG_SCATTER = 2 };

// Y = W . X for token rows of X, X given as fp16 planes (x ~= hi + lo, the
// rounding of x to fp16 and of the remainder), rows of kp halfs (kp = 256 *
// slices of W, zero past K).
//   dense:   ngroups = 1, cnt = null: tokens 0 .. T-1 against all n_rows
//            rows of mats[0].
//   grouped: ngroups experts; group g's tokens are rows [start_g, start_g +
//            cnt[g]) of X (start = exclusive prefix of cnt, device memory),
//            against rows [g * n_rows, (g+1) * n_rows) of each of the
//            nmat matrices.
// Asynchronous on s; launched with programmatic dependent launch.
struct QgLaunch {
    const QMat *mats[2] = {nullptr, nullptr};
    int nmat = 1;
    int n_rows = 0;
    int ngroups = 1;
    const int *cnt = nullptr;
    int T = 0;
    const __half *xh = nullptr, *xl = nullptr;
    long x_rows = 0;   // rows of the X planes
    int mode = QG_STORE;
    float *out = nullptr;
    long ldo = 0;
    const int *pair_at = nullptr;
};
int launch_qgemm(DevCtx *c, const QgLaunch &L, cudaStream_t s);

// hi / lo fp16 planes [rows][kp] of fp32 rows src [rows] (row pitch lds,
// first K values used, zero from K to kp).  With nw the rows are RMS-normed
// first, x * nw / sqrt(mean(x^2) + eps) (qwen_moe_q3k.c:1166); f32_out (may
// be null) then also receives the normed fp32 rows [rows][K].
int launch_split_rows(const float *src, long lds, int K, int kp, int rows, const float *nw, float eps, __half *hi,
                      __half *lo, float *f32_out, cudaStream_t s);

// h = silu(g) * u (qwen_moe.c:309) of gu [rows][2 * ffn] (gate then up) into
// fp16 hi / lo planes [rows][kp] (zero from ffn to kp).
int launch_swiglu_split(const float *gu, int ffn, int kp, int rows, __half *hi, __half *lo, cudaStream_t s);

}  // namespace x100
