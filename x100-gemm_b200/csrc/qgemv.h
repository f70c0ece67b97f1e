// qgemv.h -- resident block-quantised matrices and the dequant-GEMV launcher
// (qgemv.cu), shared by the x100q_lin_* and x100q_moe_* entry points.
#pragma once
#include <cuda_runtime.h>

#include "qformats.cuh"
#include "runtime.h"

namespace x100 {

// A block-quantised N x K matrix resident in HBM in the device layout of
// qformats.cuh (weights at w, Q4_0/Q8_0 block scales at d).
struct QMat {
    int qtype = 0, N = 0, K = 0;
    void *w = nullptr;
    __half *d = nullptr;
    size_t bytes = 0;
};

size_t qtype_block_elems(int qt);
size_t qtype_block_bytes(int qt);
// Upload N rows of GGUF-native blocks (host pointer) and re-lay them out on
// the device; synchronous on `s`.  Returns false with the error recorded.
bool qmat_upload(DevCtx *c, int qt, int N, int K, const void *blocks, QMat &m, cudaStream_t s);
// Device view of rows [row0, N) of m.
q::QView qmat_view(const QMat &m, long row0);
// y[b*N + n] = sum_k W[n][k] x[b*K + k], b < batch (<= 16); x, y device.
int launch_qgemv(DevCtx *c, const q::QView &v, const float *x, float *y, int batch, cudaStream_t s);

namespace q {
int lanes_per_row(int units);
}

}  // namespace x100
