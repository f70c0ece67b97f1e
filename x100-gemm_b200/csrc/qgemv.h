// qgemv.h -- resident block-quantised matrices and the dequant-GEMV launcher
// (qgemv.cu), shared by the x100q_lin_* and x100q_moe_* entry points.
#pragma once
#include <cuda_runtime.h>

#include "qformats.cuh"
#include "runtime.h"

namespace x100 {

// A block-quantised N x K matrix resident in HBM in the slice layout of
// qformats.cuh: N contiguous rows of ns slices (row_bytes each).
struct QMat {
    int qtype = 0, N = 0, K = 0, ns = 0;
    long row_bytes = 0;
    uint8_t *w = nullptr;
    size_t bytes = 0;
    const uint8_t *row(long r) const { return w + r * row_bytes; }
};


size_t qtype_block_elems(int qt);
size_t qtype_block_bytes(int qt);
// Upload N rows of GGUF-native blocks (host or device pointer) and re-lay
// them out on the device; synchronous on `s`.  Returns false with the error
// recorded.
bool qmat_upload(DevCtx *c, int qt, int N, int K, const void *blocks, QMat &m, cudaStream_t s);
// y[b*N + n] = sum_k W[n][k] x[b*K + k], b < batch (<= 16); x, y device.
int launch_qgemv(DevCtx *c, const QMat &m, const float *x, float *y, int batch, cudaStream_t s);
// Options of one GEMV launch: norm_w (device, K floats) applies the RMS norm
// x * nw / sqrt(mean(x^2) + eps) to every token first; accum adds into y.
struct GemvOpts {
    const float *norm_w = nullptr;
    float eps = 1e-6f;
    bool accum = false;
    bool pdl = true;   // false: launch behind a full barrier (see launch_k)
    bool indep = false;   // x, y untouched by running kernels: prepare x before the dependency wait
    int a8 = 0;           // activations packed as the reference's IME path: 1 pack_A_i8, 2 pack_A_q3k
    // Scratch of qgemv_prep_bytes(16, K) bytes (or null): with it, a call of
    // 2..16 tokens on the tensor-core kernel prepares the tokens' activations
    // once, in a kernel of its own, instead of in every CTA.  One buffer per
    // stream of calls (the model's own).
    uint8_t *prep = nullptr;
    // prep already holds the call's prepared activations, written by the
    // kernel that produced x in the layout the preparation kernel writes
    // (groups of qgemv_prep_group tokens): the call launches no preparation.
    bool prepared = false;
};
size_t qgemv_prep_bytes(int batch, int K);
// Tokens per block-major group of the prepared activations when the call
// prepares them once in o.prep (the tensor-core kernel with o.prep, no A8
// packing, not independent), else 0.  A producer that writes x may write the
// prepared blocks too (xprep_vals of each 32-element block of x, times
// o.norm_w when the call folds an RMS norm): block j of token t at ((t / g) *
// nxb + j) * g + t % g, 80 bytes each, g = the group, nxb = 8 ceil(K / 256);
// with a norm also each block's sum of squares of x at qgemv_prep_qs(o.prep,
// K)[t * nxb + j] (four squares per lane of eight, summed as the preparation
// kernel does); and set o.prepared.
int qgemv_prep_group(const QMat &m, int batch, const GemvOpts &o);
float *qgemv_prep_qs(uint8_t *prep, int K);
int qgemv_mma_prep_group(const QMat &m, int batch, const GemvOpts &o);   // qgemv_mma.cu
int launch_qgemv_ex(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const GemvOpts &o,
                    cudaStream_t s);
// Several tokens of a Q4_0 / Q8_0 matrix on the tensor cores (qgemv_mma.cu):
// the same integer block dots and summation order as the dp4a kernel.
// launch_qgemv_ex uses it for batch > 1 and for one token on a matrix of
// 65536 rows or more, when qgemv_mma_ok, except for independent calls of up
// to 4 tokens (X100_GEMV_DP4A=1 keeps the dp4a kernel everywhere).
bool qgemv_mma_ok(int qt, int K);
int launch_qgemv_mma(DevCtx *c, const QMat &m, const float *x, float *y, int batch, const GemvOpts &o,
                     cudaStream_t s);

// Launch `kernel` on `s` with programmatic stream serialization (the kernel
// may start while the previous kernel of the stream runs; it orders itself
// with griddepcontrol.wait).  X100_NO_PDL=1 launches without the attribute.
bool pdl_enabled();

// One-time kernel attributes for the quantised path: allow `smem_max` bytes
// of dynamic shared memory and ask for the maximum shared-memory carveout, so
// consecutive kernels of a decode step share one L1/shared split and the SM
// need not be reconfigured (drained) between them.
template <typename F>
void set_qkernel_attrs(F *kernel, int smem_max = 200 * 1024) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
    cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}
// launch_k with pdl = false is an ordinary launch: the kernel starts only
// after all earlier work of the stream has completed (a full barrier).
template <typename... KArgs, typename... Args>
int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
             Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
    return check_cuda(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), X100_E_LAUNCH);
}
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    return launch_k(kernel, grid, block, smem, s, true, args...);
}

}  // namespace x100
