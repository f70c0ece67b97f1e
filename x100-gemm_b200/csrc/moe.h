// moe.h -- resident mixture-of-experts layer and its launcher (moe.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "qgemv.h"

namespace x100 {

namespace q {
constexpr int kMaxDXB = 256;   // hidden size up to 8192 (256 activation blocks)
}

// Weights of one MoE layer resident in HBM: fp32 router [n_exp][d] and the
// local experts [lo, hi): gate/up rows (hi-lo)*ffn x d, down (hi-lo)*d x ffn.
struct MoeLayer {
    int d = 0, n_exp = 0, n_act = 0, ffn = 0, qtype = 0, lo = 0, hi = 0;
    float *router = nullptr;
    QMat gate, up, down;
    // plan of the fused one-token expert kernel (moe_fused_plan): grid,
    // dynamic shared memory and the bytes of it that hold staged rows;
    // fused_ok false when it does not fit
    bool fused_ok = false;
    int fused_grid = 0, fused_tiles = 0;
    size_t fused_smem = 0;
};

// Device scratch of one call (batch <= 16): routing logits, selection,
// weights, SwiGLU intermediates h[token][slot][ffn], the counters, and for
// the batched path the expert groups, the prepared activations of every token
// and the per-slot partial outputs part[token][slot][d].
struct MoeScratch {
    unsigned *ticket = nullptr;
    float *logits = nullptr;
    int *sel = nullptr;
    float *w = nullptr;
    float *h = nullptr;
    int *cnt = nullptr;   // completion counter of the fused expert kernel
    // groups: [0, n_exp) tokens per local expert, [n_exp] active experts,
    // [n_exp + 1, 2 n_exp + 1) active expert list, then pairs[n_exp][16]
    int *grp = nullptr;
    uint8_t *xq = nullptr;   // prepared activations, one token after the other
    float *part = nullptr;
    uint8_t *hq = nullptr;   // prepared h of the (expert, token) slots, slot after slot
};

bool moe_shapes_ok(int d, int n_exp, int n_act, int ffn, int qtype);
// Fill L.fused_* for a device with sm_count SMs (after the weights are uploaded).
void moe_fused_plan(MoeLayer &L, int sm_count);
size_t moe_scratch_bytes(int d, int n_exp, int n_act, int ffn);
MoeScratch moe_scratch_carve(void *base, int d, int n_exp, int n_act, int ffn);
// eout[b][:] for b < batch; hn, eout device pointers; asynchronous on s.
int launch_moe(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *hn, float *eout, int batch,
               cudaStream_t s);
// Options of a MoE call inside a decode step: norm_w (d floats) makes the
// input the residual stream x, RMS-normed by the router kernel into hn_out
// (batch x d) for the experts; accum adds the block output into eout.
struct MoeOpts {
    const float *norm_w = nullptr;
    float eps = 1e-6f;
    float *hn_out = nullptr;
    bool accum = false;
    // step timing: mark(mark_ctx, bucket, s) before the router, expert and
    // combine launches (buckets of x100q_model_timing)
    void (*mark)(void *ctx, int bucket, cudaStream_t s) = nullptr;
    void *mark_ctx = nullptr;
    // batch > 1, eout summed in one process: the combine also prepares the
    // next GEMV's activations from the rows it writes (qgemv_prep_group's
    // layout: groups of next_ntok tokens, next_nxb blocks a token, blocks of
    // row * next_nw and each block's sum of squares of the row in next_qs);
    // next_xbm null: not
    uint8_t *next_xbm = nullptr;
    float *next_qs = nullptr;
    const float *next_nw = nullptr;
    int next_ntok = 0, next_nxb = 0;
};
// Scratch of the many-token (prefill) MoE path for up to `tmax` tokens:
// routing, the (token, slot) pairs sorted by expert, their activations as
// fp16 hi / lo planes, the gate / up outputs, h planes and per-pair outputs.
struct MoeBigScratch {
    int tmax = 0;
    float *hn = nullptr;          // [tmax][d] normed tokens (router input)
    __half *xt_hi = nullptr, *xt_lo = nullptr;   // [tmax][kp_d] token planes
    float *logits = nullptr;      // [tmax][n_exp]
    int *sel = nullptr;           // [tmax][n_act]
    float *w = nullptr;           // [tmax][n_act]
    int *cnt = nullptr;           // [n_exp] tokens per local expert, then [n_exp] fill counters
    int *pair_at = nullptr;       // [tmax * n_act] pair (token * n_act + slot) at each sorted position
    __half *xg_hi = nullptr, *xg_lo = nullptr;   // [tmax * n_act][kp_d] planes of each pair's token
    float *gu = nullptr;          // [tmax * n_act][2 ffn] gate then up outputs
    __half *hh_hi = nullptr, *hh_lo = nullptr;   // [tmax * n_act][kp_f] silu(g) * u planes
    float *part = nullptr;        // [tmax * n_act][d] unweighted expert outputs per pair
};
size_t moe_big_scratch_bytes(int d, int n_exp, int n_act, int ffn, int tmax);
MoeBigScratch moe_big_scratch_carve(void *base, int d, int n_exp, int n_act, int ffn, int tmax);
// h[t] += MoE(rmsnorm(h[t], norm_w)) for T <= S.tmax tokens (the experts this
// layer holds; with a partial range, h receives this process's share): router
// logits, top-k per token, the pairs sorted by expert, the experts' gate / up
// and down layers as grouped tensor-core GEMMs (launch_qgemm), combine in
// slot order.
int launch_moe_prefill(DevCtx *c, const MoeLayer &L, const MoeBigScratch &S, float *h, int T, const float *norm_w,
                       float eps, cudaStream_t s);

int launch_moe_ex(DevCtx *c, const MoeLayer &L, const MoeScratch &S, const float *x, float *eout, int batch,
                  const MoeOpts &o, cudaStream_t s);
// Upload router [n_exp][d] and experts [lo, hi) of GGUF-native gate/up/down
// blocks (host or device pointers, the full [n_exp] tensors) into L and plan
// the fused kernel; synchronous.  On failure L holds nothing and the error is
// recorded.
bool moe_layer_upload(DevCtx *c, MoeLayer &L, int d, int n_exp, int n_act, int ffn, int qtype, const float *router,
                      const void *gate_exps, const void *up_exps, const void *down_exps, int lo, int hi);
void moe_layer_free(MoeLayer &L);

}  // namespace x100
