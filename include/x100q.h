/*
 * x100q.h -- C ABI of the block-quantised decode path (dequant-GEMV and the
 * top-k SwiGLU mixture-of-experts FFN) served by sm_100a CUDA kernels in
 * libx100gemm_b200.so.
 *
 * The reference keeps this path inside its single-file engines as static
 * functions called from forward():
 *   Lin lin_new_{hp,i8,q3k}(...)        qwen_moe_q3k.c:843,872,897 (qwen_moe.c:66)
 *   pack_act_{hp,i8,q3k}(x, K, Abuf)    qwen_moe_q3k.c:860,887,624
 *   lin_mm_{hp,i8,q3k}(&lin, Abuf, y)   qwen_moe_q3k.c:1029,1040,1048
 *   MoE block in forward()              qwen_moe.c:295-311, qwen_moe_q3k.c:1916-1978
 * This header exposes the same steps as a library: a linear is created once
 * from GGUF-native quantised blocks (weights live in HBM afterwards), then
 * applied to fp32 activations; the MoE call does router -> softmax -> top-k
 * -> renormalise -> SwiGLU experts -> weighted combine in one call.
 *
 * Activations stay fp32 end to end (no int8 activation packing): the parity
 * target is the reference's scalar fp32 path.  Calls with host pointers are
 * synchronous; *_dev calls take device pointers and a cudaStream_t and are
 * asynchronous.  Every call returns 0 or an X100_E* code (see x100_gemm.h);
 * constructors return NULL and set x100_last_error() on failure.
 * Handles are not thread-safe: one caller thread per handle at a time.
 */
#ifndef X100Q_H
#define X100Q_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* GGUF / ggml tensor type ids, the values the reference's GGUF reader
 * switches on (qwen_moe.c:158-177, qwen_moe_q3k.c:531).                     */
enum {
    X100Q_F32  = 0,
    X100Q_Q4_0 = 2,    /* 18 B / 32 weights: fp16 d, 16 B nibbles (q-8)*d      */
    X100Q_Q8_0 = 8,    /* 34 B / 32 weights: fp16 d, int8[32]   q*d            */
    X100Q_Q3_K = 11,   /* 110 B / 256: hmask[32] qs[64] scales[12] fp16 d      */
    X100Q_Q4_K = 12    /* 144 B / 256: fp16 d, fp16 dmin, scales[12], qs[128]  */
};

/* Bytes of one GGUF-native row of K weights of type qtype (0 if K is not a
 * multiple of the type's block size or qtype is unknown).                   */
size_t x100q_row_bytes(int qtype, int K);

/* ---- quantised linear ---------------------------------------------------- */
typedef struct x100q_lin x100q_lin;

/* Create an N x K linear from N rows of GGUF-native blocks (host pointer,
 * row-major, K/blocksize blocks per row).  Replaces lin_new_q3k
 * (qwen_moe_q3k.c:897-909, which also reads raw GGUF blocks) and lin_new_hp /
 * lin_new_i8 (:843, :872).  Blocks are uploaded once and re-laid-out on the
 * device for 16-byte vector loads.                                          */
x100q_lin *x100q_lin_create(int qtype, int N, int K, const void *blocks);
void       x100q_lin_destroy(x100q_lin *lin);
int        x100q_lin_info(const x100q_lin *lin, int *qtype, int *N, int *K,
                          size_t *device_bytes);

/* y[b*N + n] = sum_k W[n][k] * x[b*K + k] for b < batch (1 <= batch <= 16).
 * Replaces pack_act_* + lin_mm_* (qwen_moe_q3k.c:1029-1082): one call per
 * linear per step.  x and y may be host or device pointers.                 */
int x100q_lin_gemv(const x100q_lin *lin, const float *x, float *y, int batch);
int x100q_lin_gemv_dev(const x100q_lin *lin, const float *x, float *y, int batch,
                       void *stream);
/* As x100q_lin_gemv_dev, with flags.  X100Q_GEMV_INDEPENDENT: the caller
 * guarantees that x and y are neither written nor read by work still running
 * on `stream` (e.g. the q, k and v projections of one activation, or repeated
 * calls as the reference's bench/q4_gemv.c times them); the call then reads x
 * without waiting for the previous kernel, so consecutive independent calls
 * overlap and stream their weights back to back.  Calls still complete in
 * stream order.                                                             */
#define X100Q_GEMV_INDEPENDENT 1
/* X100Q_GEMV_A8: the activations are first quantised as the reference packs
 * them for its IME kernels -- pack_A_i8 (qwen_moe_q3k.c:420-426, int8 per 32
 * values) for Q8_0 weights, pack_A_q3k (:613-623, int8 per 256) for Q3_K,
 * pack_A_hp (qwen_moe_hp.c:131-180, int8 per 32 under fp16 scales relative
 * to a per-256 average) for Q4_0 (K % 256 == 0), the format of the int4
 * "HP" engine -- and the integer block dots are scaled by the packed scales
 * (HP: fp16 sub-scale x fp16 average), so the result follows the
 * reference's A8 numerics instead of the fp32-activation oracle (a few 1e-3
 * relative apart).  Other weight types: X100_E_UNSUPPORTED.                 */
#define X100Q_GEMV_A8 2
int x100q_lin_gemv_dev_flags(const x100q_lin *lin, const float *x, float *y, int batch,
                             int flags, void *stream);
/* pack_act_i8 / pack_act_q3k / pack_act_hp (qwen_moe_q3k.c:887, :624;
 * qwen_moe_hp.c:530) on the device: rows x [batch][K] (fp32, device, 16-byte
 * aligned) into the reference's packed records, bit for bit: mode
 * X100Q_PACK_I8 writes K/32 records of 38 bytes (fp32 scale, int16 sum of
 * q, int8 q[32]) per row, X100Q_PACK_Q3K K/256 records of 292 bytes (fp32
 * scale, int16 negated sums of 16, int8 q[256]), X100Q_PACK_HP K/256
 * records of 290 bytes (8 x [fp16 sub-scale / average, int8 q[32]], 8 fp16
 * -8 * sum(q), fp16 average scale; fp16 by the engine's truncating
 * conversion, qwen_moe_hp.c:71-79); rows follow each other in out.
 * Asynchronous on `stream`.                                                 */
#define X100Q_PACK_I8  1
#define X100Q_PACK_Q3K 2
#define X100Q_PACK_HP  3
int x100q_pack_act_dev(int mode, const float *x, int K, int batch, void *out, void *stream);

/* ---- mixture-of-experts FFN ---------------------------------------------- */
typedef struct x100q_moe x100q_moe;

/* d: hidden size; n_exp experts, n_act active per token (top-k, k <= 16);
 * ffn: expert intermediate size; qtype: expert weight type (Q4_0, Q4_K,
 * Q3_K or Q8_0).  router: fp32 [n_exp][d] (ffn_gate_inp.weight).
 * gate_exps / up_exps: GGUF-native blocks [n_exp][ffn][d]; down_exps:
 * [n_exp][d][ffn] -- the reference's blk.N.ffn_{gate,up,down}_exps tensors
 * (qwen_moe.c:215-222).  Only experts [expert_lo, expert_hi) are uploaded and
 * evaluated by this handle (expert parallelism: each process holds a slice;
 * the router is replicated so every process knows the full top-k).          */
x100q_moe *x100q_moe_create(int d, int n_exp, int n_act, int ffn, int qtype,
                            const float *router, const void *gate_exps,
                            const void *up_exps, const void *down_exps,
                            int expert_lo, int expert_hi);
void       x100q_moe_destroy(x100q_moe *moe);

/* For each of `batch` tokens (1 <= batch <= 16), hn[b][d] -> eout[b][d]:
 *   logits = router . hn;  p = softmax(logits);  top-k by p (strict >, lowest
 *   index wins ties);  w = p_sel / sum(p_sel);
 *   eout = sum over selected experts held by this handle of
 *          w_a * down_a( silu(gate_a . hn) * (up_a . hn) )
 * (qwen_moe.c:295-311).  sel_out [batch][n_act] and w_out [batch][n_act]
 * receive the routing (may be NULL).  With a partial expert range, eout is
 * this process's partial sum; summing eout over all processes (NCCL reduce)
 * gives the full block output.                                              */
int x100q_moe_ffn(const x100q_moe *moe, const float *hn, float *eout, int batch,
                  int *sel_out, float *w_out);
int x100q_moe_ffn_dev(const x100q_moe *moe, const float *hn, float *eout, int batch,
                      int *sel_out, float *w_out, void *stream);

/* No counterpart in the reference.  Router -> softmax -> top-k ->
 * renormalise for `batch` tokens, the routing step of x100q_moe_ffn, for
 * callers that may not allocate GPU memory: code whose device memory is owned
 * by a framework pool or a fixed, pre-committed budget, and hot loops that
 * cannot afford cudaMalloc/cudaFree (which may synchronise the device).  The
 * library allocates nothing here, not even its per-device context: the
 * routing logits and the completion ticket live in a fixed static device
 * array of 256 + 8192 bytes that every GPU which loads the library holds
 * until exit.  Limit: batch * n_exp <= 2048 (e.g. 16 tokens x 128 experts),
 * larger requests return X100_E_TOO_LARGE; also 1 <= batch <= 16,
 * 1 <= n_exp <= 256, 1 <= n_act <= min(16, n_exp), d % 4 == 0.
 * router [n_exp][d] and hn [batch][d] (fp32, 16-byte aligned), sel_out
 * [batch][n_act] and w_out [batch][n_act] are device pointers on the calling
 * thread's current CUDA device; the work is enqueued on `stream` and the call
 * returns without synchronising.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  The address is cached per device together with the id
 * of the CUDA context it was taken in; after a device reset (a new context)
 * the next call looks it up again, so that call too should come before any
 * capture.  All calls share the one array: calls whose work
 * overlaps on the GPU (other streams, other threads) race and must be
 * serialised by the caller.                                                 */
int x100q_router_topk_noalloc(const float *router, const float *hn, int d, int n_exp,
                              int n_act, int batch, int *sel_out, float *w_out,
                              void *stream);

/* ---- decode step of a whole model ----------------------------------------- */
/* The reference's forward(Model*, tok, pos, Kv*, logits, ...)
 * (qwen_moe_q3k.c:1842-1983) for a Qwen3-MoE-shaped model: per layer
 *   hn = rmsnorm(h, attn_norm);  q, k, v = Wq/Wk/Wv . hn;
 *   q, k per head: rmsnorm(., q_norm / k_norm) then NEOX RoPE (base rope_base);
 *   k, v stored to the KV cache at pos;  att = softmax(q.K^T / sqrt(hd)) . V
 *   over positions 0..pos (query head hh uses kv head hh / (n_heads/n_kv_heads));
 *   h += Wo . att;  h += MoE(rmsnorm(h, ffn_norm))  (the x100q_moe_ffn block);
 * then logits = Wlm . rmsnorm(h, out_norm).
 * Differences from the reference, by design: the KV cache is fp16 (the
 * reference keeps fp32), activations are never int8-packed, and up to
 * max_batch independent sequences (slots 0..batch-1) advance together.     */
typedef struct x100q_model x100q_model;

typedef struct {
    int n_layers, d, n_heads, n_kv_heads, head_dim, vocab;
    int n_exp, n_act, moe_ffn;
    int attn_qtype;      /* q/k/v/o weights (Q8_0 in the BASELINE config)       */
    int expert_qtype;    /* expert gate/up/down (Q3_K)                          */
    int lm_qtype;        /* lm_head                                             */
    int ctx;             /* KV positions per sequence                           */
    int max_batch;       /* sequences stepped together, 1..16                   */
    int expert_lo, expert_hi;   /* experts held by this process ([0, n_exp): all) */
    float rope_base, eps;
} x100q_model_cfg;

/* Allocates the KV caches (2 * n_layers * max_batch * n_kv_heads * ctx *
 * head_dim fp16, zeroed) and scratch; weights are added with set_layer /
 * set_output.  head_dim must be 128, n_heads / n_kv_heads <= 8, d and
 * n_heads * head_dim multiples of 256, ctx <= 131072.                       */
x100q_model *x100q_model_create(const x100q_model_cfg *cfg);
void         x100q_model_destroy(x100q_model *m);

/* Weights of one layer (host or device pointers, uploaded once):
 * attn_norm/ffn_norm fp32 [d]; q_norm/k_norm fp32 [head_dim];
 * wq [n_heads*head_dim][d], wk/wv [n_kv_heads*head_dim][d],
 * wo [d][n_heads*head_dim] as GGUF-native attn_qtype blocks;
 * router fp32 [n_exp][d]; gate/up [n_exp][moe_ffn][d], down [n_exp][d][moe_ffn]
 * as expert_qtype blocks (only [expert_lo, expert_hi) are kept).            */
int x100q_model_set_layer(x100q_model *m, int layer, const float *attn_norm,
                          const void *wq, const void *wk, const void *wv,
                          const float *q_norm, const float *k_norm, const void *wo,
                          const float *ffn_norm, const float *router,
                          const void *gate_exps, const void *up_exps,
                          const void *down_exps);
/* tok_embd fp32 [vocab][d] (may be NULL: callers then pass hidden states),
 * out_norm fp32 [d], lm [vocab][d] lm_qtype blocks (may be NULL: no logits). */
int x100q_model_set_output(x100q_model *m, const float *tok_embd,
                           const float *out_norm, const void *lm);

/* Copy positions [pos0, pos0+npos) of sequence slot `slot`, layer `layer`
 * between the cache and k, v (host or device), each laid out
 * [n_kv_heads][npos][head_dim] fp16: to_cache = 1 writes the cache (e.g. a
 * prompt's keys and values), 0 reads it.  Synchronous.                      */
int x100q_model_kv_copy(x100q_model *m, int layer, int slot, int pos0, int npos,
                        void *k, void *v, int to_cache);

/* Device-pointer steps, asynchronous on `stream` (calling thread's current
 * device).  h: [batch][d] residual stream, updated in place; pos: [batch]
 * positions (each < ctx; a larger one leaves h undefined and makes the next
 * synchronising call report X100_E_ARG).
 * layer_dev with eout == NULL adds the MoE output into h (all experts
 * held); with eout set it writes this process's experts' share to eout
 * [batch][d] and the caller sums eout over processes and adds it to h.
 * sel_out / w_out [batch][n_act] (may be NULL) receive the routing.         */
int x100q_model_embed_dev(x100q_model *m, const int *tokens, float *h, int batch,
                          void *stream);
int x100q_model_layer_dev(x100q_model *m, int layer, float *h, const int *pos,
                          int batch, float *eout, int *sel_out, float *w_out,
                          void *stream);
int x100q_model_head_dev(x100q_model *m, const float *h, float *logits, int batch,
                         void *stream);
/* embed (when tokens != NULL) + every layer + head (when logits != NULL).   */
int x100q_model_forward_dev(x100q_model *m, const int *tokens, float *h,
                            const int *pos, float *logits, int batch, void *stream);
/* Synchronous host-pointer step: tokens, pos [batch] -> logits [batch][vocab]
 * (needs tok_embd and lm).                                                  */
int x100q_model_forward(x100q_model *m, const int *tokens, const int *pos,
                        float *logits, int batch);
/* Per-token sequence slots: as x100q_model_forward_dev, with token b using
 * the cache of slot[b] (a device array of batch ints, each in
 * [0, max_batch)) instead of slot b, so several tokens of one sequence, at
 * different positions, can step together.  Every token's k and v are
 * written to the cache before any token attends, and token b attends over
 * positions 0 .. pos[b] of its slot, which takes in the step's own earlier
 * positions (causal, as the reference's prefill).  Two tokens with the same
 * slot and position are the caller's error; a slot out of range writes
 * nothing and makes the next synchronising call report X100_E_ARG.          */
int x100q_model_forward_slots_dev(x100q_model *m, const int *tokens, float *h, const int *pos,
                                  const int *slot, float *logits, int batch, void *stream);
/* Prefill: the reference's prefill_chunk4 (qwen_moe_hp.c:1748-1858) for
 * n >= 1 tokens -- tokens[0 .. n) of the sequence in `slot` at positions
 * pos0 .. pos0 + n - 1 (pos0 + n <= ctx), their k and v left in the cache;
 * logits [n][vocab] (host, or NULL for none).  Up to max_batch tokens run as
 * one decode step; more run in chunks (1024 tokens, X100_PREFILL_CHUNK
 * overrides, 32 .. 4096) whose linear layers are tensor-core GEMMs over all
 * the chunk's tokens.  Synchronous.                                         */
int x100q_model_prefill(x100q_model *m, int slot, const int *tokens, int n, int pos0, float *logits);

/* ---- per-bucket step timing ------------------------------------------------ */
/* The reference's decode-step buckets (qwen_moe_q3k.c:910-941, printed per
 * token at :2295-2327: act-pack, linear {qkv, o, expert, lm_head},
 * attention, rope+qknorm, router, swiglu, rest) at this library's kernel
 * boundaries.  Activation packing is fused into each linear's kernel,
 * rope + q/k norm into the attention kernel and swiglu into the expert
 * kernels, so those time under their hosts:
 *   EMBED    token embedding
 *   QKV      rmsnorm + packing + the q/k/v linear
 *   ATTN     k/v cache write, q/k norm, rope, attention, split merge
 *   O        the output linear (+ residual)
 *   ROUTER   rmsnorm + router logits + top-k (+ grouping at batch > 1)
 *   EXPERT   gate / up / swiglu / down of the routed experts
 *   COMBINE  weighted sum of the experts' outputs into the residual
 *   LM       final rmsnorm + lm_head
 * x100q_model_timing(m, 1) clears the totals and starts timing; every
 * forward call (x100q_model_forward, _forward_dev, _forward_slots_dev and
 * _layer_dev) then records a CUDA event at each bucket boundary (which
 * serialises the kernels on either side, so the sum runs a little above an
 * untimed step), and x100q_model_timing(m, 0) stops.  Calls made while the
 * stream is being captured into a graph record nothing.
 * x100q_model_timing_read waits for the recorded events and writes the
 * totals since the start, in milliseconds, to ms[X100Q_NBUCKETS] and the
 * number of timed calls to *steps (either may be NULL).                    */
enum {
    X100Q_T_EMBED = 0, X100Q_T_QKV, X100Q_T_ATTN, X100Q_T_O, X100Q_T_ROUTER,
    X100Q_T_EXPERT, X100Q_T_COMBINE, X100Q_T_LM, X100Q_NBUCKETS
};
int x100q_model_timing(x100q_model *m, int on);
int x100q_model_timing_read(x100q_model *m, double *ms, long *steps);
/* "embed", "qkv", "attention", "o", "router", "expert", "combine", "lm";
 * NULL out of range.                                                        */
const char *x100q_timing_bucket_name(int bucket);

/* ---- expert-parallel combine over peer memory ------------------------------ */
/* With experts split over `world` processes (one per GPU, x100q_moe_create
 * with [expert_lo, expert_hi) or a model with a partial expert range), each
 * process's eout is a partial sum; the reference's single-process block
 * (qwen_moe.c:305-310) is their sum.  x100q_ep_* sums them with one kernel
 * over NVLink peer memory instead of a library all-reduce: each process
 * writes its partial into every process's receive buffer, raises a flag, and
 * adds the world partials in process order once all flags are up, so every
 * process ends with the same bits.  Setup: create on every process (same
 * world, max_floats), exchange the X100Q_EP_HANDLE_BYTES handles (e.g. an
 * all-gather over the host), then open with all handles in rank order.  The
 * waits are bounded (1 s): a missing process makes the next synchronising
 * call report X100_E_TIMEOUT instead of hanging.  Every process must make the
 * same sequence of calls with the same n.                                   */
#define X100Q_EP_HANDLE_BYTES 64
typedef struct x100q_ep x100q_ep;

/* world <= 8; max_floats (a multiple of 4) bounds n of every call.          */
x100q_ep *x100q_ep_create(int world, int rank, int max_floats);
int       x100q_ep_handle(const x100q_ep *ep, void *handle_out);
int       x100q_ep_open(x100q_ep *ep, const void *all_handles);
/* dst[i] = (accum ? dst[i] : 0) + sum over processes of their src[i], i < n
 * (n a multiple of 4, src/dst 16-byte aligned device pointers; dst may be
 * src when accum = 0).  Asynchronous on `stream`.                           */
int       x100q_ep_allreduce_dev(x100q_ep *ep, const float *src, float *dst, int n,
                                 int accum, void *stream);
void      x100q_ep_destroy(x100q_ep *ep);

/* ---- GGUF ingest ----------------------------------------------------------
 * Replaces the reference's GGUF reader and model loader (gguf_open /
 * gguf_find / gguf_dequant_into / model_load, qwen_moe_q3k.c:1086-1159 and
 * :1742-1787; qwen_moe.c:110-181).  The file is mapped read-only; every
 * offset and length read from it is checked against the file size, and a
 * malformed file, a missing tensor or an unusable type is reported as
 * X100_E_FORMAT (the reference prints and exits).  Tensor data is decoded or
 * re-quantised on the device when loaded.                                   */

/* The further ggml tensor types the loader decodes (with those above).      */
enum {
    X100Q_F16  = 1,
    X100Q_Q4_1 = 3,    /* 20 B / 32: fp16 d, fp16 m, 16 B nibbles  nib*d + m   */
    X100Q_Q5_K = 13,   /* 176 B / 256: d, dmin, scales[12], qh[32], qs[128]    */
    X100Q_Q6_K = 14    /* 210 B / 256: ql[128], qh[64], int8 scales[16], d     */
};

typedef struct x100q_gguf x100q_gguf;

typedef struct {
    const char *name;     /* NUL-terminated, owned by the handle              */
    int type;             /* ggml type id                                     */
    int n_dims;           /* 1..4                                             */
    uint64_t dims[4];     /* dims[0] is the contiguous row length             */
    uint64_t n_elems;
    uint64_t bytes;       /* size of the data; 0 for a type without a known size */
    const void *data;     /* inside the mapped file (host memory)            */
} x100q_gguf_tensor;

/* Map and parse a GGUF file (versions 2 and 3).  NULL + x100_last_error()
 * on failure (X100_E_FORMAT for a malformed file, X100_E_ARG for a path that
 * cannot be opened).  No GPU is needed until a model is loaded.             */
x100q_gguf *x100q_gguf_open(const char *path);
void        x100q_gguf_close(x100q_gguf *g);
int         x100q_gguf_n_tensors(const x100q_gguf *g);
/* Tensor i in file order, or the tensor called `name`: 0, X100_E_ARG (index
 * out of range), X100_E_FORMAT (no such tensor).                           */
int         x100q_gguf_tensor_at(const x100q_gguf *g, int i, x100q_gguf_tensor *out);
int         x100q_gguf_find(const x100q_gguf *g, const char *name, x100q_gguf_tensor *out);
/* Byte offset of the tensor data section in the file.                      */
uint64_t    x100q_gguf_data_offset(const x100q_gguf *g);
/* tokenizer.ggml.tokens: count, and token `id` (NULL when out of range).   */
int         x100q_gguf_n_tokens(const x100q_gguf *g);
const char *x100q_gguf_token(const x100q_gguf *g, int id);
/* Metadata by key: 0, X100_E_FORMAT (absent or not convertible).  get_int
 * reads any integer or bool type; get_f32 reads F32 or F64; get_str returns
 * a NUL-terminated copy owned by the handle.                               */
int         x100q_gguf_get_int(const x100q_gguf *g, const char *key, int64_t *out);
int         x100q_gguf_get_f32(const x100q_gguf *g, const char *key, float *out);
int         x100q_gguf_get_str(const x100q_gguf *g, const char *key, const char **out);

/* Model configuration of a qwen3moe file, read as the reference reads it
 * (qwen_moe_q3k.c:1098-1126, :1742-1744): qwen3moe.{block_count,
 * embedding_length, attention.head_count, attention.head_count_kv,
 * attention.key_length, expert_count (default 128), expert_used_count (8),
 * expert_feed_forward_length (768), rope.freq_base (1e6)}; eps 1e-6; vocab =
 * dims[1] of token_embd.weight.  Weight types: attn_qtype is the type every
 * layer's attn_q/k/v/output share when the decode GEMV takes it, else Q8_0;
 * expert_qtype likewise for the expert tensors; lm_qtype is output.weight's
 * type when the GEMV takes it, else Q8_0 (also for a tied lm_head).  ctx =
 * 4096, max_batch = 1, all experts: edit these before loading.             */
int x100q_gguf_model_cfg(const x100q_gguf *g, x100q_model_cfg *cfg);

/* Create a model with `cfg` (dimensions as x100q_gguf_model_cfg reads them)
 * and upload every layer's weights from the file: a tensor whose type is the
 * slot's is uploaded as it is; any other decodable type is decoded to fp32
 * on the device and, for a weight slot, re-quantised to Q8_0 as the
 * reference's lin_new_i8 does (quantize_q8_0_native, qwen_moe_q3k.c:409-414),
 * so a slot of another type takes only its own type.  fp32 slots (norms,
 * router, token embeddings) take any decodable type.  A missing
 * output.weight ties the lm_head to the token embeddings (Q8_0 of them,
 * qwen_moe_q3k.c:1747-1750).  NULL + x100_last_error() on failure.         */
x100q_model *x100q_model_load_gguf(const x100q_gguf *g, const x100q_model_cfg *cfg);

/* Device decoders used by the loader, asynchronous on `stream`:
 * n elements of GGUF `type` data (device pointer, n a whole number of
 * blocks) to fp32, bit-identical to the reference's gguf_dequant_into
 * (qwen_moe_q3k.c:1129-1158; Q4_K as its Q5_K decoder with a zero fifth bit);
 * and n fp32 values (n % 32 == 0) to Q8_0 blocks as quantize_q8_0_native.  */
int x100q_gguf_dequant_dev(int type, const void *data, long n, float *out, void *stream);
int x100q_quantize_q8_0_dev(const float *x, long n, void *blocks, void *stream);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* X100Q_H */
