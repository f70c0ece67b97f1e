/*
 * x100_oracle.h -- CPU restatement of the reference's scalar algorithms for
 * the x100-gemm hot path.  TEST INFRASTRUCTURE ONLY: the parity tests, the
 * smoke check and bench.py's CPU-baseline leg call it as the checker.  It is
 * never linked into libx100gemm_b200.so and never used as a product path.
 *
 * Every function cites the reference file:line it restates (paths relative
 * to the docdailey/x100-gemm tree).
 */
#ifndef X100_ORACLE_H
#define X100_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dense GEMM (C += A*B, row-major, beta = 1) ------------------------- */
void orc_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C);
void orc_gemm_f32(int M, int N, int K, const float *A, const float *B, float *C);
/* row-sliced over `nthreads` POSIX threads (same per-row arithmetic)       */
void orc_gemm_i8_mt(int M, int N, int K, const int8_t *A, const int8_t *B, int32_t *C, int nthreads);
void orc_gemm_f32_mt(int M, int N, int K, const float *A, const float *B, float *C, int nthreads);
/* IME-2 packed layouts of src/gemm_ime2_i8.c:40-56 */
void orc_ime2_pack_a(int M, int K, const int8_t *A, int8_t *pa);
void orc_ime2_pack_b(int K, int N, const int8_t *B, int8_t *pb);

/* ---- fp16 ---------------------------------------------------------------- */
float    orc_f16_to_f32(uint16_t h);          /* qwen_moe.c:115-118          */
uint16_t orc_f32_to_f16_rne(float f);         /* IEEE round-to-nearest-even  */
uint16_t orc_f32_to_f16_trunc(float f);       /* qwen_moe_hp.c:71-79         */

/* ---- block formats: sizes ------------------------------------------------ */
enum { ORC_F32 = 0, ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q3_K = 11, ORC_Q4_K = 12 };
/* further ggml types a GGUF file may hold (decode only) */
enum { ORC_F16 = 1, ORC_Q4_1 = 3, ORC_Q5_K = 13, ORC_Q6_K = 14 };
int    orc_block_elems(int qtype);            /* 32 or 256                    */
int    orc_block_bytes(int qtype);            /* 18, 34, 110, 144             */
size_t orc_row_bytes(int qtype, int K);

/* ---- block formats: decode (n elements = whole blocks) ------------------ */
void orc_dequant_row(int qtype, const void *blocks, int K, float *out);
/* n elements (a whole number of blocks) of a GGUF tensor of any type
 * gguf_dequant_into decodes (qwen_moe_q3k.c:1129-1158): F32, F16, Q4_0,
 * Q4_1, Q8_0, Q3_K, Q4_K, Q5_K, Q6_K.  Returns 0, or -1 for another type.  */
int orc_dequant_gguf(int type, const void *data, size_t n, float *out);
/* Bytes of n elements of a GGUF tensor of `type` (0: unknown type or n not a
 * whole number of blocks). */
size_t orc_gguf_bytes(int type, size_t n);
/* quantize_q8_0_native (qwen_moe_q3k.c:409-414) over n floats (n % 32 == 0):
 * amax from 1e-6, d = amax/127, q = lrint(w/d) clamped to [-128, 127], d
 * stored as the truncating fp16 of qwen_moe_q3k.c:71-79.                    */
void orc_quantize_q8_0_ref(const float *x, size_t n, void *blocks);

/* The reference's activation packers for its IME kernels ("A8"):
 * pack_A_i8 (qwen_moe_q3k.c:420-426), 38 B per 32 values: fp32 scale =
 * max(|x|, 1e-6)/127, int16 sum of q, int8 q = lrint(x/scale) clamped;
 * pack_A_q3k (:613-623), 292 B per 256: fp32 scale = max|x|/127, 16 int16
 * negated sums of 16, int8 q = roundf(x/scale) clamped.  K % 32 / K % 256.  */
void orc_pack_a_i8(const float *x, int K, void *out);
void orc_pack_a_q3k(const float *x, int K, void *out);
/* pack_A_hp (qwen_moe_hp.c:131-180), 290 B per 256 values: 8 x [fp16
 * sub-scale / average, int8 q[32]], 8 fp16 -8*sum(q), fp16 average scale;
 * fp16 by the engine's truncating f32_to_f16 (qwen_moe_hp.c:71-79).  K%256. */
void orc_pack_a_hp(const float *x, int K, void *out);
/* quantize_q4_0_native (qwen_moe_hp.c:102-109): the HP kernels' Q4_0 weights
 * (d = max(|w|,1e-6)/8 truncated to fp16, q in [-8, 7]); n % 32 == 0.       */
void orc_quantize_q4_0_hp(const float *x, size_t n, void *blocks);
/* y[b][n] = W[n] . (x[b] packed as above): Q8_0 weights with pack_A_i8,
 * Q3_K with pack_A_q3k, Q4_0 with pack_A_hp; exact integer block dots, each
 * block's (Q8_0, Q4_0) or sub-block's (Q3_K) term scaled in fp32 (Q4_0:
 * d * ((fp16 sub-scale * fp16 average) * dot)) and summed in double in k
 * order.                                                                     */
void orc_qgemv_a8(int qtype, int N, int K, const void *blocks, const float *x, float *y, int batch);
/* scale/min pair j of a K-quant 12-byte scale array (qwen_moe_q3k.c:534-538,
 * repack.cpp:222-233)                                                      */
void orc_kq_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m);

/* ---- block formats: encode (own encoders; the reference has no Q4_K/Q3_K
 * encoder).  w has K elements per row, N rows.                             */
void orc_quantize(int qtype, int N, int K, const float *w, void *blocks);

/* ---- dequant-GEMV (fp32 x, fp32 accumulate in k order) ------------------- */
/* y[b*N+n] = sum_k dequant(W)[n][k] * x[b*K+k]                             */
void orc_qgemv(int qtype, int N, int K, const void *blocks, const float *x, float *y, int batch);
void orc_qgemv_mt(int qtype, int N, int K, const void *blocks, const float *x, float *y,
                  int batch, int nthreads);

/* ---- MoE block (qwen_moe.c:295-311) -------------------------------------- */
void orc_softmax(float *x, int n);            /* qwen_moe.c:189              */
/* greedy top-k over p: strict >, lowest index wins, sentinel -1e30 (or -1
 * for the qwen_moe.c variant -- identical for softmax probabilities).      */
void orc_topk(const float *p, int n, int k, int *sel, float *w);
float orc_silu(float x);                      /* x/(1+expf(-x)), qwen_moe.c:309 */
void orc_moe_ffn(int d, int n_exp, int n_act, int ffn, int qtype,
                 const float *router, const void *gate_exps, const void *up_exps,
                 const void *down_exps, int expert_lo, int expert_hi,
                 const float *hn, float *eout, int batch, int *sel_out, float *w_out,
                 int nthreads);

/* ---- decode-step pieces (qwen_moe_q3k.c:1166-1175, qwen_moe.c:186-189) -- */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps);
void orc_rope_neox(float *v, int hd, int pos, float base);
/* one layer of forward() for one token (qwen_moe_q3k.c:1849-1978), fp16
 * KV cache [nkv][ctx][hd] updated at pos; h updated in place              */
void orc_decode_layer(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                      int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                      const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                      const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                      const float *router, const void *gate_exps, const void *up_exps,
                      const void *down_exps, uint16_t *kc, uint16_t *vc, float *h,
                      int *sel_out, float *w_out, int nthreads);
/* the same layer with an fp32 cache [nkv][ctx][hd] (the reference's own
 * cache precision): the variant pinned against the reference's forward()    */
void orc_decode_layer_f32kv(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                            int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                            const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                            const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                            const float *router, const void *gate_exps, const void *up_exps,
                            const void *down_exps, float *kc, float *vc, float *h,
                            int *sel_out, float *w_out, int nthreads);
/* orc_decode_layer that also writes the router's softmax probabilities
 * (probs_out, n_exp floats): how close the top-k came to a tie.             */
void orc_decode_layer_probs(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                            int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                            const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                            const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                            const float *router, const void *gate_exps, const void *up_exps,
                            const void *down_exps, uint16_t *kc, uint16_t *vc, float *h,
                            int *sel_out, float *w_out, float *probs_out, int nthreads);
/* logits = lm . rmsnorm(h, out_norm)  (qwen_moe_q3k.c:1980-1981)          */
void orc_decode_head(int d, int vocab, float eps, int lm_qtype, const float *out_norm, const void *lm,
                     const float *h, float *logits, int nthreads);

/* ---- seeded generators (xorshift64 13/7/17 of bench/q3k_probe.c:403-405) */
uint64_t orc_rng_seed(uint64_t s);
uint32_t orc_rng_u32(uint64_t *state);
void     orc_fill_u8(uint64_t seed, uint8_t *dst, size_t n);

#ifdef __cplusplus
}
#endif
#endif
