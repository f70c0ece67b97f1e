/*
 * oracle_quant.c -- CPU restatement of the reference's block-quantised
 * formats (GGUF Q4_0 / Q8_0 / Q4_K / Q3_K), its scalar dequant-GEMV and its
 * scalar MoE block.  TEST INFRASTRUCTURE ONLY (checker for tests/, smoke()
 * and bench.py's cpu_baseline); never part of the product library.
 *
 * Built with -ffp-contract=off and without -ffast-math so every multiply and
 * add rounds separately, as the reference's scalar C does on x86-64.
 */
#include "x100_oracle.h"
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- fp16 ----------------------------------------------------------------*/

/* qwen_moe.c:115-118 (f16f): sign/exponent/mantissa unpack, subnormals
 * renormalised, exponent 31 -> inf/nan.                                    */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1fu, m = h & 0x3ffu, b;
    if (e == 0) {
        if (m == 0) b = s << 31;
        else {
            int ee = -14;
            while (!(m & 0x400u)) { m <<= 1; ee--; }
            m &= 0x3ffu;
            b = (s << 31) | ((uint32_t)(ee + 127) << 23) | (m << 13);
        }
    } else if (e == 0x1f) b = (s << 31) | (0xffu << 23) | (m << 13);
    else b = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* IEEE-754 binary16 conversion with round-to-nearest-even (what ggml's
 * GGML_FP32_TO_FP16 does); gcc implements the _Float16 cast that way.      */
uint16_t orc_f32_to_f16_rne(float f)
{
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

/* qwen_moe_hp.c:71-79 (f32_to_f16): truncating conversion used by the
 * reference's own Q4_0 encoder for the stored block scale.                  */
uint16_t orc_f32_to_f16_trunc(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t)((x >> 23) & 0xffu) - 127 + 15;
    uint32_t mant = x & 0x7fffffu;
    if (exp <= 0) {
        if (exp < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - exp);
        return (uint16_t)(sign | (mant >> shift));
    }
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)exp << 10) | (mant >> 13));
}

static inline float rd_f16(const uint8_t *p) { uint16_t h; memcpy(&h, p, 2); return orc_f16_to_f32(h); }
static inline void  wr_f16(uint8_t *p, float f) { uint16_t h = orc_f32_to_f16_rne(f); memcpy(p, &h, 2); }

/* ---- sizes ----------------------------------------------------------------*/
int orc_block_elems(int qtype)
{
    switch (qtype) {
    case ORC_F32: return 1;
    case ORC_Q4_0: case ORC_Q8_0: return 32;
    case ORC_Q3_K: case ORC_Q4_K: return 256;
    default: return 0;
    }
}
int orc_block_bytes(int qtype)
{
    switch (qtype) {
    case ORC_F32: return 4;
    case ORC_Q4_0: return 18;   /* fp16 d + 16 B               (qwen_moe.c:164) */
    case ORC_Q8_0: return 34;   /* fp16 d + 32 B               (qwen_moe.c:162) */
    case ORC_Q3_K: return 110;  /* block_q3_K                  (qwen_moe_q3k.c:531) */
    case ORC_Q4_K: return 144;  /* block_q4_K, ggml QK_K = 256 */
    default: return 0;
    }
}
size_t orc_row_bytes(int qtype, int K)
{
    int be = orc_block_elems(qtype);
    if (be <= 0 || K % be) return 0;
    return (size_t)(K / be) * (size_t)orc_block_bytes(qtype);
}

/* ---- decode ---------------------------------------------------------------*/

/* qwen_moe_q3k.c:534-538 == repack.cpp:222-233 (get_scale_min_k4). */
void orc_kq_scale_min(int j, const uint8_t *q, uint8_t *sc, uint8_t *m)
{
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* qwen_moe.c:164-165: element j < 16 is the low nibble of qs[j], j >= 16 the
 * high nibble of qs[j-16]; w = (nib - 8) * d.                               */
static void dq_q4_0(const uint8_t *blk, float *y)
{
    float d = rd_f16(blk);
    const uint8_t *qs = blk + 2;
    for (int j = 0; j < 32; j++) {
        int nib = (j < 16) ? (qs[j] & 0xf) : (qs[j - 16] >> 4);
        y[j] = (float)(nib - 8) * d;
    }
}

/* qwen_moe.c:162-163: w = (int8)q * d. */
static void dq_q8_0(const uint8_t *blk, float *y)
{
    float d = rd_f16(blk);
    for (int j = 0; j < 32; j++) y[j] = (float)(int8_t)blk[2 + j] * d;
}

/* Q4_K superblock: fp16 d @0, fp16 dmin @2, scales[12] @4, qs[128] @16.
 * 64-element chunk c uses scale/min pairs 2c (low nibbles of qs[32c..+31])
 * and 2c+1 (high nibbles) -- the order of repack.cpp:262-283 and of the
 * reference's K-quant decoder qwen_moe_q3k.c:541-552 (which is Q4_K when the
 * fifth bit plane qh is zero).  w = d*sc*q - dmin*m.                        */
static void dq_q4_k(const uint8_t *blk, float *y)
{
    float d = rd_f16(blk), dmin = rd_f16(blk + 2);
    const uint8_t *sc = blk + 4, *qs = blk + 16;
    for (int c = 0; c < 4; c++) {
        uint8_t s0, m0, s1, m1;
        orc_kq_scale_min(2 * c, sc, &s0, &m0);
        orc_kq_scale_min(2 * c + 1, sc, &s1, &m1);
        float d1 = d * (float)s0, mm1 = dmin * (float)m0;
        float d2 = d * (float)s1, mm2 = dmin * (float)m1;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++) y[64 * c + l] = d1 * (float)(q[l] & 0xF) - mm1;
        for (int l = 0; l < 32; l++) y[64 * c + 32 + l] = d2 * (float)(q[l] >> 4) - mm2;
    }
}

/* The 16 six-bit Q3_K sub-block scales (biased by 32) packed in 12 bytes:
 * scale i has low nibble in byte i (i < 8, low half) or byte i-8 (high half),
 * and its top two bits in byte 8 + i%4 at bit 2*(i/4).  This is the unpacking
 * done with kmask1/kmask2 in qwen_moe_q3k.c:560-564.                        */
static void q3k_scales(const uint8_t *s12, int *out)
{
    for (int i = 0; i < 16; i++) {
        int lo = (i < 8) ? (s12[i] & 0xF) : (s12[i - 8] >> 4);
        int hi = (s12[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
        out[i] = (int)(int8_t)(uint8_t)(lo | (hi << 4));
    }
}

/* qwen_moe_q3k.c:557-577: block_q3_K = hmask[32] @0, qs[64] @32,
 * scales[12] @96, fp16 d @108.  Element 128h + 32j + l (h < 2, j < 4,
 * l < 32): 2-bit value (qs[32h+l] >> 2j) & 3, minus 4 when bit (4h+j) of
 * hmask[l] is clear, times d*(scale[8h + 2j + (l >= 16)] - 32).             */
static void dq_q3_k(const uint8_t *blk, float *y)
{
    const uint8_t *hm = blk, *qs = blk + 32;
    float d_all = rd_f16(blk + 108);
    int sc[16];
    q3k_scales(blk + 96, sc);
    for (int h = 0; h < 2; h++) {
        const uint8_t *q = qs + 32 * h;
        for (int j = 0; j < 4; j++) {
            int shift = 2 * j;
            uint8_t m = (uint8_t)(1u << (4 * h + j));
            float dl = d_all * (float)(sc[8 * h + 2 * j] - 32);
            for (int l = 0; l < 16; l++)
                y[128 * h + 32 * j + l] = dl * (float)((int)((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4));
            dl = d_all * (float)(sc[8 * h + 2 * j + 1] - 32);
            for (int l = 16; l < 32; l++)
                y[128 * h + 32 * j + l] = dl * (float)((int)((q[l] >> shift) & 3) - ((hm[l] & m) ? 0 : 4));
        }
    }
}

void orc_dequant_row(int qtype, const void *blocks, int K, float *out)
{
    const uint8_t *b = (const uint8_t *)blocks;
    int be = orc_block_elems(qtype), bb = orc_block_bytes(qtype);
    if (qtype == ORC_F32) { memcpy(out, blocks, (size_t)K * 4); return; }
    for (int i = 0; i < K / be; i++) {
        const uint8_t *blk = b + (size_t)i * bb;
        float *y = out + (size_t)i * be;
        switch (qtype) {
        case ORC_Q4_0: dq_q4_0(blk, y); break;
        case ORC_Q8_0: dq_q8_0(blk, y); break;
        case ORC_Q4_K: dq_q4_k(blk, y); break;
        case ORC_Q3_K: dq_q3_k(blk, y); break;
        }
    }
}

/* ---- the other GGUF tensor types (decode only; loader conversions) -------*/

/* qwen_moe.c:115-118 bit-for-bit; F16 tensors hold plain IEEE halves. */
static void dq_f16(const uint8_t *p, float *y) { *y = rd_f16(p); }

/* qwen_moe_q3k.c:1138 (typ 3): 20 B per 32: fp16 d, fp16 m, 16 B nibbles
 * laid out as Q4_0; w = nib * d + m (two roundings, no fused multiply-add). */
static void dq_q4_1(const uint8_t *blk, float *y)
{
    float d = rd_f16(blk), m = rd_f16(blk + 2);
    const uint8_t *qs = blk + 4;
    for (int j = 0; j < 32; j++) {
        int nib = (j < 16) ? (qs[j] & 0xf) : (qs[j - 16] >> 4);
        float t = (float)nib * d;
        y[j] = t + m;
    }
}

/* qwen_moe_q3k.c:540-551 (dequantize_q5_K_block): block_q5_K = fp16 d @0,
 * fp16 dmin @2, scales[12] @4, qh[32] @16, qs[128] @48.  Chunk c of 64
 * elements: scale/min pairs 2c (low nibbles of qs[32c..+31]) and 2c+1 (high
 * nibbles); the fifth bit of element l of the low half is bit 2c of qh[l], of
 * the high half bit 2c+1.  w = (d*sc)*q - dmin*m.                           */
static void dq_q5_k(const uint8_t *blk, float *y)
{
    float d = rd_f16(blk), dmin = rd_f16(blk + 2);
    const uint8_t *sc = blk + 4, *qh = blk + 16, *qs = blk + 48;
    for (int c = 0; c < 4; c++) {
        uint8_t s0, m0, s1, m1;
        orc_kq_scale_min(2 * c, sc, &s0, &m0);
        orc_kq_scale_min(2 * c + 1, sc, &s1, &m1);
        float d1 = d * (float)s0, mm1 = dmin * (float)m0;
        float d2 = d * (float)s1, mm2 = dmin * (float)m1;
        const uint8_t *q = qs + 32 * c;
        for (int l = 0; l < 32; l++) {
            int v = (q[l] & 0xF) + ((qh[l] >> (2 * c)) & 1) * 16;
            y[64 * c + l] = d1 * (float)v - mm1;
        }
        for (int l = 0; l < 32; l++) {
            int v = (q[l] >> 4) + ((qh[l] >> (2 * c + 1)) & 1) * 16;
            y[64 * c + 32 + l] = d2 * (float)v - mm2;
        }
    }
}

/* qwen_moe_q3k.c:1148-1157 (typ 14): block_q6_K = ql[128] @0, qh[64] @128,
 * int8 scales[16] @192, fp16 d @208.  Half h (128 elements) uses ql[64h..],
 * qh[32h..], scales[8h..]; its quarter t (32 elements, l < 32) takes the low
 * (t = 0, 1) or high (t = 2, 3) nibble of ql[64h + l + 32*(t & 1)], bits
 * 2t..2t+1 of qh[32h + l] as bits 4-5, minus 32, times d * scale[8h + 2t +
 * l/16].                                                                    */
static void dq_q6_k(const uint8_t *blk, float *y)
{
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    float d = rd_f16(blk + 208);
    for (int h = 0; h < 2; h++)
        for (int t = 0; t < 4; t++)
            for (int l = 0; l < 32; l++) {
                int lo = ql[64 * h + l + 32 * (t & 1)];
                lo = (t < 2) ? (lo & 0xF) : (lo >> 4);
                int q = (lo | (((qh[32 * h + l] >> (2 * t)) & 3) << 4)) - 32;
                float ds = d * (float)sc[8 * h + 2 * t + l / 16];
                y[128 * h + 32 * t + l] = ds * (float)q;
            }
}

static int gguf_block(int type, int *elems, int *bytes)
{
    switch (type) {
    case ORC_F32: *elems = 1; *bytes = 4; return 0;
    case ORC_F16: *elems = 1; *bytes = 2; return 0;
    case ORC_Q4_0: *elems = 32; *bytes = 18; return 0;
    case ORC_Q4_1: *elems = 32; *bytes = 20; return 0;
    case ORC_Q8_0: *elems = 32; *bytes = 34; return 0;
    case ORC_Q3_K: *elems = 256; *bytes = 110; return 0;
    case ORC_Q4_K: *elems = 256; *bytes = 144; return 0;
    case ORC_Q5_K: *elems = 256; *bytes = 176; return 0;
    case ORC_Q6_K: *elems = 256; *bytes = 210; return 0;
    default: return -1;
    }
}

size_t orc_gguf_bytes(int type, size_t n)
{
    int be, bb;
    if (gguf_block(type, &be, &bb) || n % (size_t)be) return 0;
    return n / (size_t)be * (size_t)bb;
}

int orc_dequant_gguf(int type, const void *data, size_t n, float *out)
{
    int be, bb;
    if (gguf_block(type, &be, &bb) || n % (size_t)be) return -1;
    const uint8_t *b = (const uint8_t *)data;
    for (size_t i = 0; i < n / (size_t)be; i++) {
        const uint8_t *blk = b + i * (size_t)bb;
        float *y = out + i * (size_t)be;
        switch (type) {
        case ORC_F32: memcpy(y, blk, 4); break;
        case ORC_F16: dq_f16(blk, y); break;
        case ORC_Q4_0: dq_q4_0(blk, y); break;
        case ORC_Q4_1: dq_q4_1(blk, y); break;
        case ORC_Q8_0: dq_q8_0(blk, y); break;
        case ORC_Q3_K: dq_q3_k(blk, y); break;
        case ORC_Q4_K: dq_q4_k(blk, y); break;
        case ORC_Q5_K: dq_q5_k(blk, y); break;
        case ORC_Q6_K: dq_q6_k(blk, y); break;
        }
    }
    return 0;
}

void orc_quantize_q8_0_ref(const float *x, size_t n, void *blocks)
{
    uint8_t *out = (uint8_t *)blocks;
    for (size_t b = 0; b < n / 32; b++) {
        const float *w = x + 32 * b;
        uint8_t *blk = out + 34 * b;
        float amax = 1e-6f;
        for (int i = 0; i < 32; i++) {
            float v = fabsf(w[i]);
            if (v > amax) amax = v;
        }
        float d = amax / 127.0f;
        float inv = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t h = orc_f32_to_f16_trunc(d);
        memcpy(blk, &h, 2);
        for (int i = 0; i < 32; i++) {
            long q = lrintf(w[i] * inv);
            blk[2 + i] = (uint8_t)(int8_t)(q > 127 ? 127 : (q < -128 ? -128 : q));
        }
    }
}

/* ---- the reference's activation packing ("A8") ---------------------------*/

void orc_pack_a_i8(const float *x, int K, void *out)
{
    uint8_t *o = (uint8_t *)out;
    for (int kg = 0; kg < K / 32; kg++) {
        const float *a = x + 32 * kg;
        uint8_t *r = o + 38 * kg;
        float amax = 1e-6f;
        for (int i = 0; i < 32; i++) {
            float v = fabsf(a[i]);
            if (v > amax) amax = v;
        }
        float scale = amax / 127.0f;
        float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
        int32_t sum = 0;
        for (int i = 0; i < 32; i++) {
            long q = lrintf(a[i] * inv);
            q = q > 127 ? 127 : (q < -128 ? -128 : q);
            r[6 + i] = (uint8_t)(int8_t)q;
            sum += (int32_t)q;
        }
        int16_t s16 = (int16_t)sum;
        memcpy(r, &scale, 4);
        memcpy(r + 4, &s16, 2);
    }
}

void orc_pack_a_q3k(const float *x, int K, void *out)
{
    uint8_t *o = (uint8_t *)out;
    for (int sb = 0; sb < K / 256; sb++) {
        const float *a = x + 256 * sb;
        uint8_t *r = o + 292 * sb;
        float amax = 0.0f;
        for (int i = 0; i < 256; i++) {
            float v = fabsf(a[i]);
            if (v > amax) amax = v;
        }
        float scale = amax / 127.0f;
        float rep = scale != 0.0f ? 1.0f / scale : 0.0f;
        memcpy(r, &scale, 4);
        for (int b = 0; b < 16; b++) {
            int32_t sum = 0;
            for (int l = 0; l < 16; l++) {
                int q = (int)roundf(a[16 * b + l] * rep);
                q = q > 127 ? 127 : (q < -128 ? -128 : q);
                r[36 + 16 * b + l] = (uint8_t)(int8_t)q;
                sum += q;
            }
            int16_t s16 = (int16_t)(-sum);
            memcpy(r + 4 + 2 * b, &s16, 2);
        }
    }
}

/* pack_A_hp (qwen_moe_hp.c:131-180), the activation packer of the engine's
 * int4 "HP" kernels, in the scalar form the engine's RVV code was checked
 * byte-identical against (bench/vendor_ime_actpack_probe.c:37-62), with the
 * engine's own truncating f32_to_f16 (qwen_moe_hp.c:71-79).  290 bytes per
 * 256 values: 8 x [fp16 sub-scale relative to the record's average scale,
 * int8 q[32]], 8 fp16 values -8 * (sum of the sub-block's q), the fp16
 * average scale.  Sub-block scale = max(|x|, 1e-6) / 127, average = their
 * in-order sum / 8, q = lrint(x / sub-block scale) clamped to int8.         */
void orc_pack_a_hp(const float *x, int K, void *out)
{
    uint8_t *o = (uint8_t *)out;
    for (int sb = 0; sb < K / 256; sb++) {
        const float *a = x + 256 * sb;
        uint8_t *r = o + 290 * sb;
        float st[8], avg = 0.0f;
        for (int kk = 0; kk < 8; kk++) {
            float amax = 1e-6f;
            for (int i = 0; i < 32; i++) {
                float v = fabsf(a[32 * kk + i]);
                if (v > amax) amax = v;
            }
            st[kk] = amax / 127.0f;
            avg += st[kk];
        }
        avg /= 8;
        const float fac = avg != 0.0f ? 1.0f / avg : 0.0f;
        for (int kk = 0; kk < 8; kk++) {
            const float rep = st[kk] != 0.0f ? 1.0f / st[kk] : 0.0f;
            int32_t sum = 0;
            for (int i = 0; i < 32; i++) {
                long q = lrintf(a[32 * kk + i] * rep);
                q = q > 127 ? 127 : (q < -128 ? -128 : q);
                r[34 * kk + 2 + i] = (uint8_t)(int8_t)q;
                sum += (int32_t)q;
            }
            const uint16_t ss = orc_f32_to_f16_trunc(st[kk] * fac);
            const uint16_t as = orc_f32_to_f16_trunc(-(float)(int16_t)sum * 8.0f);
            memcpy(r + 34 * kk, &ss, 2);
            memcpy(r + 272 + 2 * kk, &as, 2);
        }
        const uint16_t bs = orc_f32_to_f16_trunc(avg);
        memcpy(r + 288, &bs, 2);
    }
}

/* quantize_q4_0_native (qwen_moe_hp.c:102-109): the engine re-quantises its
 * Q4_0 linears for the HP kernels with d = max(|w|, 1e-6) / 8 (stored by the
 * truncating f32_to_f16), q = lrint(w / d) clamped to [-8, 7], nibble q + 8
 * (element l < 16 low nibble of byte l, element l + 16 its high nibble): an
 * ordinary GGUF Q4_0 block.  n % 32 == 0.                                   */
void orc_quantize_q4_0_hp(const float *x, size_t n, void *blocks)
{
    uint8_t *o = (uint8_t *)blocks;
    for (size_t b = 0; b < n / 32; b++) {
        const float *w = x + 32 * b;
        uint8_t *blk = o + 18 * b;
        float amax = 1e-6f;
        for (int i = 0; i < 32; i++) {
            float v = fabsf(w[i]);
            if (v > amax) amax = v;
        }
        const float d = amax / 8.0f, inv = d != 0.0f ? 1.0f / d : 0.0f;
        int q[32];
        for (int i = 0; i < 32; i++) {
            long v = lrintf(w[i] * inv);
            q[i] = (int)(v > 7 ? 7 : (v < -8 ? -8 : v));
        }
        const uint16_t dh = orc_f32_to_f16_trunc(d);
        memcpy(blk, &dh, 2);
        for (int l = 0; l < 16; l++) blk[2 + l] = (uint8_t)(((q[l] + 8) & 15) | (((q[l + 16] + 8) & 15) << 4));
    }
}

/* Effective scale of sub-block kk of an HP record: fp16 sub-scale x fp16
 * average scale, one fp32 product.                                          */
static float hp_scale(const uint8_t *rec, int kk) { return rd_f16(rec + 34 * kk) * rd_f16(rec + 288); }

void orc_qgemv_a8(int qtype, int N, int K, const void *blocks, const float *x, float *y, int batch)
{
    const size_t rb = orc_row_bytes(qtype, K);
    const int rec = qtype == ORC_Q8_0 ? 38 : (qtype == ORC_Q4_0 ? 290 : 292), per = qtype == ORC_Q8_0 ? 32 : 256;
    uint8_t *pa = (uint8_t *)malloc((size_t)(K / per) * rec);
    for (int b = 0; b < batch; b++) {
        if (qtype == ORC_Q8_0) orc_pack_a_i8(x + (size_t)b * K, K, pa);
        else if (qtype == ORC_Q4_0) orc_pack_a_hp(x + (size_t)b * K, K, pa);
        else orc_pack_a_q3k(x + (size_t)b * K, K, pa);
        for (int n = 0; n < N; n++) {
            const uint8_t *w = (const uint8_t *)blocks + (size_t)n * rb;
            double acc = 0.0;
            if (qtype == ORC_Q4_0) {
                for (int kg = 0; kg < K / 32; kg++) {
                    const uint8_t *blk = w + 18 * kg, *r = pa + 290 * (kg / 8);
                    const int kk = kg % 8;
                    int32_t dot = 0;
                    for (int i = 0; i < 32; i++) {
                        const int nib = i < 16 ? (blk[2 + i] & 15) : (blk[2 + i - 16] >> 4);
                        dot += (nib - 8) * (int8_t)r[34 * kk + 2 + i];
                    }
                    acc += (double)(rd_f16(blk) * (hp_scale(r, kk) * (float)dot));
                }
            } else if (qtype == ORC_Q8_0) {
                for (int kg = 0; kg < K / 32; kg++) {
                    const uint8_t *blk = w + 34 * kg, *r = pa + 38 * kg;
                    float sa;
                    memcpy(&sa, r, 4);
                    int32_t dot = 0;
                    for (int i = 0; i < 32; i++) dot += (int8_t)blk[2 + i] * (int8_t)r[6 + i];
                    acc += (double)(rd_f16(blk) * (sa * (float)dot));
                }
            } else {
                for (int sb = 0; sb < K / 256; sb++) {
                    const uint8_t *blk = w + 110 * sb, *r = pa + 292 * sb, *hm = blk, *qs = blk + 32;
                    float sa;
                    memcpy(&sa, r, 4);
                    const float d = rd_f16(blk + 108);
                    int sc[16];
                    q3k_scales(blk + 96, sc);
                    for (int e = 0; e < 256; e += 16) {   /* sub-block e / 16 */
                        int32_t dot = 0;
                        for (int k = e; k < e + 16; k++) {
                            const int h = k >> 7, t = (k >> 5) & 3, l = k & 31;
                            const int q = (int)((qs[32 * h + l] >> (2 * t)) & 3) - ((hm[l] >> (4 * h + t)) & 1 ? 0 : 4);
                            dot += q * (int8_t)r[36 + k];
                        }
                        const int i = 8 * (e >> 7) + 2 * ((e >> 5) & 3) + ((e >> 4) & 1);
                        acc += (double)(d * (float)(sc[i] - 32) * (sa * (float)dot));
                    }
                }
            }
            y[(size_t)b * N + n] = (float)acc;
        }
    }
    free(pa);
}

/* ---- encode (own encoders, written from the format definitions) ---------*/

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Q4_0 with the BASELINE rule: d = max|w|/7 (fp32, floor 1e-6 as in
 * qwen_moe.c:70-72), q = lrintf(w/d) clamped to +-7, stored nibble q+8 and
 * fp16(d).                                                                  */
static void enc_q4_0(const float *w, uint8_t *blk)
{
    float amax = 1e-6f;
    for (int i = 0; i < 32; i++) { float a = fabsf(w[i]); if (a > amax) amax = a; }
    float s = amax / 7.0f, inv = 1.0f / s;
    int q[32];
    for (int i = 0; i < 32; i++) q[i] = clampi((int)lrintf(w[i] * inv), -7, 7) + 8;
    wr_f16(blk, s);
    for (int l = 0; l < 16; l++) blk[2 + l] = (uint8_t)((q[l] & 0xF) | ((q[l + 16] & 0xF) << 4));
}

static void enc_q8_0(const float *w, uint8_t *blk)
{
    float amax = 1e-6f;
    for (int i = 0; i < 32; i++) { float a = fabsf(w[i]); if (a > amax) amax = a; }
    float s = amax / 127.0f, inv = 1.0f / s;
    wr_f16(blk, s);
    for (int i = 0; i < 32; i++) blk[2 + i] = (uint8_t)(int8_t)clampi((int)lrintf(w[i] * inv), -127, 127);
}

/* Q4_K: per 32-element sub-block an affine (scale, min) pair; the pairs are
 * quantised to 6 bits against the superblock's fp16 d and dmin.            */
static void enc_q4_k(const float *w, uint8_t *blk)
{
    float scl[8], mns[8], maxs = 0.f, maxm = 0.f;
    for (int j = 0; j < 8; j++) {
        float mn = w[32 * j], mx = w[32 * j];
        for (int l = 1; l < 32; l++) { float v = w[32 * j + l]; if (v < mn) mn = v; if (v > mx) mx = v; }
        if (mn > 0.f) mn = 0.f;
        scl[j] = (mx - mn) / 15.0f;
        mns[j] = -mn;
        if (scl[j] > maxs) maxs = scl[j];
        if (mns[j] > maxm) maxm = mns[j];
    }
    wr_f16(blk, maxs / 63.0f);
    wr_f16(blk + 2, maxm / 63.0f);
    float d = rd_f16(blk), dmin = rd_f16(blk + 2);
    int sc[8], mq[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0.f ? clampi((int)lrintf(scl[j] / d), 0, 63) : 0;
        mq[j] = dmin > 0.f ? clampi((int)lrintf(mns[j] / dmin), 0, 63) : 0;
    }
    uint8_t *s = blk + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mq[j + 4] & 0xF) << 4));
    }
    int q[256];
    for (int j = 0; j < 8; j++) {
        float dd = d * (float)sc[j], mm = dmin * (float)mq[j];
        for (int l = 0; l < 32; l++)
            q[32 * j + l] = dd > 0.f ? clampi((int)lrintf((w[32 * j + l] + mm) / dd), 0, 15) : 0;
    }
    uint8_t *qs = blk + 16;
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++)
            qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
}

/* Q3_K: per 16-element sub-block a signed scale chosen so the largest-|w|
 * element maps to -4; scales quantised to 6 bits (biased 32) against fp16 d;
 * values q in [-4, 3] stored as v = q + 4: low two bits in qs, bit 2 in
 * hmask (set bit = no -4 offset).                                            */
static void enc_q3_k(const float *w, uint8_t *blk)
{
    float s[16], maxs = 0.f;
    for (int j = 0; j < 16; j++) {
        float best = 0.f;
        for (int l = 0; l < 16; l++) { float v = w[16 * j + l]; if (fabsf(v) > fabsf(best)) best = v; }
        s[j] = -best / 4.0f;
        if (fabsf(s[j]) > maxs) maxs = fabsf(s[j]);
    }
    memset(blk, 0, 110);
    wr_f16(blk + 108, maxs / 32.0f);
    float d = rd_f16(blk + 108);
    int lsc[16];
    for (int j = 0; j < 16; j++) lsc[j] = d > 0.f ? clampi((int)lrintf(s[j] / d), -32, 31) : 0;
    uint8_t *s12 = blk + 96;
    for (int k = 0; k < 8; k++)
        s12[k] = (uint8_t)(((lsc[k] + 32) & 0xF) | (((lsc[k + 8] + 32) & 0xF) << 4));
    for (int r = 0; r < 4; r++) {
        uint8_t v = 0;
        for (int g = 0; g < 4; g++) v |= (uint8_t)((((lsc[4 * g + r] + 32) >> 4) & 3) << (2 * g));
        s12[8 + r] = v;
    }
    uint8_t *hm = blk, *qs = blk + 32;
    for (int h = 0; h < 2; h++)
        for (int j = 0; j < 4; j++)
            for (int l = 0; l < 32; l++) {
                int e = 128 * h + 32 * j + l;
                int is = 8 * h + 2 * j + (l >= 16);
                float dd = d * (float)lsc[is];
                int q = dd != 0.f ? clampi((int)lrintf(w[e] / dd), -4, 3) : 0;
                int v = q + 4;
                qs[32 * h + l] |= (uint8_t)((v & 3) << (2 * j));
                if (v & 4) hm[l] |= (uint8_t)(1u << (4 * h + j));
            }
}

void orc_quantize(int qtype, int N, int K, const float *w, void *blocks)
{
    uint8_t *b = (uint8_t *)blocks;
    int be = orc_block_elems(qtype), bb = orc_block_bytes(qtype);
    if (qtype == ORC_F32) { memcpy(blocks, w, (size_t)N * K * 4); return; }
    size_t nblk = (size_t)N * (K / be);
    for (size_t i = 0; i < nblk; i++) {
        const float *src = w + i * be;
        uint8_t *dst = b + i * bb;
        switch (qtype) {
        case ORC_Q4_0: enc_q4_0(src, dst); break;
        case ORC_Q8_0: enc_q8_0(src, dst); break;
        case ORC_Q4_K: enc_q4_k(src, dst); break;
        case ORC_Q3_K: enc_q3_k(src, dst); break;
        }
    }
}

/* ---- dequant-GEMV ----------------------------------------------------------
 * The reference's scalar fp32 path: dequantise the row, then a k-ordered fp32
 * dot product with the fp32 activation (the router loop of qwen_moe.c:296 and
 * the float loops of qwen_moe.c:97-98).                                      */
typedef struct { int qtype, N, K, batch, r0, r1; const uint8_t *W; const float *x; float *y; } gemv_job;

static void *gemv_worker(void *p)
{
    gemv_job *j = (gemv_job *)p;
    size_t rb = orc_row_bytes(j->qtype, j->K);
    float *row = (float *)malloc((size_t)j->K * sizeof(float));
    for (int n = j->r0; n < j->r1; n++) {
        orc_dequant_row(j->qtype, j->W + (size_t)n * rb, j->K, row);
        for (int b = 0; b < j->batch; b++) {
            const float *x = j->x + (size_t)b * j->K;
            float acc = 0.f;
            for (int k = 0; k < j->K; k++) acc += row[k] * x[k];
            j->y[(size_t)b * j->N + n] = acc;
        }
    }
    free(row);
    return NULL;
}

void orc_qgemv_mt(int qtype, int N, int K, const void *blocks, const float *x, float *y,
                  int batch, int nt)
{
    if (nt < 1) nt = 1;
    if (nt > N) nt = N > 0 ? N : 1;
    pthread_t *th = (pthread_t *)calloc((size_t)nt, sizeof(pthread_t));
    gemv_job *jb = (gemv_job *)calloc((size_t)nt, sizeof(gemv_job));
    for (int t = 0; t < nt; t++) {
        jb[t] = (gemv_job){qtype, N, K, batch, (int)((long)N * t / nt), (int)((long)N * (t + 1) / nt),
                           (const uint8_t *)blocks, x, y};
        if (t) pthread_create(&th[t], NULL, gemv_worker, &jb[t]);
    }
    gemv_worker(&jb[0]);
    for (int t = 1; t < nt; t++) pthread_join(th[t], NULL);
    free(th); free(jb);
}

void orc_qgemv(int qtype, int N, int K, const void *blocks, const float *x, float *y, int batch)
{
    orc_qgemv_mt(qtype, N, K, blocks, x, y, batch, 1);
}

/* ---- MoE block -------------------------------------------------------------*/

/* qwen_moe.c:189 */
void orc_softmax(float *x, int n)
{
    float m = -1e30f;
    for (int i = 0; i < n; i++) if (x[i] > m) m = x[i];
    float s = 0.f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - m); s += x[i]; }
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* qwen_moe.c:299-301 / qwen_moe_q3k.c:1934-1936: greedy selection, strict >
 * so the lowest index wins a tie, then renormalise the selected weights.   */
void orc_topk(const float *p, int n, int k, int *sel, float *w)
{
    for (int a = 0; a < k; a++) {
        int bi = -1;
        float bv = -1e30f;
        for (int e = 0; e < n; e++) {
            int used = 0;
            for (int b = 0; b < a; b++) if (sel[b] == e) used = 1;
            if (!used && p[e] > bv) { bv = p[e]; bi = e; }
        }
        sel[a] = bi;
        w[a] = bv;
    }
    float ssum = 0.f;
    for (int a = 0; a < k; a++) ssum += w[a];
    for (int a = 0; a < k; a++) w[a] /= ssum;
}

/* qwen_moe.c:309 / qwen_moe_q3k.c:1678-1680 (swiglu_exact) */
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* qwen_moe.c:295-311 with the fp32 router (router mode 0) and exact SiLU
 * (swiglu mode 0) of qwen_moe_q3k.c:1925-1973.  Expert e's gate/up matrices
 * start at row e*ffn of gate_exps/up_exps, its down matrix at row e*d of
 * down_exps.  Only experts in [expert_lo, expert_hi) contribute to eout.    */
static void moe_ffn_impl(int d, int n_exp, int n_act, int ffn, int qtype,
                         const float *router, const void *gate_exps, const void *up_exps,
                         const void *down_exps, int expert_lo, int expert_hi,
                         const float *hn_all, float *eout_all, int batch, int *sel_out, float *w_out,
                         float *probs_out, int nthreads);

void orc_moe_ffn(int d, int n_exp, int n_act, int ffn, int qtype,
                 const float *router, const void *gate_exps, const void *up_exps,
                 const void *down_exps, int expert_lo, int expert_hi,
                 const float *hn_all, float *eout_all, int batch, int *sel_out, float *w_out,
                 int nthreads)
{
    moe_ffn_impl(d, n_exp, n_act, ffn, qtype, router, gate_exps, up_exps, down_exps, expert_lo, expert_hi,
                 hn_all, eout_all, batch, sel_out, w_out, NULL, nthreads);
}

/* probs_out (may be NULL): the softmax probabilities [batch][n_exp] the
 * top-k chose from (test diagnostics: how close a selection was to a tie). */
static void moe_ffn_impl(int d, int n_exp, int n_act, int ffn, int qtype,
                         const float *router, const void *gate_exps, const void *up_exps,
                         const void *down_exps, int expert_lo, int expert_hi,
                         const float *hn_all, float *eout_all, int batch, int *sel_out, float *w_out,
                         float *probs_out, int nthreads)
{
    size_t rb_d = orc_row_bytes(qtype, d), rb_f = orc_row_bytes(qtype, ffn);
    float *rl = (float *)malloc((size_t)n_exp * sizeof(float));
    float *g = (float *)malloc((size_t)ffn * sizeof(float));
    float *u = (float *)malloc((size_t)ffn * sizeof(float));
    float *tmp = (float *)malloc((size_t)d * sizeof(float));
    int sel[64];
    float sw[64];
    for (int b = 0; b < batch; b++) {
        const float *hn = hn_all + (size_t)b * d;
        float *eout = eout_all + (size_t)b * d;
        for (int e = 0; e < n_exp; e++) {
            const float *rw = router + (size_t)e * d;
            float s = 0.f;
            for (int i = 0; i < d; i++) s += rw[i] * hn[i];
            rl[e] = s;
        }
        orc_softmax(rl, n_exp);
        if (probs_out) memcpy(probs_out + (size_t)b * n_exp, rl, (size_t)n_exp * sizeof(float));
        orc_topk(rl, n_exp, n_act, sel, sw);
        if (sel_out) memcpy(sel_out + (size_t)b * n_act, sel, (size_t)n_act * sizeof(int));
        if (w_out) memcpy(w_out + (size_t)b * n_act, sw, (size_t)n_act * sizeof(float));
        for (int i = 0; i < d; i++) eout[i] = 0.f;
        for (int a = 0; a < n_act; a++) {
            int e = sel[a];
            if (e < expert_lo || e >= expert_hi) continue;
            float w = sw[a];
            orc_qgemv_mt(qtype, ffn, d, (const uint8_t *)gate_exps + (size_t)e * ffn * rb_d, hn, g, 1, nthreads);
            orc_qgemv_mt(qtype, ffn, d, (const uint8_t *)up_exps + (size_t)e * ffn * rb_d, hn, u, 1, nthreads);
            for (int i = 0; i < ffn; i++) g[i] = orc_silu(g[i]) * u[i];
            orc_qgemv_mt(qtype, d, ffn, (const uint8_t *)down_exps + (size_t)e * d * rb_f, g, tmp, 1, nthreads);
            for (int i = 0; i < d; i++) eout[i] += w * tmp[i];
        }
    }
    free(rl); free(g); free(u); free(tmp);
}

/* ---- decode-step pieces ----------------------------------------------------*/

/* qwen_moe_q3k.c:1166 */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps)
{
    float s = 0.f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    s = 1.0f / sqrtf(s / n + eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * s * w[i];
}

/* qwen_moe.c:188 / qwen_moe_q3k.c:1170-1175: NEOX rotation of the pair
 * (i, i + hd/2) by pos * base^(-2i/hd).                                     */
void orc_rope_neox(float *v, int hd, int pos, float base)
{
    for (int i = 0; i < hd / 2; i++) {
        float fr = powf(base, -2.0f * i / hd), a = pos * fr, c = cosf(a), s = sinf(a);
        float x = v[i], y = v[i + hd / 2];
        v[i] = x * c - y * s;
        v[i + hd / 2] = x * s + y * c;
    }
}

/* ---- generators ------------------------------------------------------------*/
uint64_t orc_rng_seed(uint64_t s) { return s ? s : 0x243F6A8885A308D3ULL; }

/* bench/q3k_probe.c:403-404 (xorshift64, shifts 13/7/17) */
uint32_t orc_rng_u32(uint64_t *st)
{
    uint64_t x = *st;
    x ^= x << 13; x ^= x >> 7; x ^= x << 17;
    *st = x;
    return (uint32_t)x;
}

void orc_fill_u8(uint64_t seed, uint8_t *dst, size_t n)
{
    uint64_t st = orc_rng_seed(seed);
    for (size_t i = 0; i < n; i++) dst[i] = (uint8_t)orc_rng_u32(&st);
}

/* ---- one decode step (qwen_moe_q3k.c:1842-1983) ----------------------------
 * Restates forward()'s per-layer body for one token of one sequence, with
 * the fp32 router (router mode 0) and exact SiLU.  The cache is this layer's
 * cache of this sequence, [nkv][ctx][hd]: fp16 bits (kv_f32 = 0; the step's
 * k and v are rounded to fp16, round-to-nearest-even, when stored, as the
 * BASELINE decode configuration asks) or fp32 (kv_f32 = 1; the reference's
 * own cache precision, qwen_moe.c:282 / qwen_moe_q3k.c:1877-1880).  The
 * attention reads every position, the current one included, from the cache.
 * attn_w: the four projections as GGUF-native blocks of attn_qtype:
 * wq [nh*hd][d], wk / wv [nkv*hd][d], wo [d][nh*hd].  h (d floats) is
 * updated in place; sel_out / w_out (n_act each, may be NULL) get the
 * routing.                                                                   */
static void decode_layer_impl(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                              int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                              const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                              const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                              const float *router, const void *gate_exps, const void *up_exps,
                              const void *down_exps, void *kc_, void *vc_, int kv_f32, float *h,
                              int *sel_out, float *w_out, float *probs_out, int nthreads)
{
    const int qd = nh * hd, kvd = nkv * hd, gpr = nh / nkv;
    uint16_t *kc = (uint16_t *)kc_, *vc = (uint16_t *)vc_;
    float *kcf = (float *)kc_, *vcf = (float *)vc_;
    float *hn = (float *)malloc((size_t)d * sizeof(float));
    float *q = (float *)malloc((size_t)qd * sizeof(float));
    float *k = (float *)malloc((size_t)kvd * sizeof(float));
    float *v = (float *)malloc((size_t)kvd * sizeof(float));
    float *att = (float *)malloc((size_t)qd * sizeof(float));
    float *sc = (float *)malloc((size_t)ctx * sizeof(float));
    float *tmp = (float *)malloc((size_t)d * sizeof(float));
    float *kf = (float *)malloc((size_t)hd * sizeof(float));
    /* :1850-1860 */
    orc_rmsnorm(hn, h, attn_norm, d, eps);
    orc_qgemv_mt(attn_qtype, qd, d, wq, hn, q, 1, nthreads);
    orc_qgemv_mt(attn_qtype, kvd, d, wk, hn, k, 1, nthreads);
    orc_qgemv_mt(attn_qtype, kvd, d, wv, hn, v, 1, nthreads);
    /* :1862-1864 */
    for (int hh = 0; hh < nh; hh++) {
        orc_rmsnorm(q + hh * hd, q + hh * hd, q_norm, hd, eps);
        orc_rope_neox(q + hh * hd, hd, pos, rope_base);
    }
    for (int hh = 0; hh < nkv; hh++) {
        orc_rmsnorm(k + hh * hd, k + hh * hd, k_norm, hd, eps);
        orc_rope_neox(k + hh * hd, hd, pos, rope_base);
    }
    /* :1877-1880 head-major cache write */
    for (int kvh = 0; kvh < nkv; kvh++)
        for (int t = 0; t < hd; t++) {
            const size_t at = ((size_t)kvh * ctx + pos) * hd + t;
            if (kv_f32) {
                kcf[at] = k[kvh * hd + t];
                vcf[at] = v[kvh * hd + t];
            } else {
                kc[at] = orc_f32_to_f16_rne(k[kvh * hd + t]);
                vc[at] = orc_f32_to_f16_rne(v[kvh * hd + t]);
            }
        }
    /* :1890-1899 serial attention */
    const float scale = 1.0f / sqrtf((float)hd);
    for (int hh = 0; hh < nh; hh++) {
        const int kvh = hh / gpr;
        const float *qh = q + hh * hd;
        const size_t base = (size_t)kvh * ctx * hd;
        for (int j = 0; j <= pos; j++) {
            for (int t = 0; t < hd; t++)
                kf[t] = kv_f32 ? kcf[base + (size_t)j * hd + t] : orc_f16_to_f32(kc[base + (size_t)j * hd + t]);
            float s = 0.f;
            for (int t = 0; t < hd; t++) s += qh[t] * kf[t];
            sc[j] = s * scale;
        }
        orc_softmax(sc, pos + 1);
        float *oh = att + hh * hd;
        for (int t = 0; t < hd; t++) oh[t] = 0.f;
        for (int j = 0; j <= pos; j++)
            for (int t = 0; t < hd; t++)
                oh[t] += sc[j] * (kv_f32 ? vcf[base + (size_t)j * hd + t] : orc_f16_to_f32(vc[base + (size_t)j * hd + t]));
    }
    /* :1912-1915 */
    orc_qgemv_mt(attn_qtype, d, qd, wo, att, tmp, 1, nthreads);
    for (int i = 0; i < d; i++) h[i] += tmp[i];
    /* :1916-1978 */
    orc_rmsnorm(hn, h, ffn_norm, d, eps);
    moe_ffn_impl(d, n_exp, n_act, ffn, expert_qtype, router, gate_exps, up_exps, down_exps, 0, n_exp,
                 hn, tmp, 1, sel_out, w_out, probs_out, nthreads);
    for (int i = 0; i < d; i++) h[i] += tmp[i];
    free(hn); free(q); free(k); free(v); free(att); free(sc); free(tmp); free(kf);
}

void orc_decode_layer(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                      int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                      const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                      const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                      const float *router, const void *gate_exps, const void *up_exps,
                      const void *down_exps, uint16_t *kc, uint16_t *vc, float *h,
                      int *sel_out, float *w_out, int nthreads)
{
    decode_layer_impl(d, nh, nkv, hd, ctx, pos, rope_base, eps, attn_qtype, attn_norm, wq, wk, wv, q_norm, k_norm,
                      wo, ffn_norm, n_exp, n_act, ffn, expert_qtype, router, gate_exps, up_exps, down_exps, kc, vc,
                      0, h, sel_out, w_out, NULL, nthreads);
}

void orc_decode_layer_f32kv(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                            int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                            const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                            const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                            const float *router, const void *gate_exps, const void *up_exps,
                            const void *down_exps, float *kc, float *vc, float *h,
                            int *sel_out, float *w_out, int nthreads)
{
    decode_layer_impl(d, nh, nkv, hd, ctx, pos, rope_base, eps, attn_qtype, attn_norm, wq, wk, wv, q_norm, k_norm,
                      wo, ffn_norm, n_exp, n_act, ffn, expert_qtype, router, gate_exps, up_exps, down_exps, kc, vc,
                      1, h, sel_out, w_out, NULL, nthreads);
}

/* qwen_moe_q3k.c:1980-1981: logits = lm . rmsnorm(h, out_norm) */
void orc_decode_head(int d, int vocab, float eps, int lm_qtype, const float *out_norm, const void *lm,
                     const float *h, float *logits, int nthreads)
{
    float *hn = (float *)malloc((size_t)d * sizeof(float));
    orc_rmsnorm(hn, h, out_norm, d, eps);
    orc_qgemv_mt(lm_qtype, vocab, d, lm, hn, logits, 1, nthreads);
    free(hn);
}

/* orc_decode_layer that also returns the router's softmax probabilities
 * (n_exp floats): test diagnostics of how close the top-k came to a tie.    */
void orc_decode_layer_probs(int d, int nh, int nkv, int hd, int ctx, int pos, float rope_base, float eps,
                            int attn_qtype, const float *attn_norm, const void *wq, const void *wk,
                            const void *wv, const float *q_norm, const float *k_norm, const void *wo,
                            const float *ffn_norm, int n_exp, int n_act, int ffn, int expert_qtype,
                            const float *router, const void *gate_exps, const void *up_exps,
                            const void *down_exps, uint16_t *kc, uint16_t *vc, float *h,
                            int *sel_out, float *w_out, float *probs_out, int nthreads)
{
    decode_layer_impl(d, nh, nkv, hd, ctx, pos, rope_base, eps, attn_qtype, attn_norm, wq, wk, wv, q_norm, k_norm,
                      wo, ffn_norm, n_exp, n_act, ffn, expert_qtype, router, gate_exps, up_exps, down_exps, kc, vc,
                      0, h, sel_out, w_out, probs_out, nthreads);
}
