"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree is available (REF_ROOT, by default the directory
`reference` beside this repository); the fixtures it writes are committed so
that the tests never need the reference at run time.

What it pins, and from which reference code:
  gemm_golden.npz   gemm_ref_i8 / gemm_ref_f32 of the reference's
                    src/gemm_ref.c (compiled unchanged by oracle/Makefile into
                    oracle/_ref/libx100ref.so) on xorshift64 inputs, C != 0
                    on entry (beta = 1).
  quant_golden.npz  the reference's own block decoders, compiled in a
                    temporary directory straight out of its engine sources:
                      Q4_0 / Q8_0  gguf_dequant_into   qwen_moe.c:156-179
                      Q3_K         dequantize_q3_K_block qwen_moe_q3k.c:557-577
                      Q4_K         dequantize_q5_K_block qwen_moe_q3k.c:541-552
                                   on blocks whose fifth bit plane qh is zero
                                   (a Q5_K block with qh = 0 decodes exactly
                                   as the Q4_K block with the same d, dmin,
                                   scales and qs)
                    applied to random well-formed blocks (random bytes, fp16
                    scales in a bounded range, as bench/q3k_probe.c:418-425
                    builds its test blocks) plus edge blocks.
  gguf_golden.npz   the GGUF tensor decoders of the reference's Q3_K engine
                    (gguf_dequant_into, qwen_moe_q3k.c:1129-1158: F32, F16,
                    Q4_0, Q4_1, Q8_0, Q3_K, Q5_K, Q6_K) on random well-formed
                    blocks plus edge blocks, and its Q8_0 requantiser
                    (quantize_q8_0_native, qwen_moe_q3k.c:409-414, with the
                    truncating f32_to_f16 of :71-79) on fp32 rows.
  gguf_parse.json   what the reference's GGUF reader (gguf_open,
                    qwen_moe_q3k.c:1098-1126) reads from a synthetic file made
                    by tests/gguf_writer.py (make_parse_file below): model
                    dimensions, defaults, tokens, tensor infos, data start.
  a8_golden.npz     the reference's activation packers for its IME kernels,
                    pack_A_i8 (qwen_moe_q3k.c:420-426), pack_A_q3k
                    (:613-623) and pack_A_hp (qwen_moe_hp.c:131-180, in the
                    scalar form of bench/vendor_ime_actpack_probe.c:37-62
                    with the engine's truncating f32_to_f16,
                    qwen_moe_hp.c:71-79), compiled from the reference and
                    run on fp32 rows (normal values, rounding ties, zeros,
                    tiny and large values); and the HP kernels' Q4_0 weight
                    quantiser quantize_q4_0_native (qwen_moe_hp.c:102-109).
  meta.json         struct-size known answers (block_q3_K 110 B,
                    block_q5_K 176 B, bench/q3k_probe.c:410-413) and the
                    x100_caps_t layout of the reference header.
  moe_golden.npz    the reference's routing and layer-body functions on
                    edge-case inputs: softmax (qwen_moe.c:189, the scalar
                    branch of qwen_moe_q3k.c:1221-1248 is the same text),
                    the greedy top-k and renormalisation lines of forward()
                    (qwen_moe.c:299-301) after that softmax (ties included),
                    rmsnorm (qwen_moe.c:187 = qwen_moe_q3k.c:1166), rope
                    (qwen_moe.c:188) and rope_table / rope_apply
                    (qwen_moe_q3k.c:1170-1175) at positions 0 .. 4095, and
                    swiglu_exact (qwen_moe_q3k.c:1678-1680).
  forward_golden.npz  logits of the reference's whole forward()
                    (qwen_moe.c:272-315: rmsnorm, q/k/v, per-head q/k norm and
                    RoPE, fp32 KV cache, serial softmax attention, Wo,
                    residual, router, softmax, top-k, renormalise, SwiGLU
                    experts, weighted sum, residual, output norm, lm_head)
                    compiled unchanged, with its linear layers (the RISC-V
                    IME kernels lin_mm / lin_mm_packed / pack_act) replaced by
                    the scalar fp32 dequant-GEMV -- the BASELINE's oracle
                    definition -- over weights dequantised by the reference's
                    own decoders.  Inputs: tests/golden/golden_inputs.py.
The extracted reference functions are compiled under a temporary directory
and never written into this repository.  REF_ROOT (environment) names the
reference tree; by default the directory `reference` beside this repository.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import py_oracle as po  # noqa: E402

REF_ROOT = os.environ.get("REF_ROOT") or os.path.normpath(os.path.join(REPO, "..", "reference"))

GEMM_SHAPES = [(1, 1, 1), (3, 5, 7), (7, 9, 33), (16, 16, 16), (33, 17, 5),
               (64, 48, 40), (128, 64, 96), (129, 130, 131)]
GEMM_HASH_SHAPES = [(256, 256, 256)]


def extract_function(src: str, signature_regex: str) -> str:
    m = re.search(signature_regex, src)
    if not m:
        raise RuntimeError("signature not found: " + signature_regex)
    start = m.start()
    i = src.index("{", m.end() - 1)
    depth = 0
    for j in range(i, len(src)):
        if src[j] == "{":
            depth += 1
        elif src[j] == "}":
            depth -= 1
            if depth == 0:
                return src[start:j + 1]
    raise RuntimeError("unbalanced braces")


def extract_line(src: str, regex: str) -> str:
    m = re.search(regex, src, re.M)
    if not m:
        raise RuntimeError("line not found: " + regex)
    return m.group(0)


def build_ref_decoders(tmp: str) -> C.CDLL:
    moe = open(os.path.join(REF_ROOT, "qwen_moe.c")).read()
    q3k = open(os.path.join(REF_ROOT, "qwen_moe_q3k.c")).read()
    parts = [
        "#include <stdio.h>\n#include <stdlib.h>\n#include <stdint.h>\n#include <string.h>\n#include <math.h>\n",
        # qwen_moe.c: f16 decode, GGUF tensor structs, generic dequant
        extract_function(moe, r"static float f16f\(uint16_t h\)\{"),
        extract_line(moe, r"^typedef struct \{ uint32_t typ;.*\} TInfo;$"),
        extract_line(moe, r"^typedef struct \{ unsigned char\*p;[^\n]*\n[^\n]*\} Gguf;$"),
        extract_function(moe, r"static void gguf_dequant_into\(Gguf\*g,TInfo\*ti,size_t elem0,size_t n,float\*out\)\{"),
        # qwen_moe_q3k.c: K-quant block types and decoders
        extract_line(q3k, r"^typedef struct \{ uint8_t hmask\[32\];.*\} block_q3_K;.*$"),
        extract_line(q3k, r"^typedef struct \{ _Float16 d; _Float16 dmin;.*\} block_q5_K;.*$"),
        extract_function(q3k, r"static inline void q5k_get_scale_min\(int j,const uint8_t\*q,uint8_t\*d,uint8_t\*m\)\{"),
        extract_function(q3k, r"static void dequantize_q5_K_block\(const block_q5_K\*x,float\*y\)\{"),
        extract_function(q3k, r"static void dequantize_q3_K_block\(const block_q3_K\*x,float\*y\)\{"),
        # thin exported wrappers (written here, not reference code)
        """
size_t golden_sizeof_q3k(void){ return sizeof(block_q3_K); }
size_t golden_sizeof_q5k(void){ return sizeof(block_q5_K); }
void golden_dq_q3k(const void*b,int nblk,float*out){ for(int i=0;i<nblk;i++) dequantize_q3_K_block((const block_q3_K*)b+i,out+256*i); }
void golden_dq_q5k(const void*b,int nblk,float*out){ for(int i=0;i<nblk;i++) dequantize_q5_K_block((const block_q5_K*)b+i,out+256*i); }
void golden_dq_gguf(unsigned typ,const void*data,size_t n,float*out){
  Gguf g; memset(&g,0,sizeof g); g.p=(unsigned char*)data; g.data_start=0;
  TInfo t; memset(&t,0,sizeof t); t.typ=typ; t.off=0; gguf_dequant_into(&g,&t,0,n,out); }
""",
    ]
    path = os.path.join(tmp, "refdec.c")
    with open(path, "w") as f:
        f.write("\n".join(parts))
    so = os.path.join(tmp, "librefdec.so")
    subprocess.check_call(["gcc", "-std=gnu11", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
                           "-o", so, path, "-lm"])
    L = C.CDLL(so)
    L.golden_dq_q3k.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.golden_dq_q5k.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.golden_dq_gguf.argtypes = [C.c_uint, C.c_void_p, C.c_size_t, C.c_void_p]
    L.golden_sizeof_q3k.restype = C.c_size_t
    L.golden_sizeof_q5k.restype = C.c_size_t
    return L


def build_ref_gguf(tmp: str) -> C.CDLL:
    """The Q3_K engine's GGUF reader, tensor decoders and Q8_0 requantiser,
    extracted unchanged from qwen_moe_q3k.c and compiled under tmp."""
    q3k = open(os.path.join(REF_ROOT, "qwen_moe_q3k.c")).read()
    parts = [
        "#include <stdio.h>\n#include <stdlib.h>\n#include <stdint.h>\n#include <string.h>\n#include <math.h>\n"
        "#include <fcntl.h>\n#include <sys/mman.h>\n#include <sys/stat.h>\n#include <unistd.h>\n",
        extract_function(q3k, r"static uint16_t f32_to_f16\(float f\)\{"),
        extract_line(q3k, r"^typedef struct \{ uint16_t d; int8_t qs\[32\]; \} q8_0_native;$"),
        extract_function(q3k, r"static void quantize_q8_0_native\(const float\*w /\*32 elems\*/, q8_0_native\*out\)\{"),
        extract_line(q3k, r"^typedef struct \{ uint8_t hmask\[32\];.*\} block_q3_K;.*$"),
        extract_line(q3k, r"^typedef struct \{ _Float16 d; _Float16 dmin;.*\} block_q5_K;.*$"),
        extract_function(q3k, r"static inline void q5k_get_scale_min\(int j,const uint8_t\*q,uint8_t\*d,uint8_t\*m\)\{"),
        extract_function(q3k, r"static void dequantize_q5_K_block\(const block_q5_K\*x,float\*y\)\{"),
        extract_function(q3k, r"static void dequantize_q3_K_block\(const block_q3_K\*x,float\*y\)\{"),
        extract_line(q3k, r"^typedef struct \{ uint32_t typ;.*\} TInfo;$"),
        extract_line(q3k, r"^typedef struct \{ unsigned char\*p;[^\n]*\n[^\n]*\} Gguf;$"),
        extract_function(q3k, r"static uint64_t U64\(unsigned char\*b\)\{"),
        extract_function(q3k, r"static uint32_t U32\(unsigned char\*b\)\{"),
        extract_function(q3k, r"static float f16f\(uint16_t h\)\{"),
        extract_function(q3k, r"static size_t skipval\(unsigned char\*p,uint32_t t\)\{"),
        extract_function(q3k, r"static void gguf_open\(Gguf\*g,const char\*path\)\{"),
        extract_function(q3k, r"static void gguf_dequant_into\(Gguf\*g,TInfo\*ti,size_t elem0,size_t n,float\*out\)\{"),
        # thin exported wrappers (written here, not reference code)
        """
void golden_dq(unsigned typ,const void*data,size_t n,float*out){
  Gguf g; memset(&g,0,sizeof g); g.p=(unsigned char*)data; g.data_start=0;
  TInfo t; memset(&t,0,sizeof t); t.typ=typ; t.off=0; gguf_dequant_into(&g,&t,0,n,out); }
void golden_q8(const float*w,size_t n,void*out){ for(size_t b=0;b<n/32;b++) quantize_q8_0_native(w+32*b,(q8_0_native*)out+b); }
size_t golden_sizeof_q8(void){ return sizeof(q8_0_native); }
static Gguf G;
void golden_open(const char*path,long*ints,float*rope){ memset(&G,0,sizeof G); gguf_open(&G,path);
  ints[0]=G.block_count; ints[1]=G.embd; ints[2]=G.ffn; ints[3]=G.nh; ints[4]=G.nkv; ints[5]=G.hd;
  ints[6]=G.vocab; ints[7]=G.n_exp; ints[8]=G.n_act; ints[9]=G.moe_ffn; ints[10]=G.nt; ints[11]=(long)G.data_start;
  ints[12]=G.ntok; *rope=G.rope_base; }
const char*golden_token(int i){ return G.tok[i]; }
void golden_tensor(int i,char*name,long*v){ TInfo*t=&G.t[i]; strcpy(name,t->name); v[0]=t->typ; v[1]=t->nd;
  for(int d=0;d<4;d++) v[2+d]=(long)t->dims[d]; v[6]=(long)t->off; }
""",
    ]
    path = os.path.join(tmp, "refgguf.c")
    with open(path, "w") as f:
        f.write("\n".join(parts))
    so = os.path.join(tmp, "librefgguf.so")
    subprocess.check_call(["gcc", "-std=gnu11", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
                           "-o", so, path, "-lm"])
    L = C.CDLL(so)
    L.golden_dq.argtypes = [C.c_uint, C.c_void_p, C.c_size_t, C.c_void_p]
    L.golden_q8.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p]
    L.golden_sizeof_q8.restype = C.c_size_t
    L.golden_open.argtypes = [C.c_char_p, C.c_void_p, C.c_void_p]
    L.golden_token.argtypes = [C.c_int]
    L.golden_token.restype = C.c_char_p
    L.golden_tensor.argtypes = [C.c_int, C.c_char_p, C.c_void_p]
    return L


def caps_layout(tmp: str) -> dict:
    prog = os.path.join(tmp, "caps.c")
    with open(prog, "w") as f:
        f.write('#include <stdio.h>\n#include <stddef.h>\n#include "x100_gemm.h"\n'
                'int main(void){printf("%zu %zu %zu %zu\\n", sizeof(x100_caps_t),'
                ' offsetof(x100_caps_t, has_ime), offsetof(x100_caps_t, mvendorid),'
                ' offsetof(x100_caps_t, isa)); return 0;}\n')
    exe = os.path.join(tmp, "caps")
    subprocess.check_call(["gcc", "-I", os.path.join(REF_ROOT, "include"), "-o", exe, prog])
    s, hi, mv, isa = map(int, subprocess.check_output([exe]).split())
    return {"sizeof": s, "has_ime": hi, "mvendorid": mv, "isa": isa}


def f16_bytes(vals) -> np.ndarray:
    return np.asarray(vals, np.float16).view(np.uint8).reshape(-1, 2)


def random_blocks(qtype: int, n: int, seed: int) -> np.ndarray:
    """Random well-formed blocks: random payload bytes, fp16 scales drawn from
    +-[0.001, 0.08] (plus a few edge blocks appended by the caller)."""
    rng = np.random.default_rng(seed)
    bb = po.BLOCK_BYTES[qtype]
    blk = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    mag = rng.uniform(0.001, 0.08, size=n) * rng.choice([-1.0, 1.0], size=n)
    if qtype in (po.Q4_0, po.Q8_0):
        blk[:, 0:2] = f16_bytes(mag)
    elif qtype == po.Q4_K:
        blk[:, 0:2] = f16_bytes(np.abs(mag))
        blk[:, 2:4] = f16_bytes(rng.uniform(0.0, 0.05, size=n))
    elif qtype == po.Q3_K:
        blk[:, 108:110] = f16_bytes(mag)
    return blk


def edge_blocks(qtype: int) -> np.ndarray:
    bb = po.BLOCK_BYTES[qtype]
    out = []
    z = np.zeros(bb, np.uint8)
    out.append(z.copy())                                     # all zero
    f = np.full(bb, 0xFF, np.uint8)                          # all ones payload
    dpos = {po.Q4_0: [0], po.Q8_0: [0], po.Q4_K: [0, 2], po.Q3_K: [108]}[qtype]
    for p in dpos:
        f[p:p + 2] = f16_bytes([1.0])[0]
    out.append(f)
    sub = np.full(bb, 0x5A, np.uint8)                        # subnormal scale
    for p in dpos:
        sub[p:p + 2] = np.array([0x01, 0x00], np.uint8)
    out.append(sub)
    big = np.full(bb, 0xA5, np.uint8)                        # large scale
    for p in dpos:
        big[p:p + 2] = f16_bytes([-1024.0])[0]
    out.append(big)
    return np.stack(out)


def to_q5k_layout(q4k: np.ndarray) -> np.ndarray:
    """block_q4_K (d, dmin, scales[12], qs[128]) -> block_q5_K with qh = 0
    (d, dmin, scales[12], qh[32], qs[128])."""
    n = q4k.shape[0]
    out = np.zeros((n, 176), np.uint8)
    out[:, 0:16] = q4k[:, 0:16]
    out[:, 48:176] = q4k[:, 16:144]
    return out


GGUF_TYPES = ((po.Q_F32, "F32"), (po.F16, "F16"), (po.Q4_0, "Q4_0"), (po.Q4_1, "Q4_1"), (po.Q8_0, "Q8_0"),
              (po.Q3_K, "Q3_K"), (po.Q5_K, "Q5_K"), (po.Q6_K, "Q6_K"))


def gguf_edge_blocks(gtype: int) -> np.ndarray:
    """Zero, all-ones payload with unit scales, subnormal and large scales."""
    be, bb = po.GGUF_BLOCK[gtype]
    if gtype == po.Q_F32:
        return np.array([0.0, -0.0, 1e-40, -3.4e38, 1.0], np.float32).view(np.uint8).reshape(-1, 4)
    if gtype == po.F16:
        return np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x7BFF, 0xFBFF, 0x3C00], np.uint16).view(np.uint8).reshape(-1, 2)
    dpos = {po.Q4_0: [0], po.Q8_0: [0], po.Q4_1: [0, 2], po.Q5_K: [0, 2], po.Q3_K: [108], po.Q6_K: [208]}[gtype]
    out = [np.zeros(bb, np.uint8)]
    for fill, val in ((0xFF, [1.0]), (0x5A, None), (0xA5, [-1024.0])):
        b = np.full(bb, fill, np.uint8)
        for p in dpos:
            b[p:p + 2] = f16_bytes(val)[0] if val else np.array([0x01, 0x00], np.uint8)
        out.append(b)
    return np.stack(out)


def make_parse_file(path: str) -> None:
    """A synthetic qwen3moe GGUF: every metadata value type (scalars, strings,
    arrays of scalars, of strings and of arrays), the keys the reader takes,
    a token list, and tensors of several types and ranks."""
    import gguf_writer as gw
    rng = np.random.default_rng(2025)
    toks = [f"tok{i}" for i in range(40)] + ["", "\u00e9t\u00e9", " Tokyo"]
    kv = [("general.architecture", gw.STR, "qwen3moe"), ("general.alignment", gw.U32, 32),
          ("general.flag", gw.BOOL, True), ("general.u8", gw.U8, 7), ("general.i8", gw.I8, -7),
          ("general.u16", gw.U16, 700), ("general.i16", gw.I16, -700), ("general.u64", gw.U64, 1 << 40),
          ("general.i64", gw.I64, -(1 << 40)), ("general.f64", gw.F64, 0.25),
          ("qwen3moe.block_count", gw.U32, 2), ("qwen3moe.embedding_length", gw.U32, 256),
          ("qwen3moe.feed_forward_length", gw.U32, 512), ("qwen3moe.attention.head_count", gw.U32, 4),
          ("qwen3moe.attention.head_count_kv", gw.I32, 2), ("qwen3moe.attention.key_length", gw.U32, 128),
          ("qwen3moe.expert_count", gw.U32, 4), ("qwen3moe.expert_used_count", gw.U32, 2),
          ("qwen3moe.expert_feed_forward_length", gw.U32, 256), ("qwen3moe.rope.freq_base", gw.F32, 5e5),
          ("qwen3moe.attention.layer_norm_rms_epsilon", gw.F32, 1e-6),
          ("tokenizer.ggml.scores", gw.ARR, (gw.F32, [float(i) for i in range(len(toks))])),
          ("tokenizer.ggml.tokens", gw.ARR, (gw.STR, toks)),
          ("tokenizer.ggml.merges", gw.ARR, (gw.ARR, [(gw.U16, [1, 2, 3]), (gw.U16, [])])),
          ("tokenizer.ggml.token_type", gw.ARR, (gw.I32, [1] * len(toks)))]
    specs = [("token_embd.weight", po.Q8_0, [256, 43]), ("output_norm.weight", po.Q_F32, [256]),
             ("blk.0.attn_q.weight", po.Q3_K, [256, 512]), ("blk.0.attn_k.weight", po.Q8_0, [256, 256]),
             ("blk.0.attn_output.weight", po.Q5_K, [512, 256]), ("blk.1.ffn_gate_exps.weight", po.Q4_0, [256, 256, 4]),
             ("output.weight", po.Q6_K, [256, 43]), ("blk.0.attn_norm.weight", po.F16, [256])]
    tensors = []
    for name, gt, dims in specs:
        n = int(np.prod(dims))
        be, _ = po.GGUF_BLOCK[gt]
        tensors.append((name, gt, dims, gw.random_blocks(gt, n // be, rng).tobytes()))
    gw.write_gguf(path, kv, tensors)


def make_gguf_golden() -> None:
    sys.path.insert(0, os.path.dirname(HERE))
    with tempfile.TemporaryDirectory() as tmp:
        ref = build_ref_gguf(tmp)
        import gguf_writer as gw
        out = {}
        for gt, name in GGUF_TYPES:
            be, _ = po.GGUF_BLOCK[gt]
            blk = np.concatenate([gw.random_blocks(gt, 64 if be > 1 else 512, np.random.default_rng(500 + gt)),
                                  gguf_edge_blocks(gt)])
            blk = np.ascontiguousarray(blk)
            n = blk.shape[0] * be
            vals = np.zeros(n, np.float32)
            ref.golden_dq(gt, blk.ctypes.data, n, vals.ctypes.data)
            out[f"{name}_blocks"] = blk.reshape(-1)
            out[f"{name}_values"] = vals
        rng = np.random.default_rng(77)
        rows = [rng.standard_normal(32 * 64).astype(np.float32),
                (rng.standard_normal(32 * 16) * 1e-3).astype(np.float32),
                np.zeros(32, np.float32),                                     # amax stays 1e-6
                np.tile(np.array([127.0, -127.0, 63.5, -63.5, 0.5, -0.5, 1.5, 2.5], np.float32), 4),  # ties
                np.full(32, 7e-7, np.float32),                                # below the amax floor
                (rng.standard_normal(32 * 8) * 3e4).astype(np.float32)]
        x = np.concatenate(rows)
        assert ref.golden_sizeof_q8() == 34
        q = np.zeros(x.size // 32 * 34, np.uint8)
        ref.golden_q8(x.ctypes.data, x.size, q.ctypes.data)
        out["Q8REQ_input"] = x
        out["Q8REQ_blocks"] = q
        np.savez_compressed(os.path.join(HERE, "gguf_golden.npz"), **out)

        path = os.path.join(tmp, "parse.gguf")
        make_parse_file(path)
        ints = np.zeros(13, np.int64)
        rope = np.zeros(1, np.float32)
        ref.golden_open(path.encode(), ints.ctypes.data, rope.ctypes.data)
        names = ["block_count", "embd", "ffn", "nh", "nkv", "hd", "vocab", "n_exp", "n_act", "moe_ffn",
                 "n_tensors", "data_start", "n_tokens"]
        parse = {k: int(v) for k, v in zip(names, ints)}
        parse["rope_base"] = float(rope[0])
        parse["tokens"] = [ref.golden_token(i).decode() for i in range(parse["n_tokens"])]
        tens = []
        for i in range(parse["n_tensors"]):
            nm = C.create_string_buffer(64)
            v = np.zeros(7, np.int64)
            ref.golden_tensor(i, nm, v.ctypes.data)
            tens.append({"name": nm.value.decode(), "type": int(v[0]), "n_dims": int(v[1]),
                         "dims": [int(d) for d in v[2:2 + int(v[1])]], "offset": int(v[6])})
        parse["tensors"] = tens
        parse["file_sha256"] = hashlib.sha256(open(path, "rb").read()).hexdigest()
        with open(os.path.join(HERE, "gguf_parse.json"), "w") as f:
            json.dump(parse, f, indent=1, sort_keys=True)
    print("wrote gguf_golden.npz, gguf_parse.json")


def make_a8_golden() -> None:
    q3k = open(os.path.join(REF_ROOT, "qwen_moe_q3k.c")).read()
    hp = open(os.path.join(REF_ROOT, "qwen_moe_hp.c")).read()
    probe = open(os.path.join(REF_ROOT, "bench", "vendor_ime_actpack_probe.c")).read()
    parts = [
        "#include <stdint.h>\n#include <string.h>\n#include <math.h>\n",
        extract_line(q3k, r"^#define AREC_Q3K 292$"),
        extract_function(q3k, r"static void pack_A_i8\(const float\*x, uint8_t\*out [^)]*\)\{"),
        extract_function(q3k, r"static void pack_A_q3k\(const float\*a,uint8_t\*out\)\{"),
        # qwen_moe_hp.c: the engine's truncating f32_to_f16, the HP weight
        # quantiser, and the scalar pack_A_hp its RVV packer was checked
        # byte-identical against (kept in the probe); the engine pairs that
        # packer with this f32_to_f16
        extract_function(hp, r"static uint16_t f32_to_f16\(float f\)\{"),
        extract_line(hp, r"^#define NSUB 8 .*$"),
        extract_line(hp, r"^typedef struct \{ uint16_t d; uint8_t qs\[16\]; \} q4_0_native;$"),
        extract_function(hp, r"static void quantize_q4_0_native\(const float\*w /\*32 elems\*/, q4_0_native\*out\)\{"),
        extract_function(probe, r"static void pack_A_hp_scalar\(const float\*a, uint8_t\*out\)\{"),
        """
void golden_pack_i8(const float*x,int K,uint8_t*out){ for(int kg=0;kg<K/32;kg++) pack_A_i8(x+32*kg,out+38*kg); }
void golden_pack_q3k(const float*x,int K,uint8_t*out){ for(int sb=0;sb<K/256;sb++) pack_A_q3k(x+256*sb,out+AREC_Q3K*sb); }
void golden_pack_hp(const float*x,int K,uint8_t*out){ for(int sb=0;sb<K/256;sb++) pack_A_hp_scalar(x+256*sb,out+290*sb); }
void golden_q4_0_hp(const float*w,int n,uint8_t*out){ for(int b=0;b<n/32;b++) quantize_q4_0_native(w+32*b,(q4_0_native*)(out+18*b)); }
int golden_sizeof_q4_0_native(void){ return (int)sizeof(q4_0_native); }
""",
    ]
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "refa8.c")
        with open(path, "w") as f:
            f.write("\n".join(parts))
        so = os.path.join(tmp, "librefa8.so")
        subprocess.check_call(["gcc", "-std=gnu11", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-o", so, path,
                               "-lm"])
        L = C.CDLL(so)
        L.golden_pack_i8.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.golden_pack_q3k.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.golden_pack_hp.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        L.golden_q4_0_hp.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        assert L.golden_sizeof_q4_0_native() == 18
        rng = np.random.default_rng(88)
        rows = [rng.standard_normal(2048), rng.standard_normal(2048) * 1e-4, np.zeros(512),
                np.tile([0.5, -0.5, 1.5, -2.5, 127.0, -127.0, 63.5, 0.25], 64) * (127.0 / 127.0),
                np.full(256, 7e-7), rng.standard_normal(768) * 3e4,
                np.r_[np.ones(255), 254.0].astype(np.float64)]   # ties at x / scale = k + 0.5
        x = np.concatenate([np.asarray(r, np.float32) for r in rows])
        assert x.size % 256 == 0
        i8 = np.zeros(x.size // 32 * 38, np.uint8)
        q3 = np.zeros(x.size // 256 * 292, np.uint8)
        L.golden_pack_i8(x.ctypes.data, x.size, i8.ctypes.data)
        L.golden_pack_q3k(x.ctypes.data, x.size, q3.ctypes.data)
        hpk = np.zeros(x.size // 256 * 290, np.uint8)
        L.golden_pack_hp(x.ctypes.data, x.size, hpk.ctypes.data)
        # HP weight rows: N(0, 0.02) weights, zeros, values under the 1e-6
        # floor, rounding ties at w / d = k + 0.5 and the clamp at -8 / +7
        w_rows = [rng.normal(0, 0.02, 4096), np.zeros(64), np.full(32, 5e-7), rng.normal(0, 300.0, 256),
                  np.r_[np.full(31, 0.25), 0.8] * np.tile([1, -1], 16), np.r_[np.full(31, -0.5), 1.0]]
        w = np.concatenate([np.asarray(r, np.float32) for r in w_rows])
        q4hp = np.zeros(w.size // 32 * 18, np.uint8)
        L.golden_q4_0_hp(w.ctypes.data, w.size, q4hp.ctypes.data)
        np.savez_compressed(os.path.join(HERE, "a8_golden.npz"), x=x, pack_i8=i8, pack_q3k=q3, pack_hp=hpk,
                            w_hp=w, q4_0_hp=q4hp)
    print("wrote a8_golden.npz")


# ---- routing and layer-body functions, and the whole forward() ------------------------
FWD_STUBS = r"""
/* ---- written here, not reference code: the linear layers as fp32 row-major
 * matrices, y[n] = sum_k W[n][k] * x[k] in k order (the scalar dequant-GEMV),
 * in place of the reference's IME kernels.  pack_act keeps the fp32 vector
 * (in the caller's activation buffer) instead of quantising it. */
typedef struct { int N, K; const float *W; } Lin;
static void pack_act(const float *x, int K, int8_t *xt, float *xs_out) { memcpy(xt, x, (size_t)K * 4); *xs_out = 1.0f; }
static void lin_mm_packed(const Lin *l, const int8_t *xt, float xs, float *y, int nt) {
    const float *x = (const float *)xt; (void)xs; (void)nt;
    for (int n = 0; n < l->N; n++) { const float *w = l->W + (size_t)n * l->K; float acc = 0;
        for (int k = 0; k < l->K; k++) acc += w[k] * x[k]; y[n] = acc; }
}
static void lin_mm(const Lin *l, const float *x, float *y, int nt, int8_t *xt) {
    float xs; pack_act(x, l->K, xt, &xs); lin_mm_packed(l, xt, xs, y, nt);
}
"""

FWD_EXPORTS = r"""
/* ---- written here: exported wrappers ---- */
void golden_softmax(float *x, int n) { softmax(x, n); }
void golden_rmsnorm(float *o, const float *x, const float *w, int n, float eps) { rmsnorm(o, x, w, n, eps); }
void golden_rope(float *v, int hd, int pos, float base) { rope(v, hd, pos, base); }
void golden_rope_table(float *c, float *s, int hd, int pos, float base) { rope_table(c, s, hd, pos, base); }
void golden_rope_apply(float *v, int hd, const float *c, const float *s) { rope_apply(v, hd, c, s); }
void golden_swiglu(float *g, const float *u, int n) { swiglu_exact(g, u, n); }
void golden_topk(const float *logits, int ne, int na, int *sel, float *sw) {
    float rl[256]; memcpy(rl, logits, (size_t)ne * 4); softmax(rl, ne);
    TOPK_LINE
    RENORM_LINE
}
static Model M;
void golden_setup(int d, int nl, int nh, int nkv, int hd, int vocab, int n_exp, int n_act, int moe, float rope_base,
                  float eps, float *tok_embd, float *out_norm, float *lm, float *attn_norm, float *ffn_norm,
                  float *q_norm, float *k_norm, float *router, float *wq, float *wk, float *wv, float *wo,
                  float *eg, float *eu, float *ed) {
    const int qd = nh * hd, kvd = nkv * hd;
    M.d = d; M.nl = nl; M.nh = nh; M.nkv = nkv; M.hd = hd; M.vocab = vocab; M.nt = 1; M.n_exp = n_exp;
    M.n_act = n_act; M.moe = moe; M.rope_base = rope_base; M.eps = eps; M.tok_embd = tok_embd; M.out_norm = out_norm;
    M.lm = (Lin){vocab, d, lm};
    M.L = calloc((size_t)nl, sizeof(Layer));
    for (int l = 0; l < nl; l++) { Layer *y = &M.L[l];
        y->attn_norm = attn_norm + (size_t)l * d; y->ffn_norm = ffn_norm + (size_t)l * d;
        y->q_norm = q_norm + (size_t)l * hd; y->k_norm = k_norm + (size_t)l * hd;
        y->router = router + (size_t)l * n_exp * d;
        y->q = (Lin){qd, d, wq + (size_t)l * qd * d}; y->k = (Lin){kvd, d, wk + (size_t)l * kvd * d};
        y->v = (Lin){kvd, d, wv + (size_t)l * kvd * d}; y->o = (Lin){d, qd, wo + (size_t)l * d * qd};
        y->eg = calloc((size_t)n_exp, sizeof(Lin)); y->eu = calloc((size_t)n_exp, sizeof(Lin));
        y->ed = calloc((size_t)n_exp, sizeof(Lin));
        for (int e = 0; e < n_exp; e++) { size_t i = (size_t)l * n_exp + e;
            y->eg[e] = (Lin){moe, d, eg + i * moe * d}; y->eu[e] = (Lin){moe, d, eu + i * moe * d};
            y->ed[e] = (Lin){d, moe, ed + i * d * moe}; } }
}
/* one forward() step; Kc / Vc in the reference's layout [layer][ctx][nkv*hd] */
void golden_step(int tok, int pos, float *Kc, float *Vc, int ctx, float *logits) {
    const int d = M.d, qd = M.nh * M.hd, kvd = M.nkv * M.hd;
    size_t big = (size_t)(d > qd ? d : qd); if (big < (size_t)M.moe) big = M.moe; if (big < (size_t)ctx) big = ctx;
    float *hn = malloc(d * 4), *q = malloc(qd * 4), *k = malloc(kvd * 4), *vv = malloc(kvd * 4), *att = malloc(qd * 4);
    float *tmp = malloc(big * 4), *g = malloc(M.moe * 4), *u = malloc(M.moe * 4), *eout = malloc(d * 4);
    int8_t *xt = malloc(big * 4), *xt2 = malloc(big * 4);
    Kv kv = {Kc, Vc, kvd, ctx};
    forward(&M, tok, pos, &kv, logits, hn, q, k, vv, att, tmp, g, u, eout, xt, xt2);
    free(hn); free(q); free(k); free(vv); free(att); free(tmp); free(g); free(u); free(eout); free(xt); free(xt2);
}
"""


def build_ref_forward(tmp: str, tag: str) -> C.CDLL:
    """qwen_moe.c's forward() and its helpers, and qwen_moe_q3k.c's RoPE table
    and exact SwiGLU, extracted unchanged and compiled under tmp with the fp32
    linear-layer stubs above.  `tag` names the library file: forward() keeps
    a static residual buffer sized by the first model's d, so every model
    size gets its own copy of the library."""
    moe = open(os.path.join(REF_ROOT, "qwen_moe.c")).read()
    q3k = open(os.path.join(REF_ROOT, "qwen_moe_q3k.c")).read()
    rms_moe = extract_line(moe, r"^static void rmsnorm\(float\*o,const float\*x,const float\*w,int n,float eps\).*$")
    rms_q3k = extract_line(q3k, r"^static void rmsnorm\(float\*o,const float\*x,const float\*w,int n,float eps\).*$")
    assert rms_moe == rms_q3k, "the engines' rmsnorm differ"
    sm_moe = extract_line(moe, r"^static void softmax\(float\*x,int n\)\{ float m=-1e30f;.*$")
    body = sm_moe[sm_moe.index("{") + 1:sm_moe.rindex("}")].strip()
    q3k_soft = extract_function(q3k, r"static void softmax\(float\*x,int n\)\{")
    assert body in q3k_soft, "qwen_moe_q3k.c softmax's scalar branch is not qwen_moe.c's softmax"
    exports = FWD_EXPORTS.replace(
        "TOPK_LINE", extract_line(moe, r"^\s*for\(int a=0;a<na;a\+\+\)\{ int bi=-1; float bv=-1;.*$").strip()).replace(
        "RENORM_LINE", extract_line(moe, r"^\s*float ssum=0; for\(int a=0;a<na;a\+\+\)ssum\+=sw\[a\];.*$").strip())
    parts = [
        "#include <stdio.h>\n#include <stdlib.h>\n#include <stdint.h>\n#include <string.h>\n#include <math.h>\n"
        "#include <time.h>\n",
        FWD_STUBS,
        extract_function(moe, r"static double now\(void\)\{"),
        extract_line(moe, r"^static double gT_actpack=0, gT_lin=0, gT_attn=0, gT_rest=0;.*$"),
        extract_line(moe, r"^typedef struct \{ float\*attn_norm,\*ffn_norm,\*q_norm,\*k_norm,\*router;.*\} Layer;$"),
        extract_line(moe, r"^typedef struct \{ int d,nl,nh,nkv,hd,vocab,nt,n_exp,n_act,moe;.*\} Model;$"),
        rms_moe,
        extract_line(moe, r"^static void rope\(float\*v,int hd,int pos,float base\).*$"),
        sm_moe,
        extract_line(moe, r"^typedef struct \{ float\*Kc,\*Vc; int kvd,ctx; \} Kv;$"),
        extract_function(moe, r"static void forward\(Model\*m,int tok,int pos,Kv\*kv,float\*logits,"),
        extract_function(q3k, r"static void rope_table\(float\*cosb,float\*sinb,int hd,int pos,float base\)\{"),
        extract_function(q3k, r"static void rope_apply\(float\*v,int hd,const float\*cosb,const float\*sinb\)\{"),
        extract_function(q3k, r"static void swiglu_exact\(float\*g,const float\*u,int n\)\{"),
        exports,
    ]
    path = os.path.join(tmp, f"reffwd_{tag}.c")
    with open(path, "w") as f:
        f.write("\n".join(parts))
    so = os.path.join(tmp, f"libreffwd_{tag}.so")
    subprocess.check_call(["gcc", "-std=gnu11", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-w",
                           "-o", so, path, "-lm"])
    L = C.CDLL(so)
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    L.golden_softmax.argtypes = [vp, i]
    L.golden_rmsnorm.argtypes = [vp, vp, vp, i, f]
    L.golden_rope.argtypes = [vp, i, i, f]
    L.golden_rope_table.argtypes = [vp, vp, i, i, f]
    L.golden_rope_apply.argtypes = [vp, i, vp, vp]
    L.golden_swiglu.argtypes = [vp, vp, i]
    L.golden_topk.argtypes = [vp, i, i, vp, vp]
    L.golden_setup.argtypes = [i] * 9 + [f, f] + [vp] * 15
    L.golden_step.argtypes = [i, i, vp, vp, i, vp]
    return L


def _p(a):
    return C.c_void_p(a.ctypes.data)


def make_moe_golden() -> None:
    rng = np.random.default_rng(4242)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        L = build_ref_forward(tmp, "fn")
        # softmax: router-sized, attention-sized, ties, huge and tiny logits, n = 1
        vecs = [rng.standard_normal(128) * 3, np.full(8, 0.5), np.array([1e4, -1e4, 0.0, 1e4]), np.array([42.0]),
                rng.standard_normal(4096) * 10, np.array([1.0, np.nextafter(np.float32(1), np.float32(2)), 1.0]),
                np.array([-1e4, -1e4 + 1, -3e4]), rng.standard_normal(256) * 40]
        vecs = [np.asarray(v, np.float32) for v in vecs]
        x = np.concatenate(vecs)
        off = np.cumsum([0] + [v.size for v in vecs]).astype(np.int64)
        y = x.copy()
        for a, b in zip(off[:-1], off[1:]):
            seg = np.ascontiguousarray(y[a:b])
            L.golden_softmax(_p(seg), int(b - a))
            y[a:b] = seg
        out.update(softmax_x=x, softmax_off=off, softmax_y=y)
        # top-k after softmax: random routers, exact ties at the selection
        # boundary, all-equal logits, duplicates above the boundary
        cases = []
        for t in range(6):
            cases.append((128, 8, rng.standard_normal(128) * (0.2 + t)))
        tie = rng.standard_normal(128) - 5.0
        tie[[3, 5, 9, 100]] = 2.0                              # four equal maxima, two slots
        cases.append((128, 2, tie))
        bnd = rng.standard_normal(128) - 5.0
        bnd[:6] = np.arange(6) + 3.0
        bnd[[40, 7, 99, 64]] = 1.5                             # four tied for the last two of eight
        cases.append((128, 8, bnd))
        cases.append((16, 4, np.zeros(16)))                    # all equal
        cases.append((128, 16, rng.standard_normal(128)))
        dup = rng.standard_normal(64)
        dup[10] = dup[20] = dup[30] = dup.max() + 1.0          # tied maxima
        cases.append((64, 8, dup))
        tl, tn, tk, ts, tw = [], [], [], [], []
        for ne, na, lg in cases:
            lg = np.ascontiguousarray(np.asarray(lg, np.float32))
            sel = np.zeros(na, np.int32)
            sw = np.zeros(na, np.float32)
            L.golden_topk(_p(lg), ne, na, _p(sel), _p(sw))
            tl.append(lg), tn.append(ne), tk.append(na), ts.append(sel), tw.append(sw)
        out.update(topk_logits=np.concatenate(tl), topk_ne=np.array(tn, np.int32), topk_na=np.array(tk, np.int32),
                   topk_sel=np.concatenate(ts), topk_w=np.concatenate(tw))
        # rmsnorm: hidden-sized, head-sized, zero and large vectors
        rx = [rng.standard_normal(2048), rng.standard_normal(128), np.zeros(128), rng.standard_normal(2048) * 1e3,
              rng.standard_normal(256) * 1e-4]
        rx = [np.asarray(v, np.float32) for v in rx]
        rw = [np.asarray(1 + 0.1 * rng.standard_normal(v.size), np.float32) for v in rx]
        ro = []
        for v, w in zip(rx, rw):
            o = np.zeros_like(v)
            L.golden_rmsnorm(_p(o), _p(v), _p(w), v.size, C.c_float(1e-6))
            ro.append(o)
        out.update(rms_x=np.concatenate(rx), rms_w=np.concatenate(rw), rms_y=np.concatenate(ro),
                   rms_off=np.cumsum([0] + [v.size for v in rx]).astype(np.int64))
        # RoPE: head_dim 128, base 1e6 (the decode configuration) and 64 / 1e4
        rp = [(128, 1e6, p) for p in (0, 1, 2, 63, 64, 1000, 2047, 4095)] + [(64, 1e4, p) for p in (0, 7, 511)]
        cs, vin, vt, vr = [], [], [], []
        for hd, base, pos in rp:
            c = np.zeros(hd // 2, np.float32)
            s_ = np.zeros(hd // 2, np.float32)
            L.golden_rope_table(_p(c), _p(s_), hd, pos, C.c_float(base))
            v = np.asarray(rng.standard_normal(hd), np.float32)
            a1 = v.copy()
            L.golden_rope_apply(_p(a1), hd, _p(c), _p(s_))
            a2 = v.copy()
            L.golden_rope(_p(a2), hd, pos, C.c_float(base))
            cs.append(np.concatenate([c, s_])), vin.append(v), vt.append(a1), vr.append(a2)
        out.update(rope_cfg=np.array(rp, np.float64), rope_cossin=np.concatenate(cs), rope_v=np.concatenate(vin),
                   rope_table_apply=np.concatenate(vt), rope_inline=np.concatenate(vr))
        # SwiGLU: a grid over the range where expf under/overflows, plus random
        g = np.concatenate([np.linspace(-120, 120, 481), rng.standard_normal(1000) * 4, [0.0, -0.0, 88.7, -88.7, -104.0]])
        g = np.asarray(g, np.float32)
        u = np.asarray(rng.standard_normal(g.size), np.float32)
        gy = g.copy()
        L.golden_swiglu(_p(gy), _p(u), g.size)
        out.update(swiglu_g=g, swiglu_u=u, swiglu_y=gy)
    np.savez_compressed(os.path.join(HERE, "moe_golden.npz"), **out)
    print("wrote moe_golden.npz")


def make_forward_golden() -> None:
    import golden_inputs as gi
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        dec = build_ref_decoders(tmp)

        def deq(qt, blk, n):
            y = np.zeros(n, np.float32)
            if qt == po.Q3_K:
                dec.golden_dq_q3k(blk.ctypes.data, n // 256, y.ctypes.data)
            else:
                dec.golden_dq_gguf(qt, blk.ctypes.data, n, y.ctypes.data)
            return y

        for case, c in gi.CASES.items():
            m = gi.model(case)
            d, hd, E, F, V = c["d"], c["head_dim"], c["n_exp"], c["moe_ffn"], c["vocab"]
            qd, kvd, nl = c["n_heads"] * hd, c["n_kv_heads"] * hd, c["n_layers"]
            at, et = c["attn_qtype"], c["expert_qtype"]
            cat = lambda key: np.ascontiguousarray(np.concatenate([ly[key].reshape(-1) for ly in m["layers"]]))  # noqa: E731
            dq = lambda key, qt, n: np.ascontiguousarray(np.concatenate(  # noqa: E731
                [deq(qt, ly[key], n) for ly in m["layers"]]))
            arrs = dict(tok_embd=np.ascontiguousarray(m["tok_embd"]), out_norm=m["out_norm"],
                        lm=deq(c["lm_qtype"], m["lm"], V * d),
                        attn_norm=cat("attn_norm"), ffn_norm=cat("ffn_norm"), q_norm=cat("q_norm"),
                        k_norm=cat("k_norm"), router=cat("router"),
                        wq=dq("wq", at, qd * d), wk=dq("wk", at, kvd * d), wv=dq("wv", at, kvd * d),
                        wo=dq("wo", at, d * qd), eg=dq("gate", et, E * F * d), eu=dq("up", et, E * F * d),
                        ed=dq("down", et, E * d * F))
            L = build_ref_forward(tmp, case)
            L.golden_setup(d, nl, c["n_heads"], c["n_kv_heads"], hd, V, E, c["n_act"], F,
                           C.c_float(c["rope_base"]), C.c_float(c["eps"]),
                           *(_p(arrs[k]) for k in ("tok_embd", "out_norm", "lm", "attn_norm", "ffn_norm", "q_norm",
                                                   "k_norm", "router", "wq", "wk", "wv", "wo", "eg", "eu", "ed")))
            ctx = c["ctx"]
            Kc = np.zeros((nl, ctx, kvd), np.float32)
            Vc = np.zeros((nl, ctx, kvd), np.float32)
            logits = []
            for st, (tok, pos) in enumerate(c["steps"]):
                if c["prefill"]:
                    for li in range(nl):   # oracle layout [nkv][ctx][hd] -> the reference's [ctx][nkv*hd]
                        k, v = gi.prefill_cache(case, li, st)
                        Kc[li] = k.transpose(1, 0, 2).reshape(ctx, kvd)
                        Vc[li] = v.transpose(1, 0, 2).reshape(ctx, kvd)
                lg = np.zeros(V, np.float32)
                L.golden_step(tok, pos, _p(Kc), _p(Vc), ctx, _p(lg))
                logits.append(lg)
            out[f"{case}_logits"] = np.stack(logits)
            print(f"forward case {case}: {len(logits)} steps")
    np.savez_compressed(os.path.join(HERE, "forward_golden.npz"), **out)
    print("wrote forward_golden.npz")


def main():
    if "--only-moe" in sys.argv:
        po.build()
        make_moe_golden()
        make_forward_golden()
        return
    if "--only-a8" in sys.argv:
        po.build()
        make_a8_golden()
        return
    if "--only-gguf" in sys.argv:
        po.build()
        make_gguf_golden()
        return
    po.build()
    ref = po.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libx100ref.so missing: the reference tree is needed")
    meta = {"ref_root": os.path.relpath(REF_ROOT, REPO), "gemm_shapes": GEMM_SHAPES,
            "gemm_hash_shapes": GEMM_HASH_SHAPES}
    gem = {}
    for (M, N, K) in GEMM_SHAPES + GEMM_HASH_SHAPES:
        seed = 1000003 * M + 1009 * N + K
        A = po.rand_i8(seed, M * K).reshape(M, K)
        B = po.rand_i8(seed + 1, K * N).reshape(K, N)
        C0 = po.rand_i8(seed + 2, M * N).astype(np.int32).reshape(M, N) * 1000
        Ci = C0.copy()
        ref.gemm_ref_i8(M, N, K, A.ctypes.data, B.ctypes.data, Ci.ctypes.data)
        Af = po.rand_f32(seed + 3, M * K).reshape(M, K)
        Bf = po.rand_f32(seed + 4, K * N).reshape(K, N)
        Cf = po.rand_f32(seed + 5, M * N).reshape(M, N)
        ref.gemm_ref_f32(M, N, K, Af.ctypes.data, Bf.ctypes.data, Cf.ctypes.data)
        key = f"{M}x{N}x{K}"
        if (M, N, K) in GEMM_SHAPES:
            gem[f"i8_{key}"] = Ci
            gem[f"f32_{key}"] = Cf
        else:
            meta[f"sha256_i8_{key}"] = hashlib.sha256(Ci.tobytes()).hexdigest()
            meta[f"sha256_f32_{key}"] = hashlib.sha256(Cf.tobytes()).hexdigest()
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **gem)

    with tempfile.TemporaryDirectory() as tmp:
        dec = build_ref_decoders(tmp)
        meta["sizeof_block_q3_K"] = int(dec.golden_sizeof_q3k())
        meta["sizeof_block_q5_K"] = int(dec.golden_sizeof_q5k())
        meta["caps_layout"] = caps_layout(tmp)
        qg = {}
        for qtype, name in ((po.Q4_0, "Q4_0"), (po.Q8_0, "Q8_0"), (po.Q3_K, "Q3_K"), (po.Q4_K, "Q4_K")):
            blk = np.concatenate([random_blocks(qtype, 96, 77 + qtype), edge_blocks(qtype)])
            blk = np.ascontiguousarray(blk)
            nb = blk.shape[0]
            be = po.BLOCK_ELEMS[qtype]
            out = np.zeros(nb * be, np.float32)
            if qtype in (po.Q4_0, po.Q8_0):
                dec.golden_dq_gguf(qtype, blk.ctypes.data, nb * be, out.ctypes.data)
            elif qtype == po.Q3_K:
                dec.golden_dq_q3k(blk.ctypes.data, nb, out.ctypes.data)
            else:
                q5 = np.ascontiguousarray(to_q5k_layout(blk))
                dec.golden_dq_q5k(q5.ctypes.data, nb, out.ctypes.data)
            qg[f"{name}_blocks"] = blk
            qg[f"{name}_values"] = out
        np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **qg)
    with open(os.path.join(HERE, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote gemm_golden.npz, quant_golden.npz, meta.json")
    make_gguf_golden()
    make_a8_golden()
    make_moe_golden()
    make_forward_golden()


if __name__ == "__main__":
    main()
