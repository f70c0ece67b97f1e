"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container where the reference tree is mounted (REF_ROOT, default
/root/reference); the fixtures it writes are committed so that the tests never
need the reference at run time.

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
                    pack_A_i8 (qwen_moe_q3k.c:420-426) and pack_A_q3k
                    (:613-623), compiled from the reference and run on fp32
                    rows (normal values, rounding ties, zeros, tiny and large
                    values).
  meta.json         struct-size known answers (block_q3_K 110 B,
                    block_q5_K 176 B, bench/q3k_probe.c:410-413) and the
                    x100_caps_t layout of the reference header.
The extracted reference functions are compiled under a temporary directory
and never written into this repository.
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

REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")

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
    parts = [
        "#include <stdint.h>\n#include <string.h>\n#include <math.h>\n",
        extract_line(q3k, r"^#define AREC_Q3K 292$"),
        extract_function(q3k, r"static void pack_A_i8\(const float\*x, uint8_t\*out [^)]*\)\{"),
        extract_function(q3k, r"static void pack_A_q3k\(const float\*a,uint8_t\*out\)\{"),
        """
void golden_pack_i8(const float*x,int K,uint8_t*out){ for(int kg=0;kg<K/32;kg++) pack_A_i8(x+32*kg,out+38*kg); }
void golden_pack_q3k(const float*x,int K,uint8_t*out){ for(int sb=0;sb<K/256;sb++) pack_A_q3k(x+256*sb,out+AREC_Q3K*sb); }
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
        np.savez_compressed(os.path.join(HERE, "a8_golden.npz"), x=x, pack_i8=i8, pack_q3k=q3)
    print("wrote a8_golden.npz")


def main():
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
    meta = {"ref_root": REF_ROOT, "gemm_shapes": GEMM_SHAPES, "gemm_hash_shapes": GEMM_HASH_SHAPES}
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


if __name__ == "__main__":
    main()
