"""ctypes view of oracle/liboracle.so and oracle/_ref/libx100ref.so.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker; the product library never calls
it.  liboracle.so is this repository's C restatement of the reference's
scalar paths (see x100_oracle.h for the file:line each function follows);
libx100ref.so is the reference's own src/gemm_ref.c etc. compiled unchanged
(built by oracle/Makefile when the reference tree is present).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

Q_F32, Q4_0, Q8_0, Q3_K, Q4_K = 0, 2, 8, 11, 12
BLOCK_ELEMS = {Q_F32: 1, Q4_0: 32, Q8_0: 32, Q3_K: 256, Q4_K: 256}
BLOCK_BYTES = {Q_F32: 4, Q4_0: 18, Q8_0: 34, Q3_K: 110, Q4_K: 144}
QNAMES = {Q4_0: "Q4_0", Q8_0: "Q8_0", Q3_K: "Q3_K", Q4_K: "Q4_K", Q_F32: "F32"}
# further GGUF tensor types (decode only): id -> (elements, bytes) per block
F16, Q4_1, Q5_K, Q6_K = 1, 3, 13, 14
GGUF_BLOCK = {Q_F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q8_0: (32, 34), Q3_K: (256, 110),
              Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}

_lib = None
_ref = None


def _ptr(a):
    return C.c_void_p(a.ctypes.data) if a is not None else C.c_void_p(0)


def build():
    """Build liboracle.so (and _ref/ when the reference tree exists)."""
    subprocess.check_call(["make", "-s", "-C", HERE, "all"])


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        for name, args in {
            "orc_gemm_i8": [i, i, i, vp, vp, vp],
            "orc_gemm_f32": [i, i, i, vp, vp, vp],
            "orc_gemm_i8_mt": [i, i, i, vp, vp, vp, i],
            "orc_gemm_f32_mt": [i, i, i, vp, vp, vp, i],
            "orc_ime2_pack_a": [i, i, vp, vp],
            "orc_ime2_pack_b": [i, i, vp, vp],
            "orc_dequant_row": [i, vp, i, vp],
            "orc_quantize": [i, i, i, vp, vp],
            "orc_qgemv_mt": [i, i, i, vp, vp, vp, i, i],
            "orc_softmax": [vp, i],
            "orc_topk": [vp, i, i, vp, vp],
            "orc_moe_ffn": [i, i, i, i, i, vp, vp, vp, vp, i, i, vp, vp, i, vp, vp, i],
            "orc_rmsnorm": [vp, vp, vp, i, f],
            "orc_rope_neox": [vp, i, i, f],
            "orc_decode_layer": [i, i, i, i, i, i, f, f, i] + [vp] * 8 + [i, i, i, i] + [vp] * 4 +
                                [vp, vp, vp, vp, vp, i],
            "orc_decode_layer_f32kv": [i, i, i, i, i, i, f, f, i] + [vp] * 8 + [i, i, i, i] + [vp] * 4 +
                                      [vp, vp, vp, vp, vp, i],
            "orc_decode_layer_probs": [i, i, i, i, i, i, f, f, i] + [vp] * 8 + [i, i, i, i] + [vp] * 4 +
                                      [vp, vp, vp, vp, vp, vp, i],
            "orc_decode_head": [i, i, f, i, vp, vp, vp, vp, i],
            "orc_fill_u8": [C.c_uint64, vp, C.c_size_t],
            "orc_kq_scale_min": [i, vp, vp, vp],
        }.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f32_to_f16_rne.argtypes = [C.c_float]
        L.orc_f32_to_f16_rne.restype = C.c_uint16
        L.orc_f32_to_f16_trunc.argtypes = [C.c_float]
        L.orc_f32_to_f16_trunc.restype = C.c_uint16
        L.orc_dequant_gguf.argtypes = [i, vp, C.c_size_t, vp]
        L.orc_dequant_gguf.restype = C.c_int
        L.orc_gguf_bytes.argtypes = [i, C.c_size_t]
        L.orc_gguf_bytes.restype = C.c_size_t
        L.orc_quantize_q8_0_ref.argtypes = [vp, C.c_size_t, vp]
        L.orc_quantize_q8_0_ref.restype = None
        L.orc_pack_a_i8.argtypes = [vp, i, vp]
        L.orc_pack_a_i8.restype = None
        L.orc_pack_a_q3k.argtypes = [vp, i, vp]
        L.orc_pack_a_q3k.restype = None
        L.orc_pack_a_hp.argtypes = [vp, i, vp]
        L.orc_pack_a_hp.restype = None
        L.orc_quantize_q4_0_hp.argtypes = [vp, C.c_size_t, vp]
        L.orc_quantize_q4_0_hp.restype = None
        L.orc_qgemv_a8.argtypes = [i, i, i, vp, vp, vp, i]
        L.orc_qgemv_a8.restype = None
        L.orc_silu.argtypes = [C.c_float]
        L.orc_silu.restype = C.c_float
        _lib = L
    return _lib


def ref_lib():
    """The reference's own GEMM sources compiled unchanged, or None."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libx100ref.so")
        if not os.path.exists(path):
            return None
        L = C.CDLL(path)
        for n in ("gemm_ref_i8", "gemm_ref_f32", "gemm_ime_i8", "gemm_rvv_f32"):
            getattr(L, n).argtypes = [C.c_int] * 3 + [C.c_void_p] * 3
            getattr(L, n).restype = None
        _ref = L
    return _ref


def ref_gemm_i8_mt(A, B, C, nthreads):
    """C += A @ B by the reference's own gemm_ref_i8 (oracle/_ref/libx100ref.so,
    src/gemm_ref.c compiled unchanged) on row slices, one host thread each
    (ctypes releases the GIL for the call).  Raises if the library is absent."""
    from concurrent.futures import ThreadPoolExecutor
    ref = ref_lib()
    if ref is None:
        raise FileNotFoundError("oracle/_ref/libx100ref.so missing (build it where the reference tree exists)")
    M, K = A.shape
    N = B.shape[1]
    assert A.flags.c_contiguous and B.flags.c_contiguous and C.flags.c_contiguous and C.shape == (M, N)
    per = [(M * t) // nthreads for t in range(nthreads + 1)]

    def work(t):
        r0, r1 = per[t], per[t + 1]
        if r1 > r0:
            ref.gemm_ref_i8(r1 - r0, N, K, A[r0:].ctypes.data, B.ctypes.data, C[r0:].ctypes.data)
    with ThreadPoolExecutor(nthreads) as ex:
        list(ex.map(work, range(nthreads)))
    return C


# ---- generators ------------------------------------------------------------
def fill_u8(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().orc_fill_u8(seed, _ptr(out), n)
    return out


def rand_i8(seed: int, n: int) -> np.ndarray:
    """Uniform int8 in [-128, 127] from the reference's xorshift64 stream."""
    return fill_u8(seed, n).view(np.int8)


def rand_f32(seed: int, n: int, lo=-1.0, hi=1.0) -> np.ndarray:
    """Uniform fp32 in [lo, hi) with 24-bit resolution (exactly representable)."""
    u = fill_u8(seed, 4 * n).view(np.uint32)
    return (lo + (hi - lo) * ((u >> 8).astype(np.float64) / float(1 << 24))).astype(np.float32)


# ---- GGUF tensor types ---------------------------------------------------------
def gguf_bytes(gtype: int, n: int) -> int:
    return int(lib().orc_gguf_bytes(gtype, n))


def dequant_gguf(gtype: int, data: np.ndarray, n: int) -> np.ndarray:
    """n elements of a GGUF tensor of any decodable type, as fp32."""
    data = np.ascontiguousarray(data).view(np.uint8)
    assert data.nbytes >= gguf_bytes(gtype, n) > 0
    out = np.empty(n, np.float32)
    assert lib().orc_dequant_gguf(gtype, _ptr(data), n, _ptr(out)) == 0
    return out


def quantize_q8_0_ref(x: np.ndarray) -> np.ndarray:
    """The reference's Q8_0 requantisation of fp32 values (n % 32 == 0)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().orc_quantize_q8_0_ref(_ptr(x), x.size, _ptr(out))
    return out


# ---- the reference's activation packing ("A8") ----------------------------------
def pack_a(mode: str, x: np.ndarray) -> np.ndarray:
    """pack_A_i8 ('i8', 38 B per 32), pack_A_q3k ('q3k', 292 B per 256) or
    pack_A_hp ('hp', 290 B per 256) of one fp32 row."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    if mode == "i8":
        out = np.empty(x.size // 32 * 38, np.uint8)
        lib().orc_pack_a_i8(_ptr(x), x.size, _ptr(out))
    elif mode == "hp":
        out = np.empty(x.size // 256 * 290, np.uint8)
        lib().orc_pack_a_hp(_ptr(x), x.size, _ptr(out))
    else:
        out = np.empty(x.size // 256 * 292, np.uint8)
        lib().orc_pack_a_q3k(_ptr(x), x.size, _ptr(out))
    return out


def quantize_q4_0_hp(w: np.ndarray) -> np.ndarray:
    """quantize_q4_0_native (qwen_moe_hp.c:102-109) of fp32 weights (rows of a
    multiple of 32): GGUF Q4_0 blocks with d = max|w| / 8, q in [-8, 7]."""
    w = np.ascontiguousarray(w, np.float32).reshape(-1)
    out = np.empty(w.size // 32 * 18, np.uint8)
    lib().orc_quantize_q4_0_hp(_ptr(w), w.size, _ptr(out))
    return out


def qgemv_a8(qtype: int, blocks: np.ndarray, N: int, K: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), np.float32)
    lib().orc_qgemv_a8(qtype, N, K, _ptr(blocks), _ptr(x), _ptr(y), x.shape[0])
    return y


# ---- GEMM -------------------------------------------------------------------
def gemm_i8(A, B, C, nthreads=1):
    M, K = A.shape
    N = B.shape[1]
    assert A.dtype == np.int8 and B.dtype == np.int8 and C.dtype == np.int32
    lib().orc_gemm_i8_mt(M, N, K, _ptr(A), _ptr(B), _ptr(C), nthreads)
    return C


def gemm_f32(A, B, C, nthreads=1):
    M, K = A.shape
    N = B.shape[1]
    assert A.dtype == np.float32 and B.dtype == np.float32 and C.dtype == np.float32
    lib().orc_gemm_f32_mt(M, N, K, _ptr(A), _ptr(B), _ptr(C), nthreads)
    return C


def ime2_pack(A, B):
    M, K = A.shape
    N = B.shape[1]
    pa = np.empty(M * K, np.int8)
    pb = np.empty(K * N, np.int8)
    lib().orc_ime2_pack_a(M, K, _ptr(A), _ptr(pa))
    lib().orc_ime2_pack_b(K, N, _ptr(B), _ptr(pb))
    return pa, pb


# ---- quantised formats --------------------------------------------------------
def row_bytes(qtype: int, K: int) -> int:
    be = BLOCK_ELEMS[qtype]
    assert K % be == 0
    return K // be * BLOCK_BYTES[qtype]


def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    out = np.zeros(N * row_bytes(qtype, K), np.uint8)
    lib().orc_quantize(qtype, N, K, _ptr(w), _ptr(out))
    return out


def dequant(qtype: int, blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    out = np.empty((N, K), np.float32)
    rb = row_bytes(qtype, K)
    blocks = np.ascontiguousarray(blocks, np.uint8)
    for n in range(N):
        lib().orc_dequant_row(qtype, C.c_void_p(blocks.ctypes.data + n * rb), K,
                              C.c_void_p(out.ctypes.data + n * K * 4))
    return out


def qgemv(qtype: int, blocks: np.ndarray, N: int, K: int, x: np.ndarray, nthreads=1):
    x = np.ascontiguousarray(x, np.float32).reshape(-1, K)
    y = np.empty((x.shape[0], N), np.float32)
    lib().orc_qgemv_mt(qtype, N, K, _ptr(blocks), _ptr(x), _ptr(y), x.shape[0], nthreads)
    return y


def moe_ffn(d, n_exp, n_act, ffn, qtype, router, gate, up, down, hn,
            expert_lo=0, expert_hi=None, nthreads=1):
    expert_hi = n_exp if expert_hi is None else expert_hi
    hn = np.ascontiguousarray(hn, np.float32).reshape(-1, d)
    B = hn.shape[0]
    eout = np.empty((B, d), np.float32)
    sel = np.empty((B, n_act), np.int32)
    w = np.empty((B, n_act), np.float32)
    lib().orc_moe_ffn(d, n_exp, n_act, ffn, qtype, _ptr(router), _ptr(gate), _ptr(up), _ptr(down),
                      expert_lo, expert_hi, _ptr(hn), _ptr(eout), B, _ptr(sel), _ptr(w), nthreads)
    return eout, sel, w


def route(router, hn, n_act):
    """Routing only (qwen_moe.c:296-301): fp32 router logits in k order,
    softmax, greedy top-n_act, renormalised weights.  router [n_exp][d],
    hn [batch][d]; returns (sel, w), each [batch][n_act].  Runs orc_moe_ffn
    with an empty expert range, so no expert weights are touched."""
    router = np.ascontiguousarray(router, np.float32)
    n_exp, d = router.shape
    hn = np.ascontiguousarray(hn, np.float32).reshape(-1, d)
    B = hn.shape[0]
    eout = np.empty((B, d), np.float32)
    sel = np.empty((B, n_act), np.int32)
    w = np.empty((B, n_act), np.float32)
    lib().orc_moe_ffn(d, n_exp, n_act, 32, Q4_0, _ptr(router), None, None, None, 0, 0,
                      _ptr(hn), _ptr(eout), B, _ptr(sel), _ptr(w), 1)
    return sel, w


def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def rel_l2(y, ref) -> float:
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30))


# ---- decode step (qwen_moe_q3k.c:1842-1983) ------------------------------------------
def top_margin(probs, k):
    """Relative gap between the k-th and (k+1)-th largest routing
    probabilities: how far the top-k was from a tie."""
    srt = np.sort(np.asarray(probs, np.float64))[::-1]
    return float((srt[k - 1] - srt[k]) / srt[k - 1])


def decode_layer(cfg, lw, kc, vc, h, pos, nthreads=1, probs=None):
    """One layer of forward() for one token: cfg is a dict of the model shape
    (d, n_heads, n_kv_heads, head_dim, ctx, rope_base, eps, attn_qtype, n_exp,
    n_act, moe_ffn, expert_qtype); lw a dict of the layer's weights (numpy:
    attn_norm, wq, wk, wv, q_norm, k_norm, wo, ffn_norm, router, gate, up,
    down); kc / vc uint16 [n_kv_heads][ctx][head_dim] fp16 caches, updated at
    pos; h [d] float32 updated in place.  Returns (sel, w) of the router."""
    assert h.dtype == np.float32 and h.flags.c_contiguous
    assert kc.dtype == np.uint16 and kc.flags.c_contiguous and vc.flags.c_contiguous
    sel = np.empty(cfg["n_act"], np.int32)
    w = np.empty(cfg["n_act"], np.float32)
    c = lambda a: np.ascontiguousarray(a)
    ws = {k: c(v) for k, v in lw.items()}
    args = [cfg["d"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ctx"], pos,
            cfg["rope_base"], cfg["eps"], cfg["attn_qtype"],
            *(_ptr(ws[k]) for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "ffn_norm")),
            cfg["n_exp"], cfg["n_act"], cfg["moe_ffn"], cfg["expert_qtype"],
            *(_ptr(ws[k]) for k in ("router", "gate", "up", "down")),
            _ptr(kc), _ptr(vc), _ptr(h), _ptr(sel), _ptr(w)]
    if probs is None:
        lib().orc_decode_layer(*args, nthreads)
    else:
        assert probs.dtype == np.float32 and probs.size >= cfg["n_exp"]
        lib().orc_decode_layer_probs(*args, _ptr(probs), nthreads)
    return sel, w


def decode_layer_f32kv(cfg, lw, kc, vc, h, pos, nthreads=1):
    """decode_layer with an fp32 cache (float32 [n_kv_heads][ctx][head_dim]),
    the reference's own cache precision."""
    assert h.dtype == np.float32 and h.flags.c_contiguous
    assert kc.dtype == np.float32 and kc.flags.c_contiguous and vc.flags.c_contiguous
    sel = np.empty(cfg["n_act"], np.int32)
    w = np.empty(cfg["n_act"], np.float32)
    ws = {k: np.ascontiguousarray(v) for k, v in lw.items()}
    lib().orc_decode_layer_f32kv(cfg["d"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ctx"], pos,
                                 cfg["rope_base"], cfg["eps"], cfg["attn_qtype"],
                                 *(_ptr(ws[k]) for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo",
                                                         "ffn_norm")),
                                 cfg["n_exp"], cfg["n_act"], cfg["moe_ffn"], cfg["expert_qtype"],
                                 *(_ptr(ws[k]) for k in ("router", "gate", "up", "down")),
                                 _ptr(kc), _ptr(vc), _ptr(h), _ptr(sel), _ptr(w), nthreads)
    return sel, w


def decode_head(cfg, out_norm, lm, h, nthreads=1):
    """logits = lm . rmsnorm(h, out_norm) (qwen_moe_q3k.c:1980-1981)."""
    logits = np.empty(cfg["vocab"], np.float32)
    lib().orc_decode_head(cfg["d"], cfg["vocab"], cfg["eps"], cfg["lm_qtype"], _ptr(np.ascontiguousarray(out_norm)),
                          _ptr(np.ascontiguousarray(lm)), _ptr(np.ascontiguousarray(h, np.float32)),
                          _ptr(logits), nthreads)
    return logits
