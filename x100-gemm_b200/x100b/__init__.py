"""Python binding of libx100gemm_b200.so (ctypes over the C ABI).

The library is the product: hand-written sm_100a kernels behind the C ABI
declared in include/x100_gemm.h and include/x100q.h.  This module only loads
it, declares the signatures and offers numpy / torch conveniences for the
tests and bench.py.  There is no fallback: if the shared library is missing
or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os
import re

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libx100gemm_b200.so")
HEADERS = [os.path.join(REPO, "include", "x100_gemm.h"), os.path.join(REPO, "include", "x100q.h")]

X100_OK, X100_E_ARG, X100_E_NODEV, X100_E_ARCH, X100_E_ALLOC, X100_E_COPY, X100_E_LAUNCH, \
    X100_E_TIMEOUT, X100_E_COMM, X100_E_INJECTED, X100_E_UNSUPPORTED, X100_E_TOO_LARGE, X100_E_FORMAT = range(13)

Q_F32, Q4_0, Q8_0, Q3_K, Q4_K = 0, 2, 8, 11, 12


class X100Error(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        super().__init__(f"{what}: x100 error {code} ({strerror(code)})")


class Caps(C.Structure):
    _fields_ = [("vlen_bits", C.c_int), ("vlenb", C.c_int), ("has_v", C.c_int), ("has_zvfh", C.c_int),
                ("has_zvbb", C.c_int), ("has_ime", C.c_int), ("mvendorid", C.c_ulong), ("isa", C.c_char * 1024)]


_lib = None
vp, i32, i64 = C.c_void_p, C.c_int, C.c_long

_SIGS = {
    # reference signatures (void)
    "gemm_ref_f32": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_rvv_f32": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_rvv_f16": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_f16_f32acc": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_ref_i8": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_ime_i8": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_ime2_pack_a": ([i32, i32, vp, vp], None),
    "gemm_ime2_pack_b": ([i32, i32, vp, vp], None),
    "gemm_ime2_i8_st": ([i32, i32, i32, vp, vp, vp], None),
    "gemm_ime2_i8_mt": ([i32, i32, i32, vp, vp, vp, i32], None),
    "x100_detect": ([vp], None),
    "x100_caps_print": ([vp], None),
    # device variants
    "gemm_ime_i8_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_ref_i8_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_f16_f32acc_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_f16_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_f32_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_ref_f32_dev": ([i32, i32, i32, vp, vp, vp, vp], i32),
    "gemm_ime_i8_dev_ld": ([i32, i32, i32, vp, i64, vp, i64, vp, i64, vp], i32),
    "x100_sync": ([vp], i32),
    "x100_last_error": ([], i32),
    "x100_strerror": ([i32], C.c_char_p),
    "x100_set_device": ([i32], i32),
    # quantised path
    "x100q_row_bytes": ([i32, i32], C.c_size_t),
    "x100q_lin_create": ([i32, i32, i32, vp], vp),
    "x100q_lin_destroy": ([vp], None),
    "x100q_lin_info": ([vp, vp, vp, vp, vp], i32),
    "x100q_lin_gemv": ([vp, vp, vp, i32], i32),
    "x100q_lin_gemv_dev": ([vp, vp, vp, i32, vp], i32),
    "x100q_lin_gemv_dev_flags": ([vp, vp, vp, i32, i32, vp], i32),
    "x100q_moe_create": ([i32, i32, i32, i32, i32, vp, vp, vp, vp, i32, i32], vp),
    "x100q_moe_destroy": ([vp], None),
    "x100q_moe_ffn": ([vp, vp, vp, i32, vp, vp], i32),
    "x100q_moe_ffn_dev": ([vp, vp, vp, i32, vp, vp, vp], i32),
    "x100q_router_topk_noalloc": ([vp, vp, i32, i32, i32, i32, vp, vp, vp], i32),
    # decode step
    "x100q_model_create": ([vp], vp),
    "x100q_model_destroy": ([vp], None),
    "x100q_model_set_layer": ([vp, i32] + [vp] * 12, i32),
    "x100q_model_set_output": ([vp, vp, vp, vp], i32),
    "x100q_model_kv_copy": ([vp, i32, i32, i32, i32, vp, vp, i32], i32),
    "x100q_model_embed_dev": ([vp, vp, vp, i32, vp], i32),
    "x100q_model_layer_dev": ([vp, i32, vp, vp, i32, vp, vp, vp, vp], i32),
    "x100q_model_head_dev": ([vp, vp, vp, i32, vp], i32),
    "x100q_model_forward_dev": ([vp, vp, vp, vp, vp, i32, vp], i32),
    "x100q_model_forward": ([vp, vp, vp, vp, i32], i32),
    "x100q_model_forward_slots_dev": ([vp, vp, vp, vp, vp, vp, i32, vp], i32),
    "x100q_model_prefill": ([vp, i32, vp, i32, i32, vp], i32),
    "x100q_model_timing": ([vp, i32], i32),
    "x100q_model_timing_read": ([vp, vp, vp], i32),
    "x100q_timing_bucket_name": ([i32], C.c_char_p),
    # expert-parallel combine
    "x100q_ep_create": ([i32, i32, i32], vp),
    "x100q_ep_handle": ([vp, vp], i32),
    "x100q_ep_open": ([vp, vp], i32),
    "x100q_ep_allreduce_dev": ([vp, vp, vp, i32, i32, vp], i32),
    "x100q_ep_destroy": ([vp], None),
    # GGUF ingest
    "x100q_gguf_open": ([C.c_char_p], vp),
    "x100q_gguf_close": ([vp], None),
    "x100q_gguf_n_tensors": ([vp], i32),
    "x100q_gguf_tensor_at": ([vp, i32, vp], i32),
    "x100q_gguf_find": ([vp, C.c_char_p, vp], i32),
    "x100q_gguf_data_offset": ([vp], C.c_uint64),
    "x100q_gguf_n_tokens": ([vp], i32),
    "x100q_gguf_token": ([vp, i32], C.c_char_p),
    "x100q_gguf_get_int": ([vp, C.c_char_p, vp], i32),
    "x100q_gguf_get_f32": ([vp, C.c_char_p, vp], i32),
    "x100q_gguf_get_str": ([vp, C.c_char_p, vp], i32),
    "x100q_gguf_model_cfg": ([vp, vp], i32),
    "x100q_model_load_gguf": ([vp, vp], vp),
    "x100q_gguf_dequant_dev": ([i32, vp, C.c_long, vp, vp], i32),
    "x100q_quantize_q8_0_dev": ([vp, C.c_long, vp, vp], i32),
    "x100q_pack_act_dev": ([i32, vp, i32, i32, vp, vp], i32),
}


class GgufTensor(C.Structure):
    """x100q_gguf_tensor (include/x100q.h)."""
    _fields_ = [("name", C.c_char_p), ("type", C.c_int), ("n_dims", C.c_int), ("dims", C.c_uint64 * 4),
                ("n_elems", C.c_uint64), ("bytes", C.c_uint64), ("data", C.c_void_p)]


class ModelCfg(C.Structure):
    """x100q_model_cfg (include/x100q.h)."""
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d", "n_heads", "n_kv_heads", "head_dim", "vocab", "n_exp",
                                       "n_act", "moe_ffn", "attn_qtype", "expert_qtype", "lm_qtype", "ctx",
                                       "max_batch", "expert_lo", "expert_hi")] + \
               [("rope_base", C.c_float), ("eps", C.c_float)]


def lib():
    """Load libx100gemm_b200.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} missing: run __graft_entry__.build() (make -C x100-gemm_b200)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


TIMING_BUCKETS = 8   # X100Q_NBUCKETS


def timing_bucket_name(i: int) -> str | None:
    """Name of step-timing bucket i (x100q_timing_bucket_name)."""
    n = lib().x100q_timing_bucket_name(i)
    return n.decode() if n else None


def header_functions() -> list[str]:
    """Names of every function declared in include/*.h."""
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, flags=re.M):
            if m.group(1) not in ("defined",):
                names.append(m.group(1))
    return sorted(set(names))


def strerror(code: int) -> str:
    return lib().x100_strerror(code).decode()


def last_error() -> int:
    return lib().x100_last_error()


def check(code: int, what: str = "x100") -> None:
    if code != X100_OK:
        raise X100Error(code, what)


def check_last(what: str) -> None:
    check(last_error(), what)


def detect() -> Caps:
    caps = Caps()
    lib().x100_detect(C.byref(caps))
    return caps


def _p(a):
    """Raw pointer of a numpy array or torch tensor."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


# ---- host-pointer (reference-signature) calls ------------------------------------
def gemm_host(fn: str, A, B, Cm) -> None:
    """Call a void reference-signature GEMM (gemm_ime_i8, gemm_ref_f32, ...)
    on numpy arrays (or torch tensors); C += A @ B in place."""
    M, K = A.shape
    N = B.shape[1]
    getattr(lib(), fn)(M, N, K, _p(A), _p(B), _p(Cm))
    check_last(fn)


# ---- device-pointer calls (torch tensors) ----------------------------------------------
def gemm_dev(fn: str, A, B, Cm, stream=None) -> None:
    M, K = A.shape
    N = B.shape[1]
    check(getattr(lib(), fn)(M, N, K, _p(A), _p(B), _p(Cm), _stream(stream)), fn)


def sync(stream=None) -> None:
    check(lib().x100_sync(_stream(stream)), "x100_sync")


# ---- quantised linear / MoE -----------------------------------------------------------
class Lin:
    """x100q_lin handle: an N x K block-quantised linear resident in HBM."""

    def __init__(self, qtype: int, N: int, K: int, blocks: np.ndarray):
        blocks = np.ascontiguousarray(blocks, np.uint8)
        self.qtype, self.N, self.K = qtype, N, K
        self.h = lib().x100q_lin_create(qtype, N, K, blocks.ctypes.data)
        if not self.h:
            check_last("x100q_lin_create")

    def gemv(self, x, y, batch: int) -> None:
        check(lib().x100q_lin_gemv(self.h, _p(x), _p(y), batch), "x100q_lin_gemv")

    def gemv_dev(self, x, y, batch: int, stream=None, independent: bool = False, a8: bool = False) -> None:
        flags = (1 if independent else 0) | (2 if a8 else 0)
        check(lib().x100q_lin_gemv_dev_flags(self.h, _p(x), _p(y), batch, flags, _stream(stream)),
              "x100q_lin_gemv_dev_flags")

    def device_bytes(self) -> int:
        b = C.c_size_t()
        check(lib().x100q_lin_info(self.h, None, None, None, C.byref(b)), "x100q_lin_info")
        return b.value

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.x100q_lin_destroy(self.h)
            self.h = None

    __del__ = close


class Moe:
    """x100q_moe handle: router + top-k + SwiGLU experts [lo, hi) in HBM."""

    def __init__(self, d, n_exp, n_act, ffn, qtype, router, gate, up, down, expert_lo=0, expert_hi=None):
        expert_hi = n_exp if expert_hi is None else expert_hi
        self.d, self.n_exp, self.n_act, self.ffn = d, n_exp, n_act, ffn
        router = np.ascontiguousarray(router, np.float32)
        self.h = lib().x100q_moe_create(d, n_exp, n_act, ffn, qtype, router.ctypes.data, _p(gate), _p(up),
                                        _p(down), expert_lo, expert_hi)
        if not self.h:
            check_last("x100q_moe_create")

    def ffn_host(self, hn: np.ndarray):
        hn = np.ascontiguousarray(hn, np.float32).reshape(-1, self.d)
        B = hn.shape[0]
        eout = np.empty_like(hn)
        sel = np.empty((B, self.n_act), np.int32)
        w = np.empty((B, self.n_act), np.float32)
        check(lib().x100q_moe_ffn(self.h, hn.ctypes.data, eout.ctypes.data, B, sel.ctypes.data, w.ctypes.data),
              "x100q_moe_ffn")
        return eout, sel, w

    def ffn_dev(self, hn, eout, batch, sel=None, w=None, stream=None):
        check(lib().x100q_moe_ffn_dev(self.h, _p(hn), _p(eout), batch, _p(sel), _p(w), _stream(stream)),
              "x100q_moe_ffn_dev")

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.x100q_moe_destroy(self.h)
            self.h = None

    __del__ = close


class Model:
    """x100q_model handle: a Qwen3-MoE-shaped decode model (weights, fp16 KV
    cache, scratch) resident on the current device."""

    def __init__(self, **cfg):
        self.cfg = ModelCfg(**cfg)
        self.h = lib().x100q_model_create(C.byref(self.cfg))
        if not self.h:
            check_last("x100q_model_create")

    def set_layer(self, layer, attn_norm, wq, wk, wv, q_norm, k_norm, wo, ffn_norm, router, gate, up, down):
        check(lib().x100q_model_set_layer(self.h, layer, *(_p(a) for a in (attn_norm, wq, wk, wv, q_norm, k_norm,
                                                                            wo, ffn_norm, router, gate, up, down))),
              "x100q_model_set_layer")

    def set_output(self, tok_embd, out_norm, lm):
        check(lib().x100q_model_set_output(self.h, _p(tok_embd), _p(out_norm), _p(lm)), "x100q_model_set_output")

    def kv_write(self, layer, slot, pos0, k, v):
        npos = k.shape[1]
        check(lib().x100q_model_kv_copy(self.h, layer, slot, pos0, npos, _p(k), _p(v), 1), "x100q_model_kv_copy")

    def kv_read(self, layer, slot, pos0, npos):
        c = self.cfg
        k = np.empty((c.n_kv_heads, npos, c.head_dim), np.uint16)
        v = np.empty_like(k)
        check(lib().x100q_model_kv_copy(self.h, layer, slot, pos0, npos, _p(k), _p(v), 0), "x100q_model_kv_copy")
        return k, v

    def layer_dev(self, layer, h, pos, batch, eout=None, sel=None, w=None, stream=None):
        check(lib().x100q_model_layer_dev(self.h, layer, _p(h), _p(pos), batch, _p(eout), _p(sel), _p(w),
                                          _stream(stream)), "x100q_model_layer_dev")

    def head_dev(self, h, logits, batch, stream=None):
        check(lib().x100q_model_head_dev(self.h, _p(h), _p(logits), batch, _stream(stream)), "x100q_model_head_dev")

    def embed_dev(self, tokens, h, batch, stream=None):
        check(lib().x100q_model_embed_dev(self.h, _p(tokens), _p(h), batch, _stream(stream)),
              "x100q_model_embed_dev")

    def forward_dev(self, tokens, h, pos, logits, batch, stream=None):
        check(lib().x100q_model_forward_dev(self.h, _p(tokens), _p(h), _p(pos), _p(logits), batch,
                                            _stream(stream)), "x100q_model_forward_dev")

    def forward_slots_dev(self, tokens, h, pos, slot, logits, batch, stream=None):
        check(lib().x100q_model_forward_slots_dev(self.h, _p(tokens), _p(h), _p(pos), _p(slot), _p(logits), batch,
                                                  _stream(stream)), "x100q_model_forward_slots_dev")

    def prefill(self, slot: int, tokens, pos0: int, logits: bool = True):
        """n tokens of the sequence in `slot` at positions pos0 .. pos0+n-1 in
        one step; returns their logits [n][vocab] (or None)."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        n = tokens.shape[0]
        out = np.empty((n, self.cfg.vocab), np.float32) if logits else None
        check(lib().x100q_model_prefill(self.h, slot, _p(tokens), n, pos0, _p(out)), "x100q_model_prefill")
        return out

    def forward(self, tokens, pos):
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        B = tokens.shape[0]
        logits = np.empty((B, self.cfg.vocab), np.float32)
        check(lib().x100q_model_forward(self.h, _p(tokens), _p(pos), _p(logits), B), "x100q_model_forward")
        return logits

    def timing(self, on: bool):
        """Start (clearing the totals) or stop per-bucket step timing."""
        check(lib().x100q_model_timing(self.h, 1 if on else 0), "x100q_model_timing")

    def timing_read(self) -> tuple[dict, int]:
        """({bucket name: total ms}, timed calls) since timing started."""
        ms = np.zeros(TIMING_BUCKETS, np.float64)
        steps = C.c_long(0)
        check(lib().x100q_model_timing_read(self.h, _p(ms), C.byref(steps)), "x100q_model_timing_read")
        return {timing_bucket_name(i): float(ms[i]) for i in range(TIMING_BUCKETS)}, steps.value

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.x100q_model_destroy(self.h)
            self.h = None

    __del__ = close


class Gguf:
    """x100q_gguf handle: a GGUF file mapped and parsed (no GPU needed)."""

    def __init__(self, path: str):
        self.h = lib().x100q_gguf_open(os.fsencode(path))
        if not self.h:
            check_last("x100q_gguf_open")

    def _info(self, t: GgufTensor) -> dict:
        return {"name": t.name.decode(), "type": t.type, "n_dims": t.n_dims, "dims": list(t.dims[: t.n_dims]),
                "n_elems": t.n_elems, "bytes": t.bytes, "data": t.data}

    def tensors(self) -> list[dict]:
        out = []
        for i in range(lib().x100q_gguf_n_tensors(self.h)):
            t = GgufTensor()
            check(lib().x100q_gguf_tensor_at(self.h, i, C.byref(t)), "x100q_gguf_tensor_at")
            out.append(self._info(t))
        return out

    def find(self, name: str) -> dict:
        t = GgufTensor()
        check(lib().x100q_gguf_find(self.h, name.encode(), C.byref(t)), "x100q_gguf_find")
        return self._info(t)

    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's raw data (a copy out of the mapping)."""
        t = self.find(name)
        return np.ctypeslib.as_array((C.c_uint8 * t["bytes"]).from_address(t["data"])).copy()

    @property
    def data_offset(self) -> int:
        return int(lib().x100q_gguf_data_offset(self.h))

    def tokens(self) -> list[str]:
        L = lib()
        return [L.x100q_gguf_token(self.h, i).decode() for i in range(L.x100q_gguf_n_tokens(self.h))]

    def get_int(self, key: str) -> int:
        v = C.c_int64()
        check(lib().x100q_gguf_get_int(self.h, key.encode(), C.byref(v)), key)
        return v.value

    def get_f32(self, key: str) -> float:
        v = C.c_float()
        check(lib().x100q_gguf_get_f32(self.h, key.encode(), C.byref(v)), key)
        return v.value

    def get_str(self, key: str) -> str:
        v = C.c_char_p()
        check(lib().x100q_gguf_get_str(self.h, key.encode(), C.byref(v)), key)
        return v.value.decode()

    def model_cfg(self) -> dict:
        c = ModelCfg()
        check(lib().x100q_gguf_model_cfg(self.h, C.byref(c)), "x100q_gguf_model_cfg")
        return {n: getattr(c, n) for n, _ in ModelCfg._fields_}

    def load_model(self, **overrides) -> "Model":
        """x100q_model_load_gguf with the file's configuration, fields such as
        ctx, max_batch or expert_lo / expert_hi replaced by `overrides`."""
        cfg = dict(self.model_cfg(), **overrides)
        m = Model.__new__(Model)
        m.cfg = ModelCfg(**cfg)
        m.h = lib().x100q_model_load_gguf(self.h, C.byref(m.cfg))
        if not m.h:
            check_last("x100q_model_load_gguf")
        return m

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.x100q_gguf_close(self.h)
            self.h = None

    __del__ = close


def gguf_dequant_dev(gtype: int, data, n: int, out, stream=None) -> None:
    check(lib().x100q_gguf_dequant_dev(gtype, _p(data), n, _p(out), _stream(stream)), "x100q_gguf_dequant_dev")


PACK_I8, PACK_Q3K, PACK_HP = 1, 2, 3
GEMV_INDEPENDENT, GEMV_A8 = 1, 2


def pack_act_dev(mode: int, x, K: int, batch: int, out, stream=None) -> None:
    """The reference's pack_act_i8 (mode PACK_I8) / pack_act_q3k (PACK_Q3K) /
    pack_act_hp (PACK_HP)."""
    check(lib().x100q_pack_act_dev(mode, _p(x), K, batch, _p(out), _stream(stream)), "x100q_pack_act_dev")


def quantize_q8_0_dev(x, n: int, blocks, stream=None) -> None:
    check(lib().x100q_quantize_q8_0_dev(_p(x), n, _p(blocks), _stream(stream)), "x100q_quantize_q8_0_dev")


EP_HANDLE_BYTES = 64


class EpGroup:
    """x100q_ep handle: the peer-memory combine of expert-parallel partials.
    `exchange(bytes) -> list[bytes]` must return every process's handle in
    rank order (e.g. torch.distributed.all_gather_object)."""

    def __init__(self, world: int, rank: int, max_floats: int, exchange):
        self.h = lib().x100q_ep_create(world, rank, max_floats)
        if not self.h:
            check_last("x100q_ep_create")
        mine = C.create_string_buffer(EP_HANDLE_BYTES)
        check(lib().x100q_ep_handle(self.h, mine), "x100q_ep_handle")
        allh = b"".join(exchange(mine.raw))
        assert len(allh) == world * EP_HANDLE_BYTES
        buf = C.create_string_buffer(allh, len(allh))
        check(lib().x100q_ep_open(self.h, buf), "x100q_ep_open")

    def allreduce_dev(self, src, dst, n: int, accum: bool = False, stream=None):
        check(lib().x100q_ep_allreduce_dev(self.h, _p(src), _p(dst), n, 1 if accum else 0, _stream(stream)),
              "x100q_ep_allreduce_dev")

    def close(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.x100q_ep_destroy(self.h)
            self.h = None

    __del__ = close
