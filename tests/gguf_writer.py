"""Minimal GGUF (version 3) writer for tests: synthetic model files.

Test infrastructure.  The layout follows the published GGUF format, which the
reference's reader walks (qwen_moe_q3k.c:1086-1126): magic "GGUF", u32
version, u64 tensor count, u64 metadata count; metadata entries (u64-length
key, u32 value type, value); tensor infos (u64-length name, u32 n_dims, u64
dims[n_dims] with dims[0] the contiguous row length, u32 ggml type, u64 data
offset); zero padding to the alignment; tensor data, each tensor at its
offset (a multiple of the alignment).  The output is a deterministic function
of the arguments.
"""
from __future__ import annotations

import struct

import numpy as np

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], v)
    if vtype == STR:
        return _str(v)
    if vtype == ARR:
        etype, items = v
        return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)
    raise ValueError(vtype)


def gguf_bytes(kv, tensors, alignment: int = 32, version: int = 3) -> bytes:
    """kv: [(key, vtype, value)] (arrays: value = (elem_type, [items]));
    tensors: [(name, ggml_type, dims, payload bytes)]."""
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    meta = b"".join(_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in kv)
    infos, off = [], 0
    for name, gtype, dims, payload in tensors:
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<IQ", gtype, off))
        off += (len(payload) + alignment - 1) // alignment * alignment
    out = bytearray(head + meta + b"".join(infos))
    out += bytes((-len(out)) % alignment)
    for _, _, _, payload in tensors:
        out += bytes(payload)
        out += bytes((-len(out)) % alignment)
    return bytes(out)


def write_gguf(path: str, kv, tensors, alignment: int = 32) -> None:
    with open(path, "wb") as f:
        f.write(gguf_bytes(kv, tensors, alignment))


def f16_bytes(vals) -> np.ndarray:
    return np.asarray(vals, np.float16).view(np.uint8).reshape(-1, 2)


def random_blocks(gtype: int, nblocks: int, rng, scale=(0.001, 0.08)) -> np.ndarray:
    """Random well-formed blocks of a GGUF type: random payload bytes, fp16
    scales drawn from +-[scale] (as bench/q3k_probe.c:418-425 builds its
    test blocks); F32 / F16 tensors get N(0, scale[1]) values."""
    import py_oracle as po
    be, bb = po.GGUF_BLOCK[gtype]
    if gtype == po.Q_F32:
        return rng.normal(0, scale[1], nblocks).astype(np.float32).view(np.uint8).reshape(nblocks, 4)
    if gtype == po.F16:
        return rng.normal(0, scale[1], nblocks).astype(np.float16).view(np.uint8).reshape(nblocks, 2)
    blk = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    mag = rng.uniform(scale[0], scale[1], size=nblocks) * rng.choice([-1.0, 1.0], size=nblocks)
    pos = rng.uniform(scale[0], scale[1], size=nblocks)
    if gtype in (po.Q4_0, po.Q8_0):
        blk[:, 0:2] = f16_bytes(mag)
    elif gtype == po.Q4_1:
        blk[:, 0:2] = f16_bytes(pos)
        blk[:, 2:4] = f16_bytes(-8 * pos)
    elif gtype in (po.Q4_K, po.Q5_K):
        blk[:, 0:2] = f16_bytes(pos)
        blk[:, 2:4] = f16_bytes(rng.uniform(0.0, scale[1] * 0.6, size=nblocks))
    elif gtype == po.Q3_K:
        blk[:, 108:110] = f16_bytes(mag)
    elif gtype == po.Q6_K:
        blk[:, 192:208] = (rng.integers(-64, 64, size=(nblocks, 16))).astype(np.int8).view(np.uint8)
        blk[:, 208:210] = f16_bytes(pos / 16)
    return blk


# The tensor set of a qwen3moe file, as the reference's model_load reads it
# (qwen_moe_q3k.c:1742-1787): name suffix, [rows, row length] from the
# dimensions, and the type key in `types`.
def qwen3moe_tensors(c: dict):
    d, qd, kvd, hd = c["d"], c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"], c["head_dim"]
    E, F = c["n_exp"], c["moe_ffn"]
    per_layer = [("attn_norm.weight", [d], "norm"), ("attn_q.weight", [d, qd], "q"), ("attn_k.weight", [d, kvd], "k"),
                 ("attn_v.weight", [d, kvd], "v"), ("attn_q_norm.weight", [hd], "norm"),
                 ("attn_k_norm.weight", [hd], "norm"), ("attn_output.weight", [qd, d], "o"),
                 ("ffn_norm.weight", [d], "norm"), ("ffn_gate_inp.weight", [d, E], "router"),
                 ("ffn_gate_exps.weight", [d, F, E], "exp"), ("ffn_up_exps.weight", [d, F, E], "exp"),
                 ("ffn_down_exps.weight", [F, d, E], "exp")]
    out = []
    for l in range(c["n_layers"]):
        out += [(f"blk.{l}.{s}", dims, key) for s, dims, key in per_layer]
    out += [("token_embd.weight", [d, c["vocab"]], "embd"), ("output_norm.weight", [d], "norm")]
    return out


def qwen3moe_file(path: str, c: dict, types: dict, seed: int = 0, tied: bool = False):
    """Write a synthetic qwen3moe GGUF with dimensions `c` (the x100q_model_cfg
    field names) and one ggml type per tensor role in `types` (q, k, v, o,
    exp, router, norm, embd, lm).  Norm tensors are 1 + N(0, 0.1) values, the
    router N(0, 0.02), token embeddings N(0, 1) in their type; quantised
    weights are random well-formed blocks.  Returns {name: (type, payload)}."""
    import py_oracle as po
    rng = np.random.default_rng(seed)
    specs = qwen3moe_tensors(c)
    if not tied:
        specs.append(("output.weight", [c["d"], c["vocab"]], "lm"))
    tensors, data = [], {}
    for name, dims, key in specs:
        gt = types[key]
        n = int(np.prod(dims))
        be, _ = po.GGUF_BLOCK[gt]
        if key in ("norm", "router", "embd") and gt in (po.Q_F32, po.F16):
            sd = {"norm": 0.1, "router": 0.02, "embd": 1.0}[key]
            v = rng.normal(0, sd, n) + (1.0 if key == "norm" else 0.0)
            payload = v.astype(np.float32 if gt == po.Q_F32 else np.float16).view(np.uint8)
        else:
            scale = (0.02, 0.3) if key == "embd" else (0.0002, 0.002)
            payload = random_blocks(gt, n // be, rng, scale).reshape(-1)
        tensors.append((name, gt, dims, payload.tobytes()))
        data[name] = (gt, payload)
    kv = [("general.architecture", STR, "qwen3moe"),
          ("qwen3moe.block_count", U32, c["n_layers"]), ("qwen3moe.embedding_length", U32, c["d"]),
          ("qwen3moe.feed_forward_length", U32, 6144), ("qwen3moe.attention.head_count", U32, c["n_heads"]),
          ("qwen3moe.attention.head_count_kv", U32, c["n_kv_heads"]),
          ("qwen3moe.attention.key_length", U32, c["head_dim"]), ("qwen3moe.expert_count", U32, c["n_exp"]),
          ("qwen3moe.expert_used_count", U32, c["n_act"]),
          ("qwen3moe.expert_feed_forward_length", U32, c["moe_ffn"]),
          ("qwen3moe.rope.freq_base", F32, c.get("rope_base", 1e6)),
          ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(c["vocab"])]))]
    write_gguf(path, kv, tensors)
    return data
