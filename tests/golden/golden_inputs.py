"""Deterministic inputs of the decode-step pins (forward_golden.npz).

make_golden.py builds these models, runs the reference's own forward() on
them and stores only the outputs; tests/test_oracle_golden.py rebuilds the
same models here and replays them through the oracle.  Every byte and float
comes from the oracle's xorshift64 stream (py_oracle.fill_u8 / rand_f32), so
both sides see identical inputs without committing megabytes of weights.
"""
from __future__ import annotations

import numpy as np

import py_oracle as po

# Case "small": two layers, eight steps from an empty cache.
# Case "c5": the BASELINE decode configuration's attention shape (d 2048,
# 32 query / 4 KV heads, head_dim 128, RoPE base 1e6, a 4096-position cache
# filled with random values below pos) with 16 Q3_K experts of ffn 768, one
# layer, one step at each of several positions (fresh cache each time).
CASES = {
    "small": dict(n_layers=2, d=256, n_heads=4, n_kv_heads=2, head_dim=128, vocab=96, n_exp=16, n_act=4,
                  moe_ffn=256, attn_qtype=po.Q8_0, expert_qtype=po.Q3_K, lm_qtype=po.Q8_0, ctx=8,
                  rope_base=1e6, eps=1e-6, seed=7100,
                  steps=[(3, 0), (17, 1), (90, 2), (5, 3), (5, 4), (60, 5), (41, 6), (0, 7)], prefill=False),
    "c5": dict(n_layers=1, d=2048, n_heads=32, n_kv_heads=4, head_dim=128, vocab=64, n_exp=16, n_act=8,
               moe_ffn=768, attn_qtype=po.Q8_0, expert_qtype=po.Q3_K, lm_qtype=po.Q8_0, ctx=4096,
               rope_base=1e6, eps=1e-6, seed=7200, steps=[(11, 0), (12, 1000), (13, 4095)], prefill=True),
}

SCALE_AT = {po.Q8_0: 0, po.Q4_0: 0, po.Q3_K: 108}


def blocks(qtype: int, nblocks: int, seed: int, lo: float = 0.0002, hi: float = 0.002) -> np.ndarray:
    """Well-formed GGUF blocks: payload bytes from the xorshift stream, the
    fp16 block scale set to +-(lo + (hi - lo) * u), u and the sign from a
    second stream (the magnitudes N(0, 0.02) weights give)."""
    bb = po.BLOCK_BYTES[qtype]
    blk = po.fill_u8(seed, nblocks * bb).reshape(nblocks, bb).copy()
    u = po.fill_u8(seed + 0x9E3779B9, 2 * nblocks).reshape(nblocks, 2)
    mag = lo + (hi - lo) * (u[:, 0].astype(np.float64) / 255.0)
    val = np.where(u[:, 1] & 1, -mag, mag).astype(np.float16)
    at = SCALE_AT[qtype]
    blk[:, at:at + 2] = val.view(np.uint8).reshape(-1, 2)
    return np.ascontiguousarray(blk.reshape(-1))


def model(case: str) -> dict:
    """The case's weights: per-layer dicts of GGUF-native blocks and fp32
    vectors (the layout py_oracle.decode_layer takes), plus tok_embd,
    out_norm and the lm_head blocks."""
    c = CASES[case]
    s = c["seed"]
    d, hd, E, F = c["d"], c["head_dim"], c["n_exp"], c["moe_ffn"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    at, et = c["attn_qtype"], c["expert_qtype"]
    nb = lambda qt, n, k: n * k // po.BLOCK_ELEMS[qt]   # noqa: E731
    layers = []
    for li in range(c["n_layers"]):
        b = s + 100 * li
        layers.append(dict(
            attn_norm=po.rand_f32(b + 1, d, 0.9, 1.1),
            wq=blocks(at, nb(at, qd, d), b + 2), wk=blocks(at, nb(at, kvd, d), b + 3),
            wv=blocks(at, nb(at, kvd, d), b + 4),
            q_norm=po.rand_f32(b + 5, hd, 0.9, 1.1), k_norm=po.rand_f32(b + 6, hd, 0.9, 1.1),
            wo=blocks(at, nb(at, d, qd), b + 7),
            ffn_norm=po.rand_f32(b + 8, d, 0.9, 1.1),
            router=po.rand_f32(b + 9, E * d, -0.05, 0.05).reshape(E, d),
            gate=blocks(et, E * nb(et, F, d), b + 10), up=blocks(et, E * nb(et, F, d), b + 11),
            down=blocks(et, E * nb(et, d, F), b + 12)))
    return dict(layers=layers,
                tok_embd=po.rand_f32(s + 90, c["vocab"] * d).reshape(c["vocab"], d),
                out_norm=po.rand_f32(s + 91, d, 0.9, 1.1),
                lm=blocks(c["lm_qtype"], nb(c["lm_qtype"], c["vocab"], d), s + 92))


def prefill_cache(case: str, layer: int, step: int):
    """fp32 K and V caches [n_kv_heads][ctx][head_dim] of one layer for one
    step of a prefilled case: uniform [-1, 1) below the step's position,
    zero from it on (the reference's forward reads only positions <= pos and
    writes pos itself)."""
    c = CASES[case]
    pos = c["steps"][step][1]
    shape = (c["n_kv_heads"], c["ctx"], c["head_dim"])
    n = int(np.prod(shape))
    k = po.rand_f32(c["seed"] + 1000 + 10 * layer + step, n).reshape(shape)
    v = po.rand_f32(c["seed"] + 2000 + 10 * layer + step, n).reshape(shape)
    k[:, pos:] = 0.0
    v[:, pos:] = 0.0
    return np.ascontiguousarray(k), np.ascontiguousarray(v)


def oracle_logits(case: str, nthreads: int = 8) -> np.ndarray:
    """The oracle's logits for every step of the case (fp32 cache, as the
    reference keeps it), [steps][vocab]."""
    c = CASES[case]
    m = model(case)
    out = []
    caches = None
    if not c["prefill"]:
        shape = (c["n_kv_heads"], c["ctx"], c["head_dim"])
        caches = [(np.zeros(shape, np.float32), np.zeros(shape, np.float32)) for _ in range(c["n_layers"])]
    for st, (tok, pos) in enumerate(c["steps"]):
        h = m["tok_embd"][tok].copy()
        for li, lw in enumerate(m["layers"]):
            kc, vc = caches[li] if caches else prefill_cache(case, li, st)
            po.decode_layer_f32kv(c, lw, kc, vc, h, pos, nthreads=nthreads)
        out.append(po.decode_head(c, m["out_norm"], m["lm"], h, nthreads=nthreads))
    return np.stack(out)
