"""CPU checks of the decode-step oracle (no GPU).

orc_decode_layer / orc_decode_head (oracle/oracle_quant.c) restate
forward() of qwen_moe_q3k.c:1842-1983 in C.  Here they are compared with a
second, independent numpy statement of the same steps on a small model
(dequantised weights, float64 arithmetic), and the pieces they rest on are
checked for the properties the reference's code has: RoPE is a rotation
(norm preserving, identity at position 0), attention over a single position
returns that position's value, and the fp16 cache write rounds to nearest.
"""
import numpy as np
import pytest

import py_oracle as po

SMALL = dict(d=256, n_heads=4, n_kv_heads=2, head_dim=128, ctx=12, rope_base=1e6, eps=1e-6, attn_qtype=po.Q8_0,
             n_exp=4, n_act=2, moe_ffn=256, expert_qtype=po.Q3_K, vocab=64, lm_qtype=po.Q8_0)


def _layer(rng, c):
    d, qd, kvd = c["d"], c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"]
    q = lambda qt, n, k: po.quantize(qt, rng.normal(0, 0.05, (n, k)).astype(np.float32))  # noqa: E731
    E, F = c["n_exp"], c["moe_ffn"]
    return dict(attn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
                wq=q(po.Q8_0, qd, d), wk=q(po.Q8_0, kvd, d), wv=q(po.Q8_0, kvd, d),
                q_norm=(1 + 0.1 * rng.standard_normal(c["head_dim"])).astype(np.float32),
                k_norm=(1 + 0.1 * rng.standard_normal(c["head_dim"])).astype(np.float32),
                wo=q(po.Q8_0, d, qd), ffn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
                router=(0.3 * rng.standard_normal((E, d))).astype(np.float32),
                gate=q(po.Q3_K, E * F, d), up=q(po.Q3_K, E * F, d), down=q(po.Q3_K, E * d, F))


def _np_layer(c, lw, kc, vc, h, pos):
    """Independent float64 statement of one layer (same steps, numpy)."""
    d, nh, nkv, hd = c["d"], c["n_heads"], c["n_kv_heads"], c["head_dim"]
    deq = lambda qt, b, n, k: po.dequant(qt, b, n, k).astype(np.float64)  # noqa: E731
    rms = lambda x, w: x / np.sqrt(np.mean(x * x) + c["eps"]) * w  # noqa: E731

    def rope(v):
        i = np.arange(hd // 2)
        a = pos * np.float64(c["rope_base"]) ** (-2.0 * i / hd)
        x, y = v[: hd // 2].copy(), v[hd // 2:].copy()
        return np.concatenate([x * np.cos(a) - y * np.sin(a), x * np.sin(a) + y * np.cos(a)])

    h = h.astype(np.float64)
    hn = rms(h, lw["attn_norm"])
    q = deq(c["attn_qtype"], lw["wq"], nh * hd, d) @ hn
    k = deq(c["attn_qtype"], lw["wk"], nkv * hd, d) @ hn
    v = deq(c["attn_qtype"], lw["wv"], nkv * hd, d) @ hn
    q = np.concatenate([rope(rms(q[i * hd:(i + 1) * hd], lw["q_norm"])) for i in range(nh)])
    k = np.concatenate([rope(rms(k[i * hd:(i + 1) * hd], lw["k_norm"])) for i in range(nkv)])
    kc[:, pos] = np.float16(k.reshape(nkv, hd)).view(np.uint16)
    vc[:, pos] = np.float16(v.reshape(nkv, hd)).view(np.uint16)
    K = kc.view(np.float16).astype(np.float64)
    V = vc.view(np.float16).astype(np.float64)
    att = np.zeros(nh * hd)
    for hh in range(nh):
        kvh = hh // (nh // nkv)
        s = K[kvh, : pos + 1] @ q[hh * hd:(hh + 1) * hd] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        att[hh * hd:(hh + 1) * hd] = p @ V[kvh, : pos + 1]
    h = h + deq(c["attn_qtype"], lw["wo"], d, nh * hd) @ att
    hn = rms(h, lw["ffn_norm"])
    lg = lw["router"].astype(np.float64) @ hn
    p = np.exp(lg - lg.max())
    p /= p.sum()
    sel = np.argsort(-p, kind="stable")[: c["n_act"]]
    w = p[sel] / p[sel].sum()
    E, F = c["n_exp"], c["moe_ffn"]
    G = deq(c["expert_qtype"], lw["gate"], E * F, d).reshape(E, F, d)
    U = deq(c["expert_qtype"], lw["up"], E * F, d).reshape(E, F, d)
    D = deq(c["expert_qtype"], lw["down"], E * d, F).reshape(E, d, F)
    for a, e in enumerate(sel):
        g, u = G[e] @ hn, U[e] @ hn
        h = h + w[a] * (D[e] @ (g / (1 + np.exp(-g)) * u))
    return h, sel


@pytest.mark.parametrize("pos", [0, 5, 11])
def test_decode_layer_matches_numpy_statement(pos):
    c = SMALL
    rng = np.random.default_rng(pos + 1)
    lw = _layer(rng, c)
    shape = (c["n_kv_heads"], c["ctx"], c["head_dim"])
    kc = np.float16(rng.standard_normal(shape)).view(np.uint16)
    vc = np.float16(rng.standard_normal(shape)).view(np.uint16)
    h = rng.standard_normal(c["d"]).astype(np.float32)
    kc2, vc2, h2 = kc.copy(), vc.copy(), h.copy()
    sel, _ = po.decode_layer(c, lw, kc, vc, h, pos)
    ref, rsel = _np_layer(c, lw, kc2, vc2, h2, pos)
    assert np.array_equal(sel, rsel)
    assert po.rel_l2(h, ref) <= 1e-5
    # the cache rows written at pos agree to within one fp16 rounding step
    kf, kr = kc[:, pos].view(np.float16).astype(np.float64), kc2[:, pos].view(np.float16).astype(np.float64)
    assert np.max(np.abs(kf - kr)) <= 2e-3 * np.max(np.abs(kr))
    others = np.ones(c["ctx"], bool)
    others[pos] = False
    assert np.array_equal(kc[:, others], kc2[:, others])


def test_decode_head_is_norm_then_lm():
    c = SMALL
    rng = np.random.default_rng(9)
    lm = po.quantize(po.Q8_0, rng.normal(0, 0.05, (c["vocab"], c["d"])).astype(np.float32))
    out_norm = (1 + 0.1 * rng.standard_normal(c["d"])).astype(np.float32)
    h = rng.standard_normal(c["d"]).astype(np.float32)
    got = po.decode_head(c, out_norm, lm, h)
    hn = np.empty_like(h)
    po.lib().orc_rmsnorm(po._ptr(hn), po._ptr(h), po._ptr(out_norm), c["d"], c["eps"])
    assert np.array_equal(got, po.qgemv(po.Q8_0, lm, c["vocab"], c["d"], hn)[0])


def test_rope_is_a_rotation():
    rng = np.random.default_rng(3)
    v0 = rng.standard_normal(128).astype(np.float32)
    for pos in (0, 1, 4095):
        v = v0.copy()
        po.lib().orc_rope_neox(po._ptr(v), 128, pos, 1e6)
        assert abs(np.linalg.norm(v) - np.linalg.norm(v0)) <= 1e-5 * np.linalg.norm(v0)
        if pos == 0:
            assert np.array_equal(v, v0)


def test_attention_over_one_position_returns_its_value():
    """At pos 0 softmax has one entry, so att = v of the token: the layer's
    attention output (before Wo) is the fp16-rounded v."""
    c = dict(SMALL, n_exp=4)
    rng = np.random.default_rng(4)
    lw = _layer(rng, c)
    lw["wo"] = po.quantize(po.Q8_0, np.eye(c["d"], c["n_heads"] * c["head_dim"], dtype=np.float32))
    lw["down"] = np.zeros_like(lw["down"])       # experts contribute nothing
    shape = (c["n_kv_heads"], c["ctx"], c["head_dim"])
    kc, vc = np.zeros(shape, np.uint16), np.zeros(shape, np.uint16)
    h0 = rng.standard_normal(c["d"]).astype(np.float32)
    h = h0.copy()
    po.decode_layer(c, lw, kc, vc, h, 0)
    v = vc[:, 0].view(np.float16).astype(np.float32).reshape(-1)       # kv head of query heads 0, 1 then 2, 3
    gpr = c["n_heads"] // c["n_kv_heads"]
    att = np.concatenate([v[(hh // gpr) * 128:(hh // gpr + 1) * 128] for hh in range(c["n_heads"])])
    assert po.rel_l2(h - h0, att[: c["d"]]) <= 1e-4   # Q8_0 stores 1.0 as 127 * fp16(1/127)
