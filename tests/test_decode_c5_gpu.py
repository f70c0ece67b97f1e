"""GPU parity of one decode layer and the lm_head at the BASELINE decode
configuration (config 5) against the CPU oracle.

Shape: d 2048, GQA 32 query / 4 KV heads of 128, RoPE base 1e6, Q8_0 q/k/v/o,
128 Q3_K experts (top-8, ffn 768) behind the fp32 router, a 4096-position
fp16 KV cache per sequence, 16 sequences in one step (batch 16), and the
Q8_0 lm_head over a vocabulary of 151,936.  Each sequence sits at its own
position, from 0 to 4095, so the attention runs from one to all 64 of its
64-position splits.  Every slot is compared with orc_decode_layer /
orc_decode_head (the per-layer body of forward(), qwen_moe_q3k.c:1849-1981):
expert selection exact, hidden state and logits within relative L2 1e-3,
the step's k / v written at the sequence's position and nothing else moved.
"""
import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu

REL = 1e-3
CFG = dict(n_layers=1, d=2048, n_heads=32, n_kv_heads=4, head_dim=128, vocab=151936, n_exp=128, n_act=8,
           moe_ffn=768, attn_qtype=po.Q8_0, expert_qtype=po.Q3_K, lm_qtype=po.Q8_0, ctx=4096, max_batch=16,
           expert_lo=0, expert_hi=128, rope_base=1e6, eps=1e-6)
POS = [4095, 0, 1, 63, 64, 65, 127, 128, 1000, 2047, 2048, 3000, 4032, 4094, 511, 4033]


def blocks(qtype, nblocks, rng):
    """Random well-formed GGUF blocks with the scale magnitudes N(0, 0.02)
    weights give."""
    bb = po.BLOCK_BYTES[qtype]
    blk = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    f16 = lambda v: np.asarray(v, np.float16).view(np.uint8).reshape(-1, 2)  # noqa: E731
    at = 0 if qtype == po.Q8_0 else 108
    blk[:, at:at + 2] = f16(rng.uniform(0.0002, 0.0006 if qtype == po.Q8_0 else 0.002, nblocks)
                            * rng.choice([-1, 1], nblocks))
    return np.ascontiguousarray(blk.reshape(-1))


@pytest.fixture(scope="module")
def c5():
    c = CFG
    rng = np.random.default_rng(5005)
    d, hd, E, F = c["d"], c["head_dim"], c["n_exp"], c["moe_ffn"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    lw = dict(attn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
              wq=blocks(po.Q8_0, qd * d // 32, rng), wk=blocks(po.Q8_0, kvd * d // 32, rng),
              wv=blocks(po.Q8_0, kvd * d // 32, rng),
              q_norm=(1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
              k_norm=(1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
              wo=blocks(po.Q8_0, d * qd // 32, rng),
              ffn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
              router=(0.02 * rng.standard_normal((E, d))).astype(np.float32),
              gate=blocks(po.Q3_K, E * F * d // 256, rng), up=blocks(po.Q3_K, E * F * d // 256, rng),
              down=blocks(po.Q3_K, E * d * F // 256, rng))
    out_norm = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    lm = blocks(po.Q8_0, c["vocab"] * d // 32, rng)
    emb = np.zeros((c["vocab"], d), np.float32)          # not used: the test starts from hidden states
    kv = [tuple(np.ascontiguousarray(rng.standard_normal((c["n_kv_heads"], c["ctx"], hd)).astype(np.float16))
                .view(np.uint16) for _ in range(2)) for _ in range(c["max_batch"])]
    m = x100b.Model(**c)
    m.set_layer(0, *(lw[k] for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "ffn_norm", "router",
                                     "gate", "up", "down")))
    m.set_output(emb, out_norm, lm)
    for s, (k, v) in enumerate(kv):
        m.kv_write(0, s, 0, k, v)
    yield dict(c=c, lw=lw, out_norm=out_norm, lm=lm, kv=kv, model=m)
    m.close()


def test_c5_layer_and_head_batch16(c5):
    import torch
    c, m = c5["c"], c5["model"]
    B = c["max_batch"]
    h0 = np.random.default_rng(77).standard_normal((B, c["d"])).astype(np.float32)
    hd = torch.from_numpy(h0.copy()).cuda()
    pos = torch.tensor(POS, dtype=torch.int32, device="cuda")
    sel = torch.empty((B, c["n_act"]), dtype=torch.int32, device="cuda")
    logits = torch.empty((B, c["vocab"]), device="cuda")
    m.layer_dev(0, hd, pos, B, sel=sel)
    m.head_dev(hd, logits, B)
    x100b.sync()
    hg, selg, lg = hd.cpu().numpy(), sel.cpu().numpy(), logits.cpu().numpy()
    union = set()
    kf = lambda a: a.view(np.float16).astype(np.float32)   # noqa: E731
    for b in range(B):
        k, v = (x.copy() for x in c5["kv"][b])
        h = h0[b].copy()
        rsel, _ = po.decode_layer(c, c5["lw"], k, v, h, POS[b], nthreads=16)
        assert np.array_equal(selg[b], rsel), (b, selg[b], rsel)
        union |= set(rsel.tolist())
        assert po.rel_l2(hg[b], h) <= REL, (b, POS[b], po.rel_l2(hg[b], h))
        ref = po.decode_head(c, c5["out_norm"], c5["lm"], h, nthreads=16)
        assert po.rel_l2(lg[b], ref) <= REL, (b, po.rel_l2(lg[b], ref))
        kg, vg = m.kv_read(0, b, 0, c["ctx"])
        p = POS[b]
        assert po.rel_l2(kf(kg[:, p]), kf(k[:, p])) <= REL and po.rel_l2(kf(vg[:, p]), kf(v[:, p])) <= REL
        keep = np.ones(c["ctx"], bool)
        keep[p] = False
        assert np.array_equal(kg[:, keep], c5["kv"][b][0][:, keep])
        assert np.array_equal(vg[:, keep], c5["kv"][b][1][:, keep])
    assert len(union) > 40          # the batch spreads over many experts, as at decode batch 16
