"""GPU parity of the decode attention for every split size it may choose.

The attention kernel cuts a (token, kv head) row of the cache into splits of
cps chunks of 64 positions and merges the splits' partial softmax states;
cps (1..8) is chosen per batch from the device's SM count and the kernel's
occupancy, so another device or batch can pick any of them, and with a
context that is not a multiple of 64 * cps the last split is ragged.  Each
child process (X100_ATTN_CPS is read once per process) runs one decode layer
of the same model on the same hidden states with one forced cps; every
result must match the oracle (expert selection exact, hidden state within
relative L2 1e-3, the step's k / v written at its position) and the runs
must agree with one another to within 2e-4: the splits change only the
order of the softmax sums and the running maximum against which each
split's probabilities are rounded to fp16 for the P.V product.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import py_oracle as po

pytestmark = pytest.mark.gpu

REL = 1e-3
CFG = dict(n_layers=1, d=1024, n_heads=16, n_kv_heads=2, head_dim=128, vocab=256, n_exp=16, n_act=4,
           moe_ffn=256, attn_qtype=po.Q8_0, expert_qtype=po.Q3_K, lm_qtype=po.Q8_0, ctx=1000, max_batch=6,
           expert_lo=0, expert_hi=16, rope_base=1e6, eps=1e-6)
POS = [999, 0, 63, 64, 500, 937]        # 1 to all 16 chunks, ragged last chunk and split
CPS = [1, 2, 3, 5, 8]


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


def world():
    c = CFG
    rng = np.random.default_rng(4242)
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
    kv = [tuple(np.ascontiguousarray(rng.standard_normal((c["n_kv_heads"], c["ctx"], hd)).astype(np.float16))
                .view(np.uint16) for _ in range(2)) for _ in range(c["max_batch"])]
    h0 = rng.standard_normal((c["max_batch"], d)).astype(np.float32)
    return lw, kv, h0


CHILD = r"""
import sys, numpy as np
sys.path[:0] = [{paths}]
sys.path.insert(0, {here!r})
import torch, x100b
import test_attn_splits_gpu as t
c = t.CFG
lw, kv, h0 = t.world()
m = x100b.Model(**c)
m.set_layer(0, *(lw[k] for k in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "ffn_norm", "router",
                                 "gate", "up", "down")))
m.set_output(np.zeros((c["vocab"], c["d"]), np.float32), np.ones(c["d"], np.float32),
             np.zeros(c["vocab"] * c["d"] // 32 * 34, np.uint8))
for s, (k, v) in enumerate(kv):
    m.kv_write(0, s, 0, k, v)
B = c["max_batch"]
hd = torch.from_numpy(h0.copy()).cuda()
pos = torch.tensor(t.POS, dtype=torch.int32, device="cuda")
sel = torch.empty((B, c["n_act"]), dtype=torch.int32, device="cuda")
m.layer_dev(0, hd, pos, B, sel=sel)
x100b.sync()
ks, vs = [], []
for b in range(B):
    kg, vg = m.kv_read(0, b, 0, c["ctx"])
    ks.append(kg[:, t.POS[b]])
    vs.append(vg[:, t.POS[b]])
np.savez({path!r}, h=hd.cpu().numpy(), sel=sel.cpu().numpy(), k=np.stack(ks), v=np.stack(vs))
m.close()
"""


def test_every_split_size_matches_the_oracle(tmp_path):
    c = CFG
    lw, kv, h0 = world()
    paths = ", ".join(repr(p) for p in sys.path if p)
    here = os.path.dirname(os.path.abspath(__file__))
    res = {}
    for cps in CPS:
        path = str(tmp_path / f"cps{cps}.npz")
        env = dict(os.environ)
        env["X100_ATTN_CPS"] = str(cps)
        subprocess.run([sys.executable, "-c", CHILD.format(paths=paths, here=here, path=path)], env=env,
                       check=True, timeout=300)
        res[cps] = np.load(path)
    kf = lambda a: a.view(np.float16).astype(np.float32)   # noqa: E731
    for b in range(c["max_batch"]):
        k, v = (x.copy() for x in kv[b])
        h = h0[b].copy()
        rsel, _ = po.decode_layer(c, lw, k, v, h, POS[b], nthreads=16)
        p = POS[b]
        for cps in CPS:
            r = res[cps]
            assert np.array_equal(r["sel"][b], rsel), (cps, b, r["sel"][b], rsel)
            assert po.rel_l2(r["h"][b], h) <= REL, (cps, b, p, po.rel_l2(r["h"][b], h))
            assert po.rel_l2(kf(r["k"][b]), kf(k[:, p])) <= REL and po.rel_l2(kf(r["v"][b]), kf(v[:, p])) <= REL
            assert po.rel_l2(r["h"][b], res[CPS[0]]["h"][b]) <= 2e-4, (cps, b)
