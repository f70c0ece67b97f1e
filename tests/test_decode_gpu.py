"""GPU parity of the whole decode step (x100q_model_*) against the CPU oracle.

The oracle (orc_decode_layer / orc_decode_head) restates forward() of
qwen_moe_q3k.c:1842-1983 for one token: rmsnorm, Q8_0 q/k/v projections,
per-head q/k rmsnorm + NEOX RoPE, fp16 KV cache write at pos, serial softmax
attention over 0..pos, Wo, residual, the fp32-router MoE block with Q3_K
experts, residual; then the output norm and the lm_head.  Outputs must stay
within relative L2 1e-3 of it (the bar of the dequant-GEMV and MoE path) and
the selected experts must be the oracle's.  All calls go through the C ABI.
"""
import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu

REL = 1e-3
CFG = dict(n_layers=2, d=2048, n_heads=32, n_kv_heads=4, head_dim=128, vocab=640, n_exp=32, n_act=8,
           moe_ffn=768, attn_qtype=po.Q8_0, expert_qtype=po.Q3_K, lm_qtype=po.Q8_0, ctx=160, max_batch=4,
           expert_lo=0, expert_hi=32, rope_base=1e6, eps=1e-6)


def blocks(qtype, nblocks, rng):
    """Random well-formed GGUF blocks: random payload, fp16 scales of the size
    N(0, 0.02) weights give."""
    bb = po.BLOCK_BYTES[qtype]
    blk = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    f16 = lambda v: np.asarray(v, np.float16).view(np.uint8).reshape(-1, 2)  # noqa: E731
    if qtype == po.Q8_0:
        blk[:, 0:2] = f16(rng.uniform(0.0002, 0.0006, nblocks) * rng.choice([-1, 1], nblocks))
    else:   # Q3_K
        blk[:, 108:110] = f16(rng.uniform(0.0002, 0.002, nblocks) * rng.choice([-1, 1], nblocks))
    return np.ascontiguousarray(blk.reshape(-1))


def make_layer(rng, c):
    d, qd, kvd, E, F = c["d"], c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"], c["n_exp"], c["moe_ffn"]
    nb8 = lambda n, k: n * k // 32          # noqa: E731  Q8_0 blocks
    nb3 = lambda n, k: n * k // 256         # noqa: E731  Q3_K blocks
    return dict(
        attn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
        wq=blocks(po.Q8_0, nb8(qd, d), rng), wk=blocks(po.Q8_0, nb8(kvd, d), rng), wv=blocks(po.Q8_0, nb8(kvd, d), rng),
        q_norm=(1 + 0.1 * rng.standard_normal(c["head_dim"])).astype(np.float32),
        k_norm=(1 + 0.1 * rng.standard_normal(c["head_dim"])).astype(np.float32),
        wo=blocks(po.Q8_0, nb8(d, qd), rng),
        ffn_norm=(1 + 0.1 * rng.standard_normal(d)).astype(np.float32),
        router=(0.02 * rng.standard_normal((E, d))).astype(np.float32),
        gate=blocks(po.Q3_K, E * nb3(F, d), rng), up=blocks(po.Q3_K, E * nb3(F, d), rng),
        down=blocks(po.Q3_K, E * nb3(d, F), rng))


def f16_bits(a):
    return np.ascontiguousarray(np.asarray(a, np.float16)).view(np.uint16)


@pytest.fixture(scope="module")
def world():
    rng = np.random.default_rng(2024)
    c = CFG
    layers = [make_layer(rng, c) for _ in range(c["n_layers"])]
    emb = rng.standard_normal((c["vocab"], c["d"])).astype(np.float32)
    out_norm = (1 + 0.1 * rng.standard_normal(c["d"])).astype(np.float32)
    lm = blocks(po.Q8_0, c["vocab"] * c["d"] // 32, rng)
    # past keys / values of every (layer, slot): [nkv][ctx][hd] fp16, zero past `ctx`
    kv = [[(f16_bits(rng.standard_normal((c["n_kv_heads"], c["ctx"], c["head_dim"]))),
            f16_bits(rng.standard_normal((c["n_kv_heads"], c["ctx"], c["head_dim"]))))
           for _ in range(c["max_batch"])] for _ in range(c["n_layers"])]
    m = x100b.Model(**c)
    for li, lw in enumerate(layers):
        m.set_layer(li, lw["attn_norm"], lw["wq"], lw["wk"], lw["wv"], lw["q_norm"], lw["k_norm"], lw["wo"],
                    lw["ffn_norm"], lw["router"], lw["gate"], lw["up"], lw["down"])
    m.set_output(emb, out_norm, lm)
    return dict(c=c, layers=layers, emb=emb, out_norm=out_norm, lm=lm, kv=kv, model=m)


def load_kv(w, model=None):
    m = model or w["model"]
    for li in range(w["c"]["n_layers"]):
        for s in range(w["c"]["max_batch"]):
            k, v = w["kv"][li][s]
            m.kv_write(li, s, 0, k, v)


def oracle_layer(w, li, slot, h, pos):
    k, v = (x.copy() for x in w["kv"][li][slot])
    sel, wt = po.decode_layer(w["c"], w["layers"][li], k, v, h, pos, nthreads=8)
    return sel, wt, k, v


@pytest.mark.parametrize("pos", [[0], [77], [159], [5, 159, 0, 64]])
def test_layer_matches_oracle(world, pos):
    import torch
    c, m = world["c"], world["model"]
    load_kv(world)
    B = len(pos)
    rng = np.random.default_rng(sum(pos) + B)
    h0 = rng.standard_normal((B, c["d"])).astype(np.float32)
    hd = torch.from_numpy(h0.copy()).cuda()
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    sel = torch.empty((B, c["n_act"]), dtype=torch.int32, device="cuda")
    m.layer_dev(1, hd, pd, B, sel=sel)
    x100b.sync()
    hg, selg = hd.cpu().numpy(), sel.cpu().numpy()
    for b in range(B):
        h = h0[b].copy()
        rsel, _, k, v = oracle_layer(world, 1, b, h, pos[b])
        assert np.array_equal(selg[b], rsel), (b, selg[b], rsel)
        assert po.rel_l2(hg[b], h) <= REL, (b, po.rel_l2(hg[b], h))
        # the step's k and v landed in the cache at pos (fp16), the rest untouched
        kg, vg = m.kv_read(1, b, 0, c["ctx"])
        p = pos[b]
        kf = lambda a: a.view(np.float16).astype(np.float32)   # noqa: E731
        assert po.rel_l2(kf(kg[:, p]), kf(k[:, p])) <= REL
        assert po.rel_l2(kf(vg[:, p]), kf(v[:, p])) <= REL
        others = np.ones(c["ctx"], bool)
        others[p] = False
        assert np.array_equal(kg[:, others], k[:, others]) and np.array_equal(vg[:, others], v[:, others])


def test_forward_host_api_matches_oracle(world):
    """Two tokens through embed -> 2 layers -> head via the synchronous host
    call x100q_model_forward, against the oracle chain."""
    c, m = world["c"], world["model"]
    load_kv(world)
    toks, pos = np.array([3, 611], np.int32), np.array([40, 159], np.int32)
    logits = m.forward(toks, pos)
    for b in range(2):
        h = world["emb"][toks[b]].copy()
        for li in range(c["n_layers"]):
            k, v = (x.copy() for x in world["kv"][li][b])
            po.decode_layer(c, world["layers"][li], k, v, h, int(pos[b]), nthreads=8)
        ref = po.decode_head(c, world["out_norm"], world["lm"], h, nthreads=8)
        assert po.rel_l2(logits[b], ref) <= REL, po.rel_l2(logits[b], ref)
        assert int(np.argmax(logits[b])) == int(np.argmax(ref))


def test_forward_dev_equals_layer_by_layer(world):
    """forward_dev (embed + layers + head in one call) gives the same bits as
    the same steps called one by one."""
    import torch
    c, m = world["c"], world["model"]
    B = 3
    toks = torch.tensor([1, 2, 3], dtype=torch.int32, device="cuda")
    pos = torch.tensor([10, 20, 30], dtype=torch.int32, device="cuda")
    h1 = torch.empty((B, c["d"]), device="cuda")
    l1 = torch.empty((B, c["vocab"]), device="cuda")
    load_kv(world)
    m.forward_dev(toks, h1, pos, l1, B)
    x100b.sync()
    load_kv(world)
    h2 = torch.empty_like(h1)
    l2 = torch.empty_like(l1)
    m.embed_dev(toks, h2, B)
    for li in range(c["n_layers"]):
        m.layer_dev(li, h2, pos, B)
    m.head_dev(h2, l2, B)
    x100b.sync()
    assert torch.equal(h1, h2) and torch.equal(l1, l2)


@pytest.mark.parametrize("B", [1, 4])
def test_step_timing_buckets(world, B):
    """Per-bucket timing (the reference's decode buckets, qwen_moe_q3k.c:
    910-941): timing leaves the results bit-identical, counts the calls,
    charges every layer bucket, and its buckets sum to about the wall time of
    the timed calls (the events serialise the kernels around each boundary,
    so the sum may exceed an untimed step, never the timed wall time)."""
    import time
    c, m = world["c"], world["model"]
    toks = np.arange(B, dtype=np.int32) + 5
    pos = np.arange(B, dtype=np.int32) * 7 + 30
    load_kv(world)
    ref = m.forward(toks, pos)
    m.timing(True)
    t0 = time.perf_counter()
    for _ in range(3):
        load_kv(world)
        got = m.forward(toks, pos)
        assert np.array_equal(got, ref)
    wall = (time.perf_counter() - t0) * 1e3
    ms, steps = m.timing_read()
    m.timing(False)
    assert steps == 3
    assert list(ms) == ["embed", "qkv", "attention", "o", "router", "expert", "combine", "lm"]
    for b in ("embed", "qkv", "attention", "o", "router", "expert", "lm"):
        assert ms[b] > 0, (b, ms)
    if B > 1:   # batch 1 fuses routing's top-k, the experts and the combine into one kernel
        assert ms["combine"] > 0, ms
    assert 0 < sum(ms.values()) <= wall, (ms, wall)
    # stopped: further calls add nothing
    load_kv(world)
    m.forward(toks, pos)
    ms2, steps2 = m.timing_read()
    assert steps2 == 3 and ms2 == ms


def test_expert_parallel_split_sums_to_full(world):
    """Two handles holding experts [0, 16) and [16, 32): h + eout_a + eout_b
    equals the full layer (the sum an NCCL all-reduce of eout forms)."""
    import torch
    c = dict(world["c"])
    halves = []
    for lo, hi in ((0, 16), (16, 32)):
        cc = dict(c, expert_lo=lo, expert_hi=hi, n_layers=1)
        mm = x100b.Model(**cc)
        lw = world["layers"][1]
        mm.set_layer(0, lw["attn_norm"], lw["wq"], lw["wk"], lw["wv"], lw["q_norm"], lw["k_norm"], lw["wo"],
                     lw["ffn_norm"], lw["router"], lw["gate"], lw["up"], lw["down"])
        k, v = world["kv"][1][0]
        mm.kv_write(0, 0, 0, k, v)
        halves.append(mm)
    rng = np.random.default_rng(5)
    h0 = rng.standard_normal((1, c["d"])).astype(np.float32)
    pos = torch.tensor([99], dtype=torch.int32, device="cuda")
    outs = []
    for mm in halves:
        hd = torch.from_numpy(h0.copy()).cuda()
        eo = torch.empty_like(hd)
        mm.layer_dev(0, hd, pos, 1, eout=eo)
        x100b.sync()
        outs.append((hd.cpu().numpy(), eo.cpu().numpy()))
    assert np.array_equal(outs[0][0], outs[1][0])   # attention part identical
    got = outs[0][0] + outs[0][1] + outs[1][1]
    h = h0[0].copy()
    oracle_layer(world, 1, 0, h, 99)
    assert po.rel_l2(got[0], h) <= REL
    # a partial expert range cannot add into h by itself
    with pytest.raises(x100b.X100Error):
        halves[0].layer_dev(0, torch.from_numpy(h0.copy()).cuda(), pos, 1)
    for mm in halves:
        mm.close()


def test_position_past_cache_is_reported(world):
    """pos >= ctx: the attention kernel's own bounds check refuses it (the
    reference aborts on KV overflow) and the next sync reports X100_E_ARG;
    the cache is not written."""
    import torch
    c, m = world["c"], world["model"]
    load_kv(world)
    hd = torch.zeros((1, c["d"]), device="cuda") + 0.5
    pos = torch.tensor([c["ctx"]], dtype=torch.int32, device="cuda")
    m.layer_dev(0, hd, pos, 1)
    with pytest.raises(x100b.X100Error) as e:
        x100b.sync()
    assert e.value.code == x100b.X100_E_ARG
    kg, _ = m.kv_read(0, 0, 0, c["ctx"])
    assert np.array_equal(kg, world["kv"][0][0][0])
    # the context stays usable
    pos = torch.tensor([3], dtype=torch.int32, device="cuda")
    m.layer_dev(0, hd, pos, 1)
    x100b.sync()


def test_prefill_matches_token_by_token_oracle(world):
    """x100q_model_prefill of 4 tokens of the sequence in slot 2 at positions
    40..43 (the reference's prefill_chunk4) in one step: each token's logits
    equal, within 1e-3, the oracle stepping the tokens one by one (each
    attending over the cache the earlier ones extended); the chunk's k and v
    land at positions 40..43 of slot 2 and nothing else in the cache moves."""
    c, m = world["c"], world["model"]
    load_kv(world)
    toks, slot, pos0 = np.array([7, 100, 300, 5], np.int32), 2, 40
    logits = m.prefill(slot, toks, pos0)
    caches = [[x.copy() for x in world["kv"][li][slot]] for li in range(c["n_layers"])]
    for i, t in enumerate(toks):
        h = world["emb"][t].copy()
        for li in range(c["n_layers"]):
            po.decode_layer(c, world["layers"][li], caches[li][0], caches[li][1], h, pos0 + i, nthreads=8)
        ref = po.decode_head(c, world["out_norm"], world["lm"], h, nthreads=8)
        assert po.rel_l2(logits[i], ref) <= REL, (i, po.rel_l2(logits[i], ref))
    kf = lambda a: a.view(np.float16).astype(np.float32)   # noqa: E731
    for li in range(c["n_layers"]):
        kg, vg = m.kv_read(li, slot, 0, c["ctx"])
        rows = slice(pos0, pos0 + len(toks))
        assert po.rel_l2(kf(kg[:, rows]), kf(caches[li][0][:, rows])) <= REL
        assert po.rel_l2(kf(vg[:, rows]), kf(caches[li][1][:, rows])) <= REL
        keep = np.ones(c["ctx"], bool)
        keep[rows] = False
        assert np.array_equal(kg[:, keep], world["kv"][li][slot][0][:, keep])
        for other in (0, 1, 3):   # other sequences untouched
            ko, _ = m.kv_read(li, other, 0, c["ctx"])
            assert np.array_equal(ko, world["kv"][li][other][0])


def test_forward_slots_identity_equals_forward_dev(world):
    """With slot[b] = b the slot path (k and v written by their own kernel,
    attention reading them back from the cache) gives the bits of the fused
    path."""
    import torch
    c, m = world["c"], world["model"]
    B = 3
    toks = torch.tensor([11, 22, 33], dtype=torch.int32, device="cuda")
    pos = torch.tensor([15, 64, 159], dtype=torch.int32, device="cuda")
    slot = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    h1, h2 = (torch.empty((B, c["d"]), device="cuda") for _ in range(2))
    l1, l2 = (torch.empty((B, c["vocab"]), device="cuda") for _ in range(2))
    load_kv(world)
    m.forward_dev(toks, h1, pos, l1, B)
    x100b.sync()
    k1 = m.kv_read(1, 1, 0, c["ctx"])
    load_kv(world)
    m.forward_slots_dev(toks, h2, pos, slot, l2, B)
    x100b.sync()
    k2 = m.kv_read(1, 1, 0, c["ctx"])
    assert torch.equal(h1, h2) and torch.equal(l1, l2)
    assert np.array_equal(k1[0], k2[0]) and np.array_equal(k1[1], k2[1])


def test_slot_out_of_range_is_reported(world):
    import torch
    c, m = world["c"], world["model"]
    load_kv(world)
    toks = torch.tensor([1], dtype=torch.int32, device="cuda")
    pos = torch.tensor([3], dtype=torch.int32, device="cuda")
    slot = torch.tensor([c["max_batch"]], dtype=torch.int32, device="cuda")
    h = torch.empty((1, c["d"]), device="cuda")
    m.forward_slots_dev(toks, h, pos, slot, None, 1)
    with pytest.raises(x100b.X100Error) as e:
        x100b.sync()
    assert e.value.code == x100b.X100_E_ARG
    for s_ in range(c["max_batch"]):
        kg, _ = m.kv_read(0, s_, 0, c["ctx"])
        assert np.array_equal(kg, world["kv"][0][s_][0])
    with pytest.raises(x100b.X100Error):
        m.prefill(0, np.array([1, 2], np.int32), c["ctx"] - 1)   # runs past the cache


def test_model_rejects_bad_config():
    with pytest.raises(x100b.X100Error):
        x100b.Model(**dict(CFG, head_dim=64))
    with pytest.raises(x100b.X100Error):
        x100b.Model(**dict(CFG, n_heads=36))
