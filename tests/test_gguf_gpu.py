"""GPU checks of GGUF ingest through the C ABI.

* x100q_gguf_dequant_dev decodes every GGUF type the reference's loader reads
  bit-identically to the reference's gguf_dequant_into (gguf_golden.npz) and
  Q4_K to its K-quant decoder (quant_golden.npz).
* x100q_quantize_q8_0_dev equals the reference's quantize_q8_0_native
  (gguf_golden.npz) and the oracle on a large array.
* x100q_model_load_gguf of a synthetic file with the reference checkpoint's
  Q3_K_S type mix (q, v, experts and token embeddings Q3_K, k Q8_0, output
  projection Q5_K, lm_head Q6_K, norms and router F32) gives the same bits as
  the same model built with x100q_model_set_* from the oracle's conversions,
  and stays within relative L2 1e-3 of the oracle's forward() chain; a tied
  lm_head is the Q8_0 of the decoded token embeddings.
"""
import os

import numpy as np
import pytest

import gguf_writer as gw
import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu

NAMES = {po.Q_F32: "F32", po.F16: "F16", po.Q4_0: "Q4_0", po.Q4_1: "Q4_1", po.Q8_0: "Q8_0", po.Q3_K: "Q3_K",
         po.Q5_K: "Q5_K", po.Q6_K: "Q6_K"}


@pytest.fixture(scope="module")
def gold(golden_dir):
    return np.load(os.path.join(golden_dir, "gguf_golden.npz"))


def _dev_dequant(gtype, blocks, n):
    import torch
    d = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    x100b.gguf_dequant_dev(gtype, d, n, out)
    x100b.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("gtype", list(NAMES))
def test_device_decoders_equal_reference(gold, gtype):
    name = NAMES[gtype]
    ref = gold[f"{name}_values"]
    got = _dev_dequant(gtype, gold[f"{name}_blocks"], ref.size)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_device_q4k_decoder_equals_reference(golden_dir):
    q = np.load(os.path.join(golden_dir, "quant_golden.npz"))
    ref = q["Q4_K_values"]
    got = _dev_dequant(po.Q4_K, q["Q4_K_blocks"], ref.size)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_device_decoders_large_against_oracle():
    rng = np.random.default_rng(8)
    for gtype in (po.Q3_K, po.Q5_K, po.Q6_K, po.Q4_1, po.F16):
        be, _ = po.GGUF_BLOCK[gtype]
        n = 256 * 4099   # odd number of blocks, several grid strides
        blk = gw.random_blocks(gtype, n // be, rng).reshape(-1)
        got = _dev_dequant(gtype, blk, n)
        np.testing.assert_array_equal(got.view(np.uint32), po.dequant_gguf(gtype, blk, n).view(np.uint32))


def test_device_q8_requant_equals_reference(gold):
    import torch
    x = gold["Q8REQ_input"]
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    x100b.quantize_q8_0_dev(xd, x.size, out)
    x100b.sync()
    np.testing.assert_array_equal(out.cpu().numpy(), gold["Q8REQ_blocks"])
    x = (np.random.default_rng(9).standard_normal(32 * 100003) * 0.05).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    x100b.quantize_q8_0_dev(xd, x.size, out)
    x100b.sync()
    np.testing.assert_array_equal(out.cpu().numpy(), po.quantize_q8_0_ref(x))
    with pytest.raises(x100b.X100Error):
        x100b.quantize_q8_0_dev(xd, 33, out)


CFG = dict(n_layers=2, d=2048, n_heads=32, n_kv_heads=4, head_dim=128, vocab=640, n_exp=32, n_act=8, moe_ffn=768)
MIX = dict(q=po.Q3_K, k=po.Q8_0, v=po.Q3_K, o=po.Q5_K, exp=po.Q3_K, router=po.Q_F32, norm=po.Q_F32,
           embd=po.Q3_K, lm=po.Q6_K)


def _converted(data, name, n):
    """What the loader puts in a Q8_0 slot: the block data itself when it is
    Q8_0, else the reference's Q8_0 of the decoded values."""
    gt, payload = data[name]
    if gt == po.Q8_0:
        return payload
    return po.quantize_q8_0_ref(po.dequant_gguf(gt, payload, n))


def _f32(data, name, n):
    gt, payload = data[name]
    return po.dequant_gguf(gt, payload, n)


def _oracle_layers(data, c):
    d, qd, kvd, E, F, hd = c["d"], c["n_heads"] * c["head_dim"], c["n_kv_heads"] * c["head_dim"], c["n_exp"], \
        c["moe_ffn"], c["head_dim"]
    out = []
    for l in range(c["n_layers"]):
        b = f"blk.{l}."
        out.append(dict(
            attn_norm=_f32(data, b + "attn_norm.weight", d), wq=_converted(data, b + "attn_q.weight", qd * d),
            wk=_converted(data, b + "attn_k.weight", kvd * d), wv=_converted(data, b + "attn_v.weight", kvd * d),
            q_norm=_f32(data, b + "attn_q_norm.weight", hd), k_norm=_f32(data, b + "attn_k_norm.weight", hd),
            wo=_converted(data, b + "attn_output.weight", d * qd), ffn_norm=_f32(data, b + "ffn_norm.weight", d),
            router=_f32(data, b + "ffn_gate_inp.weight", E * d), gate=data[b + "ffn_gate_exps.weight"][1],
            up=data[b + "ffn_up_exps.weight"][1], down=data[b + "ffn_down_exps.weight"][1]))
    return out


@pytest.fixture(scope="module")
def mixed(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf") / "mix.gguf")
    data = gw.qwen3moe_file(p, CFG, MIX, seed=21)
    g = x100b.Gguf(p)
    yield g, data
    g.close()


def test_load_mixed_types_equals_set_layer_model_and_oracle(mixed):
    g, data = mixed
    cfg = g.model_cfg()
    assert (cfg["attn_qtype"], cfg["expert_qtype"], cfg["lm_qtype"]) == (po.Q8_0, po.Q3_K, po.Q8_0)
    m = g.load_model(ctx=160, max_batch=2)
    c = dict(cfg, ctx=160, max_batch=2)
    layers = _oracle_layers(data, c)
    emb = _f32(data, "token_embd.weight", c["vocab"] * c["d"]).reshape(c["vocab"], c["d"])
    out_norm = _f32(data, "output_norm.weight", c["d"])
    lm = _converted(data, "output.weight", c["vocab"] * c["d"])
    ref = x100b.Model(**c)
    for li, lw in enumerate(layers):
        ref.set_layer(li, lw["attn_norm"], lw["wq"], lw["wk"], lw["wv"], lw["q_norm"], lw["k_norm"], lw["wo"],
                      lw["ffn_norm"], lw["router"], lw["gate"], lw["up"], lw["down"])
    ref.set_output(emb, out_norm, lm)
    toks, pos = np.array([5, 600], np.int32), np.array([0, 0], np.int32)
    got = m.forward(toks, pos)
    want = ref.forward(toks, pos)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # the oracle chain, position 0 of an empty cache
    for b in range(2):
        h = emb[toks[b]].copy()
        for li in range(c["n_layers"]):
            shape = (c["n_kv_heads"], c["ctx"], c["head_dim"])
            kc, vc = np.zeros(shape, np.uint16), np.zeros(shape, np.uint16)
            po.decode_layer(c, layers[li], kc, vc, h, 0, nthreads=8)
        r = po.decode_head(c, out_norm, lm, h, nthreads=8)
        assert po.rel_l2(got[b], r) <= 1e-3, po.rel_l2(got[b], r)
    m.close()
    ref.close()


def test_load_tied_lm_head_and_expert_range(tmp_path):
    c = dict(CFG, n_layers=1)
    p = str(tmp_path / "tied.gguf")
    types = dict(MIX, q=po.Q8_0, k=po.Q8_0, v=po.Q8_0, o=po.Q8_0, embd=po.F16)
    data = gw.qwen3moe_file(p, c, types, seed=4, tied=True)
    g = x100b.Gguf(p)
    cfg = g.model_cfg()
    assert (cfg["attn_qtype"], cfg["lm_qtype"]) == (po.Q8_0, po.Q8_0)
    m = g.load_model(ctx=64)
    emb = _f32(data, "token_embd.weight", c["vocab"] * c["d"])
    layers = _oracle_layers(data, dict(cfg))
    ref = x100b.Model(**dict(cfg, ctx=64))
    lw = layers[0]
    ref.set_layer(0, lw["attn_norm"], lw["wq"], lw["wk"], lw["wv"], lw["q_norm"], lw["k_norm"], lw["wo"],
                  lw["ffn_norm"], lw["router"], lw["gate"], lw["up"], lw["down"])
    ref.set_output(emb, _f32(data, "output_norm.weight", c["d"]), po.quantize_q8_0_ref(emb))
    toks, pos = np.array([17], np.int32), np.array([0], np.int32)
    np.testing.assert_array_equal(m.forward(toks, pos).view(np.uint32), ref.forward(toks, pos).view(np.uint32))
    m.close()
    ref.close()
    # half the experts: loads, and a model of a different shape is refused
    half = g.load_model(ctx=64, expert_lo=0, expert_hi=16)
    half.close()
    with pytest.raises(x100b.X100Error):
        g.load_model(d=1024)
    g.close()
