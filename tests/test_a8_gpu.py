"""GPU checks of the reference-numerics ("A8") activation path.

The reference's IME kernels consume activations packed to int8 by
pack_A_i8 (qwen_moe_q3k.c:420-426, one scale per 32 values, for its int8 /
Q8_0 path), pack_A_q3k (:613-623, one scale per 256 values, for Q3_K) and
pack_A_hp (qwen_moe_hp.c:131-180, fp16 scales per 32 relative to a per-256
average, for the int4 "HP" engine's Q4_0 weights).
x100q_pack_act_dev writes those records on the device and must equal the
reference's own packers bit for bit (a8_golden.npz, compiled from the
reference).  x100q_lin_gemv_dev_flags(X100Q_GEMV_A8) runs the GEMV on
activations packed that way (the single-token dp4a kernel and the several-
token tensor-core kernel) and must match the oracle's A8 GEMV
(orc_qgemv_a8: exact integer block dots, fp32 block terms summed in double)
to within fp32 summation rounding; against the fp32-activation oracle it
stays inside the reference's own kernel tolerance (0.05 relative,
bench/q3k_probe.c:467).
"""
import os

import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gold(golden_dir):
    return np.load(os.path.join(golden_dir, "a8_golden.npz"))


@pytest.mark.parametrize("mode, key, per, rec", [(x100b.PACK_I8, "pack_i8", 32, 38),
                                                 (x100b.PACK_Q3K, "pack_q3k", 256, 292),
                                                 (x100b.PACK_HP, "pack_hp", 256, 290)])
def test_pack_act_equals_reference(gold, mode, key, per, rec):
    import torch
    x = gold["x"]
    ref = gold[key]
    for rows in (1, 4):   # the same values as one row or as several rows
        K = x.size // rows
        K -= K % 256
        xd = torch.from_numpy(x[: K * rows].copy()).cuda()
        out = torch.zeros(K * rows // per * rec, dtype=torch.uint8, device="cuda")
        x100b.pack_act_dev(mode, xd, K, rows, out)
        x100b.sync()
        np.testing.assert_array_equal(out.cpu().numpy(), ref[: K * rows // per * rec])


def _gemv_a8(qt, N, K, B, seed):
    import torch
    rng = np.random.default_rng(seed)
    W = po.quantize(qt, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(B, K)).astype(np.float32)
    lin = x100b.Lin(qt, N, K, W)
    y = torch.empty(B, N, device="cuda")
    lin.gemv_dev(torch.from_numpy(x).cuda(), y, B, a8=True)
    x100b.sync()
    return W, x, y.cpu().numpy()


@pytest.mark.parametrize("qt, shape", [(po.Q8_0, (5120, 2048)), (po.Q8_0, (37, 256)), (po.Q3_K, (768, 2048)),
                                       (po.Q3_K, (2048, 768))])
@pytest.mark.parametrize("batch", [1, 3, 16])
def test_a8_gemv_matches_a8_oracle(qt, shape, batch):
    N, K = shape
    W, x, y = _gemv_a8(qt, N, K, batch, N + K + batch)
    ref = po.qgemv_a8(qt, W, N, K, x)
    assert po.rel_l2(y, ref) <= 1e-5, po.rel_l2(y, ref)
    # against the fp32-activation path: the A8 quantisation error, inside the
    # reference's own oracle-vs-kernel bar
    f32 = po.qgemv(qt, W, N, K, x, nthreads=8)
    assert 1e-5 < po.rel_l2(y, f32) <= 0.05


@pytest.mark.parametrize("shape", [(6144, 2048), (768, 2048), (2048, 768), (40, 256)])
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_hp_gemv_matches_hp_oracle(shape, batch):
    """The int4 HP engine's linear (qwen_moe_hp.c:513-533, 680): weights
    re-quantised by its quantize_q4_0_native (d = max|w| / 8, q in [-8, 7]),
    activations packed by pack_A_hp; the GEMV on those against the oracle's
    HP product (exact integer block dots, d * (fp16 sub-scale x fp16
    average) per 32-block, summed in double), and against the fp32 path."""
    import torch
    N, K = shape
    rng = np.random.default_rng(N * 7 + K + batch)
    W = po.quantize_q4_0_hp(rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(batch, K)).astype(np.float32)
    lin = x100b.Lin(po.Q4_0, N, K, W)
    y = torch.empty(batch, N, device="cuda")
    lin.gemv_dev(torch.from_numpy(x).cuda(), y, batch, a8=True)
    x100b.sync()
    y = y.cpu().numpy()
    ref = po.qgemv_a8(po.Q4_0, W, N, K, x)
    assert po.rel_l2(y, ref) <= 1e-5, po.rel_l2(y, ref)
    f32 = po.qgemv(po.Q4_0, W, N, K, x, nthreads=8)
    assert 1e-5 < po.rel_l2(y, f32) <= 0.05


def test_a8_rejects_other_weight_types():
    import torch
    K = 512
    W = po.quantize(po.Q4_K, np.random.default_rng(0).normal(0, 0.02, size=(64, K)).astype(np.float32))
    lin = x100b.Lin(po.Q4_K, 64, K, W)
    x = torch.zeros(1, K, device="cuda")
    y = torch.empty(1, 64, device="cuda")
    with pytest.raises(x100b.X100Error) as e:
        lin.gemv_dev(x, y, 1, a8=True)
    assert e.value.code == x100b.X100_E_UNSUPPORTED
    with pytest.raises(x100b.X100Error):
        x100b.pack_act_dev(x100b.PACK_Q3K, x, 100, 1, y)   # K not a multiple of 256
    with pytest.raises(x100b.X100Error):
        x100b.pack_act_dev(x100b.PACK_HP, x, 96, 1, y)     # K not a multiple of 256
    # HP packs whole 256-value records: a Q4_0 row of 96 weights has none
    W0 = po.quantize(po.Q4_0, np.zeros((8, 96), np.float32))
    lin0 = x100b.Lin(po.Q4_0, 8, 96, W0)
    with pytest.raises(x100b.X100Error) as e:
        lin0.gemv_dev(torch.zeros(1, 96, device="cuda"), torch.empty(1, 8, device="cuda"), 1, a8=True)
    assert e.value.code == x100b.X100_E_UNSUPPORTED
