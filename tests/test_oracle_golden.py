"""Pin the CPU oracle against fixtures produced by the reference's own code.

The fixtures (tests/golden/*.npz, meta.json) were written by
tests/golden/make_golden.py from the reference's src/gemm_ref.c, its block
decoders (qwen_moe.c:156-179, qwen_moe_q3k.c:541-577), its routing and
layer-body functions (qwen_moe.c:187-189, 297-301; qwen_moe_q3k.c:1170-1175,
1678) and its whole forward() (qwen_moe.c:272-315).  Every check here is
bit-exact.
"""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

import py_oracle as po

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))

QT = {"Q4_0": po.Q4_0, "Q8_0": po.Q8_0, "Q3_K": po.Q3_K, "Q4_K": po.Q4_K}


@pytest.fixture(scope="module")
def meta(golden_dir):
    with open(os.path.join(golden_dir, "meta.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def gemm_golden(golden_dir):
    return np.load(os.path.join(golden_dir, "gemm_golden.npz"))


@pytest.fixture(scope="module")
def quant_golden(golden_dir):
    return np.load(os.path.join(golden_dir, "quant_golden.npz"))


def gemm_inputs(M, N, K):
    seed = 1000003 * M + 1009 * N + K
    A = po.rand_i8(seed, M * K).reshape(M, K)
    B = po.rand_i8(seed + 1, K * N).reshape(K, N)
    C0 = po.rand_i8(seed + 2, M * N).astype(np.int32).reshape(M, N) * 1000
    Af = po.rand_f32(seed + 3, M * K).reshape(M, K)
    Bf = po.rand_f32(seed + 4, K * N).reshape(K, N)
    Cf = po.rand_f32(seed + 5, M * N).reshape(M, N)
    return A, B, C0, Af, Bf, Cf


def test_struct_sizes(meta):
    # bench/q3k_probe.c:410-413 known answers
    assert meta["sizeof_block_q3_K"] == 110 == po.BLOCK_BYTES[po.Q3_K]
    assert meta["sizeof_block_q5_K"] == 176
    assert po.BLOCK_BYTES[po.Q4_K] == 144 and po.BLOCK_BYTES[po.Q4_0] == 18 and po.BLOCK_BYTES[po.Q8_0] == 34


def test_caps_layout_matches_reference_header(meta):
    import ctypes

    class Caps(ctypes.Structure):
        _fields_ = [("vlen_bits", ctypes.c_int), ("vlenb", ctypes.c_int), ("has_v", ctypes.c_int),
                    ("has_zvfh", ctypes.c_int), ("has_zvbb", ctypes.c_int), ("has_ime", ctypes.c_int),
                    ("mvendorid", ctypes.c_ulong), ("isa", ctypes.c_char * 1024)]
    lay = meta["caps_layout"]
    assert ctypes.sizeof(Caps) == lay["sizeof"]
    assert Caps.has_ime.offset == lay["has_ime"]
    assert Caps.mvendorid.offset == lay["mvendorid"]
    assert Caps.isa.offset == lay["isa"]


@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (7, 9, 33), (16, 16, 16), (33, 17, 5),
                                   (64, 48, 40), (128, 64, 96), (129, 130, 131)])
def test_oracle_gemm_matches_reference(gemm_golden, shape):
    M, N, K = shape
    A, B, C0, Af, Bf, Cf = gemm_inputs(M, N, K)
    Ci = po.gemm_i8(A, B, C0.copy())
    np.testing.assert_array_equal(Ci, gemm_golden[f"i8_{M}x{N}x{K}"])
    Co = po.gemm_f32(Af, Bf, Cf.copy())
    assert Co.tobytes() == gemm_golden[f"f32_{M}x{N}x{K}"].tobytes()


def test_oracle_gemm_256_hash(meta):
    M = N = K = 256
    A, B, C0, Af, Bf, Cf = gemm_inputs(M, N, K)
    Ci = po.gemm_i8(A, B, C0.copy(), nthreads=4)
    assert hashlib.sha256(Ci.tobytes()).hexdigest() == meta["sha256_i8_256x256x256"]
    Co = po.gemm_f32(Af, Bf, Cf.copy(), nthreads=4)
    assert hashlib.sha256(Co.tobytes()).hexdigest() == meta["sha256_f32_256x256x256"]


@pytest.mark.parametrize("name", ["Q4_0", "Q8_0", "Q3_K", "Q4_K"])
def test_oracle_decode_matches_reference(quant_golden, name):
    qt = QT[name]
    blk = quant_golden[f"{name}_blocks"]
    ref = quant_golden[f"{name}_values"]
    be = po.BLOCK_ELEMS[qt]
    nb = blk.shape[0]
    got = po.dequant(qt, blk.reshape(-1), 1, nb * be).reshape(-1)
    # bit-exact, NaN-aware (edge blocks may decode to inf*0 = nan)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)) or \
        np.array_equal(got, ref, equal_nan=True)


def test_f16_conversions():
    for v in (0.0, 1.0, -2.5, 65504.0, 6.1e-5, 5.96e-8, 0.1):
        h = po.lib().orc_f32_to_f16_rne(v)
        assert np.float16(v).view(np.uint16) == h
        assert po.f16_to_f32(h) == float(np.float16(v))
    # the reference's truncating encoder (qwen_moe_hp.c:71-79) rounds toward zero
    t = po.lib().orc_f32_to_f16_trunc(0.1)
    assert po.f16_to_f32(t) <= 0.1 and po.f16_to_f32(t) > 0.0999


@pytest.mark.parametrize("qt", [po.Q4_0, po.Q8_0, po.Q3_K, po.Q4_K])
def test_encoder_roundtrip(qt):
    """Own encoders: quantise N(0, 0.02) weights, decode, bounded error."""
    rng = np.random.default_rng(5)
    N, K = 8, 512
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    blk = po.quantize(qt, w)
    assert blk.size == N * po.row_bytes(qt, K)
    wd = po.dequant(qt, blk, N, K)
    err = po.rel_l2(wd, w)
    bound = {po.Q8_0: 0.01, po.Q4_0: 0.15, po.Q4_K: 0.12, po.Q3_K: 0.30}[qt]
    assert err < bound, (po.QNAMES[qt], err)
    # idempotence: re-encoding the decoded weights reproduces the same values
    wd2 = po.dequant(qt, po.quantize(qt, wd), N, K)
    assert po.rel_l2(wd2, wd) < bound


def test_q4_0_encoder_follows_baseline_rule():
    """scale = max|w|/7 stored as fp16, q = round(w/scale) in [-7, 7]."""
    rng = np.random.default_rng(9)
    w = rng.normal(0, 0.02, size=(1, 32)).astype(np.float32)
    blk = po.quantize(po.Q4_0, w)
    d = np.frombuffer(blk[:2].tobytes(), np.float16)[0]
    assert abs(float(d) - np.abs(w).max() / 7) <= 1e-3 * abs(float(d)) + 1e-7
    qs = blk[2:18]
    nibs = np.concatenate([qs & 0xF, qs >> 4]).astype(int) - 8
    assert nibs.min() >= -7 and nibs.max() <= 7


def test_topk_tie_break_and_renorm():
    p = np.array([0.1, 0.3, 0.3, 0.05, 0.25], np.float32)
    sel = np.zeros(3, np.int32)
    w = np.zeros(3, np.float32)
    po.lib().orc_topk(po._ptr(p), 5, 3, po._ptr(sel), po._ptr(w))
    assert list(sel) == [1, 2, 4]          # strict >: lower index first on a tie
    assert abs(w.sum() - 1.0) < 1e-6


def test_moe_oracle_partial_experts_sum_to_full():
    """Expert-parallel property: partial eouts over disjoint expert ranges
    add up to the full block output (same routing everywhere)."""
    rng = np.random.default_rng(3)
    d, E, k, ffn = 256, 16, 4, 256
    router = rng.normal(0, 0.02, size=(E, d)).astype(np.float32)
    gate = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * ffn, d)).astype(np.float32))
    up = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * ffn, d)).astype(np.float32))
    down = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * d, ffn)).astype(np.float32))
    hn = rng.normal(0, 1, size=(2, d)).astype(np.float32)
    full, sel, w = po.moe_ffn(d, E, k, ffn, po.Q4_K, router, gate, up, down, hn)
    parts = [po.moe_ffn(d, E, k, ffn, po.Q4_K, router, gate, up, down, hn, lo, lo + 4)[0]
             for lo in range(0, E, 4)]
    assert po.rel_l2(sum(parts), full) < 1e-6
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)


def test_oracle_a8_packers_equal_reference(golden_dir):
    """pack_A_i8 / pack_A_q3k restated in the oracle give the reference's
    packed bytes (a8_golden.npz, from the reference's own code)."""
    g = np.load(os.path.join(golden_dir, "a8_golden.npz"))
    np.testing.assert_array_equal(po.pack_a("i8", g["x"]), g["pack_i8"])
    np.testing.assert_array_equal(po.pack_a("q3k", g["x"]), g["pack_q3k"])


def test_oracle_hp_packer_and_weight_quantiser_equal_reference(golden_dir):
    """pack_A_hp and quantize_q4_0_native of the int4 HP engine
    (qwen_moe_hp.c:102-109, 131-180, with its truncating f32_to_f16 :71-79)
    restated in the oracle give the reference's bytes (a8_golden.npz)."""
    g = np.load(os.path.join(golden_dir, "a8_golden.npz"))
    np.testing.assert_array_equal(po.pack_a("hp", g["x"]), g["pack_hp"])
    np.testing.assert_array_equal(po.quantize_q4_0_hp(g["w_hp"]), g["q4_0_hp"])


def test_oracle_hp_gemv_is_the_packed_product():
    """orc_qgemv_a8 for Q4_0 = sum over 32-blocks of d * (fp16 sub-scale *
    fp16 average) * (integer dot of the packed activations with q = nibble -
    8), against a numpy statement from the packed bytes."""
    rng = np.random.default_rng(12)
    N, K = 20, 768
    W = po.quantize_q4_0_hp(rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(2, K)).astype(np.float32)
    y = po.qgemv_a8(po.Q4_0, W, N, K, x)
    blk = W.reshape(N, K // 32, 18)
    d = blk[:, :, 0:2].copy().view(np.float16)[:, :, 0].astype(np.float32)
    qs = blk[:, :, 2:]
    qw = np.concatenate([qs & 15, qs >> 4], axis=2).astype(np.int64) - 8        # [N][K/32][32]
    for b in range(2):
        rec = po.pack_a("hp", x[b]).reshape(-1, 290)
        ss = np.stack([rec[:, 34 * k:34 * k + 2].copy().view(np.float16)[:, 0] for k in range(8)], 1)
        avg = rec[:, 288:290].copy().view(np.float16)[:, 0]
        eff = (ss.astype(np.float32) * avg.astype(np.float32)[:, None]).reshape(-1)   # per 32-block
        qa = np.stack([rec[:, 34 * k + 2:34 * k + 34].view(np.int8) for k in range(8)], 1).reshape(-1, 32)
        dots = np.einsum("nbk,bk->nb", qw, qa.astype(np.int64))
        ref = (d * (eff[None, :] * dots.astype(np.float32))).astype(np.float64).sum(axis=1)
        np.testing.assert_allclose(y[b], ref, rtol=1e-6, atol=1e-7)


def test_oracle_a8_gemv_is_the_packed_product():
    """orc_qgemv_a8 = sum over blocks of d * scale * (integer dot of the packed
    values), checked against a numpy statement from the packed bytes."""
    rng = np.random.default_rng(6)
    N, K = 24, 512
    W = po.quantize(po.Q8_0, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(2, K)).astype(np.float32)
    y = po.qgemv_a8(po.Q8_0, W, N, K, x)
    for b in range(2):
        rec = po.pack_a("i8", x[b]).reshape(-1, 38)
        sa = rec[:, 0:4].copy().view(np.float32)[:, 0].astype(np.float64)
        qa = rec[:, 6:].view(np.int8).astype(np.int64)
        blk = W.reshape(N, K // 32, 34)
        d = blk[:, :, 0:2].copy().view(np.float16)[:, :, 0].astype(np.float64)
        qw = blk[:, :, 2:].view(np.int8).astype(np.int64)
        ref = (d * sa[None, :] * np.einsum("nbk,bk->nb", qw, qa)).sum(axis=1)
        np.testing.assert_allclose(y[b], ref, rtol=1e-6, atol=1e-7)


def test_oracle_a8_gemv_q3k_is_the_packed_product():
    """orc_qgemv_a8 for Q3_K = sum over 16-element sub-blocks of
    d * (scale - 32) * sa * (integer dot of the packed activations with the
    3-bit weights), against a numpy statement: the 3-bit values are the
    dequantised weights divided by their sub-block scale (exact small
    integers), the packed values come from pack_A_q3k's bytes."""
    rng = np.random.default_rng(8)
    N, K = 12, 512
    W = po.quantize(po.Q3_K, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(2, K)).astype(np.float32)
    y = po.qgemv_a8(po.Q3_K, W, N, K, x)
    deq = po.dequant(po.Q3_K, W, N, K).astype(np.float64)          # [N][K]
    blk = W.reshape(N, K // 256, 110)
    d = blk[:, :, 108:110].copy().view(np.float16)[:, :, 0].astype(np.float64)
    for b in range(2):
        rec = po.pack_a("q3k", x[b]).reshape(-1, 292)
        sa = rec[:, 0:4].copy().view(np.float32)[:, 0].astype(np.float64)
        qa = rec[:, 36:].view(np.int8).astype(np.float64)             # [K/256][256]
        ref = np.zeros(N)
        for n in range(N):
            for sb in range(K // 256):
                w = deq[n, 256 * sb:256 * (sb + 1)]
                ref[n] += sa[sb] * np.dot(w, qa[sb])                 # = sum d*sc*q_w * sa*q_a
        np.testing.assert_allclose(y[b], ref, rtol=1e-5, atol=1e-7)


# ---- routing and decode-layer pins (moe_golden.npz, forward_golden.npz) ----------------
# Outputs of the reference's own softmax, top-k lines, rmsnorm, rope /
# rope_table / rope_apply, swiglu_exact and whole forward(), compiled from
# its sources by tests/golden/make_golden.py.  The oracle must reproduce them
# bit for bit (same fp32 operations in the same order, same libm).
@pytest.fixture(scope="module")
def moe_golden(golden_dir):
    return np.load(os.path.join(golden_dir, "moe_golden.npz"))


def test_softmax_equals_reference(moe_golden):
    g = moe_golden
    off = g["softmax_off"]
    for a, b in zip(off[:-1], off[1:]):
        x = np.ascontiguousarray(g["softmax_x"][a:b])
        po.lib().orc_softmax(po._ptr(x), int(b - a))
        np.testing.assert_array_equal(x, g["softmax_y"][a:b])


def test_topk_equals_reference_lines(moe_golden):
    """orc_softmax + orc_topk against qwen_moe.c:297-301 (softmax, greedy
    top-k with strict > so the lowest index wins a tie, renormalisation),
    including exact ties at the selection boundary and all-equal logits."""
    g = moe_golden
    lo = ko = 0
    for ne, na in zip(g["topk_ne"], g["topk_na"]):
        p = np.ascontiguousarray(g["topk_logits"][lo:lo + ne])
        po.lib().orc_softmax(po._ptr(p), int(ne))
        sel = np.zeros(na, np.int32)
        w = np.zeros(na, np.float32)
        po.lib().orc_topk(po._ptr(p), int(ne), int(na), po._ptr(sel), po._ptr(w))
        np.testing.assert_array_equal(sel, g["topk_sel"][ko:ko + na])
        np.testing.assert_array_equal(w, g["topk_w"][ko:ko + na])
        lo += ne
        ko += na
    # the tie cases select the lowest indices among equals
    assert list(g["topk_sel"][6 * 8:6 * 8 + 2]) == [3, 5]


def test_rmsnorm_equals_reference(moe_golden):
    g = moe_golden
    off = g["rms_off"]
    for a, b in zip(off[:-1], off[1:]):
        o = np.zeros(b - a, np.float32)
        x, w = np.ascontiguousarray(g["rms_x"][a:b]), np.ascontiguousarray(g["rms_w"][a:b])
        po.lib().orc_rmsnorm(po._ptr(o), po._ptr(x), po._ptr(w), int(b - a), 1e-6)
        np.testing.assert_array_equal(o, g["rms_y"][a:b])


def test_rope_equals_reference_table_and_inline(moe_golden):
    """orc_rope_neox = rope_table + rope_apply (qwen_moe_q3k.c:1170-1175) =
    rope (qwen_moe.c:188), positions 0 .. 4095."""
    g = moe_golden
    o = 0
    for hd, base, pos in g["rope_cfg"]:
        hd, pos = int(hd), int(pos)
        v = np.ascontiguousarray(g["rope_v"][o:o + hd])
        po.lib().orc_rope_neox(po._ptr(v), hd, pos, float(base))
        np.testing.assert_array_equal(v, g["rope_table_apply"][o:o + hd])
        np.testing.assert_array_equal(v, g["rope_inline"][o:o + hd])
        o += hd


def test_swiglu_equals_reference(moe_golden):
    g = moe_golden
    y = np.array([po.lib().orc_silu(float(x)) for x in g["swiglu_g"]], np.float32) * g["swiglu_u"]
    np.testing.assert_array_equal(y, g["swiglu_y"])


@pytest.mark.parametrize("case", ["small", "c5"])
def test_decode_chain_equals_reference_forward(golden_dir, case):
    """The oracle's decode chain (orc_decode_layer with the reference's fp32
    cache, then orc_decode_head) reproduces the logits of the reference's own
    forward() (qwen_moe.c:272-315) step by step: "small" runs two layers for
    eight steps from an empty cache, "c5" one layer of the decode
    configuration's attention shape at positions 0, 1000 and 4095 of a
    4096-position cache."""
    import golden_inputs as gi
    ref = np.load(os.path.join(golden_dir, "forward_golden.npz"))[f"{case}_logits"]
    got = gi.oracle_logits(case)
    np.testing.assert_array_equal(got, ref)
