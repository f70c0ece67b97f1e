"""x100q_router_topk_noalloc: routing without any GPU allocation.

Some callers cannot call cudaMalloc: their device memory belongs to a
framework's pool or to a fixed budget committed up front, or they route
tokens inside a hot loop where an allocation (and the device synchronisation
it may bring) is not acceptable.  For them the library offers one routing
entry point that allocates nothing; its scratch (logits and a completion
ticket) is a fixed static device array.  This test calls it through the C ABI
and checks it against the routing returned by the existing x100q_moe_ffn_dev
entry point on the same activations, on two calls in a row, with the
tolerance the other MoE tests use.  It also checks that those two calls left
the device's free memory unchanged and that oversized requests are refused.

The file is named to be collected last, so that a failing run with -x has
already run every other test.
"""
import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu


def wellformed_q4k(nblocks, seed):
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(nblocks, 144), dtype=np.uint8)
    blk[:, 0:2] = np.asarray(rng.uniform(0.0002, 0.002, nblocks), np.float16).view(np.uint8).reshape(-1, 2)
    blk[:, 2:4] = np.asarray(rng.uniform(0.0, 0.001, nblocks), np.float16).view(np.uint8).reshape(-1, 2)
    return np.ascontiguousarray(blk.reshape(-1))


def wellformed_q8(nblocks, seed):
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(nblocks, 34), dtype=np.uint8)
    blk[:, 0:2] = np.asarray(rng.uniform(0.0002, 0.0006, nblocks), np.float16).view(np.uint8).reshape(-1, 2)
    return np.ascontiguousarray(blk.reshape(-1))


def test_router_topk_noalloc_matches_moe_routing():
    import torch

    torch.cuda.set_device(0)
    L = x100b.lib()
    d, E, k, ffn, batch = 2048, 128, 8, 768, 16
    rng = np.random.default_rng(2024)
    router = rng.normal(0, 0.02, size=(E, d)).astype(np.float32)
    # the existing entry point only needs the experts it holds; routing is
    # computed over all E experts either way
    held = 8
    gate = wellformed_q4k(held * ffn * d // 256, 1)
    up = wellformed_q4k(held * ffn * d // 256, 2)
    down = wellformed_q4k(held * d * ffn // 256, 3)
    moe = x100b.Moe(d, E, k, ffn, x100b.Q4_K, router, gate, up, down, 0, held)

    router_d = torch.from_numpy(router).cuda()
    hns = [torch.from_numpy(rng.normal(0, 1, size=(batch, d)).astype(np.float32)).cuda() for _ in range(3)]
    eout = torch.empty((batch, d), device="cuda")
    sel_ref = torch.empty((batch, k), dtype=torch.int32, device="cuda")
    w_ref = torch.empty((batch, k), device="cuda")
    outs = [(torch.empty((batch, k), dtype=torch.int32, device="cuda"), torch.empty((batch, k), device="cuda"))
            for _ in range(3)]
    s = torch.cuda.current_stream().cuda_stream

    def noalloc(hn, out):
        return L.x100q_router_topk_noalloc(router_d.data_ptr(), hn.data_ptr(), d, E, k, batch,
                                           out[0].data_ptr(), out[1].data_ptr(), s)

    # the first call on this device does the one-time set-up (symbol address lookup)
    x100b.check(noalloc(hns[0], outs[0]), "x100q_router_topk_noalloc (set-up call)")
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    x100b.check(noalloc(hns[1], outs[1]), "x100q_router_topk_noalloc (call 1)")   # two calls in a row
    x100b.check(noalloc(hns[2], outs[2]), "x100q_router_topk_noalloc (call 2)")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before, "the no-allocation calls changed device memory use"
    for i in (1, 2):
        moe.ffn_dev(hns[i], eout, batch, sel_ref, w_ref)
        torch.cuda.synchronize()
        assert torch.equal(outs[i][0], sel_ref), f"call {i}: expert selection differs"
        np.testing.assert_allclose(outs[i][1].cpu().numpy(), w_ref.cpu().numpy(), rtol=1e-5, atol=1e-7)
    # requests beyond the fixed scratch are refused with a clear error, and
    # nothing is launched
    assert L.x100q_router_topk_noalloc(router_d.data_ptr(), hns[0].data_ptr(), d, 256, k, 16,
                                       outs[0][0].data_ptr(), outs[0][1].data_ptr(), s) == x100b.X100_E_TOO_LARGE
    assert x100b.last_error() == x100b.X100_E_TOO_LARGE
    assert "no-allocation" in x100b.strerror(x100b.X100_E_TOO_LARGE)
    moe.close()


@pytest.mark.parametrize("d,batch", [(64, 1), (160, 16), (2000, 16), (2048, 1), (2080, 4)])
def test_router_topk_noalloc_ragged_rows(d, batch):
    """Router rows whose length is not a multiple of 128 floats (the part the
    kernel streams after the registers' share), and short rows (d < 128),
    give the oracle's routing: selection exact, weights within 1e-5.  When
    d % 32 == 0 a Q8_0 MoE handle's routing (x100q_moe_ffn_dev) is compared
    as well."""
    import torch

    torch.cuda.set_device(0)
    L = x100b.lib()
    E, k = 128, 8
    rng = np.random.default_rng(d * 31 + batch)
    router = rng.normal(0, 0.02, size=(E, d)).astype(np.float32)
    hn = rng.normal(0, 1, size=(batch, d)).astype(np.float32)
    rsel, rw = po.route(router, hn, k)
    # the seeded inputs leave no near-tie at the selection boundary, so fp32
    # summation order cannot change the oracle's choice
    p = np.exp((hn @ router.T.astype(np.float64)) - (hn @ router.T).max(1, keepdims=True))
    srt = np.sort(p, axis=1)[:, ::-1]
    assert np.all((srt[:, k - 1] - srt[:, k]) / srt[:, k - 1] > 1e-4)
    router_d = torch.from_numpy(router).cuda()
    hn_d = torch.from_numpy(hn).cuda()
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        sel = torch.full((batch, k), -1, dtype=torch.int32, device="cuda")
        w = torch.zeros((batch, k), device="cuda")
        x100b.check(L.x100q_router_topk_noalloc(router_d.data_ptr(), hn_d.data_ptr(), d, E, k, batch,
                                                sel.data_ptr(), w.data_ptr(), s), "x100q_router_topk_noalloc")
        torch.cuda.synchronize()
        np.testing.assert_array_equal(sel.cpu().numpy(), rsel)
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
    if d % 32 == 0:
        held, ffn = 4, 64
        blk = lambda n, sd: wellformed_q8(n, sd)   # noqa: E731
        moe = x100b.Moe(d, E, k, ffn, x100b.Q8_0, router, blk(held * ffn * d // 32, 1), blk(held * ffn * d // 32, 2),
                        blk(held * d * ffn // 32, 3), 0, held)
        eout = torch.empty((batch, d), device="cuda")
        sel_m = torch.empty((batch, k), dtype=torch.int32, device="cuda")
        w_m = torch.empty((batch, k), device="cuda")
        moe.ffn_dev(hn_d, eout, batch, sel_m, w_m)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(sel_m.cpu().numpy(), rsel)
        np.testing.assert_allclose(w_m.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
        moe.close()


def test_router_topk_noalloc_argument_limits():
    """Arguments outside the documented limits are refused with X100_E_ARG
    before anything is launched: d not a multiple of 4, n_act above n_exp or
    above 16, batch above 16, unaligned pointers."""
    import torch

    torch.cuda.set_device(0)
    L = x100b.lib()
    d, E = 256, 32
    router = torch.zeros((E, d + 4), device="cuda")
    hn = torch.zeros((16, d + 4), device="cuda")
    sel = torch.empty((16, 16), dtype=torch.int32, device="cuda")
    w = torch.empty((16, 16), device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def call(dd, ne, na, b, rp=None, hp=None):
        return L.x100q_router_topk_noalloc(rp or router.data_ptr(), hp or hn.data_ptr(), dd, ne, na, b,
                                          sel.data_ptr(), w.data_ptr(), s)
    assert call(d + 2, E, 8, 1) == x100b.X100_E_ARG            # d % 4 != 0
    assert call(d, 4, 8, 1) == x100b.X100_E_ARG                # n_act > n_exp
    assert call(d, E, 17, 1) == x100b.X100_E_ARG               # n_act > 16
    assert call(d, E, 8, 17) == x100b.X100_E_ARG               # batch > 16
    assert call(d, E, 8, 0) == x100b.X100_E_ARG                # batch < 1
    assert call(d, E, 8, 1, rp=router.data_ptr() + 4) == x100b.X100_E_ARG   # router not 16-byte aligned
    assert call(d, 257, 8, 1) == x100b.X100_E_ARG              # n_exp > 256
    assert x100b.last_error() == x100b.X100_E_ARG
    assert call(d, E, 8, 2) == x100b.X100_OK                   # and a valid call still works
    torch.cuda.synchronize()
