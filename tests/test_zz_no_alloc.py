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

import x100b

pytestmark = pytest.mark.gpu


def wellformed_q4k(nblocks, seed):
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(nblocks, 144), dtype=np.uint8)
    blk[:, 0:2] = np.asarray(rng.uniform(0.0002, 0.002, nblocks), np.float16).view(np.uint8).reshape(-1, 2)
    blk[:, 2:4] = np.asarray(rng.uniform(0.0, 0.001, nblocks), np.float16).view(np.uint8).reshape(-1, 2)
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
