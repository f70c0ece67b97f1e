"""GPU tests of the expert-parallel combine (x100q_ep_*, peer-memory
all-reduce of the experts' partial outputs).

One process: the combine over a group of one (the kernel stores to its own
receive slot, raises and waits for its own flag) must return the input, add
into dst with accum, and keep working over many calls (epoch parities).

Two GPUs (skipped when fewer are visible): two child processes, one per GPU,
each holding half of the experts of a MoE layer; the combined output must
equal the unsplit oracle, be bit-identical on both processes and equal the
in-order sum of the two partials.  A process that skips a call makes the
other one's bounded wait run out and report X100_E_TIMEOUT (no hang).
"""
import os

import numpy as np
import pytest

import x100b

pytestmark = pytest.mark.gpu


def test_ep_group_of_one():
    import torch
    g = x100b.EpGroup(1, 0, 16384, lambda h: [h])
    for it in range(7):
        n = 2048 if it % 2 == 0 else 16384
        src = torch.randn(n, device="cuda")
        dst = torch.empty_like(src)
        g.allreduce_dev(src, dst, n)
        x100b.sync()
        assert torch.equal(dst, src)
        acc = torch.randn(n, device="cuda")
        ref = acc + src
        g.allreduce_dev(src, acc, n, accum=True)
        x100b.sync()
        assert torch.equal(acc, ref)
    # in place
    src = torch.randn(4096, device="cuda")
    ref = src.clone()
    g.allreduce_dev(src, src, 4096)
    x100b.sync()
    assert torch.equal(src, ref)
    with pytest.raises(x100b.X100Error):
        g.allreduce_dev(src, src, 4095)          # not a multiple of 4
    g.close()


def _two_gpu_child(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out
        import py_oracle as po
        g = x100b.EpGroup(world, rank, 16 * 2048, exchange)
        # 1. plain sums: in-order float adds, bit-identical on both processes
        for it in range(20):
            n = 2048 * (1 + it % 3)
            parts = [np.random.default_rng(100 * it + r).standard_normal(n).astype(np.float32) for r in range(world)]
            src = torch.from_numpy(parts[rank]).cuda()
            dst = torch.empty_like(src)
            g.allreduce_dev(src, dst, n)
            x100b.sync()
            ref = np.zeros(n, np.float32)
            for p in parts:
                ref = ref + p
            assert np.array_equal(dst.cpu().numpy(), ref), it
        # 2. a MoE layer split over the two processes
        rng = np.random.default_rng(7)
        d, E, k, ffn = 2048, 32, 8, 768
        router = (0.02 * rng.standard_normal((E, d))).astype(np.float32)
        enc = lambda n, kk: po.quantize(po.Q4_K, rng.normal(0, 0.02, (n, kk)).astype(np.float32))  # noqa: E731
        gate, up, down = enc(E * ffn, d), enc(E * ffn, d), enc(E * d, ffn)
        lo, hi = (0, E // 2) if rank == 0 else (E // 2, E)
        moe = x100b.Moe(d, E, k, ffn, po.Q4_K, router, gate, up, down, lo, hi)
        for B in (1, 3):
            hn = rng.standard_normal((B, d)).astype(np.float32)
            hd = torch.from_numpy(hn).cuda()
            eo = torch.empty_like(hd)
            moe.ffn_dev(hd, eo, B)
            g.allreduce_dev(eo, eo, B * d)
            x100b.sync()
            ref, _, _ = po.moe_ffn(d, E, k, ffn, po.Q4_K, router, gate, up, down, hn, nthreads=4)
            got = eo.cpu().numpy()
            assert po.rel_l2(got, ref) <= 1e-3
            both = [None] * world
            dist.all_gather_object(both, got.tobytes())
            assert both[0] == both[1]
        # 3. rank 1 skips a call: rank 0's wait runs out and is reported
        dist.barrier()
        if rank == 0:
            src = torch.ones(2048, device="cuda")
            g.allreduce_dev(src, src, 2048)
            try:
                x100b.sync()
                q.put((rank, "no timeout reported"))
                return
            except x100b.X100Error as e:
                assert e.code == x100b.X100_E_TIMEOUT, e.code
        dist.barrier()                       # rank 1 keeps its buffer until rank 0 is done
        g.close()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:                   # noqa: BLE001 - report to the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(not __import__("torch").cuda.is_available() or __import__("torch").cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_ep_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_two_gpu_child, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
