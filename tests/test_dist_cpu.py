"""Multi-process host logic of the sharded hot path, world size 2 on CPU (gloo).

The GPU runs use one process per GPU over NCCL (bench.py under torchrun):
the GEMM splits B and C by columns with no exchange, and the MoE layer is
expert parallel with one all-reduce of the partial outputs.  Here the same
split (x100b.shard) drives two gloo ranks that compute their parts with the
CPU oracle, and the gathered / reduced result must equal the unsplit one.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist
import torch.multiprocessing as mp

from x100b import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gemm_worker(rank, world, port, q):
    import py_oracle as po
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        M, N, K = 48, 64, 80
        A = po.rand_i8(11, M * K).reshape(M, K)
        B = po.rand_i8(12, K * N).reshape(K, N)
        n0, n1 = shard.gemm_cols(N, world, rank)
        Cr = po.gemm_i8(A, np.ascontiguousarray(B[:, n0:n1]), np.zeros((M, n1 - n0), np.int32))
        parts = [torch.empty((M, N // world), dtype=torch.int32) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(Cr))
        if rank == 0:
            C = torch.cat(parts, dim=1).numpy()
            q.put(bool(np.array_equal(C, po.gemm_i8(A, B, np.zeros((M, N), np.int32)))))
    finally:
        dist.destroy_process_group()


def _moe_worker(rank, world, port, q):
    import py_oracle as po
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        d, E, k, ffn = 256, 16, 4, 256
        rng = np.random.default_rng(5)
        router = rng.normal(0, 0.05, size=(E, d)).astype(np.float32)
        gate = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * ffn, d)).astype(np.float32))
        up = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * ffn, d)).astype(np.float32))
        down = po.quantize(po.Q4_K, rng.normal(0, 0.02, size=(E * d, ffn)).astype(np.float32))
        hn = rng.normal(0, 1, size=(3, d)).astype(np.float32)
        lo, hi = shard.expert_slice(E, world, rank)
        part, sel, _ = po.moe_ffn(d, E, k, ffn, po.Q4_K, router, gate, up, down, hn, expert_lo=lo, expert_hi=hi)
        t = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(t)
        sels = [torch.empty_like(torch.from_numpy(sel)) for _ in range(world)]
        dist.all_gather(sels, torch.from_numpy(sel))
        if rank == 0:
            full, fsel, _ = po.moe_ffn(d, E, k, ffn, po.Q4_K, router, gate, up, down, hn)
            same_sel = all(np.array_equal(s.numpy(), fsel) for s in sels)
            q.put(bool(same_sel and po.rel_l2(t.numpy(), full) <= 1e-6))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_gemm_worker, _moe_worker], ids=["gemm_nshard", "moe_expert_parallel"])
def test_two_ranks_match_unsplit(worker):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    assert q.get(timeout=5) is True


def test_shard_ranges():
    assert [shard.gemm_cols(8192, 4, r) for r in range(4)] == [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192)]
    sl = [shard.expert_slice(128, 8, r) for r in range(8)]
    assert sl[0] == (0, 16) and sl[-1] == (112, 128)
    assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
    with pytest.raises(ValueError):
        shard.gemm_cols(100, 3, 0)
    with pytest.raises(ValueError):
        shard.expert_slice(4, 8, 0)
