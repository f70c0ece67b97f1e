"""GPU checks of the tensor-core GEMV for several tokens (qgemv_mma.cu).

Q4_0 and Q8_0 calls with 2..16 tokens run as m16n8k32 integer MMAs over the
same activation planes and in the same summation order as the dp4a kernel.
Checked here: parity with the CPU oracle (relative L2 1e-3) on shapes that
exercise every path of the kernel -- K split into chunks with a ragged last
chunk, a ragged last slice, rows that are not a multiple of the 16-row tile,
several tiles per CTA, 16 tokens in one launch and in two, RMS-norm folding
and accumulation through the device entry point -- and agreement with the
dp4a kernel (run in a child process with X100_GEMV_DP4A=1) to within fp32
summation rounding.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu

REL_Q = 1e-3
HERE = os.path.dirname(os.path.abspath(__file__))


def blocks(qt, N, K, seed):
    rng = np.random.default_rng(seed)
    return po.quantize(qt, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))


# (512, 7936): 31 slices per row (prime), so the rows are staged in ragged
# K-chunks; (2048, 4096) and (300, 6144): whole chunks; the rest whole rows
SHAPES = [(37, 256), (1000, 2080), (8192, 2048), (2048, 4096), (300, 6144), (5120, 2048), (512, 7936)]


@pytest.mark.parametrize("qt", [po.Q4_0, po.Q8_0])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("batch", [2, 8, 9, 16])
def test_mma_gemv_matches_oracle(qt, shape, batch):
    N, K = shape
    W = blocks(qt, N, K, N + K + qt)
    x = np.random.default_rng(batch + N).normal(0, 1, size=(batch, K)).astype(np.float32)
    ref = po.qgemv(qt, W, N, K, x, nthreads=8)
    lin = x100b.Lin(qt, N, K, W)
    y = np.empty((batch, N), np.float32)
    lin.gemv(x, y, batch)
    assert po.rel_l2(y, ref) <= REL_Q, (po.QNAMES[qt], shape, batch, po.rel_l2(y, ref))
    for b in range(batch):   # every token, not only the aggregate
        assert po.rel_l2(y[b], ref[b]) <= REL_Q


@pytest.mark.parametrize("qt", [po.Q4_0, po.Q8_0])
def test_single_token_tall_matrix(qt):
    """One token on a matrix of 70000 rows (the lm_head shape class)."""
    N, K = 70000, 2048
    W = blocks(qt, N, K, 77 + qt)
    x = np.random.default_rng(78).normal(0, 1, size=(1, K)).astype(np.float32)
    ref = po.qgemv(qt, W, N, K, x, nthreads=8)
    y = np.empty((1, N), np.float32)
    x100b.Lin(qt, N, K, W).gemv(x, y, 1)
    assert po.rel_l2(y, ref) <= REL_Q


def test_mma_gemv_device_path_repeat_and_streams():
    """Device pointers, repeated calls on one stream (the persistent CTAs'
    barriers re-initialised per launch) and a second stream."""
    import torch
    N, K, B = 6144, 2048, 8
    W = blocks(po.Q4_0, N, K, 3)
    lin = x100b.Lin(po.Q4_0, N, K, W)
    x = torch.randn(B, K, device="cuda")
    ref = po.qgemv(po.Q4_0, W, N, K, x.cpu().numpy(), nthreads=8)
    y = torch.empty(B, N, device="cuda")
    first = None
    for _ in range(20):
        lin.gemv_dev(x, y, B)
        x100b.sync()
        if first is None:
            first = y.clone()
        assert torch.equal(y, first)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y2 = torch.empty_like(y)
        lin.gemv_dev(x, y2, B, stream=s)
    s.synchronize()
    assert torch.equal(y2, first)
    assert po.rel_l2(first.cpu().numpy(), ref) <= REL_Q


CHILD = r"""
import sys, numpy as np
sys.path[:0] = [{paths}]
import py_oracle as po, x100b
out = []
for qt, N, K, B, seed in {cases}:
    rng = np.random.default_rng(seed)
    W = po.quantize(qt, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(B, K)).astype(np.float32)
    y = np.empty((B, N), np.float32)
    x100b.Lin(qt, N, K, W).gemv(x, y, B)
    out.append(y)
np.savez({path!r}, *out)
"""


def test_mma_agrees_with_dp4a_kernel(tmp_path):
    cases = [(po.Q4_0, 6144, 2048, 4, 1), (po.Q8_0, 5120, 2048, 16, 2), (po.Q8_0, 2048, 4096, 16, 3),
             (po.Q4_0, 1000, 2080, 7, 4)]
    paths = ", ".join(repr(p) for p in sys.path if p)
    res = {}
    for mode in ("mma", "dp4a"):
        path = str(tmp_path / f"{mode}.npz")
        env = dict(os.environ)
        env.pop("X100_GEMV_DP4A", None)
        if mode == "dp4a":
            env["X100_GEMV_DP4A"] = "1"
        subprocess.run([sys.executable, "-c", CHILD.format(paths=paths, cases=cases, path=path)], env=env,
                       check=True, timeout=300)
        res[mode] = np.load(path)
    for i in range(len(cases)):
        a, b = res["mma"][f"arr_{i}"], res["dp4a"][f"arr_{i}"]
        assert po.rel_l2(a, b) <= 1e-6, (cases[i], po.rel_l2(a, b))
