"""The reference's own GEMM harness, unmodified, on this library.

oracle/Makefile compiles the reference's bench/bench.c, unchanged, against
include/x100_gemm.h twice (outputs in oracle/_ref/, built where the
reference tree exists and shipped with the repository snapshot):
  gemm_bench_b200           every x100_gemm.h symbol from libx100gemm_b200.so;
  gemm_bench_b200_refcheck  the harness's oracle side, gemm_ref_f32 and
                            gemm_ref_i8, from the reference's own
                            src/gemm_ref.c linked into the executable, and
                            only the kernels under test (gemm_rvv_f32,
                            gemm_ime_i8) and the capability calls from the
                            library -- so the harness's own check compares
                            this library against the reference's scalar C.
Each is run as `gemm_bench M N K`, the way the reference's README runs it,
and its printed verdicts are checked: the fp32 line's maxerr gate
(bench/bench.c:50-55) and the int8 line's mismatch count (:84-90).
"""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def run_bench(exe, M, N, K):
    path = os.path.join(REF, exe)
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build it with make -C oracle where the reference tree exists")
    out = subprocess.run([path, str(M), str(N), str(K), "3"], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr
    return out.stdout


@pytest.mark.parametrize("exe", ["gemm_bench_b200", "gemm_bench_b200_refcheck"])
@pytest.mark.parametrize("shape", [(256, 256, 256), (1024, 1024, 1024), (129, 130, 131)])
def test_reference_harness_passes(exe, shape):
    txt = run_bench(exe, *shape)
    assert "tcgen05   : yes" in txt, txt          # the library found the B200
    f32 = re.search(r"rvv_f32\s*:\s*([\d.]+) GFLOP/s\s+maxerr=(\S+)\s+(\w+)", txt)
    i8 = re.search(r"i8->i32\s*:\s*([\d.]+) GOP/s\s+mismatch=(\d+)\s+(\w+)", txt)
    assert f32 and i8, txt
    assert f32.group(3) == "OK" and float(f32.group(2)) < 1e-2, txt
    assert i8.group(3) == "OK" and int(i8.group(2)) == 0, txt
    if exe.endswith("refcheck"):
        # against the reference's scalar fp32 GEMM the tf32 x3 kernel stays
        # far inside the harness's 1e-2 gate
        assert float(f32.group(2)) < 1e-3, txt
