"""CPU checks of the C ABI: the product library loads, exports every function
declared in include/*.h, and reports errors through its error channel (no
GPU is touched; calls that need a device must fail cleanly here)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import x100b


def test_library_exports_every_header_function():
    names = x100b.header_functions()
    assert "gemm_ime_i8" in names and "x100q_moe_ffn" in names and len(names) >= 30
    L = x100b.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_reference_symbols_present():
    # the reference header's symbols (include/x100_gemm.h:42-61), same names
    for n in ("x100_detect", "x100_caps_print", "gemm_ref_f32", "gemm_rvv_f32", "gemm_rvv_f16",
              "gemm_ref_i8", "gemm_ime_i8"):
        assert hasattr(x100b.lib(), n)


def test_only_api_symbols_exported():
    out = subprocess.check_output(["nm", "-D", "--defined-only", x100b.LIB_PATH], text=True)
    funcs = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert funcs <= set(x100b.header_functions()), funcs - set(x100b.header_functions())


def test_caps_struct_size():
    assert ctypes.sizeof(x100b.Caps) == 1056


def test_strerror_table():
    assert x100b.strerror(0) == "ok"
    assert "timeout" in x100b.strerror(x100b.X100_E_TIMEOUT) or "wait" in x100b.strerror(x100b.X100_E_TIMEOUT)
    assert x100b.strerror(999) == "unknown error"


def test_bad_arguments_are_reported_not_fatal():
    L = x100b.lib()
    L.gemm_ime_i8(-1, 4, 4, None, None, None)
    assert x100b.last_error() == x100b.X100_E_ARG
    L.gemm_ime_i8(0, 0, 0, None, None, None)      # empty GEMM is a no-op
    assert x100b.last_error() == x100b.X100_OK
    assert L.x100_set_device(-3) == x100b.X100_E_ARG


def _run_child(code: str, env_extra: dict) -> str:
    env = dict(os.environ, **env_extra)
    env["CUDA_VISIBLE_DEVICES"] = env_extra.get("CUDA_VISIBLE_DEVICES", env.get("CUDA_VISIBLE_DEVICES", ""))
    pkg = os.path.dirname(x100b.PKG_DIR + "/")
    return subprocess.check_output(["python", "-c", f"import sys; sys.path.insert(0, {pkg!r}); " + code],
                                   env=env, text=True).strip()


def test_no_device_is_an_error_not_a_crash():
    # CUDA_VISIBLE_DEVICES="" hides every GPU: the call must record NODEV and
    # leave C untouched (no CPU fallback computes it).
    out = _run_child(
        "import numpy as np, x100b; A=np.ones((4,4),np.int8); C=np.zeros((4,4),np.int32); "
        "x100b.lib().gemm_ime_i8(4,4,4,A.ctypes.data,A.ctypes.data,C.ctypes.data); "
        "print(x100b.last_error(), int(C.sum()))", {"CUDA_VISIBLE_DEVICES": ""})
    code, csum = map(int, out.split())
    assert code == x100b.X100_E_NODEV and csum == 0


@pytest.mark.parametrize("site,fn", [("device", "gemm_ime_i8"), ("device", "gemm_rvv_f32")])
def test_fault_injection_on_host(site, fn):
    out = _run_child(
        "import numpy as np, x100b; A=np.ones((4,4),np.int8); C=np.zeros((4,4),np.int32); "
        f"x100b.lib().{fn}(4,4,4,A.ctypes.data,A.ctypes.data,C.ctypes.data); print(x100b.last_error())",
        {"X100_FAULT": site})
    assert int(out) == x100b.X100_E_INJECTED


def test_quant_row_bytes():
    L = x100b.lib()
    assert L.x100q_row_bytes(x100b.Q4_0, 2048) == 64 * 18
    assert L.x100q_row_bytes(x100b.Q4_K, 2048) == 8 * 144
    assert L.x100q_row_bytes(x100b.Q3_K, 768) == 3 * 110
    assert L.x100q_row_bytes(x100b.Q8_0, 4096) == 128 * 34
    assert L.x100q_row_bytes(x100b.Q4_K, 100) == 0


def test_quant_create_without_device_fails_cleanly():
    out = _run_child(
        "import numpy as np, x100b; L=x100b.lib(); b=np.zeros(18*64*8,np.uint8); "
        "h=L.x100q_lin_create(2,8,2048,b.ctypes.data); print(int(h is None or h==0), x100b.last_error())",
        {"CUDA_VISIBLE_DEVICES": ""})
    null, code = map(int, out.split())
    assert null == 1 and code == x100b.X100_E_NODEV


def test_step_timing_buckets_named_and_checked():
    """The timing buckets follow the header's enum order; a null model is an
    argument error (no device touched)."""
    src = open(os.path.join(os.path.dirname(x100b.LIB_PATH), "..", "include", "x100q.h")).read()
    a = src.index("X100Q_T_EMBED = 0")
    enum = src[a:src.index("X100Q_NBUCKETS", a)]
    assert enum.count("X100Q_T_") == x100b.TIMING_BUCKETS
    names = [x100b.timing_bucket_name(i) for i in range(x100b.TIMING_BUCKETS)]
    assert names == ["embed", "qkv", "attention", "o", "router", "expert", "combine", "lm"]
    assert x100b.timing_bucket_name(-1) is None and x100b.timing_bucket_name(x100b.TIMING_BUCKETS) is None
    L = x100b.lib()
    assert L.x100q_model_timing(None, 1) == 1 and L.x100q_model_timing_read(None, None, None) == 1
