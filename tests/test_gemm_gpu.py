"""GPU parity of the dense GEMM entry points against the reference's results.

int8 paths must be bit-exact (fixtures from the reference's own gemm_ref_i8,
and the C oracle elsewhere); fp32 / fp16-in-fp32-accumulate paths must stay
within relative Frobenius error 1e-5 of gemm_ref_f32 (the BASELINE bar);
gemm_ref_f32 itself is bit-exact.  All calls go through the C ABI.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import py_oracle as po
import x100b

pytestmark = pytest.mark.gpu

REL_F32 = 1e-5   # relative Frobenius error bar for fp32 and fp16->fp32 GEMM


def inputs(M, N, K):
    seed = 1000003 * M + 1009 * N + K
    A = po.rand_i8(seed, M * K).reshape(M, K)
    B = po.rand_i8(seed + 1, K * N).reshape(K, N)
    C0 = po.rand_i8(seed + 2, M * N).astype(np.int32).reshape(M, N) * 1000
    Af = po.rand_f32(seed + 3, M * K).reshape(M, K)
    Bf = po.rand_f32(seed + 4, K * N).reshape(K, N)
    Cf = po.rand_f32(seed + 5, M * N).reshape(M, N)
    return A, B, C0, Af, Bf, Cf


def frob(x, ref):
    return po.rel_l2(x, ref)


@pytest.fixture(scope="module")
def golden(golden_dir):
    return np.load(os.path.join(golden_dir, "gemm_golden.npz"))


@pytest.fixture(scope="module")
def meta(golden_dir):
    return json.load(open(os.path.join(golden_dir, "meta.json")))


def test_caps_report_tcgen05():
    caps = x100b.detect()
    assert x100b.last_error() == 0
    assert caps.has_ime == 1 and caps.mvendorid == 0x10DE
    assert b"sm_10" in caps.isa


@pytest.mark.parametrize("fn", ["gemm_ime_i8", "gemm_ref_i8"])
@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (7, 9, 33), (16, 16, 16), (33, 17, 5),
                                   (64, 48, 40), (128, 64, 96), (129, 130, 131)])
def test_i8_matches_reference_fixture(golden, fn, shape):
    M, N, K = shape
    A, B, C0, *_ = inputs(M, N, K)
    C = C0.copy()
    x100b.gemm_host(fn, A, B, C)
    np.testing.assert_array_equal(C, golden[f"i8_{M}x{N}x{K}"])


def test_i8_256_matches_reference_hash(meta):
    A, B, C0, *_ = inputs(256, 256, 256)
    C = C0.copy()
    x100b.gemm_host("gemm_ime_i8", A, B, C)
    assert hashlib.sha256(C.tobytes()).hexdigest() == meta["sha256_i8_256x256x256"]


@pytest.mark.parametrize("shape", [(128, 256, 128), (256, 512, 1024), (300, 700, 520), (1, 16, 16),
                                   (1000, 1000, 1000), (130, 260, 4096), (512, 48, 2048), (600, 528, 2912)])
def test_i8_tc_vs_oracle(shape):
    M, N, K = shape
    A, B, C0, *_ = inputs(M, N, K)
    ref = po.gemm_i8(A, B, C0.copy(), nthreads=8)
    C = C0.copy()
    x100b.gemm_host("gemm_ime_i8", A, B, C)
    np.testing.assert_array_equal(C, ref)


def test_i8_extreme_values_no_saturation():
    # all -128 x -128 at K = 8192: |sum| = 2^27 -- exercises sign and magnitude
    M, N, K = 128, 256, 8192
    A = np.full((M, K), -128, np.int8)
    B = np.full((K, N), -128, np.int8)
    B[:, ::2] = 127
    C = np.zeros((M, N), np.int32)
    x100b.gemm_host("gemm_ime_i8", A, B, C)
    exp = np.where(np.arange(N) % 2 == 0, -128 * 127 * K, 128 * 128 * K).astype(np.int64)
    np.testing.assert_array_equal(C, np.broadcast_to(exp, (M, N)).astype(np.int32))


def test_i8_8192_cubed_equals_reference_gemm_ref_i8():
    """The benched configuration in full: M = N = K = 8192, operands uniform
    in [-128, 127], C != 0 on entry, through the reference-signature host call
    gemm_ime_i8, against the reference's own gemm_ref_i8 (src/gemm_ref.c
    compiled unchanged) run row-sliced on every host thread.  Bit-exact."""
    import os
    M = N = K = 8192
    A = po.rand_i8(81, M * K).reshape(M, K)
    B = po.rand_i8(82, K * N).reshape(K, N)
    C0 = (po.rand_i8(83, M * N).astype(np.int32) * 1000).reshape(M, N)
    C = C0.copy()
    x100b.gemm_host("gemm_ime_i8", A, B, C)
    try:
        nt = len(os.sched_getaffinity(0))
    except AttributeError:
        nt = os.cpu_count() or 1
    ref = po.ref_gemm_i8_mt(A, B, C0, max(1, nt))
    assert np.array_equal(C, ref), f"{int(np.count_nonzero(C != ref))} of {M * N} entries differ"


def test_i8_device_path_large_properties():
    """4096^3 on the device: tensor-core result equals the CUDA-core exact
    kernel, and C accumulates (second call adds the same product again)."""
    import torch
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    C1 = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    C2 = torch.zeros_like(C1)
    x100b.gemm_dev("gemm_ime_i8_dev", A, B, C1)
    x100b.gemm_dev("gemm_ref_i8_dev", A, B, C2)
    x100b.sync()
    assert torch.equal(C1, C2)
    x100b.gemm_dev("gemm_ime_i8_dev", A, B, C1)
    x100b.sync()
    assert torch.equal(C1, 2 * C2)
    # spot rows against the CPU oracle
    rows = [0, 1234, 4095]
    Ah, Bh = A[rows].cpu().numpy(), B.cpu().numpy()
    ref = po.gemm_i8(Ah, Bh, np.zeros((3, N), np.int32), nthreads=8)
    np.testing.assert_array_equal(C2[rows].cpu().numpy(), ref)


@pytest.mark.parametrize("N", [1024, 2048])
def test_i8_stream_k_shard_shapes(N):
    """The column shards of the 8192^3 GEMM on 8 and 4 GPUs leave a partial
    last wave of output tiles, which the 2-SM kernel splits along K across all
    CTA pairs (several pieces reduce-added into one C tile).  The result must
    equal the CUDA-core exact kernel on a non-zero C."""
    import torch
    M = K = 8192
    g = torch.Generator(device="cuda").manual_seed(N)
    A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    C0 = torch.randint(-2**30, 2**30, (M, N), dtype=torch.int32, device="cuda", generator=g)
    C1, C2 = C0.clone(), C0.clone()
    x100b.gemm_dev("gemm_ime_i8_dev", A, B, C1)
    x100b.gemm_dev("gemm_ref_i8_dev", A, B, C2)
    x100b.sync()
    assert torch.equal(C1, C2)


def test_i8_device_unaligned_falls_back_exactly():
    import torch
    M, N, K = 37, 45, 61   # lda = 61, ldb = 45: not TMA-addressable -> CUDA-core kernel
    A, B, C0, *_ = inputs(M, N, K)
    ref = po.gemm_i8(A, B, C0.copy())
    Ad, Bd, Cd = (torch.from_numpy(x).cuda() for x in (A, B, C0))
    x100b.gemm_dev("gemm_ime_i8_dev", Ad, Bd, Cd)
    x100b.sync()
    np.testing.assert_array_equal(Cd.cpu().numpy(), ref)


def test_i8_strided_device_variant():
    import torch
    M, N, K = 256, 512, 384
    A, B, C0, *_ = inputs(M, N, K)
    big = torch.from_numpy(np.ascontiguousarray(np.pad(B, ((0, 0), (0, 128))))).cuda()   # ldb = 640
    Ad, Cd = torch.from_numpy(A).cuda(), torch.from_numpy(C0.copy()).cuda()
    L = x100b.lib()
    s = torch.cuda.current_stream().cuda_stream
    x100b.check(L.gemm_ime_i8_dev_ld(M, N, K, Ad.data_ptr(), K, big.data_ptr(), N + 128, Cd.data_ptr(), N, s))
    x100b.sync()
    np.testing.assert_array_equal(Cd.cpu().numpy(), po.gemm_i8(A, B, C0.copy()))


def test_ime2_packed_driver_overwrites_c():
    M, N, K = 64, 128, 256
    A, B, *_ = inputs(M, N, K)
    pa, pb = po.ime2_pack(A, B)
    pa2 = np.empty_like(pa)
    pb2 = np.empty_like(pb)
    x100b.lib().gemm_ime2_pack_a(M, K, A.ctypes.data, pa2.ctypes.data)
    x100b.lib().gemm_ime2_pack_b(K, N, B.ctypes.data, pb2.ctypes.data)
    assert np.array_equal(pa, pa2) and np.array_equal(pb, pb2)
    C = np.full((M, N), 12345, np.int32)           # overwritten, not accumulated
    x100b.lib().gemm_ime2_i8_mt(M, N, K, pa.ctypes.data, pb.ctypes.data, C.ctypes.data, 8)
    x100b.check_last("gemm_ime2_i8_mt")
    np.testing.assert_array_equal(C, po.gemm_i8(A, B, np.zeros((M, N), np.int32)))


@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (7, 9, 33), (16, 16, 16), (33, 17, 5),
                                   (64, 48, 40), (128, 64, 96), (129, 130, 131)])
def test_ref_f32_bit_exact(golden, shape):
    M, N, K = shape
    *_, Af, Bf, Cf = inputs(M, N, K)
    C = Cf.copy()
    x100b.gemm_host("gemm_ref_f32", Af, Bf, C)
    assert C.tobytes() == golden[f"f32_{M}x{N}x{K}"].tobytes()


@pytest.mark.parametrize("shape", [(129, 130, 131), (256, 256, 256), (1024, 1024, 1024), (1000, 333, 777)])
def test_rvv_f32_within_1e5(shape):
    M, N, K = shape
    *_, Af, Bf, Cf = inputs(M, N, K)
    ref = po.gemm_f32(Af, Bf, Cf.copy(), nthreads=8)
    C = Cf.copy()
    x100b.gemm_host("gemm_rvv_f32", Af, Bf, C)
    assert frob(C, ref) <= REL_F32


@pytest.mark.parametrize("shape", [(128, 256, 64), (129, 130, 131), (256, 512, 1024), (1024, 1024, 1024),
                                   (100, 260, 72), (37, 45, 61)])
def test_f16_f32acc_within_1e5(shape):
    """fp16 inputs; oracle = gemm_ref_f32 on the widened fp16 values."""
    M, N, K = shape
    *_, Af, Bf, Cf = inputs(M, N, K)
    A16, B16 = Af.astype(np.float16), Bf.astype(np.float16)
    ref = po.gemm_f32(A16.astype(np.float32), B16.astype(np.float32), Cf.copy(), nthreads=8)
    C = Cf.copy()
    x100b.gemm_host("gemm_f16_f32acc", A16, B16, C)
    assert frob(C, ref) <= REL_F32


@pytest.mark.parametrize("shape", [(2048, 2048, 4096), (640, 1536, 8192), (1000, 512, 1000), (256, 260, 2048)])
def test_rvv_f32_tensor_core_path(shape):
    """gemm_rvv_f32 on TMA-addressable operands runs as three tf32
    tensor-core products; the result must stay within relative Frobenius
    1e-5 of an fp64 product (C += A.B with non-zero C).  (1000, 512, 1000):
    ragged tiles in every dimension; (256, 260, 2048): C's rows are not
    16-byte aligned, so the K-pieces of a tile are added through the
    non-TMA epilogue in order."""
    import torch
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.rand((M, K), device="cuda", generator=g) * 2 - 1
    B = torch.rand((K, N), device="cuda", generator=g) * 2 - 1
    C0 = torch.rand((M, N), device="cuda", generator=g) * 2 - 1
    C = C0.clone()
    x100b.gemm_dev("gemm_f32_dev", A, B, C)
    x100b.sync()
    ref = C0.double() + A.double() @ B.double()
    err = (torch.linalg.norm(C.double() - ref) / torch.linalg.norm(ref)).item()
    assert err <= REL_F32, err


def test_f16_f32acc_long_k():
    """fp16 operands, fp32 C at K = 12288 (three 4096-k accumulator pieces):
    relative Frobenius error vs the fp64 product of the fp16 values <= 1e-5."""
    import torch
    M, N, K = 1024, 1024, 12288
    g = torch.Generator(device="cuda").manual_seed(5)
    A = (torch.rand((M, K), device="cuda", generator=g) * 2 - 1).half()
    B = (torch.rand((K, N), device="cuda", generator=g) * 2 - 1).half()
    C = torch.zeros((M, N), device="cuda")
    x100b.gemm_dev("gemm_f16_f32acc_dev", A, B, C)
    x100b.sync()
    ref = A.double() @ B.double()
    err = (torch.linalg.norm(C.double() - ref) / torch.linalg.norm(ref)).item()
    assert err <= REL_F32, err


def test_rvv_f16_fp16_c():
    M, N, K = 256, 256, 512
    *_, Af, Bf, Cf = inputs(M, N, K)
    A16, B16, C16 = Af.astype(np.float16), Bf.astype(np.float16), Cf.astype(np.float16)
    ref = po.gemm_f32(A16.astype(np.float32), B16.astype(np.float32), C16.astype(np.float32), nthreads=8)
    C = C16.copy()
    x100b.gemm_host("gemm_rvv_f16", A16, B16, C)
    # one fp16 rounding of the fp32 result
    np.testing.assert_allclose(C.astype(np.float32), ref, rtol=2 ** -10, atol=1e-3)
    # fp32 accumulate: far better than the reference's fp16-accumulate 0.15 bar (bench/bench.c:66-71)
    assert frob(C.astype(np.float32), ref) < 1e-3


def test_f16_device_tc_vs_fp64():
    import torch
    M, N, K = 512, 768, 1024
    g = torch.Generator(device="cuda").manual_seed(3)
    A = (torch.rand((M, K), device="cuda", generator=g) * 2 - 1).half()
    B = (torch.rand((K, N), device="cuda", generator=g) * 2 - 1).half()
    C1 = torch.zeros((M, N), device="cuda")
    x100b.gemm_dev("gemm_f16_f32acc_dev", A, B, C1)
    x100b.sync()
    ref = A.double() @ B.double()
    assert (torch.linalg.norm(C1.double() - ref) / torch.linalg.norm(ref)).item() < REL_F32


def test_i8_host_call_in_panels_equals_device_call():
    """A host call moving more than 32 MiB runs as row panels (copies of A and
    C, the kernel and the copy back of C overlap on three streams).  Ragged
    last panel, N whose rows are not 16-byte aligned: the result must equal
    the device-pointer call bit for bit, and spot rows of every panel the
    CPU oracle."""
    import torch
    M, N, K = 2300, 3001, 4096
    A = po.rand_i8(11, M * K).reshape(M, K)
    B = po.rand_i8(12, K * N).reshape(K, N)
    C0 = po.rand_i8(13, M * N).astype(np.int32).reshape(M, N) * 1000
    C = C0.copy()
    x100b.gemm_host("gemm_ime_i8", A, B, C)
    Cd = torch.from_numpy(C0.copy()).cuda()
    x100b.gemm_dev("gemm_ime_i8_dev", torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), Cd)
    x100b.sync()
    np.testing.assert_array_equal(C, Cd.cpu().numpy())
    rows = [0, 511, 512, 1023, 1024, 1535, 1536, 2047, 2048, 2299]   # both sides of each 512-row panel edge
    ref = po.gemm_i8(A[rows], B, C0[rows].copy(), nthreads=8)
    np.testing.assert_array_equal(C[rows], ref)


def test_f32_and_f16_host_calls_in_panels():
    """Panelled host calls of the fp32 and fp16 routes stay within their
    bars: fp32 within relative Frobenius 1e-5 of the fp64 product; fp16 with
    fp16 C within one fp16 rounding of the fp32 result."""
    M, N, K = 1500, 4096, 2048
    rng = np.random.default_rng(3)
    Af = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    Bf = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    Cf = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    C = Cf.copy()
    x100b.gemm_host("gemm_rvv_f32", Af, Bf, C)
    ref = Cf.astype(np.float64) + Af.astype(np.float64) @ Bf.astype(np.float64)
    assert frob(C, ref) <= REL_F32
    M, N, K = 2000, 8192, 2048
    A16 = rng.uniform(-1, 1, (M, K)).astype(np.float16)
    B16 = rng.uniform(-1, 1, (K, N)).astype(np.float16)
    C16 = rng.uniform(-1, 1, (M, N)).astype(np.float16)
    C = C16.copy()
    x100b.gemm_host("gemm_rvv_f16", A16, B16, C)
    ref = C16.astype(np.float32) + A16.astype(np.float32) @ B16.astype(np.float32)
    np.testing.assert_allclose(C.astype(np.float32), ref, rtol=2 ** -10, atol=2e-2)
