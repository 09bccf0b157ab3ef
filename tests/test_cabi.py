"""C ABI host logic, no GPU: the library loads, exports every symbol that
include/cek.h declares, and rejects bad arguments before touching the device.
Mirrors the reference's host-side checks (esimd_kernel.sycl:26-37, :62-73),
which this build moves below the torch layer."""
import ctypes

import pytest

from esimd_learning_b200 import cabi


def test_library_exports_every_declared_symbol():
    L = cabi.lib()
    declared = cabi.header_functions()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(L, name), f"libcek_b200.so does not export {name}"
        assert name in cabi.SIGNATURES, f"cabi.SIGNATURES lacks a prototype for {name}"


def test_status_strings_and_version():
    L = cabi.lib()
    assert L.cek_status_string(0) == b"ok"
    for s in range(1, 6):
        assert L.cek_status_string(s) not in (b"ok", b"unknown status")
    assert L.cek_status_string(99) == b"unknown status"
    assert b"sm_100a" in L.cek_version()


def _gemv(**kw):
    a = dict(x=16, w=16, s=16, y=16, M=1, N=16, K=64, xd=0, yd=0, fmt=0, sk=0, fl=0)
    a.update(kw)
    return cabi.lib().cek_gemv_fp8(a["x"], a["w"], a["s"], a["y"], a["M"], a["N"], a["K"],
                                   a["xd"], a["yd"], a["fmt"], a["sk"], a["fl"], None)


@pytest.mark.parametrize("kw", [
    dict(M=-1), dict(N=-1), dict(K=24), dict(xd=2), dict(yd=-1), dict(fmt=2), dict(sk=3),
    dict(x=0), dict(w=0), dict(s=0), dict(y=0), dict(fl=8),
])
def test_gemv_rejects_bad_arguments(kw):
    assert _gemv(**kw) == cabi.CEK_ERR_INVALID_ARG


def test_gemv_alignment_and_empty():
    assert _gemv(x=8) == cabi.CEK_ERR_ALIGNMENT
    assert _gemv(w=24) == cabi.CEK_ERR_ALIGNMENT
    # M == 0 or N == 0: nothing to do, no launch
    assert _gemv(M=0, x=0, y=0) == cabi.CEK_OK
    assert _gemv(N=0) == cabi.CEK_OK


def test_norm_and_helpers_reject_bad_arguments():
    L = cabi.lib()
    assert L.cek_fused_add_rmsnorm(16, 16, 16, 1, 12, 1e-6, 0, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_fused_add_rmsnorm(16, 16, 16, 1, 32768, 1e-6, 0, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_fused_add_rmsnorm(16, 16, 16, 0, 512, 1e-6, 0, None) == cabi.CEK_OK
    assert L.cek_fused_add_rmsnorm(8, 16, 16, 1, 512, 1e-6, 0, None) == cabi.CEK_ERR_ALIGNMENT
    assert L.cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(3, 512) == 3072
    assert L.cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes(17, 512) == 0
    assert L.cek_fused_add_rmsnorm_gemv_fp8(16, 16, 16, 1e-6, 16, 16, 16, 16, 1 << 20, 17, 64, 512, 0,
                                            0, 0, 0, None) == cabi.CEK_ERR_INVALID_ARG
    # workspace smaller than the inverse-RMS block
    assert L.cek_fused_add_rmsnorm_gemv_fp8(16, 16, 16, 1e-6, 16, 16, 16, 16, 8, 2, 64, 512, 0,
                                            0, 0, 0, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_gelu_and_mul(16, 16, -1, 16, 0, None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_gelu_and_mul(16, 16, 0, 16, 0, None) == cabi.CEK_OK
    assert L.cek_qkv_norm_rope(16, 16, 16, 16, 16, 1, 8, 1, 96, 64, 1e-6, 1, 0,
                               None) == cabi.CEK_ERR_INVALID_ARG
    assert L.cek_quant_fp8_per_token(16, 16, 16, 1, 12, 0, None) == cabi.CEK_ERR_INVALID_ARG


def test_gemm_fp8w_preferred_crossovers():
    """The per-tensor dispatch (host only, no device work): GEMV family for
    M <= 16 and shapes the GEMM does not take, the tcgen05 GEMM above 256
    tokens, and in between the measured crossovers (148 SMs)."""
    L = cabi.lib()
    pref = L.cek_gemm_fp8w_preferred
    assert pref(16, 28672, 4096) == 0 and pref(17, 28672, 4096) == 1
    assert pref(25, 14336, 4096) == 0 and pref(26, 14336, 4096) == 1
    assert pref(59, 6144, 4096) == 0 and pref(60, 6144, 4096) == 1
    assert pref(111, 4096, 14336) == 0 and pref(112, 4096, 14336) == 1
    assert pref(257, 16, 64) == 1 and pref(300, 4096, 14336) == 1
    assert pref(64, 14336, 4100) == 0 and pref(64, 14348, 4096) == 0
    assert pref(0, 14336, 4096) == 0 and pref(64, 0, 4096) == 0
