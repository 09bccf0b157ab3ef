"""ctypes binding of the C ABI in include/cek.h (libcek_b200.so).

This is the binding a non-torch caller would write; the tests use it to call
the kernels through the C ABI directly, and it checks that every symbol the
header declares is exported.  Device pointers are passed as integers, the
stream as a `cudaStream_t` integer (0 = legacy default stream).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcek_b200.so"
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "cek.h"

(CEK_OK, CEK_ERR_INVALID_ARG, CEK_ERR_UNSUPPORTED, CEK_ERR_ALIGNMENT, CEK_ERR_LAUNCH, CEK_ERR_TIMEOUT,
 CEK_ERR_SCRATCH_LIMIT) = range(7)
CEK_NOALLOC_MAX_ROWS = 16
CEK_F16, CEK_BF16 = 0, 1
CEK_E4M3, CEK_E5M2 = 0, 1
CEK_SCALE_PERN_F16, CEK_SCALE_PERN_F32, CEK_SCALE_PERT_F32 = 0, 1, 2
CEK_GEMV_EARLY_WEIGHTS = 1
CEK_GEMV_GELU_MUL_OUTPUT = 2
CEK_COMM_SYNC_BYTES = 4096  # data area offset inside a comm region (include/cek.h)

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_U = ctypes.c_uint

# name -> (restype, argtypes); must list every function include/cek.h declares.
SIGNATURES = {
    "cek_status_string": (ctypes.c_char_p, [_I]),
    "cek_version": (ctypes.c_char_p, []),
    "cek_gemv_fp8": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _I, _U, _P]),
    "cek_gemv_fp8_multi": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P),
                                ctypes.POINTER(_I64), _I, _I64, _I64, _I, _I, _I, _I, _U, _P]),
    "cek_fused_add_rmsnorm": (_I, [_P, _P, _P, _I64, _I64, _F, _I, _P]),
    "cek_fused_add_rmsnorm_gemv_fp8_workspace_bytes": (_I64, [_I64, _I64]),
    "cek_fused_add_rmsnorm_gemv_fp8": (_I, [_P, _P, _P, _F, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _U, _P]),
    "cek_fused_add_rmsnorm_gemv_fp8_noalloc": (_I, [_P, _P, _P, _F, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _U, _P]),
    "cek_gelu_and_mul": (_I, [_P, _P, _I64, _I64, _I, _P]),
    "cek_qkv_norm_rope": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _I, _I, _P]),
    "cek_quant_fp8_per_token": (_I, [_P, _P, _P, _I64, _I64, _I, _P]),
    "cek_tp_comm_bytes": (_I64, [_I64, _I]),
    "cek_comm_alloc": (_I, [_I64, ctypes.POINTER(ctypes.c_void_p)]),
    "cek_comm_free": (_I, [_P]),
    "cek_ipc_get_handle": (_I, [_P, ctypes.c_char_p]),
    "cek_ipc_open_handle": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "cek_ipc_close_handle": (_I, [_P]),
    "cek_comm_errors": (_I, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "cek_comm_reset": (_I, [_P, _I64]),
    "cek_comm_barrier": (_I, [_P, _P, _I, _I, _P]),
    "cek_gemv_fp8_allgather": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I, _I, _I, _P, _P, _I64,
                                    _I, _I, _U, _P]),
    "cek_gemv_fp8_allreduce": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _I64, _I, _I, _U, _P]),
    "cek_gemm_fp8_scaled": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "cek_gemm_fp8w_workspace_bytes": (_I64, [_I64, _I64]),
    "cek_gemm_fp8w": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _P]),
    "cek_gemm_fp8w_preferred": (_I, [_I64, _I64, _I64]),
    "cek_gemv_fp8_timeouts": (_I, [ctypes.POINTER(ctypes.c_uint64)]),
    "cek_gemm_fp8_timeouts": (_I, [ctypes.POINTER(ctypes.c_uint64)]),
}


def header_functions() -> list[str]:
    """Names of the functions declared in include/cek.h."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"CEK_API\s+[\w\s\*]*?\b(cek_\w+)\s*\(", text)))


_lib = None


def lib() -> ctypes.CDLL:
    """Load libcek_b200.so once and attach the prototypes."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise OSError(f"{LIB_PATH} not built; run `python esimd_learning_b200/build.py`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class CekError(RuntimeError):
    def __init__(self, fn: str, status: int):
        msg = lib().cek_status_string(status).decode()
        super().__init__(f"{fn}: {msg} (status {status})")
        self.status = status


def call(name: str, *args) -> int:
    """Call `name`; raise CekError on a non-zero status (int results pass through)."""
    r = getattr(lib(), name)(*args)
    if SIGNATURES[name][0] is _I and r != CEK_OK:
        raise CekError(name, r)
    return r


def ptr(t) -> int:
    """Device pointer of a torch tensor (0 for None)."""
    return 0 if t is None else int(t.data_ptr())


def current_stream() -> int:
    import torch
    return int(torch.cuda.current_stream().cuda_stream)


def io_dtype(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return CEK_F16
    if t.dtype == torch.bfloat16:
        return CEK_BF16
    raise TypeError(f"unsupported I/O dtype {t.dtype}")


def fp8_format(w) -> int:
    import torch
    return CEK_E5M2 if w.dtype == torch.float8_e5m2 else CEK_E4M3


def scale_kind(s, N: int, per_tensor: bool = False) -> int:
    import torch
    if s.dtype == torch.float16:
        return CEK_SCALE_PERN_F16
    return CEK_SCALE_PERT_F32 if (per_tensor or s.numel() == 1 and N != 1) else CEK_SCALE_PERN_F32

