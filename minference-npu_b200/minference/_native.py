"""ctypes binding of libminference_b200.so (the C ABI in include/minference_b200.h).

This is the only bridge between Python and the CUDA kernels.  There is no
fallback: if the library is missing or the tensors are not on a CUDA device,
the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_LIB_NAME = "libminference_b200.so"
_HERE = os.path.dirname(os.path.abspath(__file__))
_lock = threading.Lock()
_lib = None

MI_OK = 0
_STATUS = {
    1: "unsupported or inconsistent shape/argument",
    2: "unsupported dtype (fp16/bf16 only)",
    3: "workspace too small",
    4: "CUDA launch error",
    5: "pointer/stride alignment not usable by TMA (need 16-byte aligned rows)",
    6: "not an sm_100 device",
    7: "problem larger than the library's built-in scratch (allocation-free entry point)",
}
MI_F16, MI_BF16 = 0, 1
MAX_REPLICAS = 7


class MInferenceNativeError(RuntimeError):
    pass


class mi_tensor4(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("stride_b", ctypes.c_int64),
        ("stride_h", ctypes.c_int64),
        ("stride_s", ctypes.c_int64),
        ("stride_d", ctypes.c_int64),
        ("head_index", ctypes.c_void_p),
        ("head_extent", ctypes.c_int64),
        ("replica", ctypes.POINTER(ctypes.c_void_p)),
        ("n_replica", ctypes.c_int64),
    ]


def library_path() -> str:
    # MINFERENCE_B200_LIB points at an alternative build of the same library
    # (e.g. a tuning variant); by default the in-tree build is used.
    return os.environ.get("MINFERENCE_B200_LIB") or os.path.join(_HERE, _LIB_NAME)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not os.path.exists(path):
            raise MInferenceNativeError(
                f"{_LIB_NAME} not found at {path}; build it with `python __graft_entry__.py` "
                "(build()) or `python -m minference.build`"
            )
        L = ctypes.CDLL(path)
        T4 = mi_tensor4
        I64, P, F, I = ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_int
        SZ = ctypes.c_size_t
        L.mi_version.restype = ctypes.c_char_p
        L.mi_get_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
        L.mi_get_device_error.restype = I
        L.mi_stream_fwd.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I64, I, I64, I64, F, P]
        L.mi_stream_fwd.restype = I
        L.mi_dense_fwd.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I64, I, I, F, P]
        L.mi_dense_fwd.restype = I
        L.mi_block_pool_topk_workspace_size.argtypes = [I64, I64, I64, I64, I64]
        L.mi_block_pool_topk_workspace_size.restype = SZ
        L.mi_block_pool_topk.argtypes = [T4, T4, I64, I64, I64, I64, I64, I, I64, I, F, P, P, SZ, P]
        L.mi_block_pool_topk.restype = I
        L.mi_block_sparse_fwd_workspace_size.argtypes = [I64, I64, I64, I64]
        L.mi_block_sparse_fwd_workspace_size.restype = SZ
        L.mi_block_sparse_fwd.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I, P, I64, F, P, SZ, P]
        L.mi_block_sparse_fwd.restype = I
        L.mi_block_sparse_fwd_rows.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I, P, I64, F,
                                               I64, I64, P, SZ, P]
        L.mi_block_sparse_fwd_rows.restype = I
        L.mi_vs_estimate_workspace_size.argtypes = [I64, I64, I64]
        L.mi_vs_estimate_workspace_size.restype = SZ
        L.mi_vs_estimate.argtypes = [T4, T4, I64, I64, I64, I64, I, I64, I64, F, P, P, P, SZ, P]
        L.mi_vs_estimate.restype = I
        L.mi_vs_sparse_fwd_workspace_size.argtypes = [I64, I64, I64]
        L.mi_vs_sparse_fwd_workspace_size.restype = SZ
        L.mi_vs_sparse_fwd.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I, P, I64, P, I64, F, P, SZ, P]
        L.mi_vs_sparse_fwd.restype = I
        L.mi_vs_sparse_fwd_rows.argtypes = [T4, T4, T4, T4, I64, I64, I64, I64, I, P, I64, P, I64,
                                            F, I64, I64, P, SZ, P]
        L.mi_vs_sparse_fwd_rows.restype = I
        L.mi_vs_convert_indexes.argtypes = [P, P, I64, P, I64, I64, I64, I64, P, P, P, P, P]
        L.mi_vs_convert_indexes.restype = I
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MI_OK:
        raise MInferenceNativeError(f"{what} failed: status {rc} ({_STATUS.get(rc, 'unknown')})")


def t4(x: torch.Tensor, heads: torch.Tensor | None = None, replicas=None) -> mi_tensor4:
    """View descriptor of a BNSD tensor; `heads` (device int32) selects the
    heads a call addresses; `replicas` (output only) lists device addresses of
    the same view in other buffers, written as well (see mi_tensor4 in the
    header)."""
    s = x.stride()
    hp, he = (None, 0) if heads is None else (heads.data_ptr(), x.shape[1])
    t = mi_tensor4(x.data_ptr(), s[0], s[1], s[2], s[3], hp, he, None, 0)
    if replicas:
        if len(replicas) > MAX_REPLICAS:
            raise ValueError(f"at most {MAX_REPLICAS} output replicas")
        arr = (ctypes.c_void_p * len(replicas))(*[int(r) for r in replicas])
        t.replica = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
        t.n_replica = len(replicas)
        t._keep = arr  # the host array must outlive the call
    return t


def dtype_code(x: torch.Tensor) -> int:
    if x.dtype == torch.float16:
        return MI_F16
    if x.dtype == torch.bfloat16:
        return MI_BF16
    raise TypeError(f"minference-b200 kernels take fp16/bf16 tensors, got {x.dtype}")


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(
                "minference-b200 ops run only on CUDA (sm_100) tensors; got a tensor on "
                f"{t.device}. There is no CPU fallback."
            )


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def device_error() -> int:
    code = ctypes.c_int(0)
    check(lib().mi_get_device_error(ctypes.byref(code)), "mi_get_device_error")
    return code.value


def version() -> str:
    return lib().mi_version().decode()
