"""Shared helpers of the op wrappers: head-dim handling and softmax scale."""

from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from .. import _native

# head dims the reference's NPU kernels accept; other dims are zero-padded to
# the next one of these and the softmax scale is taken from the padded dim
# (block_sparse_kernel_npu.py:651-656 then :340, streaming_kernel_npu.py:377-381
# then :114, vertical_slash_kernel_npu.py:568-573 then :409).
_REF_ALLOWED_HEAD_DIMS = (16, 32, 64, 128, 256, 512)
# head dims the sm_100a kernels are compiled for
_KERNEL_HEAD_DIMS = (64, 96, 128)

TRUE_SCALE_ENV = "MINFERENCE_TRUE_SCALE"


def reference_padded_dim(d: int) -> int:
    for c in _REF_ALLOWED_HEAD_DIMS:
        if c >= d:
            return c
    raise ValueError(f"head_dim={d} exceeds the largest supported value {_REF_ALLOWED_HEAD_DIMS[-1]}")


def default_softmax_scale(d: int) -> float:
    """Default scale of the sparse ops: 1/sqrt(padded D), as the reference's
    sparse ops compute it after zero-padding D; 1/sqrt(D) when
    MINFERENCE_TRUE_SCALE=1.  Dense attention does not use this: its default
    is 1/sqrt(D) of the unpadded dim."""
    if os.environ.get(TRUE_SCALE_ENV, "").strip().lower() in {"1", "true", "yes", "on"}:
        return 1.0 / math.sqrt(d)
    return 1.0 / math.sqrt(reference_padded_dim(d))


def kernel_dim(d: int) -> int:
    for c in _KERNEL_HEAD_DIMS:
        if c >= d:
            return c
    raise NotImplementedError(f"head_dim={d} > 128 is not supported by the sm_100a kernels")


def prepare(x: torch.Tensor, dk: int) -> torch.Tensor:
    """Zero-pad the head dim to dk and make rows usable by TMA (unit D stride,
    16-byte aligned row starts)."""
    if x.shape[-1] != dk:
        x = F.pad(x, (0, dk - x.shape[-1]))
    s = x.stride()
    if (
        s[-1] != 1
        or (s[0] * 2) % 16
        or (s[1] * 2) % 16
        or (s[2] * 2) % 16
        or x.data_ptr() % 16
    ):
        x = x.contiguous()
    return x


def check_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    assert q.dim() == 4, f"q must be 4D [B,H,S,D], got {q.dim()}D"
    assert (
        q.shape[0] == k.shape[0] and q.shape[1] == k.shape[1] and q.shape[-1] == k.shape[-1]
    ), f"q/k B/H/D mismatch; q={tuple(q.shape)} k={tuple(k.shape)}"
    assert k.shape == v.shape, f"k/v shape mismatch; k={tuple(k.shape)} v={tuple(v.shape)}"
    _native.require_cuda(q, k, v)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q/k/v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    _native.dtype_code(q)


def output(out: torch.Tensor | None, shape: tuple, like: torch.Tensor,
           zero: bool = False) -> torch.Tensor:
    """The output tensor: a new one (zero-filled if `zero`, for calls that
    write only some heads), or a caller-provided [B,H,S,D] view (any strides
    with unit D stride and 16-byte aligned rows) written in place."""
    if out is None:
        if zero:
            return torch.zeros(shape, dtype=like.dtype, device=like.device)
        return torch.empty(shape, dtype=like.dtype, device=like.device)
    if tuple(out.shape) != tuple(shape) or out.dtype != like.dtype or out.device != like.device:
        raise ValueError(
            f"out must be {tuple(shape)} {like.dtype} on {like.device}; got "
            f"{tuple(out.shape)} {out.dtype} on {out.device}"
        )
    s = out.stride()
    if s[-1] != 1 or (s[0] * 2) % 16 or (s[1] * 2) % 16 or (s[2] * 2) % 16 or out.data_ptr() % 16:
        raise ValueError("out needs unit D stride and 16-byte aligned rows")
    return out


def replica_ptrs(out_replicas, out: torch.Tensor, D: int, dk: int):
    """Device addresses of the output view's replicas: ``out_replicas`` gives,
    per replica, the address of element 0 of ``out`` in that buffer (an int),
    or a tensor laid out like ``out``."""
    if not out_replicas:
        return None
    if dk != D:
        raise NotImplementedError("output replicas need a head dim of 64, 96 or 128")
    return [int(r.data_ptr()) if isinstance(r, torch.Tensor) else int(r) for r in out_replicas]


def row_window(rows, S: int) -> tuple[int, int]:
    """Validate an optional query-row window ``(row_begin, row_end)``: whole
    128-row tiles, except that it may end at S.  None means every row."""
    if rows is None:
        return 0, S
    r0, r1 = int(rows[0]), int(rows[1])
    if not (0 <= r0 <= r1 <= S) or r0 % 128 or (r1 % 128 and r1 != S):
        raise ValueError(f"rows={rows!r}: need 0 <= begin <= end <= S={S}, begin a multiple of "
                         "128 and end a multiple of 128 or S")
    return r0, r1


_HEAD_TABLES: dict = {}


def head_table(heads, q: torch.Tensor):
    """(device int32 table or None, number of heads the call addresses).

    ``heads`` lists heads of q's head dimension (a sequence of ints, or an
    integer tensor); the op then runs on those heads only, in place, with one
    launch (the kernels index the views through the table).  A sequence is
    checked on the host and its device table cached, so repeated calls (a
    layer's groups at every forward) neither copy nor synchronise; a tensor is
    checked on its device."""
    H = q.shape[1]
    if heads is None:
        return None, H
    if isinstance(heads, torch.Tensor):
        t = heads.to(device=q.device, dtype=torch.int32).flatten()
        if t.numel() and (bool((t < 0).any()) or bool((t >= H).any())):
            raise ValueError(f"heads must lie in [0, {H}); got {t.tolist()}")
        return t, int(t.numel())
    hs = tuple(int(h) for h in heads)
    if any(h < 0 or h >= H for h in hs):
        raise ValueError(f"heads must lie in [0, {H}); got {list(hs)}")
    key = (hs, str(q.device))
    t = _HEAD_TABLES.get(key)
    if t is None:
        t = torch.tensor(hs, dtype=torch.int32, device=q.device)
        _HEAD_TABLES[key] = t
    return t, len(hs)
