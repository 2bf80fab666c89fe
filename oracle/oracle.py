"""Test oracle: CPU restatement of the reference's sparse-prefill algorithms.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import this module; the product path
(``minference-npu_b200/minference``) never does.

Index algorithms come from ``libmi_oracle.so`` (``mi_oracle.c``), whose
fixed evaluation order makes them bit-comparable with the CUDA kernels.
Masks and fp32 masked attention are restated here in numpy.  Reference
functions followed (paths relative to the MInference-NPU project root):

* ``block_pool_topk``      block_sparse_kernel_npu.py:230-263
* ``block_sparse_mask``    block_sparse_kernel_npu.py:266-317
* ``stream_mask``          streaming_kernel_npu.py:94-146 (visible set at :131-136)
* ``vs_estimate``          minference_forward.py:124-167
* ``vs_mask``              vertical_slash_kernel_npu.py:255-369
* ``vs_convert_indexes``   backend_npu/cuda_shim.py:147-236 (legacy format)
* ``masked_attention``     block_sparse_kernel_npu.py:325-348,
                           vertical_slash_kernel_npu.py:377-415 (fp32 softmax,
                           fully masked rows -> 0)

The oracle is pinned against the reference's own outputs stored in
``tests/golden/`` (see ``tests/test_oracle_golden.py``).
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmi_oracle.so")
_lib = None


def build() -> None:
    subprocess.check_call(["sh", os.path.join(_HERE, "build_oracle.sh")])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, f32 = ctypes.c_int, ctypes.c_float
        L.oracle_block_pool_topk.argtypes = [P, P, i32, i32, i32, i32, i32, i32, f32, P]
        L.oracle_block_pool_topk.restype = i32
        L.oracle_vs_estimate.argtypes = [P, P, i32, i32, i32, i32, i32, f32, P, P, P]
        L.oracle_vs_estimate.restype = i32
        L.oracle_vs_block_row.argtypes = [P, i32, P, i32, i32, i32, P]
        L.oracle_vs_block_row.restype = None
        L.oracle_vs_convert_indexes.argtypes = [P, i32, P, i32, i32, i32, P, P, P, P]
        L.oracle_vs_convert_indexes.restype = None
        L.oracle_det_exp.argtypes = [f32]
        L.oracle_det_exp.restype = f32
        _lib = L
    return _lib


def _bits(x) -> tuple[np.ndarray, int]:
    """A torch fp16/bf16 tensor (any device) -> (uint16 numpy array, is_bf16)."""
    import torch

    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"oracle expects fp16/bf16, got {x.dtype}")
    arr = x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
    return np.ascontiguousarray(arr), int(x.dtype == torch.bfloat16)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def block_pool_topk(q, k, topk: int, score_scale: float, force_sink_diag: bool = False) -> np.ndarray:
    """Selected key blocks per query block, int64 [B, H, nbq, min(topk, nbk)], ascending."""
    qb, isbf = _bits(q)
    kb, _ = _bits(k)
    B, H, Sq, D = qb.shape
    Sk = kb.shape[2]
    nbq, nbk = -(-Sq // 64), -(-Sk // 64)
    kk = min(int(topk), nbk)
    out = np.zeros((B, H, nbq, kk), dtype=np.int64)
    for b in range(B):
        for h in range(H):
            qh = np.ascontiguousarray(qb[b, h])
            kh = np.ascontiguousarray(kb[b, h])
            o = np.zeros((nbq, kk), dtype=np.int64)
            rc = lib().oracle_block_pool_topk(_ptr(qh), _ptr(kh), Sq, Sk, D, isbf, int(topk),
                                              int(bool(force_sink_diag)), float(score_scale), _ptr(o))
            assert rc == 0
            out[b, h] = o
    return out


def vs_estimate(q, k, vertical_size: int, slash_size: int, logit_scale: float | None = None,
                return_logits: bool = False):
    """(v_idx int32 [B,H,nv] ascending, s_idx int32 [B,H,ns] descending).

    ``vertical_size``/``slash_size`` are clamped as the reference does."""
    qb, isbf = _bits(q)
    kb, _ = _bits(k)
    B, H, S, D = qb.shape
    nv = min(S, max(int(vertical_size), 30))
    ns = min(S, max(int(slash_size), 50))
    if logit_scale is None:
        logit_scale = 1.0 / math.sqrt(D)
    LQ = min(64, S)
    v_idx = np.zeros((B, H, nv), dtype=np.int32)
    s_idx = np.zeros((B, H, ns), dtype=np.int32)
    logits = np.zeros((B, H, LQ, S), dtype=np.float32) if return_logits else None
    for b in range(B):
        for h in range(H):
            qh = np.ascontiguousarray(qb[b, h])
            kh = np.ascontiguousarray(kb[b, h])
            vo = np.zeros(nv, dtype=np.int32)
            so = np.zeros(ns, dtype=np.int32)
            lo = np.zeros((LQ, S), dtype=np.float32) if return_logits else None
            rc = lib().oracle_vs_estimate(_ptr(qh), _ptr(kh), S, D, isbf, nv, ns, float(logit_scale),
                                          _ptr(vo), _ptr(so), _ptr(lo) if lo is not None else None)
            assert rc == 0
            v_idx[b, h] = vo
            s_idx[b, h] = so
            if return_logits:
                logits[b, h] = lo
    if return_logits:
        return v_idx, s_idx, logits
    return v_idx, s_idx


def vs_convert_indexes(seqlens, v_idx: np.ndarray, s_idx: np.ndarray, context_size: int):
    """Legacy (block_count, block_offset, column_count, column_index), int32,
    for v_idx [B,H,nv] ascending and s_idx [B,H,ns] descending."""
    v_idx = np.ascontiguousarray(v_idx, dtype=np.int32)
    s_idx = np.ascontiguousarray(s_idx, dtype=np.int32)
    B, H, nv = v_idx.shape
    ns = s_idx.shape[2]
    R = -(-int(context_size) // 64)
    bc = np.zeros((B, H, R), np.int32)
    bo = np.zeros((B, H, R, ns), np.int32)
    cc = np.zeros((B, H, R), np.int32)
    ci = np.zeros((B, H, R, nv), np.int32)
    for b in range(B):
        for h in range(H):
            v = np.ascontiguousarray(v_idx[b, h])
            s = np.ascontiguousarray(s_idx[b, h])
            o_bc = np.zeros(R, np.int32)
            o_bo = np.zeros((R, ns), np.int32)
            o_cc = np.zeros(R, np.int32)
            o_ci = np.zeros((R, nv), np.int32)
            lib().oracle_vs_convert_indexes(_ptr(v), nv, _ptr(s), ns, int(seqlens[b]), R,
                                            _ptr(o_bc), _ptr(o_bo), _ptr(o_cc), _ptr(o_ci))
            bc[b, h], bo[b, h], cc[b, h], ci[b, h] = o_bc, o_bo, o_cc, o_ci
    return bc, bo, cc, ci


def det_exp(y: float) -> float:
    return float(lib().oracle_det_exp(float(y)))


# ---------------------------------------------------------------------------
# Token-level visible sets (True = visible), one head: [S_q, S_k]
# ---------------------------------------------------------------------------


def causal_mask(S_q: int, S_k: int) -> np.ndarray:
    abs_i = np.arange(S_k - S_q, S_k)[:, None]
    return np.arange(S_k)[None, :] <= abs_i


def stream_mask(S_q: int, S_k: int, n_init: int, n_local: int) -> np.ndarray:
    abs_i = np.arange(S_k - S_q, S_k)[:, None]
    j = np.arange(S_k)[None, :]
    sink = j < n_init
    sliding = (j <= abs_i) & (j > abs_i - n_local)
    return (sink | sliding) & (j <= abs_i)


def block_sparse_mask(block_idx: np.ndarray, S: int) -> np.ndarray:
    """block_idx: [nb, topk] (one head) -> [S, S]; selected blocks AND causal."""
    nb = -(-S // 64)
    blk = np.zeros((nb, nb), dtype=bool)
    for bq in range(block_idx.shape[0]):
        for kb in block_idx[bq]:
            if 0 <= kb < nb:
                blk[bq, kb] = True
    tok = np.repeat(np.repeat(blk, 64, axis=0), 64, axis=1)[:S, :S]
    return tok & causal_mask(S, S)


def vs_mask(v_idx: np.ndarray, s_idx: np.ndarray, S: int) -> np.ndarray:
    """v_idx [nv], s_idx [ns] (one head) -> [S, S]."""
    v = np.ascontiguousarray(v_idx, dtype=np.int32)
    s = np.ascontiguousarray(s_idx, dtype=np.int32)
    nb = -(-S // 64)
    rows = np.zeros((nb, S), dtype=np.uint8)
    for bq in range(nb):
        r = np.zeros(S, dtype=np.uint8)
        lib().oracle_vs_block_row(_ptr(v), len(v), _ptr(s), len(s), S, bq, _ptr(r))
        rows[bq] = r
    tok = np.repeat(rows.astype(bool), 64, axis=0)[:S]
    return tok & causal_mask(S, S)


# ---------------------------------------------------------------------------
# The same visible sets for selected query rows only: [len(rows), S_k].  For
# parity checks at sizes where an [S, S] mask does not fit (64K-128K).
# ---------------------------------------------------------------------------


def stream_rows_mask(rows, S_q: int, S_k: int, n_init: int, n_local: int) -> np.ndarray:
    abs_i = (np.asarray(rows, dtype=np.int64) + (S_k - S_q))[:, None]
    j = np.arange(S_k)[None, :]
    return ((j < n_init) | (j > abs_i - n_local)) & (j <= abs_i)


def block_sparse_rows_mask(block_idx: np.ndarray, S: int, rows) -> np.ndarray:
    """block_idx: [nb, topk] (one head); rows sees the blocks of its query block."""
    rows = np.asarray(rows, dtype=np.int64)
    nb = -(-S // 64)
    out = np.zeros((len(rows), S), dtype=bool)
    for n, r in enumerate(rows):
        for kb in block_idx[r // 64]:
            if 0 <= kb < nb:
                out[n, kb * 64:min(S, kb * 64 + 64)] = True
    return out & (np.arange(S)[None, :] <= rows[:, None])


def vs_rows_mask(v_idx: np.ndarray, s_idx: np.ndarray, S: int, rows) -> np.ndarray:
    """v_idx [nv], s_idx [ns] (one head); the direct-mask row of each row's query block."""
    v = np.ascontiguousarray(v_idx, dtype=np.int32)
    s = np.ascontiguousarray(s_idx, dtype=np.int32)
    rows = np.asarray(rows, dtype=np.int64)
    cache = {}
    out = np.zeros((len(rows), S), dtype=bool)
    for n, r in enumerate(rows):
        bq = int(r // 64)
        if bq not in cache:
            b = np.zeros(S, dtype=np.uint8)
            lib().oracle_vs_block_row(_ptr(v), len(v), _ptr(s), len(s), S, bq, _ptr(b))
            cache[bq] = b.astype(bool)
        out[n] = cache[bq]
    return out & (np.arange(S)[None, :] <= rows[:, None])


def masked_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray,
                     scale: float) -> np.ndarray:
    """fp32 softmax(q k^T * scale, masked) v for one head; fully masked rows -> 0."""
    q = q.astype(np.float32)
    k = k.astype(np.float32)
    v = v.astype(np.float32)
    logits = (q @ k.T) * np.float32(scale)
    logits = np.where(mask, logits, -np.inf)
    mx = logits.max(axis=-1, keepdims=True)
    mx = np.where(np.isfinite(mx), mx, 0.0)
    p = np.exp(logits - mx)
    l = p.sum(axis=-1, keepdims=True)
    p = np.where(l > 0, p / np.where(l > 0, l, 1.0), 0.0)
    return (p @ v).astype(np.float32)
