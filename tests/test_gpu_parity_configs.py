"""GPU parity at the benchmark configurations and at 64K / 128K context.

Each case runs a few heads of a BASELINE configuration (or of the 64K / 128K
sizes the benchmark sweeps) through the public ops:

* index kernels (block selector, VS estimator) are compared whole and bit for
  bit with the C oracle (oracle/mi_oracle.c);
* attention outputs are compared with an fp32 recompute over the oracle's
  visible sets: whole heads where an [S, S] mask fits (config 0), else on
  sampled query rows (first, last and ragged tiles plus seeded random rows),
  within the same max-abs 2e-3 as the other parity tests.

These sizes reach code the small cases do not: the two-pass VS row
statistics above 65,536 keys, the 8-CTA cluster top-k over 32K-128K keys,
plans with ~100 entries per query half and triangular plan offsets at
T = 1024 tiles.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _util import gen_qkv, ref_rows

pytestmark = pytest.mark.gpu

TOL = 2e-3
SCALE = 128 ** -0.5  # sparse ops at D=96: 1/sqrt(padded D), as the reference


def _ops():
    from minference import ops

    return ops


def _oracle():
    from oracle import oracle

    return oracle


def _rows(S: int, n: int, seed: int) -> list[int]:
    g = np.random.default_rng(seed)
    fixed = [0, 1, 63, 64, 127, 128, S // 2, S - 129, S - 128, S - 65, S - 64, S - 2, S - 1]
    rnd = g.choice(S, size=n, replace=False).tolist()
    return sorted({r for r in fixed + rnd if 0 <= r < S})


def _check_rows(out, q, k, v, rows, vis_fn, what):
    r = torch.tensor(rows, device=q.device)
    ref = ref_rows(q, k, v, r, vis_fn, SCALE)
    err = (out[r].float() - ref).abs().max().item()
    assert err < TOL, f"{what}: max abs err {err} on sampled rows"


def test_config0_stream_4k_fp16_full(cuda):
    """S=4096 fp16, n_init 128, n_local 1024; whole heads."""
    ops, O = _ops(), _oracle()
    S, H = 4096, 4
    q, k, v = gen_qkv(1, H, S, 96, torch.float16, 100, device=cuda)
    out = ops.streaming_forward(q, k, v, 128, 1024)
    mask = torch.as_tensor(O.stream_mask(S, S, 128, 1024), device=cuda)
    for h in range(H):
        logits = (q[0, h].float() @ k[0, h].float().T) * SCALE
        ref = torch.softmax(logits.masked_fill(~mask, float("-inf")), -1) @ v[0, h].float()
        err = (out[0, h].float() - ref).abs().max().item()
        assert err < TOL, f"head {h}: {err}"


@pytest.mark.parametrize("S", [16384, 65536, 131072])
def test_block_sparse_selector_and_attention_large(cuda, S):
    """BASELINE config 1 (S=16384 bf16, rank-4 K bias x2, top-100 with block 0
    and the diagonal forced) and the same pattern at 64K / 128K: selector bit
    exact against the C oracle, attention on sampled rows."""
    ops, O = _ops(), _oracle()
    H = 2
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, S + 1, lowrank=2.0)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    idx = ops.select_block_sparse_topk_indices(qd, kd, 100, force_sink_diag=True)
    ref_idx = O.block_pool_topk(q, k, 100, SCALE, force_sink_diag=True)
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    out = ops.block_sparse_attention_from_indices(qd, kd, vd, idx)
    rows = _rows(S, 200, S)
    for h in range(H):
        _check_rows(out[0, h], qd[0, h], kd[0, h], vd[0, h], rows,
                    lambda r, h=h: O.block_sparse_rows_mask(ref_idx[0, h], S, r.cpu().numpy()),
                    f"block_sparse S={S} head {h}")


@pytest.mark.parametrize("S", [32768, 65536, 131072])
def test_vertical_slash_estimate_and_attention_large(cuda, S):
    """BASELINE config 2 (S=32768 bf16, 32 x4 sink keys, v=1000, s=6096) and
    the same pattern at 64K / 128K: estimator bit exact against the C oracle,
    attention with those indices on sampled rows."""
    ops, O = _ops(), _oracle()
    H = 2
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, S + 2, sinks=32)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    vi, si = ops.vertical_and_slash_estimate(qd, kd, 1000, 6096)
    rv, rs = O.vs_estimate(q, k, 1000, 6096)
    assert np.array_equal(vi.cpu().numpy(), rv)
    assert np.array_equal(si.cpu().numpy(), rs)
    out = ops.vertical_slash_sparse_attention(qd, kd, vd, vi, si)
    rows = _rows(S, 200, S + 7)
    for h in range(H):
        _check_rows(out[0, h], qd[0, h], kd[0, h], vd[0, h], rows,
                    lambda r, h=h: O.vs_rows_mask(rv[0, h], rs[0, h], S, r.cpu().numpy()),
                    f"vertical_slash S={S} head {h}")


@pytest.mark.parametrize("S", [65536, 131072])
def test_stream_large(cuda, S):
    ops, O = _ops(), _oracle()
    H = 2
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, S + 3, device=cuda)
    out = ops.streaming_forward(q, k, v, 128, 1024)
    rows = _rows(S, 200, S + 9)
    for h in range(H):
        _check_rows(out[0, h], q[0, h], k[0, h], v[0, h], rows,
                    lambda r: O.stream_rows_mask(r.cpu().numpy(), S, S, 128, 1024),
                    f"stream S={S} head {h}")


def test_dense_128k_sampled(cuda):
    """Dense causal (default scale 1/sqrt(96)) at 128K on sampled rows."""
    ops = _ops()
    S = 131072
    q, k, v = gen_qkv(1, 1, S, 96, torch.bfloat16, 5, device=cuda)
    out = ops.dense_attention(q, k, v)
    rows = torch.tensor(_rows(S, 100, 3), device=cuda)
    ref = ref_rows(q[0, 0], k[0, 0], v[0, 0], rows,
                   lambda r: (torch.arange(S, device=cuda)[None, :] <= r[:, None]).cpu().numpy(),
                   1 / math.sqrt(96))
    err = (out[0, 0][rows].float() - ref).abs().max().item()
    assert err < TOL, err


@pytest.mark.parametrize("S,nv,ns", [(8192, 1000, 1024), (8192, 64, 300), (3000, 1024, 100),
                                     (8192, 1500, 512)])
def test_vs_local_slashes_scattered_verticals(cuda, S, nv, ns):
    """Structured VS sets as real configs have them: local slashes (the ns
    nearest diagonals) plus scattered vertical columns that mostly fall
    outside the slash band (they are gathered row by row; nv > 1024 keeps
    them in block masks).  Whole heads against the fp32 masked attention."""
    ops, O = _ops(), _oracle()
    H = 2
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, S + nv, sinks=16, device=cuda)
    g = torch.Generator().manual_seed(nv)
    vi = torch.stack([torch.cat([torch.arange(30), 30 + torch.randperm(S - 30, generator=g)[:nv - 30]])
                      .sort().values for _ in range(H)])[None].int()
    si = torch.stack([torch.arange(ns - 1, -1, -1) for _ in range(H)])[None].int()
    out = ops.vertical_slash_sparse_attention(q, k, v, vi, si)
    for h in range(H):
        mask = torch.as_tensor(O.vs_mask(vi[0, h].numpy(), si[0, h].numpy(), S), device=cuda)
        logits = (q[0, h].float() @ k[0, h].float().T) * SCALE
        ref = torch.softmax(logits.masked_fill(~mask, float("-inf")), -1) @ v[0, h].float()
        err = (out[0, h].float() - ref).abs().max().item()
        assert err < TOL, f"head {h}: {err}"


@pytest.mark.parametrize("S,D,dt", [(65536, 96, torch.float16), (32768, 128, torch.bfloat16),
                                    (32768, 64, torch.float16)])
def test_other_dtypes_and_head_dims_large(cuda, S, D, dt):
    """fp16 and head dims 64 / 128 at long context: both index kernels bit exact
    against the C oracle, block_sparse and stream_llm attention on sampled rows."""
    ops, O = _ops(), _oracle()
    pd = 64 if D <= 64 else 128
    q, k, v = gen_qkv(1, 1, S, D, dt, S + D, lowrank=2.0, sinks=16)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    vi, si = ops.vertical_and_slash_estimate(qd, kd, 1000, 6096)
    rv, rs = O.vs_estimate(q, k, 1000, 6096)
    assert np.array_equal(vi.cpu().numpy(), rv) and np.array_equal(si.cpu().numpy(), rs)
    idx = ops.select_block_sparse_topk_indices(qd, kd, 64)
    ref_idx = O.block_pool_topk(q, k, 64, pd ** -0.5)
    assert np.array_equal(idx.cpu().numpy(), ref_idx)
    rows = torch.tensor(_rows(S, 100, D), device=cuda)
    out = ops.block_sparse_attention_from_indices(qd, kd, vd, idx)
    ref = ref_rows(qd[0, 0], kd[0, 0], vd[0, 0], rows,
                   lambda r: O.block_sparse_rows_mask(ref_idx[0, 0], S, r.cpu().numpy()), pd ** -0.5)
    assert (out[0, 0][rows].float() - ref).abs().max().item() < TOL
    out = ops.streaming_forward(qd, kd, vd, 128, 1024)
    ref = ref_rows(qd[0, 0], kd[0, 0], vd[0, 0], rows,
                   lambda r: O.stream_rows_mask(r.cpu().numpy(), S, S, 128, 1024), pd ** -0.5)
    assert (out[0, 0][rows].float() - ref).abs().max().item() < TOL
