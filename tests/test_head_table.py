"""Head tables (``heads=``): one launch over a non-contiguous, unordered set
of heads reads them in place and writes exactly those heads of the output,
bit for bit what the same op computes on a contiguous copy of those heads.
This is what the dispatcher uses instead of index_select / index_copy_."""

from __future__ import annotations

import pytest
import torch

from _util import gen_qkv

pytestmark = pytest.mark.gpu

HEADS = [4, 0, 2]


def _pick(t, heads):
    return t[:, heads].contiguous()


def _check(out_full, ref, heads, H):
    for i, h in enumerate(heads):
        assert torch.equal(out_full[:, h], ref[:, i]), f"head {h}"
    rest = [h for h in range(H) if h not in heads]
    assert (out_full[:, rest] == 7.0).all()


@pytest.mark.parametrize("layout", ["bnsd", "bshd"])
def test_head_table_all_ops(cuda, layout):
    from minference import ops

    H, S = 6, 1000
    q, k, v = gen_qkv(1, H, S, 96, torch.bfloat16, 9, lowrank=2.0, sinks=8, device=cuda)
    if layout == "bshd":  # [B, S, H, D] storage viewed as BNSD, as the dispatcher does
        q, k, v = (x.transpose(1, 2).contiguous().transpose(1, 2) for x in (q, k, v))
    qs, ks, vs = _pick(q, HEADS), _pick(k, HEADS), _pick(v, HEADS)
    sentinel = lambda: torch.full_like(q, 7.0)  # noqa: E731

    o = ops.streaming_forward(q, k, v, 64, 256, out=sentinel(), heads=HEADS)
    _check(o, ops.streaming_forward(qs, ks, vs, 64, 256), HEADS, H)
    o = ops.dense_attention(q, k, v, out=sentinel(), heads=HEADS)
    _check(o, ops.dense_attention(qs, ks, vs), HEADS, H)

    idx = ops.select_block_sparse_topk_indices(q, k, 5, heads=HEADS)
    ref_idx = ops.select_block_sparse_topk_indices(qs, ks, 5)
    assert torch.equal(idx, ref_idx)
    o = ops.block_sparse_attention(q, k, v, 5, out=sentinel(), heads=HEADS)
    _check(o, ops.block_sparse_attention(qs, ks, vs, 5), HEADS, H)

    vi, si = ops.vertical_and_slash_estimate(q, k, 100, 200, heads=HEADS)
    rvi, rsi = ops.vertical_and_slash_estimate(qs, ks, 100, 200)
    assert torch.equal(vi, rvi) and torch.equal(si, rsi)
    o = ops.vertical_and_slash(q, k, v, 100, 200, out=sentinel(), heads=HEADS)
    _check(o, ops.vertical_and_slash(qs, ks, vs, 100, 200), HEADS, H)


def test_head_table_rejects_bad_heads(cuda):
    from minference import ops

    q, k, v = gen_qkv(1, 3, 256, 96, torch.bfloat16, 1, device=cuda)
    with pytest.raises(ValueError):
        ops.dense_attention(q, k, v, heads=[0, 3])
