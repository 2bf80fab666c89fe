"""CPU: the oracle pinned against the reference's own outputs (tests/golden).

The golden vectors were produced by running the reference's CPU code paths
(tests/golden/make_golden.py).  Index selections must match exactly except
where the reference's torch.topk picks among tied scores (its order among
ties is unspecified); masks must match exactly; fp32 attention over the
oracle's masks must match the reference outputs to output precision.
"""

from __future__ import annotations

import numpy as np
import pytest

from _util import assert_topk_equivalent, from_bits, golden


def _oracle():
    from oracle import oracle

    return oracle


def test_block_select_matches_reference():
    O = _oracle()
    z = golden("block_select.npz")
    for ci in range(int(z["n_cases"])):
        S, D, isbf, topk, Dp = [int(x) for x in z[f"c{ci}_meta"]]
        q, k = from_bits(z[f"c{ci}_q"], isbf), from_bits(z[f"c{ci}_k"], isbf)
        mine = O.block_pool_topk(q, k, topk, Dp ** -0.5)
        ref = z[f"c{ci}_idx"]
        assert mine.shape == ref.shape
        for h in range(ref.shape[1]):
            for bq in range(ref.shape[2]):
                a = [x for x in mine[0, h, bq] if x <= bq]
                b = [x for x in ref[0, h, bq] if x <= bq]
                assert_topk_equivalent(a, b, z[f"c{ci}_scores"][0, h, bq], what=f"case {ci}")


def test_block_sparse_mask_matches_reference():
    O = _oracle()
    z = golden("block_sparse_attn.npz")
    for ci in range(int(z["n_cases"])):
        S, D, isbf, topk = [int(x) for x in z[f"c{ci}_meta"]]
        q, k = from_bits(z[f"c{ci}_q"], isbf), from_bits(z[f"c{ci}_k"], isbf)
        Dp = 64 if D <= 64 else 128
        idx = O.block_pool_topk(q, k, topk, Dp ** -0.5)
        vis = z[f"c{ci}_visible"]
        for h in range(vis.shape[1]):
            assert np.array_equal(O.block_sparse_mask(idx[0, h], S), vis[0, h])


def test_block_sparse_attention_matches_reference():
    O = _oracle()
    z = golden("block_sparse_attn.npz")
    for ci in range(int(z["n_cases"])):
        S, D, isbf, topk = [int(x) for x in z[f"c{ci}_meta"]]
        q, k, v = (from_bits(z[f"c{ci}_{n}"], isbf) for n in "qkv")
        Dp = 64 if D <= 64 else 128
        idx = O.block_pool_topk(q, k, topk, Dp ** -0.5)
        ref = from_bits(z[f"c{ci}_out"], isbf).float().numpy()
        for h in range(q.shape[1]):
            mask = O.block_sparse_mask(idx[0, h], S)
            o = O.masked_attention(q[0, h].float().numpy(), k[0, h].float().numpy(),
                                   v[0, h].float().numpy(), mask, Dp ** -0.5)
            assert np.abs(o - ref[0, h]).max() < 2e-3


def test_stream_matches_reference():
    O = _oracle()
    z = golden("stream.npz")
    for ci in range(int(z["n_cases"])):
        ni, nl, sq, sk, D, isbf = [int(x) for x in z[f"c{ci}_meta"]]
        q, k, v = (from_bits(z[f"c{ci}_{n}"], isbf) for n in "qkv")
        ref = from_bits(z[f"c{ci}_out"], isbf).float().numpy()
        Dp = 64 if D <= 64 else 128
        mask = O.causal_mask(sq, sk) if sk <= nl else O.stream_mask(sq, sk, ni, nl)
        for h in range(q.shape[1]):
            o = O.masked_attention(q[0, h].float().numpy(), k[0, h].float().numpy(),
                                   v[0, h].float().numpy(), mask, Dp ** -0.5)
            assert np.abs(o - ref[0, h]).max() < 2e-3, f"case {ci}"


def test_vs_estimate_matches_reference():
    O = _oracle()
    z = golden("vertical_slash.npz")
    for ci in range(int(z["n_cases"])):
        S, D, isbf, nv, ns = [int(x) for x in z[f"c{ci}_meta"]]
        q, k = from_bits(z[f"c{ci}_q"], isbf), from_bits(z[f"c{ci}_k"], isbf)
        vi, si, logits = O.vs_estimate(q, k, nv, ns, return_logits=True)
        # logits: the reference's bf16 matmul differs only in rare last-bit roundings
        ref_logits = from_bits(z[f"c{ci}_logits"], isbf).float().numpy()
        same = (logits == ref_logits) | (np.isinf(logits) & np.isinf(ref_logits))
        assert same.mean() > 0.999
        for h in range(vi.shape[1]):
            vert = z[f"c{ci}_vert"][0, h].copy()
            vert[:30] = np.inf
            diag = z[f"c{ci}_diag"][0, h].copy()
            diag[-100:] = np.inf
            assert_topk_equivalent(vi[0, h], z[f"c{ci}_vidx"][0, h], vert, rtol=1e-4, what="v")
            assert_topk_equivalent(S - 1 - si[0, h], S - 1 - z[f"c{ci}_sidx"][0, h], diag,
                                   rtol=1e-4, what="s")


def test_vs_mask_matches_reference():
    O = _oracle()
    for name in ("vs_mask.npz", "vertical_slash.npz"):
        z = golden(name)
        for ci in range(int(z["n_cases"])):
            if f"c{ci}_visible" not in z.files:
                continue
            S = int(z[f"c{ci}_S"]) if f"c{ci}_S" in z.files else int(z[f"c{ci}_meta"][0])
            vis = np.unpackbits(z[f"c{ci}_visible"], axis=-1)[..., :S].astype(bool)
            for h in range(vis.shape[1]):
                m = O.vs_mask(z[f"c{ci}_vidx"][0, h], z[f"c{ci}_sidx"][0, h], S)
                assert np.array_equal(m, vis[0, h]), f"{name} case {ci} head {h}"


def test_vs_attention_matches_reference():
    O = _oracle()
    z = golden("vertical_slash.npz")
    for ci in range(int(z["n_cases"])):
        S, D, isbf, nv, ns = [int(x) for x in z[f"c{ci}_meta"]]
        if S > 2048:
            continue
        q, k, v = (from_bits(z[f"c{ci}_{n}"], isbf) for n in "qkv")
        ref = from_bits(z[f"c{ci}_out"], isbf).float().numpy()
        for h in range(q.shape[1]):
            mask = O.vs_mask(z[f"c{ci}_vidx"][0, h], z[f"c{ci}_sidx"][0, h], S)
            o = O.masked_attention(q[0, h].float().numpy(), k[0, h].float().numpy(),
                                   v[0, h].float().numpy(), mask, 128 ** -0.5)
            assert np.abs(o - ref[0, h]).max() < 2e-3


@pytest.mark.parametrize("y", [0.0, -1e-8, -0.5, -1.0, -3.3, -10.0, -50.0, -86.9, -87.5, -1e30])
def test_det_exp_accuracy(y):
    import math

    O = _oracle()
    got = O.det_exp(y)
    want = math.exp(y) if y >= -87.0 else 0.0
    assert got == pytest.approx(want, rel=4e-7, abs=1e-37)


def test_vs_convert_indexes_matches_reference():
    O = _oracle()
    z = golden("vs_convert.npz")
    for ci in range(int(z["n_cases"])):
        B, H, S, nv, ns, seqlen = [int(x) for x in z[f"c{ci}_meta"]]
        got = O.vs_convert_indexes([seqlen] * B, z[f"c{ci}_vidx"], z[f"c{ci}_sidx"], S)
        for arr, name in zip(got, ("bc", "bo", "cc", "ci")):
            assert np.array_equal(arr, z[f"c{ci}_{name}"]), f"case {ci} {name}"
