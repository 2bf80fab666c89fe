"""GPU parity: sm_100a kernels (through the C ABI) vs the oracle.

Index kernels are compared bit for bit with the C restatement
(oracle/mi_oracle.c); attention outputs are compared with fp32 masked
attention over the oracle's visible sets, within max-abs 2e-3 (the bound the
build targets for fp16/bf16 against an fp32 recompute), and with the
reference's own outputs stored in tests/golden.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _util import assert_topk_equivalent, from_bits, gen_qkv, golden, ref_rows

pytestmark = pytest.mark.gpu

TOL = 2e-3  # max |out - fp32 reference| for fp16/bf16 outputs


def _ops():
    from minference import ops

    return ops


def _oracle():
    from oracle import oracle

    return oracle


def _dense_ref(q, k, v, scale, mask):
    """fp32 reference for one head with an explicit [Sq,Sk] visible mask (torch)."""
    logits = (q.float() @ k.float().T) * scale
    logits = logits.masked_fill(~mask, float("-inf"))
    p = torch.nan_to_num(torch.softmax(logits, dim=-1), nan=0.0)
    return p @ v.float()


# ---------------------------------------------------------------------------
# stream_llm / dense
# ---------------------------------------------------------------------------
STREAM_CASES = [
    # (n_init, n_local, S_q, S_k, D, dtype)
    (4, 8, 9, 9, 96, torch.float16),
    (0, 16, 32, 64, 96, torch.float16),
    (128, 512, 512, 1024, 96, torch.float16),
    (400, 128, 128, 512, 64, torch.bfloat16),
    (128, 256, 700, 700, 96, torch.bfloat16),
    (100, 300, 1000, 1000, 128, torch.bfloat16),
    (0, 64, 200, 200, 80, torch.float16),  # D=80 padded to 96
    (64, 5000, 300, 300, 96, torch.bfloat16),  # short circuit -> dense causal
]


@pytest.mark.parametrize("case", STREAM_CASES, ids=[str(c[:5]) for c in STREAM_CASES])
def test_stream_vs_fp32(cuda, case):
    n_init, n_local, sq, sk, D, dt = case
    ops, O = _ops(), _oracle()
    g = torch.Generator().manual_seed(sq * 7 + sk)
    q = (torch.randn(1, 3, sq, D, generator=g) / math.sqrt(D)).to(dt).to(cuda)
    k = (torch.randn(1, 3, sk, D, generator=g) / math.sqrt(D)).to(dt).to(cuda)
    v = (torch.randn(1, 3, sk, D, generator=g) / math.sqrt(D)).to(dt).to(cuda)
    out = ops.streaming_forward(q, k, v, n_init, n_local)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == dt
    pd = 64 if D <= 64 else 128
    scale = pd ** -0.5
    if sk <= n_local:
        mask = torch.as_tensor(O.causal_mask(sq, sk), device=cuda)
    else:
        mask = torch.as_tensor(O.stream_mask(sq, sk, n_init, n_local), device=cuda)
    for h in range(3):
        ref = _dense_ref(q[0, h], k[0, h], v[0, h], scale, mask)
        err = (out[0, h].float() - ref).abs().max().item()
        assert err < TOL, f"head {h}: max abs err {err}"


def test_stream_golden(cuda):
    z = golden("stream.npz")
    ops = _ops()
    for ci in range(int(z["n_cases"])):
        ni, nl, sq, sk, D, isbf = [int(x) for x in z[f"c{ci}_meta"]]
        q = from_bits(z[f"c{ci}_q"], isbf, cuda)
        k = from_bits(z[f"c{ci}_k"], isbf, cuda)
        v = from_bits(z[f"c{ci}_v"], isbf, cuda)
        ref = from_bits(z[f"c{ci}_out"], isbf).float()
        out = ops.streaming_forward(q, k, v, ni, nl).float().cpu()
        err = (out - ref).abs().max().item()
        assert err < TOL, f"case {ci}: max abs err vs reference output {err}"


def test_dense_causal_matches_sdpa(cuda):
    ops = _ops()
    q, k, v = gen_qkv(1, 4, 2048, 96, torch.bfloat16, 5, device=cuda)
    out = ops.dense_attention(q, k, v, causal=True)  # default scale 1/sqrt(D)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=True, scale=96 ** -0.5
    )
    err = (out.float() - ref).abs().max().item()
    assert err < TOL, err


def test_stream_strided_views(cuda):
    """BSHD storage viewed as BNSD (transpose) goes through TMA strides."""
    ops = _ops()
    S, H, D = 640, 4, 96
    g = torch.Generator().manual_seed(3)
    base = (torch.randn(3, 1, S, H, D, generator=g) / math.sqrt(D)).to(torch.bfloat16).to(cuda)
    q, k, v = (base[i].transpose(1, 2) for i in range(3))
    out = ops.streaming_forward(q, k, v, 64, 256)
    out2 = ops.streaming_forward(q.contiguous(), k.contiguous(), v.contiguous(), 64, 256)
    assert torch.equal(out, out2)


# ---------------------------------------------------------------------------
# block_sparse
# ---------------------------------------------------------------------------
SEL_CASES = [
    # (S, D, dtype, topk, lowrank, force)
    (300, 96, torch.bfloat16, 3, 0.0, False),
    (1024, 96, torch.float16, 4, 0.0, False),
    (4096, 96, torch.bfloat16, 100, 2.0, False),
    (4096, 96, torch.bfloat16, 100, 2.0, True),
    (640, 64, torch.bfloat16, 64, 0.0, False),
    (8192, 128, torch.float16, 17, 2.0, True),
]


@pytest.mark.parametrize("case", SEL_CASES, ids=[str(c) for c in SEL_CASES])
def test_block_select_bit_exact(cuda, case):
    S, D, dt, topk, lr, force = case
    ops, O = _ops(), _oracle()
    q, k, _ = gen_qkv(1, 2, S, D, dt, S + topk, lowrank=lr)
    pd = 64 if D <= 64 else 128
    mine = ops.select_block_sparse_topk_indices(q.to(cuda), k.to(cuda), topk,
                                                force_sink_diag=force).cpu().numpy()
    ref = O.block_pool_topk(q, k, topk, pd ** -0.5, force_sink_diag=force)
    assert np.array_equal(mine, ref)


def test_block_select_golden(cuda):
    z = golden("block_select.npz")
    ops = _ops()
    for ci in range(int(z["n_cases"])):
        S, D, isbf, topk, Dp = [int(x) for x in z[f"c{ci}_meta"]]
        q = from_bits(z[f"c{ci}_q"], isbf, cuda)
        k = from_bits(z[f"c{ci}_k"], isbf, cuda)
        mine = ops.select_block_sparse_topk_indices(q, k, topk).cpu().numpy()
        ref = z[f"c{ci}_idx"]
        sc = z[f"c{ci}_scores"]
        for h in range(mine.shape[1]):
            for bq in range(mine.shape[2]):
                # compare the causal (visible) part of the selections
                a = [x for x in mine[0, h, bq] if x <= bq]
                b = [x for x in ref[0, h, bq] if x <= bq]
                assert_topk_equivalent(a, b, sc[0, h, bq], what=f"case {ci} h {h} bq {bq}")


BS_CASES = [
    # (S, D, dtype, topk)
    (256, 96, torch.bfloat16, 2),
    (300, 96, torch.float16, 3),
    (1000, 96, torch.bfloat16, 5),
    (2048, 64, torch.bfloat16, 7),
    (2048, 128, torch.float16, 1),
]


@pytest.mark.parametrize("case", BS_CASES, ids=[str(c) for c in BS_CASES])
def test_block_sparse_attention_vs_fp32(cuda, case):
    S, D, dt, topk = case
    ops, O = _ops(), _oracle()
    q, k, v = gen_qkv(1, 2, S, D, dt, S + 11, lowrank=2.0)
    pd = 64 if D <= 64 else 128
    idx = O.block_pool_topk(q, k, topk, pd ** -0.5)
    out = ops.block_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), topk)
    for h in range(2):
        mask = torch.as_tensor(O.block_sparse_mask(idx[0, h], S), device=cuda)
        ref = _dense_ref(q[0, h].to(cuda), k[0, h].to(cuda), v[0, h].to(cuda), pd ** -0.5, mask)
        err = (out[0, h].float() - ref).abs().max().item()
        assert err < TOL, f"head {h}: {err}"


def test_block_sparse_golden(cuda):
    z = golden("block_sparse_attn.npz")
    ops = _ops()
    for ci in range(int(z["n_cases"])):
        S, D, isbf, topk = [int(x) for x in z[f"c{ci}_meta"]]
        q = from_bits(z[f"c{ci}_q"], isbf, cuda)
        k = from_bits(z[f"c{ci}_k"], isbf, cuda)
        v = from_bits(z[f"c{ci}_v"], isbf, cuda)
        ref = from_bits(z[f"c{ci}_out"], isbf).float()
        out = ops.block_sparse_attention(q, k, v, topk).float().cpu()
        err = (out - ref).abs().max().item()
        assert err < TOL, f"case {ci}: {err}"


def test_block_sparse_full_topk_is_dense(cuda):
    ops = _ops()
    q, k, v = gen_qkv(1, 2, 1536, 96, torch.bfloat16, 9, device=cuda)
    a = ops.block_sparse_attention(q, k, v, 10_000)
    b = ops.dense_attention(q, k, v, scale=128 ** -0.5)  # block_sparse: padded-D scale
    assert (a.float() - b.float()).abs().max().item() < 1e-6


# ---------------------------------------------------------------------------
# vertical_and_slash
# ---------------------------------------------------------------------------
VS_EST_CASES = [
    # (S, D, dtype, nv, ns, sinks)
    (200, 96, torch.bfloat16, 40, 60, 4),
    (1000, 96, torch.bfloat16, 100, 200, 8),
    (2048, 96, torch.float16, 200, 300, 8),
    (4096, 128, torch.bfloat16, 1000, 1500, 32),
    (50, 64, torch.bfloat16, 30, 50, 2),
    (1001, 64, torch.float16, 100, 150, 4),
]


@pytest.mark.parametrize("case", VS_EST_CASES, ids=[str(c) for c in VS_EST_CASES])
def test_vs_estimate_bit_exact(cuda, case):
    S, D, dt, nv, ns, sinks = case
    ops, O = _ops(), _oracle()
    q, k, _ = gen_qkv(1, 2, S, D, dt, S + 3, sinks=sinks)
    vi, si = ops.vertical_and_slash_estimate(q.to(cuda), k.to(cuda), nv, ns)
    rv, rs = O.vs_estimate(q, k, nv, ns)
    assert np.array_equal(vi.cpu().numpy(), rv)
    assert np.array_equal(si.cpu().numpy(), rs)


def test_vs_estimate_golden(cuda):
    z = golden("vertical_slash.npz")
    ops = _ops()
    for ci in range(int(z["n_cases"])):
        S, D, isbf, nv, ns = [int(x) for x in z[f"c{ci}_meta"]]
        q = from_bits(z[f"c{ci}_q"], isbf, cuda)
        k = from_bits(z[f"c{ci}_k"], isbf, cuda)
        vi, si = ops.vertical_and_slash_estimate(q, k, nv, ns)
        vi, si = vi.cpu().numpy(), si.cpu().numpy()
        for h in range(vi.shape[1]):
            vert = z[f"c{ci}_vert"][0, h].copy()
            vert[:30] = np.inf
            diag = z[f"c{ci}_diag"][0, h].copy()
            diag[-100:] = np.inf
            assert_topk_equivalent(vi[0, h], z[f"c{ci}_vidx"][0, h], vert, rtol=1e-4, what=f"v {ci}")
            assert_topk_equivalent(S - 1 - si[0, h], S - 1 - z[f"c{ci}_sidx"][0, h], diag,
                                   rtol=1e-4, what=f"s {ci}")


VS_ATT_CASES = [
    # (S, D, dtype, nv, ns)
    (200, 96, torch.bfloat16, 40, 60),
    (1000, 96, torch.bfloat16, 100, 200),
    (2048, 96, torch.float16, 64, 80),
    (1500, 128, torch.bfloat16, 300, 100),
    (37, 64, torch.bfloat16, 30, 37),
]


@pytest.mark.parametrize("case", VS_ATT_CASES, ids=[str(c) for c in VS_ATT_CASES])
def test_vs_attention_vs_fp32(cuda, case):
    S, D, dt, nv, ns = case
    ops, O = _ops(), _oracle()
    q, k, v = gen_qkv(1, 2, S, D, dt, S + 5, sinks=8)
    g = torch.Generator().manual_seed(S)
    nv, ns = min(nv, S), min(ns, S)
    vi = torch.stack([torch.randperm(S, generator=g)[:nv].sort().values for _ in range(2)])[None].int()
    si = torch.stack([torch.randperm(S, generator=g)[:ns].sort(descending=True).values for _ in range(2)])[None].int()
    out = ops.vertical_slash_sparse_attention(q.to(cuda), k.to(cuda), v.to(cuda), vi, si)
    pd = 64 if D <= 64 else 128
    for h in range(2):
        mask = torch.as_tensor(O.vs_mask(vi[0, h].numpy(), si[0, h].numpy(), S), device=cuda)
        ref = _dense_ref(q[0, h].to(cuda), k[0, h].to(cuda), v[0, h].to(cuda), pd ** -0.5, mask)
        err = (out[0, h].float() - ref).abs().max().item()
        assert err < TOL, f"head {h}: {err}"


def test_vs_golden_end_to_end(cuda):
    """Reference estimator + attention output vs this build's, on the golden inputs."""
    z = golden("vertical_slash.npz")
    ops = _ops()
    for ci in range(int(z["n_cases"])):
        S, D, isbf, nv, ns = [int(x) for x in z[f"c{ci}_meta"]]
        q = from_bits(z[f"c{ci}_q"], isbf, cuda)
        k = from_bits(z[f"c{ci}_k"], isbf, cuda)
        v = from_bits(z[f"c{ci}_v"], isbf, cuda)
        # attention with the reference's own indices
        out = ops.vertical_slash_sparse_attention(q, k, v, torch.from_numpy(z[f"c{ci}_vidx"]),
                                                  torch.from_numpy(z[f"c{ci}_sidx"]))
        ref = from_bits(z[f"c{ci}_out"], isbf).float()
        err = (out.float().cpu() - ref).abs().max().item()
        assert err < TOL, f"case {ci}: {err}"


def test_device_error_word_clear(cuda):
    from minference import _native

    assert _native.device_error() == 0


# ---------------------------------------------------------------------------
# legacy VS index format
# ---------------------------------------------------------------------------
def test_vs_convert_golden(cuda):
    from minference.backend_npu import convert_vertical_slash_indexes

    z = golden("vs_convert.npz")
    for ci in range(int(z["n_cases"])):
        B, H, S, nv, ns, seqlen = [int(x) for x in z[f"c{ci}_meta"]]
        got = convert_vertical_slash_indexes(
            torch.full((B,), seqlen, dtype=torch.int32), torch.from_numpy(z[f"c{ci}_vidx"]).to(cuda),
            torch.from_numpy(z[f"c{ci}_sidx"]).to(cuda), S, 64, 64)
        for arr, name in zip(got, ("bc", "bo", "cc", "ci")):
            assert np.array_equal(arr.cpu().numpy(), z[f"c{ci}_{name}"]), f"case {ci} {name}"


@pytest.mark.parametrize("S,nv,ns,seqlen", [(4096, 1000, 1500, 4096), (8192, 300, 2000, 7000),
                                            (1000, 64, 0, 1000), (3000, 0, 200, 3000)])
def test_vs_convert_bit_exact(cuda, S, nv, ns, seqlen):
    from minference.ops import convert_vertical_slash_indexes

    O = _oracle()
    g = torch.Generator().manual_seed(S + nv)
    v = torch.stack([torch.randperm(S, generator=g)[:nv].sort().values for _ in range(3)])[None].int()
    s = torch.stack([torch.randperm(S, generator=g)[:ns].sort(descending=True).values
                     for _ in range(3)])[None].int()
    got = convert_vertical_slash_indexes(torch.tensor([seqlen]), v.to(cuda), s.to(cuda), S)
    ref = O.vs_convert_indexes([seqlen], v.numpy(), s.numpy(), S)
    for a, r in zip(got, ref):
        assert np.array_equal(a.cpu().numpy(), r)


def test_bounded_wait_gives_up_and_reports(cuda):
    """A wait that can never complete gives up after its poll limit, records
    its code in the device error word and returns; the context stays usable
    (the next kernels run and the error word reads clean afterwards)."""
    import ctypes

    from minference import _native

    lib = _native.lib()
    lib.mi_selftest_wait_timeout.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p]
    lib.mi_selftest_wait_timeout.restype = ctypes.c_int
    assert _native.device_error() == 0
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = lib.mi_selftest_wait_timeout(1000, flag.data_ptr(),
                                      torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(flag.item()) == 1
    assert _native.device_error() == 120
    assert _native.device_error() == 0  # read-and-clear
    q, k, v = gen_qkv(1, 1, 256, 96, torch.bfloat16, 1, device=cuda)
    out = _ops().streaming_forward(q, k, v, 16, 64)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and _native.device_error() == 0
