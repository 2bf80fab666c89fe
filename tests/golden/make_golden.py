"""Generate golden vectors from the reference implementation itself.

Run where the reference checkout exists, with MINFERENCE_REF set to its
MInference-NPU directory:

    MINFERENCE_REF=<path to MInference-NPU> python tests/golden/make_golden.py

It imports the reference's own CPU code paths (the NPU paths are not
importable without torch_npu) and stores seeded inputs together with the
reference outputs as compressed .npz files next to this script.  The tests
(tests/test_oracle_golden.py, tests/test_gpu_parity.py) only read those
files; they never import the reference.

Reference functions exercised (paths relative to the project root):
  ops/block_sparse_kernel_npu.py   _select_block_sparse_topk_indices (:230),
                                   _build_block_sparse_mask (:266),
                                   block_sparse_attention (:609)
  ops/streaming_kernel_npu.py      streaming_forward (:349)
  modules/minference_forward.py    _vertical_and_slash_kernel (:140)
  ops/vertical_slash_kernel_npu.py _build_vs_mask_direct (:255),
                                   _vertical_slash_pytorch_ref (:377)
"""

from __future__ import annotations

import importlib
import importlib.util
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("MINFERENCE_REF", "")


def _load_ref_package():
    if not REF or not os.path.isdir(os.path.join(REF, "minference")):
        raise SystemExit("set MINFERENCE_REF to the reference's MInference-NPU directory")
    pkg_dir = os.path.join(REF, "minference")
    spec = importlib.util.spec_from_file_location(
        "ref_minference", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir]
    )
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_minference"] = mod
    spec.loader.exec_module(mod)

    bs = importlib.import_module("ref_minference.ops.block_sparse_kernel_npu")
    st = importlib.import_module("ref_minference.ops.streaming_kernel_npu")
    vs = importlib.import_module("ref_minference.ops.vertical_slash_kernel_npu")
    fw = importlib.import_module("ref_minference.modules.minference_forward")
    return bs, st, vs, fw


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gen_qkv(B, H, S, D, dtype, seed, lowrank=0.0, sinks=0):
    """Q,K,V ~ N(0,1)/sqrt(D); optional rank-4 bias on K and x4 'sink' rows."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    k = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    v = torch.randn(B, H, S, D, generator=g) / math.sqrt(D)
    if lowrank:
        u = torch.randn(B, H, S, 4, generator=g)
        w = torch.randn(B, H, 4, D, generator=g) / math.sqrt(4 * D)
        k = k + lowrank * (u @ w)
    if sinks:
        for b in range(B):
            for h in range(H):
                pos = torch.randperm(S, generator=g)[:sinks]
                k[b, h, pos] *= 4.0
    return q.to(dtype), k.to(dtype), v.to(dtype)


def pad128(t):
    return F.pad(t, (0, 128 - t.shape[-1])) if t.shape[-1] < 128 else t


def make_convert_fixture() -> None:
    """convert_vertical_slash_indexes (backend_npu/cuda_shim.py:147) golden vectors."""
    _load_ref_package()
    shim = importlib.import_module("ref_minference.backend_npu.cuda_shim")
    g = torch.Generator().manual_seed(51)
    out = {}
    ccases = [(1, 2, 200, 10, 20, 200), (2, 2, 300, 25, 40, 260), (1, 3, 1000, 64, 80, 1000),
              (1, 1, 130, 0, 12, 130), (1, 1, 190, 9, 0, 190)]
    for ci, (B, H, S, nv, ns, seqlen) in enumerate(ccases):
        v_idx = torch.stack([torch.stack([torch.randperm(S, generator=g)[:nv].sort().values
                                          for _ in range(H)]) for _ in range(B)]).to(torch.int32)
        s_idx = torch.stack([torch.stack([torch.randperm(S, generator=g)[:ns].sort(descending=True).values
                                          for _ in range(H)]) for _ in range(B)]).to(torch.int32)
        seqlens = torch.full((B,), seqlen, dtype=torch.int32)
        bc, bo, cc, cix = shim.convert_vertical_slash_indexes(seqlens, v_idx, s_idx, S, 64, 64)
        out[f"c{ci}_meta"] = np.array([B, H, S, nv, ns, seqlen])
        out[f"c{ci}_vidx"], out[f"c{ci}_sidx"] = v_idx.numpy(), s_idx.numpy()
        out[f"c{ci}_bc"], out[f"c{ci}_bo"] = bc.numpy(), bo.numpy()
        out[f"c{ci}_cc"], out[f"c{ci}_ci"] = cc.numpy(), cix.numpy()
    out["n_cases"] = np.array(len(ccases))
    np.savez_compressed(os.path.join(HERE, "vs_convert.npz"), **out)


HF_QK_GAIN = 4.0


def tiny_phi3(seed=0, layers=2, heads=4, head_dim=96, qk_gain=HF_QK_GAIN):
    """Seeded random tiny Phi-3 (same constructor as tests/test_hf_patch.py).

    The q and k rows of every qkv_proj are multiplied by ``qk_gain`` so the
    attention is peaked enough for the softmax scale and the sparse patterns
    to change the logits well beyond bf16 rounding."""
    from transformers import Phi3Config, Phi3ForCausalLM

    torch.manual_seed(seed)
    cfg = Phi3Config(vocab_size=128, hidden_size=heads * head_dim, intermediate_size=256,
                     num_hidden_layers=layers, num_attention_heads=heads,
                     num_key_value_heads=heads, max_position_embeddings=4096,
                     pad_token_id=0, attn_implementation="eager")
    model = Phi3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            layer.self_attn.qkv_proj.weight[: 2 * heads * head_dim] *= qk_gain
    return model


HF_MIXED_LAYERS = [
    {"0": ["stream_llm", 64, 128, 1], "1": ["block_sparse", 4, 0, 1],
     "2": ["stream_llm", 64, 128, 1], "3": ["dense", 0, 0, 1]},
    {"0": ["dense", 0, 0, 1], "1": ["vertical_and_slash", 100, 200, 1],
     "2": ["block_sparse", 4, 0, 1], "3": ["dense", 0, 0, 1]},
]


def make_hf_fixture() -> None:
    """Logits of a tiny head_dim-96 Phi-3 patched by the reference's own
    ``MInference`` (models_patch.py) under attn_type "dense" and under a mixed
    per-head config, computed by its CPU dispatcher in bf16.

    Two shims adapt the reference's forward to the installed transformers
    (the reference pins 4.57): its ``apply_rotary_pos_emb`` call passes
    ``position_ids`` in the slot that is now ``unsqueeze_dim``, and it returns
    a 3-tuple for Phi-3 where the decoder layer now unpacks 2."""
    import json as _json
    import tempfile

    _, _, _, fw = _load_ref_package()
    mp = importlib.import_module("ref_minference.models_patch")
    out = {}
    ids = torch.randint(1, 128, (1, 700), generator=torch.Generator().manual_seed(5))
    out["ids"] = ids.numpy()
    out["mixed_config"] = np.array(_json.dumps(HF_MIXED_LAYERS))
    with tempfile.TemporaryDirectory() as td:
        cfg_path = os.path.join(td, "mixed.json")
        with open(cfg_path, "w") as f:
            _json.dump(HF_MIXED_LAYERS, f)
        for name, kwargs in (("dense", dict(attn_type="dense")),
                             ("mixed", dict(attn_type="minference", config_path=cfg_path))):
            model = tiny_phi3().to(torch.bfloat16)
            out["param_sum"] = np.array(
                sum(float(p.float().sum()) for p in model.parameters()), dtype=np.float64)
            with torch.no_grad():
                out["hf_logits"] = model(ids).logits.float().numpy()
            mp.MInference(**kwargs)(model)
            for mod in model.modules():
                if mod.__class__.__name__ == "Phi3Attention":
                    fwd = mod.forward
                    mod.forward = (lambda *a, _f=fwd, **kw: tuple(_f(*a, **kw)[:2]))
                    mod.init_minference_parameters()
            # init_minference_parameters has just rebound the module-level
            # apply_rotary_pos_emb to transformers' own; wrap that one
            rope = fw.apply_rotary_pos_emb
            fw.apply_rotary_pos_emb = lambda q, k, c, s, pid=None, _r=rope: _r(q, k, c, s)
            with torch.no_grad():
                out[f"{name}_logits"] = model(ids).logits.float().numpy()
            if name == "dense":
                # the same run with dense heads at 1/sqrt(padded D): how far a
                # wrong default scale moves the logits
                dense = fw.dense_attention
                fw.dense_attention = lambda q, k, v, causal=True, _d=dense: _d(
                    q, k, v, causal=causal, scale=1.0 / math.sqrt(128))
                with torch.no_grad():
                    out["dense_padded_scale_logits"] = model(ids).logits.float().numpy()
                fw.dense_attention = dense
    np.savez_compressed(os.path.join(HERE, "hf_phi3.npz"), **out)


def main() -> None:
    bs, st, vs, fw = _load_ref_package()
    torch.set_num_threads(min(8, os.cpu_count() or 1))

    # ---- block_sparse selector ------------------------------------------------
    sel_cases = [
        # (S, D, dtype, topk, seed, lowrank)
        (300, 96, torch.bfloat16, 3, 1, 0.0),
        (1024, 96, torch.float16, 4, 2, 0.0),
        (2048, 96, torch.bfloat16, 8, 3, 2.0),
        (4096, 96, torch.bfloat16, 100, 4, 2.0),
        (640, 64, torch.bfloat16, 64, 5, 0.0),  # topk > nb: future blocks padded
    ]
    out = {}
    for ci, (S, D, dt, topk, seed, lr) in enumerate(sel_cases):
        q, k, _ = gen_qkv(1, 2, S, D, dt, seed, lowrank=lr)
        qp, kp = pad128(q), pad128(k)
        idx = bs._select_block_sparse_topk_indices(qp, kp, topk, 64)
        # reference scores (same expressions as :251-260) for tie analysis
        nb = -(-S // 64)
        padn = nb * 64 - S
        qq = F.pad(qp, (0, 0, 0, padn)) if padn else qp
        kk = F.pad(kp, (0, 0, 0, padn)) if padn else kp
        qpool = qq.reshape(1, 2, nb, 64, qp.shape[-1]).mean(dim=3).float()
        kpool = kk.reshape(1, 2, nb, 64, kp.shape[-1]).mean(dim=3).float()
        scores = torch.matmul(qpool, kpool.transpose(-2, -1)) * (qp.shape[-1] ** -0.5)
        out[f"c{ci}_q"] = bits(q)
        out[f"c{ci}_k"] = bits(k)
        out[f"c{ci}_meta"] = np.array([S, D, int(dt == torch.bfloat16), topk, qp.shape[-1]])
        out[f"c{ci}_idx"] = idx.numpy()
        out[f"c{ci}_scores"] = scores.numpy()
    out["n_cases"] = np.array(len(sel_cases))
    np.savez_compressed(os.path.join(HERE, "block_select.npz"), **out)

    # ---- block_sparse attention (op) + token mask --------------------------------
    att_cases = [
        (256, 96, torch.bfloat16, 2, 11),
        (300, 96, torch.float16, 3, 12),
        (512, 64, torch.bfloat16, 100, 13),  # full topk == dense causal
    ]
    out = {}
    for ci, (S, D, dt, topk, seed) in enumerate(att_cases):
        q, k, v = gen_qkv(1, 2, S, D, dt, seed, lowrank=2.0)
        o = bs.block_sparse_attention(q, k, v, topk)
        mask = bs._build_block_sparse_mask(pad128(q), pad128(k), topk, 64)
        out[f"c{ci}_q"], out[f"c{ci}_k"], out[f"c{ci}_v"] = bits(q), bits(k), bits(v)
        out[f"c{ci}_meta"] = np.array([S, D, int(dt == torch.bfloat16), topk])
        out[f"c{ci}_out"] = bits(o)
        out[f"c{ci}_visible"] = (~mask).numpy()
    out["n_cases"] = np.array(len(att_cases))
    np.savez_compressed(os.path.join(HERE, "block_sparse_attn.npz"), **out)

    # ---- stream_llm -------------------------------------------------------------
    stream_cases = [
        # (n_init, n_local, s_q, s_k, D, dtype, seed)
        (4, 8, 9, 9, 96, torch.float16, 21),
        (0, 16, 32, 64, 96, torch.float16, 22),
        (128, 512, 512, 1024, 96, torch.float16, 23),
        (400, 128, 128, 512, 64, torch.bfloat16, 24),
        (64, 512, 256, 256, 96, torch.bfloat16, 25),  # short circuit: dense causal
        (128, 256, 700, 700, 96, torch.float16, 26),
    ]
    out = {}
    for ci, (ni, nl, sq, sk, D, dt, seed) in enumerate(stream_cases):
        g = torch.Generator().manual_seed(seed)
        q = (torch.randn(1, 2, sq, D, generator=g) / math.sqrt(D)).to(dt)
        k = (torch.randn(1, 2, sk, D, generator=g) / math.sqrt(D)).to(dt)
        v = (torch.randn(1, 2, sk, D, generator=g) / math.sqrt(D)).to(dt)
        o = st.streaming_forward(q, k, v, ni, nl)
        out[f"c{ci}_q"], out[f"c{ci}_k"], out[f"c{ci}_v"] = bits(q), bits(k), bits(v)
        out[f"c{ci}_meta"] = np.array([ni, nl, sq, sk, D, int(dt == torch.bfloat16)])
        out[f"c{ci}_out"] = bits(o)
    out["n_cases"] = np.array(len(stream_cases))
    np.savez_compressed(os.path.join(HERE, "stream.npz"), **out)

    # ---- vertical_and_slash estimation + attention ------------------------------
    captured = {}

    def _capture(q, k, v, v_idx, s_idx):
        captured["v"] = v_idx.clone()
        captured["s"] = s_idx.clone()
        return vs.vertical_slash_sparse_attention(q, k, v, v_idx, s_idx)

    fw._vs_sparse_attention = _capture
    vs_cases = [
        # (S, D, dtype, vsize, ssize, seed, sinks)
        (200, 96, torch.bfloat16, 40, 60, 31, 4),
        (1000, 96, torch.bfloat16, 100, 200, 32, 8),
        (2048, 96, torch.float16, 200, 300, 33, 8),
        (4096, 96, torch.bfloat16, 1000, 1500, 34, 32),
    ]
    out = {}
    for ci, (S, D, dt, nv, ns, seed, sinks) in enumerate(vs_cases):
        q, k, v = gen_qkv(1, 2, S, D, dt, seed, sinks=sinks)
        o = fw._vertical_and_slash_kernel(None, q, k, v, nv, ns)
        v_idx, s_idx = captured["v"], captured["s"]
        # reference estimator intermediates (same expressions as :149-165)
        last_q = min(64, S)
        qk = torch.matmul(q[:, :, -last_q:, :], k.transpose(-2, -1)) / math.sqrt(D)
        lq = torch.arange(last_q)
        lq_mask = (lq[None, None, :, None] >= lq[None, None, None, :])
        qk[:, :, :, -last_q:] = torch.where(lq_mask, qk[:, :, :, -last_q:], float("-inf"))
        logits = qk.float()
        p = torch.softmax(qk, dim=-1, dtype=torch.float32)
        vert = p.sum(-2)
        diag = fw.sum_all_diagonal_matrix(p)
        if last_q > 1:
            diag = diag[..., : -last_q + 1]
        mask = vs._build_vs_mask_direct(v_idx, s_idx, S, S, q.device)
        out[f"c{ci}_q"], out[f"c{ci}_k"], out[f"c{ci}_v"] = bits(q), bits(k), bits(v)
        out[f"c{ci}_meta"] = np.array([S, D, int(dt == torch.bfloat16), nv, ns])
        out[f"c{ci}_vidx"] = v_idx.numpy()
        out[f"c{ci}_sidx"] = s_idx.numpy()
        out[f"c{ci}_logits"] = bits(qk)
        out[f"c{ci}_vert"] = vert.numpy()
        out[f"c{ci}_diag"] = diag.numpy()
        out[f"c{ci}_out"] = bits(o)
        if S <= 2048:  # keeps the fixture small; vs_mask.npz covers the mask rules
            out[f"c{ci}_visible"] = np.packbits((~mask).numpy(), axis=-1)
    out["n_cases"] = np.array(len(vs_cases))
    np.savez_compressed(os.path.join(HERE, "vertical_slash.npz"), **out)

    # ---- VS direct mask on ragged / adversarial index sets ------------------------
    g = torch.Generator().manual_seed(41)
    out = {}
    mcases = [(37, 5, 9), (100, 7, 20), (130, 10, 40), (257, 12, 60), (64, 3, 64), (1000, 30, 300)]
    for ci, (S, nv, ns) in enumerate(mcases):
        v_idx = torch.randperm(S, generator=g)[:nv].sort().values.to(torch.int32)[None, None]
        s_idx = torch.randperm(S, generator=g)[:ns].sort(descending=True).values.to(torch.int32)[None, None]
        mask = vs._build_vs_mask_direct(v_idx, s_idx, S, S, torch.device("cpu"))
        out[f"c{ci}_S"] = np.array(S)
        out[f"c{ci}_vidx"] = v_idx.numpy()
        out[f"c{ci}_sidx"] = s_idx.numpy()
        out[f"c{ci}_visible"] = np.packbits((~mask).numpy(), axis=-1)
    out["n_cases"] = np.array(len(mcases))
    np.savez_compressed(os.path.join(HERE, "vs_mask.npz"), **out)
    make_convert_fixture()
    make_hf_fixture()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if "--only-convert" in sys.argv:
        make_convert_fixture()
    elif "--only-hf" in sys.argv:
        make_hf_fixture()
    else:
        main()
