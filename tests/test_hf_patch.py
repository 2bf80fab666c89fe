"""HF drop-in layer: MInference(...)(model), patch_hf, pattern config, grouping.

CPU tests swap the dispatcher's op table for a recording stub (fp32 torch
attention, test-only) so the host logic -- QKV split, RoPE, grouping,
in-place writes, o_proj -- is checked against HF's own attention without a
GPU.  The GPU test runs the real sm_100a ops on a tiny random Phi-3.
"""

from __future__ import annotations

import json
import math
import types

import pytest
import torch


def tiny_phi3(num_layers=2, heads=4, head_dim=64, seed=0):
    from transformers import Phi3Config, Phi3ForCausalLM

    torch.manual_seed(seed)
    cfg = Phi3Config(vocab_size=128, hidden_size=heads * head_dim, intermediate_size=256,
                     num_hidden_layers=num_layers, num_attention_heads=heads,
                     num_key_value_heads=heads, max_position_embeddings=4096,
                     pad_token_id=0, attn_implementation="eager")
    return Phi3ForCausalLM(cfg).eval()


def _causal_fp32(q, k, v, scale):
    S_q, S_k = q.shape[2], k.shape[2]
    logits = (q.float() @ k.float().transpose(-1, -2)) * scale
    i = torch.arange(S_k - S_q, S_k)[:, None]
    j = torch.arange(S_k)[None, :]
    logits = logits.masked_fill(j > i, float("-inf"))
    return torch.softmax(logits, -1) @ v.float()


class StubOps:
    """Records calls; dense is exact fp32 causal attention with the reference scale."""

    def __init__(self):
        self.calls = []

    def _scale(self, d):
        from minference.ops._common import default_softmax_scale

        return default_softmax_scale(d)

    def _write(self, res, out):
        res = res.to(torch.float32)
        if out is not None:
            out.copy_(res.to(out.dtype))
            return out
        return res

    def dense_attention(self, q, k, v, causal=True, out=None):
        self.calls.append(("dense", q.shape[1]))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out)

    def streaming_forward(self, q, k, v, n_init, n_local, out=None):
        self.calls.append(("stream_llm", q.shape[1], n_init, n_local))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out)

    def block_sparse_attention(self, q, k, v, topk, out=None):
        self.calls.append(("block_sparse", q.shape[1], topk))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out)

    def vertical_and_slash(self, q, k, v, vs, ss, out=None):
        self.calls.append(("vertical_and_slash", q.shape[1], vs, ss))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out)


@pytest.fixture
def stub(monkeypatch):
    from minference.modules import minference_forward as mf

    s = StubOps()
    monkeypatch.setattr(mf, "OPS", s)
    return s


def _write_config(tmp_path, layers):
    p = tmp_path / "pattern.json"
    p.write_text(json.dumps(layers))
    return str(p)


def test_patched_dense_matches_hf_attention(stub, tmp_path):
    from minference import MInference

    model = tiny_phi3()
    ids = torch.randint(1, 128, (1, 50))
    with torch.no_grad():
        ref = model(ids).logits
    patched = MInference("dense")(model)
    with torch.no_grad():
        out = patched(ids).logits
    assert torch.allclose(out, ref, atol=1e-4, rtol=1e-4)
    assert all(c[0] == "dense" for c in stub.calls)


def test_grouping_follows_pattern_config(stub, tmp_path):
    from minference import MInference

    layers = [
        {"0": ["stream_llm", 4, 16, 1], "1": ["block_sparse", 3, 0, 1],
         "2": ["stream_llm", 4, 16, 1], "3": ["dense", 0, 0, 1]},
        {"1": ["vertical_and_slash", 40, 60, 1]},  # unlisted heads -> default VS (1000, 6096)
    ]
    model = tiny_phi3()
    ids = torch.randint(1, 128, (1, 40))
    with torch.no_grad():
        ref = model(ids).logits
    MInference("minference", config_path=_write_config(tmp_path, layers))(model)
    with torch.no_grad():
        out = model(ids).logits
    # every stub computes dense causal attention, so the logits must match HF
    assert torch.allclose(out, ref, atol=1e-4, rtol=1e-4)
    calls = stub.calls
    assert ("stream_llm", 2, 4, 16) in calls          # heads 0 and 2 batched (gathered)
    assert ("block_sparse", 1, 3) in calls
    assert ("dense", 1) in calls
    assert ("vertical_and_slash", 1, 40, 60) in calls
    assert ("vertical_and_slash", 3, 1000, 6096) in calls  # heads 0, 2, 3 default


def test_starting_layer_runs_dense(stub, tmp_path):
    from minference import MInference

    layers = [{"0": ["stream_llm", 4, 16, 1]}, {"0": ["stream_llm", 4, 16, 1]}]
    model = tiny_phi3()
    MInference("minference", config_path=_write_config(tmp_path, layers), starting_layer=1)(model)
    with torch.no_grad():
        model(torch.randint(1, 128, (1, 24)))
    kinds = [c[0] for c in stub.calls]
    assert kinds[0] == "dense"            # layer 0 < starting_layer: whole layer dense
    assert "stream_llm" in kinds[1:]


def test_hf_attn_type_leaves_model_untouched():
    from minference import MInference

    model = tiny_phi3()
    fwd = model.model.layers[0].self_attn.forward
    assert MInference("hf")(model) is model
    assert model.model.layers[0].self_attn.forward == fwd


def test_patch_hf_entry(stub):
    from minference import patch_hf

    model = tiny_phi3()
    patch_hf(model, "dense")
    with torch.no_grad():
        model(torch.randint(1, 128, (1, 10)))
    assert stub.calls and stub.calls[0][0] == "dense"
    with pytest.raises(NotImplementedError):
        patch_hf(tiny_phi3(), "hf")


def test_registered_model_config_loads():
    from minference.configs.model2path import MODEL2PATH
    from minference.modules.minference_forward import load_pattern_config

    cfg = load_pattern_config(MODEL2PATH["microsoft/Phi-3-mini-128k-instruct"], 32, 32)
    assert len(cfg) == 32 and all(len(layer) == 32 for layer in cfg)
    kinds = {p[0] for layer in cfg for p in layer.values()}
    assert kinds == {"vertical_and_slash", "block_sparse", "stream_llm"}


@pytest.mark.parametrize("bad", [
    {"x": ["dense", 0, 0]},
    {"0": ["triangle", 1, 1, 1]},
    {"0": ["vertical_and_slash", 0, 10, 1]},
    {"0": ["block_sparse", 0, 0, 1]},
    {"9": ["dense", 0, 0, 1]},
    {"0": "dense"},
])
def test_pattern_config_validation(bad):
    from minference.modules.minference_forward import load_pattern_config

    with pytest.raises(ValueError):
        load_pattern_config([bad], num_layers=1, num_heads=4)


def test_invalid_attn_type():
    from minference import MInference

    with pytest.raises(ValueError):
        MInference("triton")
    with pytest.raises(AssertionError):
        MInference("minference", model_name="unknown/model")


@pytest.mark.gpu
def test_patched_phi3_on_gpu(cuda, tmp_path):
    """Real kernels: all-dense patch vs HF sdpa; a mixed config runs and stays finite."""
    from minference import MInference

    model = tiny_phi3(num_layers=2, heads=4, head_dim=96).to(cuda, torch.bfloat16)
    ids = torch.randint(1, 128, (1, 700), device=cuda)
    model.config._attn_implementation = "sdpa"
    with torch.no_grad():
        ref = model(ids).logits.float()
    # HF scales by 1/sqrt(96); the reference's dense path after padding uses
    # 1/sqrt(128).  MINFERENCE_TRUE_SCALE selects 1/sqrt(D) for this comparison.
    import os

    os.environ["MINFERENCE_TRUE_SCALE"] = "1"
    try:
        MInference("dense")(model)
        with torch.no_grad():
            out = model(ids).logits.float()
    finally:
        del os.environ["MINFERENCE_TRUE_SCALE"]
    assert (out - ref).abs().max().item() < 0.1
    layers = [{"0": ["stream_llm", 64, 128, 1], "1": ["block_sparse", 3, 0, 1],
               "2": ["vertical_and_slash", 100, 200, 1], "3": ["dense", 0, 0, 1]}] * 2
    model2 = tiny_phi3(num_layers=2, heads=4, head_dim=96).to(cuda, torch.bfloat16)
    MInference("minference", config_path=_write_config(tmp_path, layers))(model2)
    with torch.no_grad():
        out2 = model2(ids).logits
    assert torch.isfinite(out2).all()
