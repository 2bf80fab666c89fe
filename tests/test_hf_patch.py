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


def tiny_phi3(num_layers=2, heads=4, head_dim=96, seed=0, qk_gain=1.0):
    """Seeded random tiny Phi-3; the same constructor as tests/golden/make_golden.py
    (whose fixtures use qk_gain=4: q/k rows of qkv_proj scaled up so attention
    is peaked enough for the softmax scale to matter)."""
    from transformers import Phi3Config, Phi3ForCausalLM

    torch.manual_seed(seed)
    cfg = Phi3Config(vocab_size=128, hidden_size=heads * head_dim, intermediate_size=256,
                     num_hidden_layers=num_layers, num_attention_heads=heads,
                     num_key_value_heads=heads, max_position_embeddings=4096,
                     pad_token_id=0, attn_implementation="eager")
    model = Phi3ForCausalLM(cfg).eval()
    if qk_gain != 1.0:
        with torch.no_grad():
            for layer in model.model.layers:
                layer.self_attn.qkv_proj.weight[: 2 * heads * head_dim] *= qk_gain
    return model


def _causal_fp32(q, k, v, scale):
    S_q, S_k = q.shape[2], k.shape[2]
    logits = (q.float() @ k.float().transpose(-1, -2)) * scale
    i = torch.arange(S_k - S_q, S_k)[:, None]
    j = torch.arange(S_k)[None, :]
    logits = logits.masked_fill(j > i, float("-inf"))
    return torch.softmax(logits, -1) @ v.float()


class StubOps:
    """Records calls.  Every op computes exact fp32 causal attention; dense
    uses the reference's dense default scale 1/sqrt(D), the sparse ops the
    package's sparse default (1/sqrt(padded D))."""

    def __init__(self):
        self.calls = []

    def _scale(self, d):
        from minference.ops._common import default_softmax_scale

        return default_softmax_scale(d)

    def _write(self, res, out, q, heads):
        res = res.to(torch.float32)
        if heads is not None:  # one call over a head table: write those heads in place
            idx = torch.as_tensor(heads, dtype=torch.long)
            full = out if out is not None else torch.zeros(q.shape, dtype=torch.float32)
            full.index_copy_(1, idx, res[:, idx].to(full.dtype))
            return full
        if out is not None:
            out.copy_(res.to(out.dtype))
            return out
        return res

    def _n(self, q, heads):
        return q.shape[1] if heads is None else len(heads)

    def dense_attention(self, q, k, v, *, scale=None, causal=True, out=None, heads=None):
        self.calls.append(("dense", self._n(q, heads)))
        sc = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
        return self._write(_causal_fp32(q, k, v, sc), out, q, heads)

    def streaming_forward(self, q, k, v, n_init, n_local, out=None, heads=None):
        self.calls.append(("stream_llm", self._n(q, heads), n_init, n_local))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out, q, heads)

    def block_sparse_attention(self, q, k, v, topk, out=None, heads=None):
        self.calls.append(("block_sparse", self._n(q, heads), topk))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out, q, heads)

    def vertical_and_slash(self, q, k, v, vs, ss, out=None, heads=None):
        self.calls.append(("vertical_and_slash", self._n(q, heads), vs, ss))
        return self._write(_causal_fp32(q, k, v, self._scale(q.shape[-1])), out, q, heads)


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
    # every stub computes dense causal attention; the sparse ones at the
    # padded-D scale, so the logits differ from HF's but stay finite
    assert torch.isfinite(out).all() and out.shape == ref.shape
    calls = stub.calls
    assert ("stream_llm", 2, 4, 16) in calls          # heads 0 and 2: one call, head table
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
    kinds = [p[0] for layer in cfg for p in layer.values()]
    # the reference's registered config: 981 dense + 43 stream_llm (128, 896)
    assert kinds.count("dense") == 981 and kinds.count("stream_llm") == 43
    assert {p[1:3] for layer in cfg for p in layer.values() if p[0] == "stream_llm"} == {(128, 896)}
    cfg = load_pattern_config(MODEL2PATH["minference-b200/Phi-3-mini-128k-seeded-mixed"], 32, 32)
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


def _golden_hf():
    import os

    import numpy as np

    return np.load(os.path.join(os.path.dirname(__file__), "golden", "hf_phi3.npz"))


def _phi3_for_golden(g):
    model = tiny_phi3(qk_gain=4.0).to(torch.bfloat16)
    psum = sum(float(p.detach().float().sum()) for p in model.parameters())
    assert abs(psum - float(g["param_sum"])) < 1e-3 * max(1.0, abs(psum)), \
        "seeded tiny Phi-3 weights differ from the ones the fixture was made with"
    return model


def test_hf_golden_fixture_discriminates():
    """The fixture's reference logits separate a 1/sqrt(padded D) dense scale
    (and the sparse patterns) from bf16 rounding, so the GPU test below can
    tell them apart."""
    g = _golden_hf()
    noise = abs(g["dense_logits"] - g["hf_logits"]).mean()
    wrong = abs(g["dense_padded_scale_logits"] - g["dense_logits"]).mean()
    sparse = abs(g["mixed_logits"] - g["dense_logits"]).mean()
    assert noise < HF_MEAN_TOL < wrong and HF_MEAN_TOL < sparse


# mean / max |logit difference| allowed against the reference's own dispatcher
HF_MEAN_TOL = 0.02
HF_MAX_TOL = 0.3


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["dense", "mixed"])
def test_patched_phi3_matches_reference_dispatcher(cuda, tmp_path, mode):
    """Tiny head_dim-96 Phi-3 patched by this package, on the sm_100a kernels,
    against logits of the reference's own CPU dispatcher on the same weights
    (tests/golden/make_golden.py, make_hf_fixture): attn_type "dense" (every
    head at 1/sqrt(96)) and a mixed dense / stream_llm / block_sparse /
    vertical_and_slash config with non-contiguous head groups."""
    from minference import MInference

    g = _golden_hf()
    model = _phi3_for_golden(g).to(cuda)
    ids = torch.from_numpy(g["ids"]).to(cuda)
    if mode == "dense":
        MInference("dense")(model)
    else:
        layers = json.loads(str(g["mixed_config"]))
        MInference("minference", config_path=_write_config(tmp_path, layers))(model)
    with torch.no_grad():
        out = model(ids).logits.float().cpu().numpy()
    ref = g[f"{mode}_logits"]
    diff = abs(out - ref)
    assert diff.mean() < HF_MEAN_TOL and diff.max() < HF_MAX_TOL, (diff.mean(), diff.max())


@pytest.mark.gpu
def test_decode_and_dense_defaults_on_gpu(cuda):
    """backend_npu.dense_attention / decode_dense default to 1/sqrt(D) of the
    unpadded dim (reference backend_npu/attention.py:209-210, :291-292);
    decode sees every cached key; non-causal prefill sees every key."""
    from minference.backend_npu import decode_dense, dense_attention

    torch.manual_seed(3)
    B, H, S, D = 1, 2, 300, 96
    q = (torch.randn(B, H, S, D) / math.sqrt(D)).to(torch.bfloat16)
    k = (torch.randn(B, H, S, D) / math.sqrt(D) * 4).to(torch.bfloat16)
    v = (torch.randn(B, H, S, D) / math.sqrt(D)).to(torch.bfloat16)

    def ref(qq, causal):
        lg = (qq.float() @ k.float().transpose(-1, -2)) / math.sqrt(D)
        if causal:
            sq = qq.shape[2]
            i = torch.arange(S - sq, S)[:, None]
            lg = lg.masked_fill(torch.arange(S)[None, :] > i, float("-inf"))
        return torch.softmax(lg, -1) @ v.float()

    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    out = dense_attention(qd, kd, vd).float().cpu()
    assert (out - ref(q, True)).abs().max() < 2e-3
    out = dense_attention(qd, kd, vd, causal=False).float().cpu()
    assert (out - ref(q, False)).abs().max() < 2e-3
    out = decode_dense(qd[:, :, -1:], kd, vd).float().cpu()
    assert (out - ref(q[:, :, -1:], False)).abs().max() < 2e-3
    q2 = q[:, :, 100:130]   # S_q < S_k, bottom-right aligned causal
    out = dense_attention(q2.to(cuda), kd, vd, scale=0.07).float().cpu()
    lg = (q2.float() @ k.float().transpose(-1, -2)) * 0.07
    i = torch.arange(S - 30, S)[:, None]
    lg = lg.masked_fill(torch.arange(S)[None, :] > i, float("-inf"))
    assert (out - torch.softmax(lg, -1) @ v.float()).abs().max() < 2e-3
