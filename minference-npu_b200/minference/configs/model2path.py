"""Registered per-head pattern configs.

A pattern config is a JSON list with one dict per layer,
``{"<head>": [type, vertical_size, slash_size, score]}`` (the reference's
format, e.g. MInference-NPU benchmarks/prepare_phi3_pathb_configs.py:103-111):
``stream_llm`` stores n_init / n_local in vertical_size / slash_size,
``block_sparse`` stores top-k key blocks in vertical_size.  Reference configs
load unchanged through ``config_path=``.

Registered names:

* ``microsoft/Phi-3-mini-128k-instruct`` resolves to the config the reference
  registers for that model (MInference-NPU minference/configs/model2path.py:
  16-20): 981 dense heads and 43 stream_llm heads (128 sink + 896 window) in
  layers 8-13, carried here as data.
* ``minference-b200/Phi-3-mini-128k-seeded-mixed`` is this package's seeded
  benchmark mix (40 % vertical_and_slash 1000/6096, 40 % block_sparse top-100,
  20 % stream_llm 128/1024; ``make_seeded_config.py``), used by the TTFT
  benchmark.
"""

from __future__ import annotations

import os

BASE_DIR = os.path.dirname(os.path.abspath(__file__))

SEEDED_MIXED_MODEL = "minference-b200/Phi-3-mini-128k-seeded-mixed"

MODEL2PATH = {
    "microsoft/Phi-3-mini-128k-instruct": os.path.join(
        BASE_DIR, "Phi_3_mini_128k_instruct_pathb_stream_llm_aligned_dense_others.json"
    ),
    SEEDED_MIXED_MODEL: os.path.join(BASE_DIR, "Phi_3_mini_128k_instruct_seeded_mixed.json"),
}


def get_support_models():
    return list(MODEL2PATH.keys())


def check_path():
    for name, path in MODEL2PATH.items():
        assert os.path.exists(path), f"{name} config does not exist: {path}"
