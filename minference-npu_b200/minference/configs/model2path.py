"""Registered per-head pattern configs.

A pattern config is a JSON list with one dict per layer,
``{"<head>": [type, vertical_size, slash_size, score]}`` (the reference's
format, e.g. MInference-NPU benchmarks/prepare_phi3_pathb_configs.py:103-111):
``stream_llm`` stores n_init / n_local in vertical_size / slash_size,
``block_sparse`` stores top-k key blocks in vertical_size.  Reference configs
load unchanged through ``config_path=``.
"""

from __future__ import annotations

import os

BASE_DIR = os.path.dirname(os.path.abspath(__file__))

MODEL2PATH = {
    "microsoft/Phi-3-mini-128k-instruct": os.path.join(
        BASE_DIR, "Phi_3_mini_128k_instruct_seeded_mixed.json"
    ),
}


def get_support_models():
    return list(MODEL2PATH.keys())
