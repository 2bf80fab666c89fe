"""Writes the seeded Phi-3-mini pattern config used by the TTFT benchmark.

Per head a pattern drawn from a seed: 40% vertical_and_slash (1000, 6096),
40% block_sparse (top-100 blocks), 20% stream_llm (n_init 128, n_local 1024).

    python -m minference.configs.make_seeded_config
"""

from __future__ import annotations

import json
import os
import random

from .model2path import MODEL2PATH, SEEDED_MIXED_MODEL


def make(num_layers: int = 32, num_heads: int = 32, seed: int = 0) -> list[dict]:
    rng = random.Random(seed)
    layers = []
    for _ in range(num_layers):
        layer = {}
        for h in range(num_heads):
            r = rng.random()
            if r < 0.4:
                layer[str(h)] = ["vertical_and_slash", 1000, 6096, 1.0]
            elif r < 0.8:
                layer[str(h)] = ["block_sparse", 100, 0, 1.0]
            else:
                layer[str(h)] = ["stream_llm", 128, 1024, 1.0]
        layers.append(layer)
    return layers


if __name__ == "__main__":
    path = MODEL2PATH[SEEDED_MIXED_MODEL]
    with open(path, "w") as f:
        json.dump(make(), f)
    print(path)
