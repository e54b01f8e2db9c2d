"""Seeded MoE test cases shared by the GPU parity tests, the golden-fixture
generator and smoke(): every input is regenerated from (seed, stream) pairs by
the oracle's splitmix64/Box-Muller generator, so the same case is bit-identical
here, on the GPU box and in the committed fixtures."""
from __future__ import annotations

import numpy as np

import oracle as o

# name -> (T, H, E, I, K, seed, variant)
CASES = {
    "small": (40, 256, 32, 128, 4, 5, "normal"),
    "ragged": (33, 256, 32, 192, 4, 6, "normal"),
    "one": (1, 256, 32, 128, 4, 7, "normal"),
    "ties": (40, 256, 32, 128, 4, 8, "ties"),
    "hot_expert": (96, 256, 32, 128, 4, 9, "hot"),
    "zipf": (512, 256, 32, 128, 4, 10, "zipf"),
    "tiny_probs": (40, 256, 32, 128, 4, 11, "tiny"),
    "config1": (64, 2048, 32, 1792, 4, 1, "normal"),
}


def build_case(name: str):
    T, H, E, I, K, seed, variant = CASES[name]
    inp = o.moe_inputs(T, H, E, I, seed)
    x, gate = inp["x"], inp["gate"]
    if variant == "ties":
        # experts come in identical pairs (2j, 2j+1): every logit ties with its
        # partner, and the bias is shared, so the lower id must win each tie
        gate[1::2] = gate[0::2]
        inp["bias"][1::2] = inp["bias"][0::2]
    elif variant == "hot":
        # expert 5 is everyone's first choice: its logit dominates
        L = np.full((T, E), -2.0, dtype=np.float32) + o.randn((T, E), seed, 50, 0.5)
        L[:, 5] = 8.0
        o.inject_logits(x, gate, L)
    elif variant == "zipf":
        o.inject_logits(x, gate, o.zipf_logits(T, E, seed))
        inp["bias"][:] = 0.0
    elif variant == "tiny":
        # every probability underflows to 0: sum <= 1e-6 path (scale = 1)
        L = np.full((T, E), -200.0, dtype=np.float32)
        o.inject_logits(x, gate, L)
    inp["K"] = K
    return inp


def expected(inp, tile=128):
    return o.moe_forward(inp["x"], inp["gate"], inp["bias"], inp["w1"], inp["w2"], inp["w3"],
                         K=inp["K"], tile=tile)
