"""Tiny model configurations of the golden fixtures, shared by the tests.

Rebuilds the seeded weights the fixture generator used (CPU, fp32) and
checks their digest against the fixture, so a drift in the weight generator
fails loudly instead of comparing different models."""

from pathlib import Path

import numpy as np

import oracle as O
from mu_b200.core.config import ModelConfig
from mu_b200.models.weights import random_state_dict, state_dict_digest

G = Path(__file__).resolve().parent / "golden"

SPECS = {
    "llama_tiny": dict(arch="llama", hidden=256, layers=4, heads=4, kv=2, head_dim=64, inter=688,
                       vocab=1024, seed=0, qk_norm=False, experts=4),
    "deep_tiny": dict(arch="deep", hidden=256, layers=2, heads=4, kv=2, head_dim=64, inter=1024,
                      vocab=1024, seed=5, qk_norm=True, experts=4),
}


def model_config(spec) -> ModelConfig:
    return ModelConfig(
        vocab_size=spec["vocab"], hidden_size=spec["hidden"], intermediate_size=spec["inter"],
        num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
        num_key_value_heads=spec["kv"], head_dim=spec["head_dim"], max_position_embeddings=2048,
        rope_theta=10000.0, rms_norm_eps=1e-6, num_experts=spec["experts"],
        use_qk_norm=spec["qk_norm"], tie_word_embeddings=True)


def load_tiny(name):
    spec = SPECS[name]
    cfg = model_config(spec)
    sd = random_state_dict(cfg, spec["arch"], spec["seed"])
    d = np.load(G / f"{name}.npz")
    assert abs(state_dict_digest(sd) - float(d["digest"])) <= 1e-9 * abs(float(d["digest"])), \
        "seeded weights drifted from the fixture"
    lens = d["prompt_lens"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    prompts = [d["prompt_ids"][offs[i]:offs[i + 1]].tolist() for i in range(len(lens))]
    shape = O.ModelShape(arch=spec["arch"], hidden=spec["hidden"], layers=spec["layers"],
                         heads=spec["heads"], kv_heads=spec["kv"], head_dim=spec["head_dim"],
                         vocab=spec["vocab"], experts=spec["experts"] if spec["arch"] == "deep" else 0,
                         qk_norm=spec["qk_norm"])
    return shape, cfg, sd, d, prompts
