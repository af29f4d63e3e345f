"""Tiny model configurations of the golden fixtures, shared by the tests.

Rebuilds the seeded weights the fixture generator used (CPU, fp32) and
checks their digest against the fixture, so a drift in the weight generator
fails loudly instead of comparing different models."""

from pathlib import Path

import numpy as np
import torch

import oracle as O
from mu_b200.core.config import ModelConfig
from mu_b200.models.weights import random_state_dict, state_dict_digest

G = Path(__file__).resolve().parent / "golden"

SPECS = {
    "llama_tiny": dict(arch="llama", hidden=256, layers=4, heads=4, kv=2, head_dim=64, inter=688,
                       vocab=1024, seed=0, qk_norm=False, experts=4),
    "deep_tiny": dict(arch="deep", hidden=256, layers=2, heads=4, kv=2, head_dim=64, inter=1024,
                      vocab=1024, seed=5, qk_norm=True, experts=4),
    "llama_decisive": dict(arch="llama", hidden=256, layers=4, heads=4, kv=2, head_dim=64,
                           inter=688, vocab=1024, seed=6, qk_norm=False, experts=4, tie=False),
}
# Generation settings of the model fixtures (prompts: seed + 100).
DECISIVE = dict(SPECS["llama_decisive"], reqs=8, plen=(16, 128), ntok=32)

# Large-vocabulary prepare_logits cases: (temperature, top_k, top_p,
# repetition_penalty).  With top_k 0 or above 1024 the GPU sampler takes its
# radix top-p path (more than 1024 survivors).
LARGE_SAMPLING_VOCABS = (32000, 128256)
LARGE_SAMPLING_CASES = ((0.7, 0, 0.5, 1.0), (0.7, 0, 0.9, 1.0), (0.7, 0, 0.99, 1.0),
                        (1.0, 2000, 0.9, 1.0), (0.7, 0, 0.9, 1.3))


def large_logits(V: int) -> np.ndarray:
    """Seeded f32 logits ~ N(0, 2.5^2) of one row of width V."""
    rng = np.random.default_rng(7000 + V)
    return (rng.standard_normal(V, dtype=np.float32) * np.float32(2.5)).astype(np.float32)


def large_past(V: int) -> list:
    """Seeded past tokens (repetition-penalty case) for a row of width V."""
    return np.random.default_rng(9000 + V).integers(0, V, 300).tolist()


# Top-p boundary band.  The reference normalises its softmax with a float32
# sum (torch CPU; measured 2.0e-5 relative error at V = 128256) and so may
# place the cut a few tokens away from exact arithmetic.  Tokens whose exact
# mass before them lies within TOP_P_BAND of top_p may differ between the
# reference and an exact implementation; every other token must agree.
TOP_P_BAND = 1e-4


def top_p_band(logits, temperature, top_k, repetition_penalty, past, top_p, delta=TOP_P_BAND):
    """Tokens whose exact (float64) descending-order mass before them is
    within ``delta`` of ``top_p`` (all False when top_p >= 1)."""
    x = O.prepare_logits(logits, temperature, top_k, 1.0, repetition_penalty, past)
    band = np.zeros(x.shape[0], dtype=bool)
    if top_p >= 1.0:
        return band
    order = np.argsort(-x, kind="stable")
    sx = x[order].astype(np.float64)
    e = np.exp(sx - sx[0])
    prev = np.concatenate([[0.0], np.cumsum(e / e.sum())[:-1]])
    band[order] = np.abs(prev - top_p) <= delta
    return band


def decisive_state_dict(cfg, seed: int):
    """Seeded Llama weights whose logits are decisive at every step.

    The layers keep the N(0, 0.02) draw of random_state_dict, but the token
    embeddings are N(0, 1), so the residual stream stays close to the current
    token's embedding, and the untied LM head is 0.02 x a row permutation of
    the embedding table: the top logit is the permuted partner of the current
    token (about 5 above the rest at H = 256).  bf16 rounding moves logits by
    ~1e-2, far inside that gap, so greedy tokens must match exactly."""
    sd = random_state_dict(cfg, "llama", seed)
    g = torch.Generator().manual_seed(seed + 1)
    emb = torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g)
    perm = torch.randperm(cfg.vocab_size, generator=g)
    sd["embed_tokens.weight"] = emb
    sd["lm_head.weight"] = (emb[perm] * 0.02).contiguous()
    return sd


def model_config(spec) -> ModelConfig:
    return ModelConfig(
        vocab_size=spec["vocab"], hidden_size=spec["hidden"], intermediate_size=spec["inter"],
        num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
        num_key_value_heads=spec["kv"], head_dim=spec["head_dim"], max_position_embeddings=2048,
        rope_theta=10000.0, rms_norm_eps=1e-6, num_experts=spec["experts"],
        use_qk_norm=spec["qk_norm"], tie_word_embeddings=spec.get("tie", True))


def load_tiny(name):
    spec = SPECS[name]
    cfg = model_config(spec)
    if name == "llama_decisive":
        sd = decisive_state_dict(cfg, spec["seed"])
    else:
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
                         qk_norm=spec["qk_norm"], tie=spec.get("tie", True))
    return shape, cfg, sd, d, prompts
