"""Generate the golden fixtures by running the reference implementation.

Runs Complexity-ML/complexity-inference (package ``mu_inference``) from
/root/reference on the CPU of this container and records its outputs for
seeded inputs.  The fixtures pin the numpy oracle (``oracle/``) and the GPU
path (``tests/test_model_gpu.py``).  /root/reference does not exist on the
GPU box, so only the .npz files travel; this script is committed so the
fixtures can be regenerated:

Contents
  mu_clamp.npz        mu_clamp / soft_clamp on fixed inputs (core/mu.py)
  paged_cache.npz     MuPagedCache block tables and lengths along an
                      allocate/append/free trace (core/cache.py)
  sampling.npz        prepare_logits outputs for several parameter sets
                      (utils/sampling.py)
  routing.npz         expert ids of MuTokenRoutedMLP incl. mu-guided routing
                      (models/layers.py:485-559)
  inl.npz             INLDynamics outputs (models/layers.py:21-127)
  llama_tiny.npz      served path (MuWorker.execute, fp32, greedy argmax) of a
  deep_tiny.npz       tiny LlamaForCausalLM / DeepForCausalLM: prompts, tokens,
                      logits at selected steps, top-2 gaps at every step
  sampling_large.npz  prepare_logits kept-token masks at V = 32000 and 128256
                      (the radix top-p path of the GPU sampler); the logits
                      are regenerated from a seed (golden_models.large_logits)
  llama_decisive.npz  served path of a C1-shaped Llama whose logits have a wide
                      top-2 gap at every step (golden_models.decisive_state_dict),
                      so greedy tokens can be compared without exceptions
Weights come from mu_b200.models.weights.random_state_dict (seeded, CPU);
each model fixture stores the weights' digest.

Usage (the reference checkout is given by argument or environment):

    python tests/golden/make_golden.py --reference <complexity-inference checkout>
    MU_REFERENCE=<checkout> python tests/golden/make_golden.py
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", default=os.environ.get("MU_REFERENCE"),
                    help="checkout of Complexity-ML/complexity-inference (or MU_REFERENCE)")
    ap.add_argument("--only", default="",
                    help="comma-separated fixture names (without .npz) to regenerate")
    args = ap.parse_args()
    if not args.reference or not (Path(args.reference) / "mu_inference").is_dir():
        ap.error("--reference (or MU_REFERENCE) must name a checkout containing mu_inference/")
    args.reference = str(Path(args.reference).resolve())
    return args


ARGS = _args() if __name__ == "__main__" else None
REFERENCE = ARGS.reference if ARGS else None
sys.path.insert(0, str(ROOT / "complexity-inference_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
if REFERENCE:
    sys.path.insert(0, REFERENCE)

from mu_b200.core.config import ModelConfig as MyModelConfig  # noqa: E402
from mu_b200.models.weights import random_state_dict, state_dict_digest, write_model_dir  # noqa: E402

import mu_inference  # noqa: E402  (the reference)
from mu_inference.core.cache import MuPagedCache  # noqa: E402
from mu_inference.core.config import EngineConfig, MuConfig  # noqa: E402
from mu_inference.core.mu import mu_clamp, soft_clamp  # noqa: E402
from mu_inference.models.layers import INLDynamics, MuTokenRoutedMLP  # noqa: E402
from mu_inference.models.loader import config_from_dict  # noqa: E402
from mu_inference.serving.worker import MuWorker, WorkerRequest  # noqa: E402
from mu_inference.utils.sampling import prepare_logits  # noqa: E402

from golden_models import (DECISIVE, LARGE_SAMPLING_CASES, LARGE_SAMPLING_VOCABS,  # noqa: E402
                           decisive_state_dict, large_logits, large_past)

assert str(Path(mu_inference.__file__).resolve()).startswith(REFERENCE), mu_inference.__file__

LLAMA_TINY = dict(arch="llama", hidden=256, layers=4, heads=4, kv=2, head_dim=64, inter=688,
                  vocab=1024, seed=0, reqs=8, plen=(16, 128), ntok=32, qk_norm=False)
DEEP_TINY = dict(arch="deep", hidden=256, layers=2, heads=4, kv=2, head_dim=64, inter=1024,
                 vocab=1024, seed=5, reqs=4, plen=(16, 96), ntok=16, qk_norm=True, experts=4)


def model_config(spec) -> MyModelConfig:
    return MyModelConfig(
        vocab_size=spec["vocab"], hidden_size=spec["hidden"], intermediate_size=spec["inter"],
        num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
        num_key_value_heads=spec["kv"], head_dim=spec["head_dim"], max_position_embeddings=2048,
        rope_theta=10000.0, rms_norm_eps=1e-6, num_experts=spec.get("experts", 4),
        use_qk_norm=spec["qk_norm"], tie_word_embeddings=spec.get("tie", True))


def prompts_for(spec):
    g = np.random.default_rng(spec["seed"] + 100)
    lo, hi = spec["plen"]
    return [g.integers(0, spec["vocab"], g.integers(lo, hi + 1)).tolist()
            for _ in range(spec["reqs"])]


def run_model(spec, out_name, make_sd=None):
    cfg = model_config(spec)
    sd = (make_sd or (lambda c, s: random_state_dict(c, spec["arch"], s)))(cfg, spec["seed"])
    with tempfile.TemporaryDirectory() as td:
        path = write_model_dir(td, cfg, spec["arch"], sd)
        import json

        cfg_dict = json.loads((path / "config.json").read_text())
        ec = EngineConfig(model=config_from_dict(cfg_dict), device="cpu", dtype="float32",
                          mu=MuConfig(enabled=True))
        worker = MuWorker(ec, device="cpu")
        worker.load_model(str(path))
    # every parameter of the reference model must come from our state dict
    ref_params = dict(worker.model.named_parameters())
    missing = [k for k in ref_params if k not in sd and k != "lm_head.weight"]
    assert not missing, missing
    for k in sd:
        assert torch.equal(ref_params[k].detach(), sd[k]), k
    prompts = prompts_for(spec)
    n = spec["ntok"]
    toks = np.zeros((len(prompts), n), dtype=np.int64)
    keep = [0, 1, n // 2 - 1, n - 1]
    logits_keep = np.zeros((len(prompts), len(keep), spec["vocab"]), dtype=np.float32)
    gaps = np.zeros((len(prompts), n), dtype=np.float32)
    for r, prompt in enumerate(prompts):
        rid = f"r{r}"
        assert worker.allocate_request(rid)
        x = torch.tensor([prompt])
        for i in range(n):
            o = worker.execute([WorkerRequest(rid, x, is_prefill=(i == 0))])[0]
            assert o.error is None, o.error
            lg = o.logits.reshape(-1).float().numpy()
            t = int(np.argmax(lg))
            s = np.sort(lg)
            gaps[r, i] = s[-1] - s[-2]
            toks[r, i] = t
            if i in keep:
                logits_keep[r, keep.index(i)] = lg
            x = torch.tensor([[t]])
        worker.free_request(rid)
    plens = np.array([len(p) for p in prompts])
    flat = np.concatenate([np.array(p) for p in prompts])
    np.savez_compressed(HERE / out_name, prompt_lens=plens, prompt_ids=flat, tokens=toks,
                        logits=logits_keep, logit_steps=np.array(keep), top2_gap=gaps,
                        digest=np.array(state_dict_digest(sd)), seed=np.array(spec["seed"]))
    print(out_name, "tokens[0]", toks[0][:8], "min gap", gaps.min())


def make_mu_clamp():
    x = torch.tensor([100.0, -50.0, 5.0, 0.0, -3.25, 9.99, 1e-3, -1e4], dtype=torch.float32)
    cases = [(0.0, -10.0, 10.0), (1.5, -2.0, 6.0), (0.0, 5.0, 5.0), (-1.0, -1.0, 3.0)]
    outs = np.stack([mu_clamp(x, mu, lo, hi).numpy() for mu, lo, hi in cases])
    sc = np.stack([soft_clamp(x, lo, hi).numpy() for _, lo, hi in cases])
    np.savez_compressed(HERE / "mu_clamp.npz", x=x.numpy(), cases=np.array(cases), mu_clamp=outs,
                        soft_clamp=sc)


def make_paged_cache():
    N, bs = 12, 16
    cache = MuPagedCache(num_layers=1, num_kv_heads=1, head_dim=2, block_size=bs,
                         max_num_blocks=N, dtype=torch.float32, device="cpu")
    ops = [("alloc", "a", 0), ("append", "a", 6), ("alloc", "b", 0), ("append", "b", 16),
           ("append", "a", 10), ("append", "a", 1), ("append", "b", 1), ("alloc", "c", 0),
           ("append", "c", 40), ("free", "a", 0), ("alloc", "d", 0), ("append", "d", 17),
           ("append", "c", 30), ("free", "b", 0), ("append", "d", 33), ("alloc", "e", 0),
           ("append", "e", 5), ("free", "c", 0), ("alloc", "f", 0), ("append", "f", 0),
           ("append", "f", 48)]
    names, results, tables, lens = [], [], [], []
    for op, rid, n in ops:
        if op == "alloc":
            res = int(cache.allocate(rid))
        elif op == "append":
            k = torch.zeros(1, n, 1, 2)
            res = cache.append(rid, 0, k, k) if n > 0 else cache.get_seq_len(rid)
        else:
            cache.free(rid)
            res = 0
        names.append(f"{op}:{rid}:{n}")
        results.append(res)
        tab = np.full((8, 8), -1, dtype=np.int64)
        for i, r in enumerate("abcdef"):
            bl = cache.request_blocks.get(r, [])
            tab[i, : len(bl)] = bl
        tables.append(tab)
        lens.append([cache.get_seq_len(r) for r in "abcdef"])
    np.savez_compressed(HERE / "paged_cache.npz", ops=np.array(names), results=np.array(results),
                        tables=np.stack(tables), lens=np.array(lens), num_blocks=N, block_size=bs,
                        free_final=np.array(cache.free_blocks))


def make_sampling():
    g = torch.Generator().manual_seed(21)
    V = 1000
    logits = torch.randn(1, V, generator=g) * 3
    past = torch.randint(0, V, (40,), generator=g).tolist()
    cases = [(1.0, 0, 1.0, 1.0), (0.7, 50, 0.9, 1.0), (1.3, 0, 0.8, 1.1), (0.5, 10, 1.0, 1.2),
             (1.0, 200, 0.95, 1.0), (0.0, 50, 0.9, 1.1), (2.0, 0, 0.5, 1.0)]
    outs = np.stack([prepare_logits(logits, t, k, p, rp, past).numpy()[0] for t, k, p, rp in cases])
    np.savez_compressed(HERE / "sampling.npz", logits=logits.numpy()[0], past=np.array(past),
                        cases=np.array(cases), out=outs)


def make_sampling_large():
    """Kept-token masks of the reference's prepare_logits at vocabulary sizes
    where the GPU sampler runs its radix top-p search; packed bits per case."""
    out = {}
    for V in LARGE_SAMPLING_VOCABS:
        x = large_logits(V)
        past = large_past(V)
        logits = torch.from_numpy(x)[None]
        masks = []
        for t, k, p, rp in LARGE_SAMPLING_CASES:
            got = prepare_logits(logits, t, k, p, rp, past).numpy()[0]
            masks.append(np.packbits(~np.isinf(got)))
        out[f"masks_{V}"] = np.stack(masks)
        out[f"checksum_{V}"] = np.array([float(x.astype(np.float64).sum()),
                                         float((x.astype(np.float64) ** 2).sum())])
    np.savez_compressed(HERE / "sampling_large.npz", cases=np.array(LARGE_SAMPLING_CASES),
                        vocabs=np.array(LARGE_SAMPLING_VOCABS), **out)


def make_routing():
    torch.manual_seed(0)
    H, E, V, T = 32, 4, 1000, 96
    mlp = MuTokenRoutedMLP(H, 4 * E, E, V, mu_config=MuConfig(enabled=False))
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        # make each expert's output reveal its index: output = silu(H*e)*(H*e)
        for e in range(E):
            mlp.gate_up_proj[e].fill_(float(e))
            mlp.down_proj[e].fill_(1.0 / mlp.expert_intermediate_size)
        mlp.mu_router.weight.copy_(torch.randn(E, H, generator=g) * 1.5)
    ids = torch.randint(-5, V + 5, (1, T), generator=g)
    mu = torch.randn(1, T, H, generator=g)
    x = torch.ones(1, T, H)
    out = mlp(x, token_ids=ids, mu=mu)[0, :, 0].detach()
    table = torch.tensor([float(torch.nn.functional.silu(torch.tensor(float(H * e))) * H * e)
                          for e in range(E)])
    eids = (out[:, None] - table[None]).abs().argmin(-1)
    base = mlp(x, token_ids=ids, mu=None)[0, :, 0].detach()
    beids = (base[:, None] - table[None]).abs().argmin(-1)
    np.savez_compressed(HERE / "routing.npz", ids=ids.numpy()[0], mu=mu.numpy()[0],
                        router=mlp.mu_router.weight.detach().numpy(), experts=eids.numpy(),
                        base_experts=beids.numpy(), vocab=V, num_experts=E)


def make_inl():
    torch.manual_seed(3)
    H, T = 48, 10
    dyn = INLDynamics(H, controller_hidden=16, dt=0.1)
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        dyn.mu_proj.weight.copy_(torch.randn(H, H, generator=g) * 0.1)
        dyn.mu.copy_(torch.randn(H, generator=g) * 0.1)
    h = torch.randn(T, H, generator=g) * 2
    v = torch.randn(T, H, generator=g) * 3
    hn, vn, mu_c = dyn(h, v)
    hn0, vn0, mu0 = dyn(h, None)
    sd = {k: t.detach().numpy() for k, t in dyn.state_dict().items()}
    np.savez_compressed(HERE / "inl.npz", h=h.numpy(), v=v.numpy(), h_next=hn.detach().numpy(),
                        v_next=vn.detach().numpy(), mu_c=mu_c.detach().numpy(),
                        h_next0=hn0.detach().numpy(), v_next0=vn0.detach().numpy(),
                        **{"p_" + k: a for k, a in sd.items()})


def main():
    torch.set_num_threads(8)
    makers = {
        "mu_clamp": make_mu_clamp,
        "paged_cache": make_paged_cache,
        "sampling": make_sampling,
        "sampling_large": make_sampling_large,
        "routing": make_routing,
        "inl": make_inl,
        "llama_tiny": lambda: run_model(LLAMA_TINY, "llama_tiny.npz"),
        "deep_tiny": lambda: run_model(DEEP_TINY, "deep_tiny.npz"),
        "llama_decisive": lambda: run_model(DECISIVE, "llama_decisive.npz", decisive_state_dict),
    }
    only = [n for n in ARGS.only.split(",") if n]
    for name, make in makers.items():
        if not only or name in only:
            make()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
