"""Pin the numpy oracle to the reference's own outputs (tests/golden/*.npz).

The fixtures were produced by running the reference (mu_inference) on CPU;
these tests show the oracle restates it: integer outputs bit-exact, float
outputs within f32 re-association noise (1e-4 relative)."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O

G = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(G / name)


def test_mu_clamp_known_answers():
    d = _load("mu_clamp.npz")
    for (mu, lo, hi), ref, sref in zip(d["cases"], d["mu_clamp"], d["soft_clamp"]):
        np.testing.assert_allclose(O.mu_clamp(d["x"], mu, lo, hi), ref, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(O.soft_clamp(d["x"], lo, hi), sref, rtol=1e-6, atol=1e-6)
    # the executed values of the mu.py docstring example (its printed values are wrong)
    np.testing.assert_allclose(O.mu_clamp(np.array([100.0, -50.0, 5.0])),
                               [10.0, -9.999092, 4.6211715], rtol=1e-6)


def test_paged_allocator_trace():
    d = _load("paged_cache.npz")
    a = O.PagedAllocatorOracle(int(d["num_blocks"]), int(d["block_size"]))
    for op, res, tab, lens in zip(d["ops"], d["results"], d["tables"], d["lens"]):
        kind, rid, n = str(op).split(":")
        n = int(n)
        if kind == "alloc":
            assert int(a.allocate(rid)) == res
        elif kind == "append":
            slots = a.append(rid, n)
            assert slots is not None and a.seq_len(rid) == res
        else:
            a.free(rid)
        for i, r in enumerate("abcdef"):
            bl = a.blocks.get(r, [])
            assert list(tab[i, : len(bl)]) == bl and (len(bl) == 8 or tab[i, len(bl)] == -1)
            assert a.seq_len(r) == lens[i]
    assert a.free_blocks == list(d["free_final"])


def test_prepare_logits_cases():
    d = _load("sampling.npz")
    for (t, k, p, rp), ref in zip(d["cases"], d["out"]):
        got = O.prepare_logits(d["logits"], t, int(k), p, rp, d["past"].tolist())
        assert np.array_equal(np.isinf(got), np.isinf(ref))
        fin = ~np.isinf(ref)
        np.testing.assert_allclose(got[fin], ref[fin], rtol=1e-6, atol=1e-6)


def test_prepare_logits_large_vocab():
    """The oracle's kept sets at V = 32000 / 128256 equal the reference's
    outside the top-p boundary band, and the masks are pinned to the seeded
    logits by their checksum."""
    from golden_models import (LARGE_SAMPLING_CASES, LARGE_SAMPLING_VOCABS, large_logits,
                               large_past, top_p_band)

    d = _load("sampling_large.npz")
    assert tuple(d["vocabs"]) == LARGE_SAMPLING_VOCABS
    for V in LARGE_SAMPLING_VOCABS:
        x = large_logits(V)
        np.testing.assert_allclose(d[f"checksum_{V}"], [x.astype(np.float64).sum(),
                                                        (x.astype(np.float64) ** 2).sum()],
                                   rtol=1e-12)
        past = large_past(V)
        for c, (t, k, p, rp) in enumerate(LARGE_SAMPLING_CASES):
            ref = np.unpackbits(d[f"masks_{V}"][c])[:V].astype(bool)
            got = ~np.isinf(O.prepare_logits(x, t, int(k), p, rp, past))
            band = top_p_band(x, t, int(k), rp, past, p)
            assert np.array_equal(ref[~band], got[~band]), (V, c)
            assert ref.sum() > 1 and band.sum() < 0.02 * ref.sum() + 2, (V, c, band.sum())


def test_routing():
    d = _load("routing.npz")
    E, V = int(d["num_experts"]), int(d["vocab"])
    assert np.array_equal(O.route_experts(d["ids"], d["mu"], d["router"], E, V), d["experts"])
    assert np.array_equal(O.route_experts(d["ids"], None, d["router"], E, V), d["base_experts"])
    # the fixture exercises the mu-guided override, not only id % E
    assert (d["experts"] != d["base_experts"]).any()


def test_inl_dynamics():
    d = _load("inl.npz")
    p = {k[2:]: d[k] for k in d.files if k.startswith("p_")}
    hn, vn, mu = O.inl_dynamics(d["h"], d["v"], p, "", 0.1)
    np.testing.assert_allclose(hn, d["h_next"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(vn, d["v_next"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(mu, d["mu_c"], rtol=1e-5, atol=1e-5)
    hn0, vn0, _ = O.inl_dynamics(d["h"], None, p, "", 0.1)
    np.testing.assert_allclose(hn0, d["h_next0"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(vn0, d["v_next0"], rtol=1e-5, atol=1e-5)


def _tiny(name):
    from golden_models import load_tiny

    return load_tiny(name)


@pytest.mark.parametrize("name", ["llama_tiny", "deep_tiny"])
def test_oracle_model_matches_reference(name):
    spec, cfg, sd, d, prompts = _tiny(name)
    model = O.OracleModel(spec, {k: v.numpy() for k, v in sd.items()}, O.MuCfg(True))
    steps = list(d["logit_steps"])
    # two requests keep the CPU time small; the GPU test covers all of them
    for r in range(2):
        toks = d["tokens"][r]
        lg = O.teacher_forced_logits(model, prompts[r], toks)
        assert int(np.argmax(lg[0])) == toks[0]
        for j, s in enumerate(steps):
            np.testing.assert_allclose(lg[s], d["logits"][r, j], rtol=1e-4, atol=2e-4)
        assert list(np.argmax(lg, -1)) == list(toks)


@pytest.mark.parametrize("name", ["llama_tiny", "deep_tiny", "llama_decisive"])
def test_oracle_batch_forward_equals_per_request(name):
    """forward_batch (ragged requests, each with its own cache) gives every
    request the logits and cache of its own batch-1 forward; the decisive
    fixture is pinned to the reference's tokens for two requests."""
    spec, cfg, sd, d, prompts = _tiny(name)
    model = O.OracleModel(spec, {k: v.numpy() for k, v in sd.items()}, O.MuCfg(True))
    singles = [model.forward(p) for p in prompts[:3]]
    lg, pasts, _ = model.forward_batch(prompts[:3])
    for r, (l1, p1) in enumerate(singles):
        np.testing.assert_allclose(lg[r], l1, rtol=1e-5, atol=1e-5)
        for (k1, v1), (k2, v2) in zip(p1, pasts[r]):
            np.testing.assert_allclose(k2, k1, rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(v2, v1, rtol=1e-5, atol=1e-5)
    toks = [int(np.argmax(x)) for x in lg]
    lg2, _, _ = model.forward_batch([[t] for t in toks], pasts)
    for r in range(3):
        l2, _ = model.forward([toks[r]], singles[r][1])
        np.testing.assert_allclose(lg2[r], l2, rtol=1e-5, atol=1e-5)
    if name == "llama_decisive":
        for r in range(2):
            got = O.teacher_forced_logits(model, prompts[r], d["tokens"][r])
            assert list(np.argmax(got, -1)) == list(d["tokens"][r])
            np.testing.assert_allclose(got[d["logit_steps"]], d["logits"][r], rtol=1e-4,
                                       atol=2e-4)
        assert float(d["top2_gap"].min()) > 1.0
