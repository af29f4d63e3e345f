"""Tensor-parallel sharding on CPU: gloo ranks, oracle math.

Two processes each take their shard of the tiny fixtures' weights
(mu_b200.models.sharding) and run the oracle's layer math on it; after each
row-parallel projection (O and down) they all-reduce the partial outputs
over gloo, exactly where the GPU model calls NCCL.  The result must equal the
unsharded oracle forward, and the shards must recombine to the full weights.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mu_oracle as O
from golden_models import load_tiny
from mu_b200.models.sharding import expert_range, shard_state_dict


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _allreduce(x):
    t = torch.from_numpy(np.ascontiguousarray(x))
    dist.all_reduce(t)
    return t.numpy()


def _tp_forward(model: O.OracleModel, ids, experts=None):
    """Prefill-only forward of a sharded OracleModel with all-reduces.

    ``experts``: (lo, hi) when the shard holds whole experts [lo, hi)
    (expert parallelism); tokens routed elsewhere contribute zero here."""
    s, p, mu = model.s, model.p, model.mu
    ids = np.asarray(ids)
    h = O._clamp(p["embed_tokens.weight"][ids].astype(np.float32), mu)
    v_state, mu_prev = None, None
    for l in range(s.layers):
        pre = f"layers.{l}."
        res = h
        x = O.rmsnorm(h, p[pre + "input_layernorm.weight"], s.eps, mu)
        # attention on the local heads; o_proj gives a partial sum
        a = pre + "self_attn."
        S = x.shape[0]
        q = x @ p[a + "q_proj.weight"].T
        k = x @ p[a + "k_proj.weight"].T
        v = x @ p[a + "v_proj.weight"].T
        if s.arch == "deep" and mu_prev is not None:
            q = q + mu_prev @ p[a + "mu_to_q.weight"].T
            k = k + mu_prev @ p[a + "mu_to_k.weight"].T
            v = v + mu_prev @ p[a + "mu_to_v.weight"].T
        q = q.reshape(S, s.heads, s.head_dim).astype(np.float32)
        k = k.reshape(S, s.kv_heads, s.head_dim).astype(np.float32)
        v = v.reshape(S, s.kv_heads, s.head_dim).astype(np.float32)
        if s.qk_norm:
            q = O.rmsnorm(q, p[a + "q_norm.weight"], 1e-6)
            k = O.rmsnorm(k, p[a + "k_norm.weight"], 1e-6)
        pos = np.arange(S)
        q = O.apply_rope(q, model.cos, model.sin, pos)
        k = O.apply_rope(k, model.cos, model.sin, pos)
        o = O.sdpa(q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2), True)
        o = o.transpose(1, 0, 2).reshape(S, -1)
        attn = O._clamp(_allreduce(o @ p[a + "o_proj.weight"].T), mu)
        if s.arch == "deep":
            h_next, v_state, mu_cur = O.inl_dynamics(attn, v_state, p, pre + "dynamics.", s.dt)
            h = res + h_next
            res = h
            x2 = O.rmsnorm(h, p[pre + "post_attention_layernorm.weight"], s.eps, mu)
            e = O.route_experts(ids, mu_cur, p[pre + "mlp.mu_router.weight"], s.experts, s.vocab)
            gu, dn = p[pre + "mlp.gate_up_proj"], p[pre + "mlp.down_proj"]
            I = dn.shape[1]
            lo, hi = experts if experts else (0, gu.shape[0])

            def mlp(t):
                if not lo <= e[t] < hi:
                    return np.zeros(dn.shape[2], np.float32)
                j = e[t] - lo
                return (O._silu(x2[t] @ gu[j][:, :I]) * (x2[t] @ gu[j][:, I:])) @ dn[j]

            part = np.stack([mlp(t) for t in range(S)])
            h = O._clamp(res + O._clamp(_allreduce(part), mu), mu)
            mu_prev = mu_cur
        else:
            h = res + attn
            res = h
            x2 = O.rmsnorm(h, p[pre + "post_attention_layernorm.weight"], s.eps, mu)
            m = pre + "mlp."
            part = (O._silu(x2 @ p[m + "gate_proj.weight"].T) * (x2 @ p[m + "up_proj.weight"].T)
                    ) @ p[m + "down_proj.weight"].T
            h = O._clamp(res + O._clamp(_allreduce(part), mu), mu)
    hn = O.rmsnorm(h, p["norm.weight"], s.eps, mu)
    return (hn[-1] @ p["lm_head.weight"].T).astype(np.float32)


def _rows_of(rank, world, S):
    """Rows [lo, hi) owned by ``rank``: contiguous shares of ceil(S / world)."""
    sr = (S + world - 1) // world
    lo = min(S, rank * sr)
    return sr, lo, min(S, lo + sr)


def _reduce_scatter_rows(part, sr, lo, hi):
    """This rank's rows of the sum over the ranks (gloo has no
    reduce-scatter: all-reduce, then keep the owned rows)."""
    return _allreduce(part)[lo:hi]


def _all_gather_rows(rows, sr, S, world):
    pad = np.zeros((sr, rows.shape[1]), np.float32)
    pad[:rows.shape[0]] = rows
    out = [torch.empty(sr, rows.shape[1]) for _ in range(world)]
    dist.all_gather(out, torch.from_numpy(pad))
    return torch.cat(out).numpy()[:S]


def _tp_forward_rs_norm(model: O.OracleModel, ids):
    """Llama prefill under tensor parallelism in the reduce-scatter form of
    muk_tp_residual_norm: after each row-parallel projection a rank keeps
    only its own rows of the sum, adds them to its rows of the residual
    (the other rows are never kept), normalises them and all-gathers the
    normalised rows; the last layer normalises with the final norm and the
    LM head reads the last row of x."""
    s, p, mu = model.s, model.p, model.mu
    ids = np.asarray(ids)
    S = len(ids)
    rank, world = dist.get_rank(), dist.get_world_size()
    sr, lo, hi = _rows_of(rank, world, S)
    h = O._clamp(p["embed_tokens.weight"][ids].astype(np.float32), mu)
    x = O.rmsnorm(h, p["layers.0.input_layernorm.weight"], s.eps, mu)
    h = h[lo:hi].copy()                      # the residual is row-sharded from here on
    for l in range(s.layers):
        pre = f"layers.{l}."
        a = pre + "self_attn."
        q = (x @ p[a + "q_proj.weight"].T).reshape(S, s.heads, s.head_dim).astype(np.float32)
        k = (x @ p[a + "k_proj.weight"].T).reshape(S, s.kv_heads, s.head_dim).astype(np.float32)
        v = (x @ p[a + "v_proj.weight"].T).reshape(S, s.kv_heads, s.head_dim).astype(np.float32)
        pos = np.arange(S)
        q = O.apply_rope(q, model.cos, model.sin, pos)
        k = O.apply_rope(k, model.cos, model.sin, pos)
        o = O.sdpa(q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2), True)
        o = o.transpose(1, 0, 2).reshape(S, -1)
        h = h + O._clamp(_reduce_scatter_rows(o @ p[a + "o_proj.weight"].T, sr, lo, hi), mu)
        x2 = _all_gather_rows(O.rmsnorm(h, p[pre + "post_attention_layernorm.weight"], s.eps, mu),
                              sr, S, world)
        m = pre + "mlp."
        part = (O._silu(x2 @ p[m + "gate_proj.weight"].T) * (x2 @ p[m + "up_proj.weight"].T)
                ) @ p[m + "down_proj.weight"].T
        h = O._clamp(h + O._clamp(_reduce_scatter_rows(part, sr, lo, hi), mu), mu)
        w = p["norm.weight"] if l + 1 == s.layers else p[f"layers.{l + 1}.input_layernorm.weight"]
        x = _all_gather_rows(O.rmsnorm(h, w, s.eps, mu), sr, S, world)
    return (x[-1] @ p["lm_head.weight"].T).astype(np.float32)


def _worker(rank, world, port, name, q, ep=False, rs_norm=False, trim=0):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, f"init failed: {e!r}"))
        return
    try:
        shape, cfg, sd, d, prompts = load_tiny(name)
        shard, local = shard_state_dict(sd, cfg, shape.arch, rank, world, expert_parallel=ep)
        lshape = O.ModelShape(shape.arch, shape.hidden, shape.layers, local.num_attention_heads,
                              local.num_key_value_heads, shape.head_dim, shape.vocab,
                              experts=shape.experts, qk_norm=shape.qk_norm)
        model = O.OracleModel(lshape, {k: v.numpy() for k, v in shard.items()}, O.MuCfg(True))
        ids = prompts[0][:len(prompts[0]) - trim]
        if rs_norm:
            logits = _tp_forward_rs_norm(model, ids)
        else:
            logits = _tp_forward(model, ids, expert_range(cfg, rank, world) if ep else None)
        q.put((rank, logits))
    except Exception as e:
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,ep,rs_norm,trim", [("llama_tiny", False, False, 0),
                                                  ("deep_tiny", False, False, 0),
                                                  ("deep_tiny", True, False, 0),
                                                  ("llama_tiny", False, True, 0),
                                                  ("llama_tiny", False, True, 1)])
def test_tp2_matches_unsharded(name, ep, rs_norm, trim):
    """rs_norm: the reduce-scatter + owned-row residual/norm + all-gather
    form; trim drops prompt tokens so the two ranks own unequal shares."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, q, ep, rs_norm, trim))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shape, cfg, sd, d, prompts = load_tiny(name)
    full = O.OracleModel(shape, {k: v.numpy() for k, v in sd.items()}, O.MuCfg(True))
    ids = prompts[0][:len(prompts[0]) - trim]
    if trim:
        assert (len(ids) % world) != 0
    ref, _ = full.forward(ids)
    for r in range(world):
        np.testing.assert_allclose(got[r], ref, rtol=1e-4, atol=1e-4)
    assert np.array_equal(got[0], got[1])  # every rank holds the same logits


def _dying_worker(rank, world, port, q):
    """Rank 1 fails (an exception, then the process exits) before its first
    all-reduce; rank 0 runs the sharded forward and must see its next
    collective end with an error, not wait forever."""
    import time

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "injected failure"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(3)  # dies without leaving the group
    shape, cfg, sd, d, prompts = load_tiny("llama_tiny")
    shard, local = shard_state_dict(sd, cfg, shape.arch, rank, world)
    lshape = O.ModelShape(shape.arch, shape.hidden, shape.layers, local.num_attention_heads,
                          local.num_key_value_heads, shape.head_dim, shape.vocab)
    model = O.OracleModel(lshape, {k: v.numpy() for k, v in shard.items()}, O.MuCfg(True))
    t0 = time.time()
    try:
        _tp_forward(model, prompts[0])
        q.put((rank, ("no error", time.time() - t0)))
    except Exception as e:  # noqa: BLE001 - the collective's failure is the result
        q.put((rank, ("error", time.time() - t0, type(e).__name__)))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_death_ends_the_peers_collective():
    """Failure detection on the host: a rank that dies between steps makes
    the survivor's next all-reduce fail within the process-group timeout."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "injected failure" and procs[1].exitcode == 3
    assert got[0][0] == "error", got[0]
    assert got[0][1] < 60.0, got[0]


@pytest.mark.parametrize("name", ["llama_tiny", "deep_tiny"])
def test_shards_recombine(name):
    shape, cfg, sd, d, prompts = load_tiny(name)
    tp = 2
    shards = [shard_state_dict(sd, cfg, shape.arch, r, tp)[0] for r in range(tp)]
    a = "layers.0.self_attn."
    assert torch.equal(torch.cat([s[a + "q_proj.weight"] for s in shards]), sd[a + "q_proj.weight"])
    assert torch.equal(torch.cat([s[a + "o_proj.weight"] for s in shards], 1), sd[a + "o_proj.weight"])
    if shape.arch == "deep":
        gu = sd["layers.0.mlp.gate_up_proj"]
        I = gu.shape[2] // 2
        g = torch.cat([s["layers.0.mlp.gate_up_proj"][:, :, : I // tp] for s in shards], 2)
        assert torch.equal(g, gu[:, :, :I])
        dn = torch.cat([s["layers.0.mlp.down_proj"] for s in shards], 1)
        assert torch.equal(dn, sd["layers.0.mlp.down_proj"])
    else:
        dn = torch.cat([s["layers.0.mlp.down_proj.weight"] for s in shards], 1)
        assert torch.equal(dn, sd["layers.0.mlp.down_proj.weight"])
    assert torch.equal(shards[1]["embed_tokens.weight"], sd["embed_tokens.weight"])
    if shape.arch == "deep":  # expert parallelism: whole experts, split over the ranks
        ep = [shard_state_dict(sd, cfg, shape.arch, r, tp, expert_parallel=True)[0]
              for r in range(tp)]
        for k in ("layers.0.mlp.gate_up_proj", "layers.0.mlp.down_proj"):
            assert torch.equal(torch.cat([s[k] for s in ep]), sd[k])
        assert ep[0]["layers.0.self_attn.q_proj.weight"].shape[0] == \
            sd["layers.0.self_attn.q_proj.weight"].shape[0] // tp


@pytest.mark.parametrize("name,ep", [("llama_tiny", False), ("deep_tiny", False), ("deep_tiny", True)])
def test_sharded_safetensors_load(tmp_path, name, ep):
    """Reading a rank's slices straight from a model dir's safetensors (with
    the reference's "model." prefix) gives exactly the in-memory shard."""
    from mu_b200.models.sharding import load_sharded_state_dict
    from safetensors.torch import save_file

    shape, cfg, sd, d, prompts = load_tiny(name)
    save_file({"model." + k: v.contiguous() for k, v in sd.items()},
              str(tmp_path / "model.safetensors"))
    for rank in range(2):
        want, wcfg = shard_state_dict(sd, cfg, shape.arch, rank, 2, expert_parallel=ep)
        got, gcfg = load_sharded_state_dict(tmp_path, cfg, shape.arch, rank, 2, expert_parallel=ep)
        assert gcfg == wcfg and sorted(got) == sorted(want)
        for k in want:
            assert torch.equal(got[k], want[k]), k


def _agree_worker(rank, world, port, q, fail_rank, fail_at):
    """One tensor-parallel rank of the CPU stand-in engine (test_engine_overlap's
    fake worker and sampler) with MuWorker's step agreement over gloo; the
    sampler of ``fail_rank`` raises a device error when the ``fail_at``-th
    step is read back."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, f"init failed: {e!r}"))
        return
    try:
        import test_engine_overlap as T
        from mu_b200 import _lib
        from mu_b200.core.config import CacheConfig, EngineConfig, SamplingParams, SchedulerConfig
        from mu_b200.serving import engine as E
        from mu_b200.serving.worker import MuWorker

        class _Bad:
            def __init__(self, toks):
                self.dev = torch.tensor(toks, dtype=torch.int32)

            def wait(self):
                raise _lib.DeviceError(5, "sampled step")

        class Sampler(T.FakeSampler):
            n = 0

            def launch(self, logits, ids, params, steps, token_rows=None, input_ids=None,
                       num_tokens=0):
                Sampler.n += 1
                if rank == fail_rank and Sampler.n == fail_at:
                    return _Bad(logits)
                return T._Handle(logits)

        E.BatchSampler = Sampler
        resets = []
        w = T.FakeWorker(64)
        w._agree_group = dist.group.WORLD
        w.tp_agree = MuWorker.tp_agree.__get__(w)
        w.tp_reset = lambda: (resets.append(1), MuWorker.tp_reset(w))
        ec = EngineConfig(cache=CacheConfig(block_size=4, max_num_blocks=64, max_num_seqs=4),
                          scheduler=SchedulerConfig(max_batch_size=4, max_num_batched_tokens=64,
                                                    max_prefill_tokens=64))
        eng = E.StepEngine(w, ec, overlap=True)
        rng = np.random.default_rng(5)
        for i in range(6):
            eng.add_request(rng.integers(0, T.V, int(rng.integers(3, 9))).tolist(),
                            SamplingParams(temperature=0.0, max_tokens=8), f"r{i}")
        reasons = {}
        while eng.has_unfinished():
            for o in eng.step():
                if o.finished:
                    reasons[o.request_id] = o.finish_reason
        out = {rid: (reasons.get(rid), list(r.output_token_ids)) for rid, r in eng.requests.items()}
        q.put((rank, (out, len(resets))))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_tp_step_failure_is_agreed_across_ranks():
    """A device error read back on one tensor-parallel rank fails the same
    step (and the one launched after it) on every rank: both ranks finish
    the same requests with "error", reset their cross-GPU flags once, and
    generate identical tokens for every other request."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, world, port, q, 1, 4))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    (out0, resets0), (out1, resets1) = got[0], got[1]
    assert out0 == out1
    assert resets0 == resets1 == 1
    errs = [rid for rid, (reason, _) in out0.items() if reason == "error"]
    assert errs and len(errs) < len(out0)
    assert all(reason in ("length", "stop") for rid, (reason, _) in out0.items() if rid not in errs)


def _ep_combine_worker(rank, world, port, q):
    """One rank of the expert-parallel combine on CPU: every rank routes all
    tokens identically, sorts them stably by expert (as muk_route_permute
    does), computes only its own experts' rows in that sorted order, and the
    ranks exchange those rows (gloo all-gather of each rank's contiguous
    range, as muk_ep_gather_bf16 does over NVLink); un-permuting gives every
    token's expert output."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, f"init failed: {e!r}"))
        return
    try:
        shape, cfg, sd, d, prompts = load_tiny("deep_tiny")
        p = {k: v.numpy() for k, v in sd.items()}
        E, V, H = shape.experts, shape.vocab, shape.hidden
        rng = np.random.default_rng(3)
        T = 97
        ids = rng.integers(0, V, T)
        x = rng.standard_normal((T, H)).astype(np.float32)
        mu = (rng.standard_normal((T, H)) * 0.3).astype(np.float32)
        pre = "layers.0.mlp."
        e = O.route_experts(ids, mu, p[pre + "mu_router.weight"], E, V)
        perm = np.argsort(e, kind="stable")          # sorted row i holds token perm[i]
        inv = np.empty(T, dtype=np.int64)
        inv[perm] = np.arange(T)                      # token t sits at sorted row inv[t]
        offs = np.concatenate([[0], np.cumsum(np.bincount(e, minlength=E))])
        lo, hi = expert_range(cfg, rank, world)
        gu, dn = p[pre + "gate_up_proj"], p[pre + "down_proj"]
        I = dn.shape[1]
        rows = np.zeros((T, H), dtype=np.float32)
        xs = x[perm]
        for ex in range(lo, hi):
            a, b = offs[ex], offs[ex + 1]
            g = xs[a:b] @ gu[ex]
            rows[a:b] = (O._silu(g[:, :I]) * g[:, I:]) @ dn[ex]
        # exchange: every rank contributes its range [offs[lo], offs[hi])
        mine = torch.from_numpy(np.ascontiguousarray(rows[offs[lo]:offs[hi]]))
        sizes = [None] * world
        dist.all_gather_object(sizes, (int(offs[lo]), int(offs[hi])))
        parts = [torch.zeros(b - a, H) for a, b in sizes]
        counts = torch.tensor([b - a for a, b in sizes])
        mx = int(counts.max())
        pad = torch.zeros(mx, H)
        pad[:mine.shape[0]] = mine
        gathered = [torch.zeros(mx, H) for _ in range(world)]
        dist.all_gather(gathered, pad)
        full = np.zeros((T, H), dtype=np.float32)
        for (a, b), gpart in zip(sizes, gathered):
            full[a:b] = gpart[:b - a].numpy()
        out = full[inv]                               # back to token order
        q.put((rank, (out, e, (lo, hi))))
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_ep_combine_bookkeeping_matches_unsharded():
    """Expert-parallel routing, stable expert sort, per-rank expert rows, the
    row exchange and the un-permute reproduce the unsharded token-routed MLP
    (layers.py:485-559, via the oracle) on both ranks, and the two ranks' expert
    ranges cover every expert exactly once."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_combine_worker, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
    shape, cfg, sd, d, prompts = load_tiny("deep_tiny")
    p = {k: v.numpy() for k, v in sd.items()}
    E, V, H = shape.experts, shape.vocab, shape.hidden
    rng = np.random.default_rng(3)
    T = 97
    ids = rng.integers(0, V, T)
    x = rng.standard_normal((T, H)).astype(np.float32)
    mu = (rng.standard_normal((T, H)) * 0.3).astype(np.float32)
    model = O.OracleModel(shape, p, O.MuCfg(False))
    ref = model._mlp(0, x, ids, mu)
    ranges = sorted(got[r][2] for r in range(world))
    assert ranges[0][0] == 0 and ranges[-1][1] == E and ranges[0][1] == ranges[1][0]
    for r in range(world):
        out, e, _ = got[r]
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=1e-5)
        assert np.array_equal(e, O.route_experts(ids, mu, p["layers.0.mlp.mu_router.weight"], E, V))
    assert len(np.unique(got[0][1])) > 1   # tokens really spread over both ranks' experts


def _greedy_combine_worker(rank, world, port, q):
    """Each rank holds the columns [r V/P, (r+1) V/P) of the same logits rows;
    it reduces them to one (value, index) pair per row with the sampler's
    penalty rule, the pairs are all-gathered and the best pair is taken
    (largest value, lowest index): muk_tp_greedy's arithmetic."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        B, V = 9, 64
        rng = np.random.default_rng(5)                      # the same rows on every rank
        x = rng.standard_normal((B, V)).astype(np.float32)
        x[1, 3] = x[1, 40] = 9.0                            # a tie across the two slices
        x[2, 17] = x[2, 21] = 9.0                           # a tie inside one slice
        x[3] = -np.inf
        seen = rng.random((B, V)) < 0.3
        seen[1, [3, 40]] = seen[2, [17, 21]] = False        # keep the planted ties exact
        rp = np.where(np.arange(B) % 2 == 0, 1.3, 1.0).astype(np.float32)
        pen = np.where(seen & (rp[:, None] != 1.0),
                       np.where(x > 0, x / rp[:, None], x * rp[:, None]), x)
        n = V // world
        c0 = rank * n
        loc = pen[:, c0:c0 + n]
        vals, idxs = [], []
        for b in range(B):
            best, bi = -np.inf, 2**31 - 1
            for i in range(n):                              # first maximum of the slice
                if loc[b, i] > best:
                    best, bi = loc[b, i], c0 + i
            vals.append(best)
            idxs.append(bi)
        mine = torch.tensor([vals, idxs], dtype=torch.float64)
        allp = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        out = []
        for b in range(B):
            best, bi = -np.inf, 2**31 - 1
            for p in allp:                                  # rank order = vocabulary order
                v, i = float(p[0, b]), int(p[1, b])
                if v > best or (v == best and i < bi):
                    best, bi = v, i
            out.append(0 if bi == 2**31 - 1 else bi)
        ref = [int(np.argmax(pen[b])) if np.isfinite(pen[b]).any() else 0 for b in range(B)]
        q.put((rank, out == ref and out[1] == 3 and out[2] == 17))
        dist.destroy_process_group()
    except Exception:
        import traceback

        q.put((rank, traceback.format_exc()))


def test_vocab_parallel_greedy_combine():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_greedy_combine_worker, args=(r, world, port, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got == {0: True, 1: True}, got
