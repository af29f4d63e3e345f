"""One rank of the tensor-parallel GPU check (launched by test_tp_gpu.py).

Each rank loads its shard of the tiny Llama / Deep fixtures through
MuWorker (tensor_parallel_size = world size, NCCL) and runs the fixtures'
requests teacher-forced with the reference's greedy tokens, then greedily
through StepEngine.  Logits must be within 2e-2 max-abs of the reference's
fp32 logits on every rank, and the ranks' generated tokens must agree.
Exit code 0 = pass.
"""

import datetime
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent / "complexity-inference_b200"))
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from golden_models import load_tiny  # noqa: E402


def check_peer_allreduce(rank, world, failures):
    """muk_allreduce_f32 alone: sums equal the NCCL reference on every rank,
    bit-identical across ranks, also when replayed from a CUDA graph."""
    from mu_b200.comm import PeerAllReduce

    comm = PeerAllReduce(dist.group.WORLD, 1 << 20, torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for n in (4, 1000, 1 << 20):
        x = comm.view(n)
        x.copy_(torch.randn(n, device="cuda", generator=g))
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.clone())
        ref = torch.stack(parts).sum(0)   # rank order, like the kernel
        comm.all_reduce_(x)
        torch.cuda.synchronize()
        if not torch.allclose(x, ref, rtol=1e-6, atol=1e-6):
            failures.append(("peer allreduce", n, float((x - ref).abs().max())))
        allx = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(allx, x)
        if not all(torch.equal(a, allx[0]) for a in allx):
            failures.append(("peer allreduce not identical across ranks", n))
    # split-K slices are folded before the exchange; the sum lands in slice 0
    n, S = 1000, 3
    x = comm.view(S * n).view(S, n)
    x.copy_(torch.randn(S, n, device="cuda", generator=g))
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.clone())
    ref = torch.stack([p.sum(0) for p in parts]).sum(0)
    out = comm.all_reduce_(x, slices=S)
    torch.cuda.synchronize()
    if out.data_ptr() != x.data_ptr() or not torch.allclose(out, ref, rtol=1e-5, atol=1e-5):
        failures.append(("peer allreduce slices", float((out - ref).abs().max())))
    # GEMM and reduce-scatter fused (muk_gemm_allreduce_f32): out = sum_r A_r W_r^T
    M, N, Kd = 37, 256, 320
    A = torch.randn(M, Kd, device="cuda", generator=g).bfloat16()
    W = (torch.randn(N, Kd, device="cuda", generator=g) * 0.05).bfloat16()
    ref = A.float() @ W.float().t()
    dist.all_reduce(ref)
    out = comm.gemm_all_reduce(A, W, M)[0]
    torch.cuda.synchronize()
    if not torch.allclose(out, ref, rtol=1e-4, atol=1e-4 * float(ref.abs().max())):
        failures.append(("fused gemm allreduce", float((out - ref).abs().max())))
    allx = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(allx, out.contiguous())
    if not all(torch.equal(a, allx[0]) for a in allx):
        failures.append(("fused gemm allreduce not identical across ranks",))
    # graph capture and replay
    n = 4096
    x = comm.view(n)
    src = torch.empty(n, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        x.copy_(src)
        comm.all_reduce_(x)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        x.copy_(src)
        comm.all_reduce_(x)
    for it in range(3):
        src.copy_(torch.full((n,), float(rank + 1 + it), device="cuda"))
        graph.replay()
        torch.cuda.synchronize()
        want = float(sum(r + 1 + it for r in range(world)))
        if not torch.all(x == want):
            failures.append(("peer allreduce graph replay", it, float(x[0])))
    del graph
    # expert-parallel combine (muk_ep_gather_bf16): rank r owns the sorted rows of
    # experts [2r, 2r + 2); afterwards every rank holds every owner's rows, also
    # when the call is replayed from a CUDA graph
    T, H, E = 37, 256, 2 * world
    offs = torch.tensor([0, 5, 5, 20, 33, 37, 37, 37, 37][:E + 1] + [37] * max(0, E + 1 - 9),
                        device="cuda", dtype=torch.int32)[:E + 1]
    offs[-1] = T
    rows = comm.rows_view(T, H)
    lo, hi = int(offs[2 * rank]), int(offs[2 * rank + 2])
    val = torch.arange(T, device="cuda", dtype=torch.float32)[:, None] + 1000.0 * torch.arange(
        H, device="cuda", dtype=torch.float32)[None, :] / H
    want = val.bfloat16()
    rows.fill_(float("nan"))
    rows[lo:hi] = want[lo:hi]
    comm.ep_gather_(rows, offs, 2 * rank, 2 * rank + 2)
    torch.cuda.synchronize()
    if not torch.equal(rows, want):
        failures.append(("ep gather", int((rows != want).sum())))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    src = torch.zeros(T, H, device="cuda", dtype=torch.bfloat16)
    with torch.cuda.stream(side):
        rows[lo:hi] = src[lo:hi]
        comm.ep_gather_(rows, offs, 2 * rank, 2 * rank + 2)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rows[lo:hi] = src[lo:hi]
        comm.ep_gather_(rows, offs, 2 * rank, 2 * rank + 2)
    for it in range(3):
        src.copy_((val + it).bfloat16())
        graph.replay()
        torch.cuda.synchronize()
        if not torch.equal(rows, (val + it).bfloat16()):
            failures.append(("ep gather graph replay", it))
    del graph
    comm.close()
    dist.barrier()


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    from mu_b200.core.config import (CacheConfig, EngineConfig, MuConfig, SamplingParams,
                                     SchedulerConfig)
    from mu_b200.serving.engine import StepEngine
    from mu_b200.serving.worker import MuWorker, WorkerRequest

    worst = {}
    failures = []
    check_peer_allreduce(rank, world, failures)
    # (model, CUDA graphs, expert parallel, all-reduce: peer memory or NCCL,
    # expert combine, Llama step form)
    # "peer": GEMM + reduce-scatter fused; "peer-split": GEMM, then the push kernel
    # expert-parallel cases combine expert outputs by the bf16 row exchange
    # ("gather", the default) or the f32 all-reduce ("allreduce").
    # Llama steps under peer memory: "rs-norm" (default: reduce-scatter, residual
    # + norm on the owned rows, all-gather of x) from the native executor or the
    # Python step, or "allreduce" (all-reduce, then the replicated residual/norm).
    # Deep steps under peer memory run the native executor ("python": the
    # per-kernel step)
    for name, graphs, ep, comm, combine, form in (
            ("llama_tiny", False, False, "nccl", "-", "-"),
            ("llama_tiny", True, False, "peer", "-", "rs-norm"),
            ("llama_tiny", False, False, "peer-split", "-", "rs-norm"),
            ("llama_tiny", False, False, "peer", "-", "rs-norm-python"),
            ("llama_tiny", False, False, "peer-split", "-", "rs-norm-python"),
            ("llama_tiny", True, False, "peer", "-", "allreduce"),
            ("deep_tiny", False, False, "nccl", "-", "-"),
            ("deep_tiny", True, False, "peer", "-", "-"),
            ("deep_tiny", True, True, "peer-split", "gather", "-"),
            ("deep_tiny", False, True, "peer", "allreduce", "-"),
            ("deep_tiny", False, True, "peer", "gather", "python")):
        os.environ["MU_TP_COMM"] = "nccl" if comm == "nccl" else "peer"
        os.environ["MU_TP_FUSED"] = "0" if comm == "peer-split" else "1"
        os.environ["MU_EP_COMBINE"] = "allreduce" if combine == "allreduce" else "gather"
        os.environ["MU_TP_NORM"] = "0" if form == "allreduce" else "1"
        os.environ["MU_NATIVE_STEP"] = "0" if form in ("rs-norm-python", "python") else "1"
        shape, cfg, sd, d, prompts = load_tiny(name)
        ec = EngineConfig(model=cfg, mu=MuConfig(enabled=True), tensor_parallel_size=world,
                          expert_parallel=ep,
                          cache=CacheConfig(max_seq_len=256, max_num_blocks=512, max_num_seqs=16),
                          scheduler=SchedulerConfig(max_batch_size=8, max_num_batched_tokens=2048))
        w = MuWorker(ec, f"cuda:{torch.cuda.current_device()}")
        w.load_state_dict(shape.arch, cfg, sd)
        w.use_graphs = graphs
        if form.startswith("rs-norm"):
            assert w.model.tp_norm(), "peer-memory TP should take the reduce-scatter + norm path"
        if comm != "nccl":
            assert w.model.vocab_slice() is not None, "peer-memory TP: vocabulary-parallel head"
        toks = d["tokens"]
        R, n = toks.shape
        steps = list(d["logit_steps"])
        for r in range(R):
            assert w.allocate_request(f"r{r}")
        err = 0.0
        step_err = []
        for i in range(n):
            if i == 0:
                reqs = [WorkerRequest(f"r{r}", torch.tensor([prompts[r]]), is_prefill=True)
                        for r in range(R)]
            else:
                reqs = [WorkerRequest(f"r{r}", torch.tensor([[int(toks[r, i - 1])]]),
                                      is_prefill=False) for r in range(R)]
            outs = w.execute(reqs)
            for r, o in enumerate(outs):
                assert o.error is None, o.error
                if i in steps:
                    lg = o.logits.float().cpu().numpy().reshape(-1)
                    e = float(np.abs(lg - d["logits"][r, steps.index(i)]).max())
                    err = max(err, e)
                    step_err.append((i, r, round(e, 5)))
        for r in range(R):
            w.free_request(f"r{r}")
        worst[f"{name}/graphs={graphs}/ep={ep}/{comm}/{combine}/{form}"] = err
        if err > 2e-2:
            failures.append((name, graphs, rank, err, [x for x in step_err if x[2] > 2e-2][:6]))
        eng = StepEngine(w, ec)
        for r in range(R):
            eng.add_request(prompts[r], SamplingParams(temperature=0.0, top_k=0, top_p=1.0,
                                                       repetition_penalty=1.0, max_tokens=n),
                            f"g{r}")
        eng.run_to_completion()
        gen = torch.tensor([eng.requests[f"g{r}"].output_token_ids for r in range(R)],
                           device="cuda")
        allg = [torch.empty_like(gen) for _ in range(world)]
        dist.all_gather(allg, gen)
        for g in allg:
            if not torch.equal(g, allg[0]):
                failures.append((name, graphs, rank, "ranks generated different tokens"))
        # greedy tokens equal the reference's up to its first near tie
        for r in range(R):
            for i, t in enumerate(gen[r].tolist()):
                if t != int(toks[r, i]):
                    if d["top2_gap"][r, i] > 0.05:
                        failures.append((name, graphs, rank, f"greedy token r{r} step {i}"))
                    break
        # sampled generation (temperature 0.8, top-p 0.9, seeded): the ranks
        # combine the vocabulary columns before sampling and draw the same tokens
        for r in range(R):
            eng.add_request(prompts[r], SamplingParams(temperature=0.8, top_k=0, top_p=0.9,
                                                       repetition_penalty=1.1, max_tokens=8,
                                                       seed=1234 + r), f"s{r}")
        eng.run_to_completion()
        smp = torch.tensor([eng.requests[f"s{r}"].output_token_ids for r in range(R)],
                           device="cuda")
        alls = [torch.empty_like(smp) for _ in range(world)]
        dist.all_gather(alls, smp)
        for g in alls:
            if not torch.equal(g, alls[0]):
                failures.append((name, graphs, rank, "ranks sampled different tokens"))
        w.close()  # graphs (which may hold NCCL calls) and peer mappings go before the group
        del eng, w
    from mu_b200 import _lib

    if _lib.device_error() != 0:
        failures.append("device error")
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if failures:
        print(f"rank {rank}: FAIL {failures} worst {worst}", flush=True)
        sys.exit(1)
    print(f"rank {rank}: tp={world} ok, worst logit max-abs {worst}", flush=True)


if __name__ == "__main__":
    main()
