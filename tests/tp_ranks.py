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
    for name, graphs, ep in (("llama_tiny", False, False), ("llama_tiny", True, False),
                             ("deep_tiny", False, False), ("deep_tiny", True, False),
                             ("deep_tiny", False, True)):
        shape, cfg, sd, d, prompts = load_tiny(name)
        ec = EngineConfig(model=cfg, mu=MuConfig(enabled=True), tensor_parallel_size=world,
                          expert_parallel=ep,
                          cache=CacheConfig(max_seq_len=256, max_num_blocks=512, max_num_seqs=16),
                          scheduler=SchedulerConfig(max_batch_size=8, max_num_batched_tokens=2048))
        w = MuWorker(ec, f"cuda:{torch.cuda.current_device()}")
        w.load_state_dict(shape.arch, cfg, sd)
        w.use_graphs = graphs
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
        worst[f"{name}/graphs={graphs}/ep={ep}"] = err
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
        w._graphs.clear()  # graphs holding NCCL calls must go before the process group
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
