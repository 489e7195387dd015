"""One rank of the peer-memory expert-parallel check (launched by
test_gpu_ep_p2p.py through torch.distributed.run, one process per GPU).

Every rank builds the same seeded layer, keeps its block of experts, and
checks its own tokens' outputs from the peer-memory exchange against the
all-to-all exchange over the process group (the same kernels on the same
rows: equal bits) and against the whole layer on one GPU (within the f32 /
bf16 bars), then repeats from a CUDA graph.  24 tokens per rank take the
one-launch route+plan of the decode front, 100 the router and plan kernels."""
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "qmoe-rs_b200", "python"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import helpers  # noqa: E402
from helpers import rel_err  # noqa: E402
from qmoe_b200 import ExpertParallelMoE, MoEConfig, QMoELayer, default_context  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    E, K, H, I, Is = 16, 4, 512, 256, 256
    cfg = MoEConfig(E, K, H, I, shared_intermediate_dim=Is)
    experts, shared, gate_w = helpers.synth_layer(E, H, I, Is, seed=5, device=dev)
    epr = E // world
    mine = experts[rank * epr:(rank + 1) * epr]
    ctx = default_context(local)
    full = QMoELayer(cfg, gate_w, experts, shared=shared, ctx=ctx)
    for T, dtype, tol in ((24, torch.float32, 1e-4), (24, torch.bfloat16, 2e-2),
                          (100, torch.float32, 1e-4)):
        g = torch.Generator().manual_seed(100 + rank)
        xs = [torch.randn(T, H, generator=g).to(dtype).to(dev) for _ in range(3)]
        p2p = ExpertParallelMoE(cfg, gate_w, mine, rank, world, shared=shared, capacity=T,
                                ctx=ctx, exchange="p2p", dtype=dtype)
        nccl = ExpertParallelMoE(cfg, gate_w, mine, rank, world, shared=shared, capacity=T, ctx=ctx)
        outs = []
        for x in xs:                        # consecutive forwards: sequence numbers advance
            a = p2p.forward(x)
            b = nccl.forward(x)
            ref = full.forward(x)
            torch.cuda.synchronize()
            assert torch.equal(a, b), f"rank {rank}: p2p and all-to-all exchanges differ"
            err = rel_err(a.float().cpu().numpy(), ref.float().cpu().numpy())
            assert err <= tol, f"rank {rank}: rel err {err} vs the one-GPU layer"
            outs.append(a.clone())
        # the whole forward from a CUDA graph (exchange flags included)
        dist.barrier()
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                og = p2p.forward(xs[0])
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(og, outs[0]), f"rank {rank}: graph replay differs"
        del graph
        p2p.layer.ctx.synchronize()        # raises if any bounded wait gave up
        dist.barrier()
        p2p.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: ok", flush=True)


if __name__ == "__main__":
    main()
