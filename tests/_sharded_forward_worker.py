"""Worker of tests/test_gpu_sharded.py, one process per GPU (torchrun):
the prefix LM with the N-sharded gate/up must give bit-identical hidden
states and KV cache to the single-GPU forward, eager and CUDA-graph
replayed."""

from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from pi05_pytorch_fast_b200 import _native as nat  # noqa: E402
from pi05_pytorch_fast_b200 import prefix_lm as plm  # noqa: E402
from pi05_pytorch_fast_b200.shard import MlpShard  # noqa: E402


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    graph = None
    try:
        cfg = plm.PrefixLMConfig(layers=2)
        full = plm.W4A4PrefixLM.random(cfg, dev, seed=11)
        sharded = plm.W4A4PrefixLM.random(cfg, dev, seed=11, shard=MlpShard(rank, world))
        embeds, pad = plm.synthetic_prefix(2, device=dev, seed=3)
        with torch.no_grad():
            ref = full.forward(embeds, pad)
            ref_h, ref_k = ref.hidden.clone(), [k.clone() for k in ref.keys]
            got = sharded.forward(embeds, pad)
            ok_eager = torch.equal(got.hidden.view(torch.int16), ref_h.view(torch.int16)) and all(
                torch.equal(a.view(torch.int16), b.view(torch.int16)) for a, b in zip(got.keys, ref_k))
            graph = plm.GraphedPrefixLM(sharded, 2, embeds.shape[1])
            out = graph.run(embeds, pad)
            torch.cuda.synchronize(dev)
            ok_graph = torch.equal(out.hidden.view(torch.int16), ref_h.view(torch.int16))
        bits = nat.device_error(clear=True)
        flag = torch.tensor([int(ok_eager), int(ok_graph), int(bits == 0)], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            print(f"sharded eager {bool(flag[0])} graph {bool(flag[1])} no-device-error {bool(flag[2])}")
            if bool(flag.all()):
                print("sharded ok")
    finally:
        del graph  # a graph holding NCCL work must go before the process group
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
