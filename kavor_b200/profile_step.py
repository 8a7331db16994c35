"""Per-kernel share of one decode step (Qwen3 decode graph, any TP).

    python -m kavor_b200.profile_step [--model Qwen3-8B --batch 256 --context 1024]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m kavor_b200.profile_step --gpus N

Builds the same runner as bench.py (random-init weights, B sequences at the
given context, TP = number of ranks), replays the captured decode graph five
times under torch.profiler (CUPTI kernel records) and prints, on rank 0, the
table of kernels by total device time. The profiler stretches absolute times:
read the shares, and take step times from bench.py.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys
import tempfile

import torch
import torch.distributed as dist


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--model", default="Qwen3-8B")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--replays", type=int, default=5)
    ap.add_argument("--microbatches", type=int, choices=[1, 2], default=1,
                    help="TP > 1: decode as two halves on two streams (Config.decode_microbatches)")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    else:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=1, rank=0, device_id=dev)
    from torch.profiler import ProfilerActivity, profile

    from kavor_b200.config import Config, write_model_dir
    from kavor_b200.engine.block_manager import BlockManager
    from kavor_b200.engine.model_runner import ModelRunner
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    B, ctx0 = a.batch, a.context
    blocks_per_seq = (ctx0 + 64 + 255) // 256
    model_dir = write_model_dir(os.path.join(tempfile.mkdtemp(prefix="kvb_prof_"), f"r{rank}"), a.model)
    cfg = Config(model_dir, load_format="dummy", seed=0, tensor_parallel_size=world,
                 max_model_len=(blocks_per_seq + 1) * 256, max_num_seqs=B, max_num_batched_tokens=4096,
                 num_kvcache_blocks=B * blocks_per_seq + 8, rdzv_port=1, graph_batch_sizes=(B,),
                 decode_microbatches=a.microbatches)
    runner = ModelRunner(cfg, rank, None)
    Sequence.block_size = 256
    bm = BlockManager(cfg.num_kvcache_blocks, 256, enable_prefix_cache=False)
    g = torch.Generator().manual_seed(0)
    seqs = []
    for _ in range(B):
        s = Sequence(torch.randint(0, 151936, (ctx0,), generator=g).tolist(),
                     SamplingParams(temperature=0.6, max_tokens=10 ** 6, ignore_eos=True))
        bm.allocate_prefill(s, 0)
        s.num_cached_tokens = ctx0 - 1
        s.is_prefill = False
        seqs.append(s)
    runner.run(seqs, False)
    graph = runner.graphs[B]
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(a.replays):
            graph.replay()
        torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=90),
              flush=True)
    del graph
    runner.exit()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
