"""All-reduce + residual add + RMSNorm microbenchmark over N GPUs of one node.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m kavor_b200.profile_allreduce [--hidden 1024,4096,5120] [--tokens 1,16,256,4096,16384]

For every (hidden, tokens) it times, on every rank with CUDA events around a
CUDA graph of ``--iters`` calls (max over ranks), the fused NVLink kernel
``kvb_allreduce_add_rmsnorm`` in its automatic mode and each explicit mode
(peer one-shot / two-shot; switch-reduced one-shot / two-shot when the area has
an NVLink multicast mapping), against the reference's sequence: NCCL
``all_reduce`` of the [T, H] bf16 partial followed by the add+RMSNorm kernel. Inputs are x ~ N(0, 1) bf16,
w ~ N(1, 0.1), eps 1e-6; consecutive calls alternate two partial buffers, as
the layers of a forward do. Prints one JSON line per case on rank 0 with the
average call time and the bus bandwidth 2 (N-1)/N T H 2 bytes / time.

``--halves``: also times the decode micro-batch form (Config.decode_microbatches
= 2): two communicators, grids capped at DecodeMicrobatches.MAX_BLOCKS, each
reducing half of the T rows, the second on another stream, both in flight
together (``halves_us`` = time per pair of half calls).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from kavor_b200 import _kernels as K
from kavor_b200 import _lib
from kavor_b200.layers.allreduce import DecodeMicrobatches, TPAllReduce


def _time_graph(fn, iters: int, warmup: int) -> float:
    """Seconds per call of ``fn`` (max over ranks), replayed from one CUDA graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(warmup):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3 / iters], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    torch.cuda.synchronize()
    dist.barrier()
    return float(t.item())


def fused_vs_nccl(ar: TPAllReduce, tokens: list[int], iters: int = 20, warmup: int = 3, seed: int = 1234) -> list[dict]:
    """Per token count: the fused kernel in its automatic mode against NCCL
    all_reduce followed by the add+RMSNorm kernel (the reference's sequence),
    on the communicator ``ar`` (its hidden size, at most ar.max_tokens rows);
    every rank calls it, rows are returned on every rank."""
    rank, world = dist.get_rank(), dist.get_world_size()
    H, dev = ar.hidden, ar.device
    g = torch.Generator(device=dev).manual_seed(seed + rank)
    tmax = max(tokens)
    w = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
    for i in range(2):
        ar.buffers[i][:tmax].copy_(torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16))
    nccl_x = [torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    res = torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(tmax, H, device=dev, dtype=torch.bfloat16)
    rows = []
    for T in tokens:
        def fused(i, T=T):
            _lib.call("kvb_allreduce_add_rmsnorm", ar.comm, i & 1, res.data_ptr(), res.data_ptr(), out.data_ptr(),
                      w.data_ptr(), T, H, 1e-6, 0, torch.cuda.current_stream().cuda_stream)

        def nccl(i, T=T):
            x = nccl_x[i & 1][:T]
            dist.all_reduce(x)
            K.add_rmsnorm(x, res[:T], w, 1e-6, out=out[:T])

        bus = 2 * (world - 1) / world * T * H * 2
        tf, tn = _time_graph(fused, iters, warmup), _time_graph(nccl, iters, warmup)
        rows.append({"hidden": H, "tokens": T, "fused_us": tf * 1e6, "nccl_plus_add_rmsnorm_us": tn * 1e6,
                     "fused_busbw_gbs": bus / tf / 1e9, "nccl_busbw_gbs": bus / tn / 1e9})
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--hidden", default="1024,4096,5120")
    ap.add_argument("--tokens", default="1,16,256,4096,16384")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--backend", default="auto", choices=["auto", "symmetric", "ipc"])
    ap.add_argument("--halves", action="store_true", help="also time two half-size calls in flight together")
    a = ap.parse_args(argv)
    hiddens = [int(x) for x in a.hidden.split(",")]
    tokens = [int(x) for x in a.tokens.split(",")]
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    for H in hiddens:
        tmax = max(tokens)
        ar = TPAllReduce(tmax, H, dev, backend=a.backend)
        halves = None
        if a.halves:  # the decode micro-batches' communicators and per-half rows
            hmax = (tmax + 1) // 2
            halves = [TPAllReduce(hmax, H, dev, backend=a.backend, max_blocks=DecodeMicrobatches.MAX_BLOCKS)
                      for _ in range(2)]
            for c in halves:
                for i in range(2):
                    c.buffers[i].copy_(torch.randn(hmax, H, device=dev, generator=g).to(torch.bfloat16))
            half_res = [torch.randn(hmax, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
            half_out = [torch.empty(hmax, H, device=dev, dtype=torch.bfloat16) for _ in range(2)]
            side = torch.cuda.Stream(dev)
        modes = (("fused_auto", 0), ("fused_one_shot", 1), ("fused_two_shot", 2))
        if ar.multicast:
            modes += (("fused_switch_one_shot", 3), ("fused_switch_two_shot", 4))
        w = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).to(torch.bfloat16)
        for i in range(2):
            ar.buffers[i].copy_(torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16))
        nccl_x = [torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
        res = torch.randn(tmax, H, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(tmax, H, device=dev, dtype=torch.bfloat16)
        for T in tokens:
            row = {"world": world, "hidden": H, "tokens": T, "backend": ar.backend,
                   "bus_bytes": 2 * (world - 1) / world * T * H * 2}

            def fused(mode):
                def fn(i):
                    _lib.call("kvb_allreduce_add_rmsnorm", ar.comm, i & 1, res.data_ptr(), res.data_ptr(),
                              out.data_ptr(), w.data_ptr(), T, H, 1e-6, mode, torch.cuda.current_stream().cuda_stream)
                return fn

            for name, mode in modes:
                t = _time_graph(fused(mode), a.iters, a.warmup)
                row[name + "_us"] = t * 1e6

            if halves is not None and T >= 2:
                def pair(i):
                    main = torch.cuda.current_stream()
                    side.wait_stream(main)
                    for m, n in enumerate((T - T // 2, T // 2)):
                        st = main if m == 0 else side
                        with torch.cuda.stream(st):
                            _lib.call("kvb_allreduce_add_rmsnorm", halves[m].comm, i & 1, half_res[m].data_ptr(),
                                      half_res[m].data_ptr(), half_out[m].data_ptr(), w.data_ptr(), n, H, 1e-6, 0,
                                      st.cuda_stream)
                    main.wait_stream(side)

                row["halves_us"] = _time_graph(pair, a.iters, a.warmup) * 1e6

            def nccl(i):
                x = nccl_x[i & 1][:T]
                dist.all_reduce(x)
                K.add_rmsnorm(x, res[:T], w, 1e-6, out=out[:T])

            t = _time_graph(nccl, a.iters, a.warmup)
            row["nccl_plus_add_rmsnorm_us"] = t * 1e6
            row["fused_auto_busbw_gbs"] = row["bus_bytes"] / (row["fused_auto_us"] * 1e-6) / 1e9
            row["nccl_busbw_gbs"] = row["bus_bytes"] / (t) / 1e9
            row["device_error_bits"] = _lib.device_error(clear=True)
            if rank == 0:
                print(json.dumps(row), flush=True)
        del nccl_x, res, out
        if halves is not None:
            for c in halves:
                c.close()
        ar.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
