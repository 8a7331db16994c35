"""Microbenchmark one kavor_b200 kernel on a synthetic case (used for ncu captures).

    python -m kavor_b200.profile_kernels decode_attn --batch 64 --context 1024 --hq 32 --hkv 8
    python -m kavor_b200.profile_kernels prefill_attn[_warp_mma] --batch 4 --context 2048 --hq 32 --hkv 8
    python -m kavor_b200.profile_kernels qknorm_rope_store|add_rmsnorm|silu_mul|sample --batch 256
    python -m kavor_b200.profile_kernels gemm --batch M --inter N --hidden K   (gemm_cublas: torch/cuBLAS)

Allocates only the kernel's own inputs (a few hundred MB at most), runs
``--warmup`` untimed launches, then ``--iters`` launches captured in one CUDA
graph and timed (one replay) with CUDA events on the launching stream — device
time without host launch overhead (``--eager`` times plain launches instead) —
rotating over ``--copies`` copies of the inputs so consecutive launches do not
hit in L2 (use enough copies that they exceed the 126 MB L2), and prints one
JSON line with the average launch time and the achieved algorithmic bandwidth.
"""
from __future__ import annotations

import argparse
import json

import torch

from kavor_b200 import _kernels as K


def _decode_attn(a, dev):
    bs, hd = 256, 128
    nb = (a.context + bs - 1) // bs
    pools = [torch.randn(a.batch * nb, 2, bs, a.hkv, hd, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    tables = torch.arange(a.batch * nb, dtype=torch.int32, device=dev).view(a.batch, nb)
    ctx = torch.full((a.batch,), a.context, dtype=torch.int32, device=dev)
    q = torch.randn(a.batch, a.hq, hd, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    nbytes = a.batch * a.context * a.hkv * hd * 2 * 2 + 2 * q.numel() * 2

    def run(i):
        p = pools[i % len(pools)]
        K.paged_decode_attention(q, p[:, 0], p[:, 1], tables, ctx, hd ** -0.5, out=out, num_splits=a.splits)

    return run, nbytes, 0


def _prefill_attn(a, dev, tensor_cores=True):
    hd = 128
    T = a.batch * a.context
    qkv = [torch.randn(T, (a.hq + 2 * a.hkv) * hd, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    cu = torch.arange(0, T + 1, a.context, dtype=torch.int32, device=dev)
    out = torch.empty(T, a.hq, hd, device=dev, dtype=torch.bfloat16)
    flops = 4 * a.hq * hd * a.batch * a.context * (a.context + 1) // 2

    def run(i):
        x = qkv[i % len(qkv)]
        K.prefill_attention(x[:, :a.hq * hd].view(T, a.hq, hd), x[:, a.hq * hd:(a.hq + a.hkv) * hd].view(T, a.hkv, hd),
                            x[:, (a.hq + a.hkv) * hd:].view(T, a.hkv, hd), cu, cu, a.context, hd ** -0.5, out=out,
                            tensor_cores=tensor_cores)

    return run, 2 * (qkv[0].numel() + out.numel()), flops


def _qknorm_rope_store(a, dev):
    from kavor_b200.layers.rotary_embedding import build_cos_sin_cache

    hd, bs = 128, 256
    T = a.batch
    qkv = [torch.randn(T, (a.hq + 2 * a.hkv) * hd, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    pool = torch.zeros((T + bs - 1) // bs, 2, bs, a.hkv, hd, device=dev, dtype=torch.bfloat16)
    slots = torch.arange(T, dtype=torch.int32, device=dev)
    pos = torch.arange(T, device=dev)
    cache = build_cos_sin_cache(hd, max(T, 2), 1e6).to(dev).contiguous()
    w = torch.ones(hd, device=dev, dtype=torch.bfloat16)

    def run(i):
        K.qknorm_rope_store(qkv[i % len(qkv)], a.hq, a.hkv, hd, w, w, 1e-6, pos, cache, False, pool[:, 0],
                            pool[:, 1], slots)

    return run, 2 * qkv[0].numel() * 2, 0


def _add_rmsnorm(a, dev):
    H = a.hidden
    xs = [torch.randn(a.batch, H, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    rs = [torch.randn(a.batch, H, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = torch.empty(a.batch, H, device=dev, dtype=torch.bfloat16)

    def run(i):
        K.add_rmsnorm(xs[i % len(xs)], rs[i % len(rs)], w, 1e-6, out=out)

    return run, 4 * a.batch * H * 2, 0


def _silu_mul(a, dev):
    xs = [torch.randn(a.batch, 2 * a.inter, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    out = torch.empty(a.batch, a.inter, device=dev, dtype=torch.bfloat16)

    def run(i):
        K.silu_mul(xs[i % len(xs)], out=out)

    return run, 3 * a.batch * a.inter * 2, 0


def _sample(a, dev):
    logits = [torch.randn(a.batch, a.vocab, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    temps = torch.full((a.batch,), 0.6, device=dev)
    seed = torch.zeros((), dtype=torch.int32, device=dev)
    out = torch.empty(a.batch, dtype=torch.int64, device=dev)

    def run(i):
        K.sample(logits[i % len(logits)], temps, seed, out=out)

    return run, a.batch * a.vocab * 2, 0


def _gemm(a, dev, use_torch=False):
    M, N, K_ = a.batch, a.inter, a.hidden
    xs = [torch.randn(M, K_, device=dev).to(torch.bfloat16) for _ in range(a.copies)]
    ws = [(torch.randn(N, K_, device=dev) * 0.02).to(torch.bfloat16) for _ in range(a.copies)]
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)

    def run(i):
        if use_torch:
            torch.matmul(xs[i % len(xs)], ws[i % len(ws)].t(), out=out)
        else:
            K.gemm(xs[i % len(xs)], ws[i % len(ws)], out=out, splits=a.splits)

    return run, 2 * (N * K_ + M * K_ + M * N), 2 * M * N * K_


CASES = {"decode_attn": _decode_attn, "prefill_attn": _prefill_attn,
         "prefill_attn_warp_mma": lambda a, dev: _prefill_attn(a, dev, tensor_cores=False),
         "qknorm_rope_store": _qknorm_rope_store,
         "add_rmsnorm": _add_rmsnorm, "silu_mul": _silu_mul, "sample": _sample, "gemm": _gemm,
         "gemm_cublas": lambda a, dev: _gemm(a, dev, use_torch=True)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("kernel", choices=sorted(CASES))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=12288)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--copies", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--eager", action="store_true", help="time eager launches (includes host overhead)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    run, nbytes, flops = CASES[a.kernel](a, dev)
    for i in range(a.warmup):
        run(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if a.eager:
        e0.record()
        for i in range(a.iters):
            run(i)
        e1.record()
    else:
        # launches captured once and replayed: device time only, no host overhead
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(a.iters):
                run(i)
        graph.replay()
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / a.iters
    res = {"kernel": a.kernel, "avg_launch_us": t * 1e6, "algorithmic_bytes": nbytes, "gbs": nbytes / t / 1e9}
    if flops:
        res["tflops"] = flops / t / 1e12
    res.update({k: v for k, v in vars(a).items() if k not in ("kernel",)})
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
