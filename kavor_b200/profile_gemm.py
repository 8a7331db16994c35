"""GEMM sweep over the Qwen3-8B decode projections: kvb_gemm_bf16 (automatic
plan and every forced K split), kvb_gemm_silu_bf16 for the gate-up shapes, and
cuBLAS (torch.matmul) on the same operands.

    python -m kavor_b200.profile_gemm [M,M,...] [--splits 1,2,3,4,8,16] [--l2-prefetch 0,4] [--pair]

(default M 1,64,256; K splits 1,2,4,8,16; L2 prefetch distance 0). Every
variant runs at every L2 prefetch distance given (kvb_gemm_set_l2_prefetch);
labels carry a "_pfN" suffix when N > 0. --pair adds the CTA-pair kernel
(kvb_gemm_pair_bf16): "pair_auto" and "pair_sN" for K splits N <= 8, and
"g_pair" (kvb_gemm_pair_silu_bf16) for the gate-up shapes. The stream-K
CTA-pair kernel (kvb_gemm_sk_bf16, "sk"; "g_sk" = kvb_gemm_sk_silu_bf16 for
the gate-up shapes) is always measured; --no-single skips the single-CTA
kernel's split sweep.

Shapes: QKV, O, gate-up, down and LM head of Qwen3-8B at TP=1 and TP=8. Each
timing is one replay of a CUDA graph of 20 launches (device time, CUDA events),
rotating over enough weight copies (>= 400 MB) that no launch finds its weight
in L2. Prints one JSON line per (M, shape): [us, GB/s of weight + x + y bytes,
token tile, max |y - cuBLAS|] per variant, then prefill-size lines (M = 2048,
8192) in TFLOP/s.
"""
from __future__ import annotations

import argparse
import json

import torch

from kavor_b200 import _kernels as K
from kavor_b200 import _lib


def _timeit(fn, iters=20):
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("ms", nargs="?", default="1,64,256")
    ap.add_argument("--splits", default="1,2,4,8,16")
    ap.add_argument("--l2-prefetch", default="0")
    ap.add_argument("--pair", action="store_true")
    ap.add_argument("--no-single", action="store_true")
    ap.add_argument("--launches", type=int, default=0,
                    help="profiler mode: only N plain launches of --impl on --shape at the first M (no timing)")
    ap.add_argument("--shape", default="lm_head_tp1")
    ap.add_argument("--impl", default="sk", choices=["sk", "sk_silu", "single", "cublas"])
    ap.add_argument("--sk-plans", default="", help="also time the stream-K GEMM at forced (token tile x pairs), "
                    "e.g. 128x32,256x64 (labels sk_<mt>x<pairs>)")
    a = ap.parse_args(argv)
    split_list = [int(v) for v in a.splits.split(",")]
    pf_list = [int(v) for v in a.l2_prefetch.split(",")]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load()
    shapes = []
    for tp in (1, 8):
        for name, N, Kd in (("qkv", 6144 // tp, 4096), ("o", 4096, 4096 // tp), ("gate_up", 24576 // tp, 4096),
                            ("down", 4096, 12288 // tp), ("lm_head", 151936 // tp, 4096)):
            shapes.append((f"{name}_tp{tp}", N, Kd))
    Ms = [int(x) for x in a.ms.split(",")]
    if a.launches:
        return _plain_launches(dict((n, (N, Kd)) for n, N, Kd in shapes)[a.shape], Ms[0], a.impl, a.launches, dev)
    for M in Ms:
        for name, N, Kd in shapes:
            wbytes = N * Kd * 2
            copies = max(2, -(-400_000_000 // wbytes))
            ws = [(torch.randn(N, Kd, device=dev) * 0.02).to(torch.bfloat16) for _ in range(min(copies, 16))]
            x = torch.randn(M, Kd, device=dev).to(torch.bfloat16)
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            ref = torch.matmul(x, ws[0].t())
            res = {"M": M, "shape": name, "N": N, "K": Kd, "copies": len(ws), "plan": K.gemm_plan(M, N, Kd)}
            nbytes = wbytes + M * Kd * 2 + M * N * 2
            K.gemm_sk(x, ws[0], out=out)
            err = (out.float() - ref.float()).abs().max().item()
            t = _timeit(lambda i: K.gemm_sk(x, ws[i % len(ws)], out=out))
            res["sk"] = [round(t, 2), round(nbytes / t / 1e3), K.gemm_sk_plan(M, N, Kd)["pairs"], round(err, 4)]
            if name.startswith("gate_up"):
                og = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16)
                t = _timeit(lambda i: K.gemm_sk_silu(x, ws[i % len(ws)], out=og))
                res["g_sk"] = [round(t, 2), round(nbytes / t / 1e3), K.gemm_sk_plan(M, N // 2, Kd, True)["pairs"]]
            for spec in [v for v in a.sk_plans.split(",") if v]:
                mt, pairs = (int(v) for v in spec.split("x"))
                if mt > 16 and mt // 2 >= M:
                    continue
                K.gemm_sk_set_plan(mt, pairs)
                try:
                    t = _timeit(lambda i: K.gemm_sk(x, ws[i % len(ws)], out=out))
                    res[f"sk_{mt}x{pairs}"] = round(t, 2)
                    if name.startswith("gate_up"):
                        t = _timeit(lambda i: K.gemm_sk_silu(x, ws[i % len(ws)], out=og))
                        res[f"g_sk_{mt}x{pairs}"] = round(t, 2)
                finally:
                    K.gemm_sk_set_plan(0, 0)
            for pf in ([] if a.no_single else pf_list):
                K.gemm_set_l2_prefetch(pf)
                sfx = f"_pf{pf}" if pf else ""
                for splits in [0] + split_list:
                    label = ("auto" if splits == 0 else f"s{splits}") + sfx
                    p = K.gemm_plan(M, N, Kd, splits)
                    if splits and p["splits"] != splits:
                        continue
                    K.gemm(x, ws[0], out=out, splits=splits)
                    err = (out.float() - ref.float()).abs().max().item()
                    t = _timeit(lambda i: K.gemm(x, ws[i % len(ws)], out=out, splits=splits))
                    res[label] = [round(t, 2), round(nbytes / t / 1e3), p["mt"], round(err, 4)]
                if name.startswith("gate_up"):
                    og = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16)
                    for splits in [0] + [s for s in split_list if s <= 8]:
                        label = ("g_auto" if splits == 0 else f"g_s{splits}") + sfx
                        p = K.gemm_plan(M, N // 2, Kd, splits, True)
                        if splits and p["splits"] != splits:
                            continue
                        t = _timeit(lambda i: K.gemm_silu(x, ws[i % len(ws)], out=og, splits=splits))
                        res[label] = [round(t, 2), round(nbytes / t / 1e3), p["mt"]]
            K.gemm_set_l2_prefetch(0)
            if a.pair:
                for splits in [0] + [s for s in split_list if s <= 8]:
                    p = K.gemm_pair_plan(M, N, Kd, splits)
                    if splits and p["splits"] != splits:
                        continue
                    label = "pair_auto" if splits == 0 else f"pair_s{splits}"
                    K.gemm_pair(x, ws[0], out=out, splits=splits)
                    err = (out.float() - ref.float()).abs().max().item()
                    t = _timeit(lambda i: K.gemm_pair(x, ws[i % len(ws)], out=out, splits=splits))
                    res[label] = [round(t, 2), round(nbytes / t / 1e3), p["mt"], round(err, 4)]
                if name.startswith("gate_up"):
                    og = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16)
                    t = _timeit(lambda i: K.gemm_pair_silu(x, ws[i % len(ws)], out=og))
                    res["g_pair"] = [round(t, 2), round(nbytes / t / 1e3), K.gemm_pair_plan(M, N // 2, Kd, 0, True)["mt"],
                                     K.gemm_pair_plan(M, N // 2, Kd, 0, True)["splits"]]
            t = _timeit(lambda i: torch.matmul(x, ws[i % len(ws)].t(), out=out))
            res["cublas"] = [round(t, 2), round(nbytes / t / 1e3)]
            res["device_error_bits"] = _lib.device_error(clear=True)
            print(json.dumps(res), flush=True)
            del ws
            torch.cuda.empty_cache()
    for M in (2048, 8192):
        for name, N, Kd in (("qkv_tp1", 6144, 4096), ("gate_up_tp1", 24576, 4096), ("down_tp1", 4096, 12288)):
            w = (torch.randn(N, Kd, device=dev) * 0.02).to(torch.bfloat16)
            x = torch.randn(M, Kd, device=dev).to(torch.bfloat16)
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            res = {"M": M, "shape": name, "N": N, "K": Kd, "plan": K.gemm_plan(M, N, Kd)}
            res["auto_us"] = _timeit(lambda i: K.gemm(x, w, out=out), 10)
            res["cublas_us"] = _timeit(lambda i: torch.matmul(x, w.t(), out=out), 10)
            for k in ("auto", "cublas"):
                res[k + "_tflops"] = 2 * M * N * Kd / res[k + "_us"] / 1e6
            print(json.dumps(res), flush=True)
    return 0


def _plain_launches(shape, M: int, impl: str, n: int, dev) -> int:
    """n back-to-back launches of one GEMM on fresh weights (for ncu: one
    shape, a few launches, a few GB on the device at most)."""
    N, Kd = shape
    x = torch.randn(M, Kd, device=dev).to(torch.bfloat16)
    ws = [(torch.randn(N, Kd, device=dev) * 0.02).to(torch.bfloat16) for _ in range(2)]
    for i in range(n):
        w = ws[i % 2]
        if impl == "sk":
            K.gemm_sk(x, w)
        elif impl == "sk_silu":
            K.gemm_sk_silu(x, w)
        elif impl == "single":
            K.gemm(x, w)
        else:
            torch.matmul(x, w.t())
    torch.cuda.synchronize()
    bits = _lib.device_error(clear=True)
    print(json.dumps({"M": M, "N": N, "K": Kd, "impl": impl, "launches": n, "device_error_bits": bits}))
    return 1 if bits else 0


if __name__ == "__main__":
    raise SystemExit(main())
