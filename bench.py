"""Decode-step benchmark of the kavor_b200 Qwen3 path (Qwen3-8B decode, the headline metric).

Workload: Qwen3-8B (random-init bf16, the reference checkpoint shapes), a
decode batch of 256 sequences whose context is 1024 tokens (block_size 256),
tensor parallel over the N GPUs of the launch (TP=N, one process per GPU,
NCCL). A step = one decode step of the whole batch: embedding, 36 layers,
LM head and sampling, replayed from the captured CUDA graph.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Printed on rank 0 as one JSON line:
* value / ms_per_step: device time (CUDA events, max over ranks) of K graph
  replays with the batch metadata already resident in HBM;
* e2e: the same metric through the public per-step API ModelRunner.run (host
  metadata build, one pinned host->device copy, graph replay, sampled token ids
  read back to the host), sequences growing by one token per step;
* roofline: the decode-attention kernel (dominant kernel: its K/V bytes are
  ~70% of the step's HBM bytes at TP1) timed alone over the layers' caches;
* step_roofline: whole-step HBM bytes (weights + KV) at the measured peak;
* cpu_baseline: the CPU oracle (reference algorithm) timed on the host cores;
* clocks: nvidia-smi samples taken during the timed region.
``--impl reference`` times the reference algorithm on the host CPU (the
oracle restatement; the reference's own GPU path needs flash-attn/Triton
kernels that are not part of this build) and prints the same line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="Qwen3-8B")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gemm", choices=["auto", "cublas", "tcgen05", "tcgen05_pair"], default="auto",
                    help="GEMM of the projections (Config.gemm_backend)")
    ap.add_argument("--gemm-l2-prefetch", type=int, default=0,
                    help="tcgen05 GEMM: weight K-steps prefetched into L2 ahead of the loads")
    ap.add_argument("--pdl", action="store_true", help="programmatic dependent launch of the package's kernels")
    ap.add_argument("--no-probes", action="store_true",
                    help="skip the one-GPU probes of the package's GEMM in place of cuBLAS")
    ap.add_argument("--microbatches", type=int, choices=[1, 2], default=1,
                    help="TP > 1: 2 runs the decode step as two halves on two streams (Config.decode_microbatches)")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the smaller decode batches (1, 16, 64) and, at TP > 1, the all-reduce microbenchmark")
    ap.add_argument("--e2e-pipelined", action="store_true",
                    help="e2e through ModelRunner.run_async with one step in flight (host work overlaps the GPU)")
    return ap.parse_args(argv)


# ----------------------------------------------------------------- helpers
def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def model_shape(name: str) -> dict:
    from kavor_b200.config import FAMILY_PRESETS, QWEN3_PRESETS

    if name in FAMILY_PRESETS:
        return dict(FAMILY_PRESETS[name])
    d = dict(QWEN3_PRESETS[name])
    d["vocab_size"] = 151936
    return d


class ClockSampler:
    """nvidia-smi samples (100 ms) of the SM clock and throttle reasons while running."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.lines: list[str] = []
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], 0.0, set()
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, f[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def max_over_ranks(x: float) -> float:
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    return x


def barrier():
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


# ----------------------------------------------------------------- CPU reference path
class CpuDecodeSample:
    """The CPU oracle (the reference algorithm restated on the CPU) on one decode
    step of the workload: one decoder layer at the full batch and context, and
    the LM-head GEMM, both run and timed by every sample; a step's time is
    extrapolated as num_layers x layer + head. Weight / KV values are cheap
    deterministic fills (the timing does not depend on them)."""

    def __init__(self, shape: dict, batch: int, context: int, threads: int):
        sys.path.insert(0, str(ROOT))
        from oracle import model as om
        from oracle import ops

        self.om, self.ops = om, ops
        torch.set_num_threads(threads)
        self.layers = shape["num_hidden_layers"]
        H, I = shape["hidden_size"], shape["intermediate_size"]
        hq, hkv, hd = shape["num_attention_heads"], shape["num_key_value_heads"], 128

        def fill(*s):
            n = math.prod(s)
            return ((torch.arange(n, dtype=torch.int32) % 251 - 125).to(torch.bfloat16) * 1e-4).view(*s)

        pre = "model.layers.0."
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16)  # noqa: E731
        self.p = {pre + "self_attn.q_proj.weight": fill(hq * hd, H), pre + "self_attn.k_proj.weight": fill(hkv * hd, H),
                  pre + "self_attn.v_proj.weight": fill(hkv * hd, H), pre + "self_attn.o_proj.weight": fill(H, hq * hd),
                  pre + "mlp.gate_proj.weight": fill(I, H), pre + "mlp.up_proj.weight": fill(I, H),
                  pre + "mlp.down_proj.weight": fill(H, I), pre + "self_attn.q_norm.weight": ones(hd),
                  pre + "self_attn.k_norm.weight": ones(hd), pre + "input_layernorm.weight": ones(H),
                  pre + "post_attention_layernorm.weight": ones(H)}
        nb = (context + 255) // 256
        self.pool = fill(batch * nb, 2, 256, hkv, hd)
        tables = torch.arange(batch * nb, dtype=torch.int32).view(batch, nb)
        ctx = torch.full((batch,), context, dtype=torch.int32)
        pos = torch.full((batch,), context - 1)
        slots = tables[:, (context - 1) // 256] * 256 + (context - 1) % 256
        self.batch = om.Batch(False, pos, slots, context_lens=ctx, block_tables=tables)
        family = shape.get("model_type", "qwen3")
        ernie = family == "ernie4_5"
        if family != "qwen3":  # Mistral / ERNIE 4.5: no q/k norm; ERNIE: optional q/k/v bias
            del self.p[pre + "self_attn.q_norm.weight"], self.p[pre + "self_attn.k_norm.weight"]
        bias = ernie and bool(shape.get("use_bias", False))
        if bias:
            for n, rows in (("q", hq), ("k", hkv), ("v", hkv)):
                self.p[pre + f"self_attn.{n}_proj.bias"] = fill(rows * hd)
        self.cache = ops.cos_sin_cache(hd, context + 1, float(shape.get("rope_theta", 1e6)))
        self.shape = om.Shape(hidden=H, inter=I, layers=1, hq=hq, hkv=hkv, qk_norm=family == "qwen3",
                              qkv_bias=bias, interleaved=ernie, separate_residual_add=ernie)
        self.h = fill(batch, H) * 100
        self.head_w = fill(shape["vocab_size"], H)
        self.layer()  # warm-up

    def layer(self) -> float:
        t0 = time.perf_counter()
        self.om.decoder_layer(self.p, 0, self.h, self.h.clone(), self.batch, (self.pool[:, 0], self.pool[:, 1]),
                              self.shape, self.cache)
        return time.perf_counter() - t0

    def head(self) -> float:
        t0 = time.perf_counter()
        self.ops.linear(self.h, self.head_w)
        return time.perf_counter() - t0

    def sample(self) -> tuple[float, float]:
        """One sampled decode step: (seconds the sample ran: one layer + the
        head, seconds of the whole step extrapolated: all layers + the head)."""
        t_layer, t_head = self.layer(), self.head()
        return t_layer + t_head, self.layers * t_layer + t_head

    def step_time(self) -> float:
        """The extrapolated time of one decode step (one new sample)."""
        return self.sample()[1]


def run_reference(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # the CPU reference runs once, on rank 0
    shape = model_shape(args.model)
    threads = os.cpu_count() or 1
    sample = CpuDecodeSample(shape, args.batch, args.context, threads)
    for _ in range(args.warmup):
        sample.sample()
    runs = [sample.sample() for _ in range(args.steps)]
    t_sample = sum(r[0] for r in runs) / len(runs)
    t_step = sum(r[1] for r in runs) / len(runs)
    value = args.batch / t_step
    sample = (f"each step: 1 of {shape['num_hidden_layers']} decoder layers + the LM head of one decode step "
              f"(B={args.batch}, ctx={args.context}) on the CPU oracle, the layer's time extrapolated "
              f"x{shape['num_hidden_layers']} for the value; ms_per_step is the sampled work each step ran; "
              f"weights and KV pages are deterministic ramp fills (the CPU time does not depend on the values)")
    line = {
        "impl": "reference", "metric": f"decode output tok/s ({args.model}, B={args.batch}, ctx={args.context})",
        "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_sample * 1e3, "ms_per_step_extrapolated": t_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "config": _config(args),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference algorithm restated on the host CPU (oracle/); the reference's own GPU kernels "
                "(flash-attn, Triton) are third-party and not part of this build",
    }
    print(json.dumps(line), flush=True)
    return 0


def gemm_dispatch(shape: dict, tp: int, batch: int, backend: str) -> dict:
    """Which GEMM each projection of the decode step runs on (this rank's shapes)."""
    from kavor_b200.layers.linear import SK_MAX_TOKENS, auto_uses_stream_k

    H, I, hd = shape["hidden_size"], shape["intermediate_size"], 128
    hq, hkv = shape["num_attention_heads"] // tp, shape["num_key_value_heads"] // tp
    shapes = {"qkv": ((hq + 2 * hkv) * hd, H), "o": (H, hq * hd), "gate_up": (2 * I // tp, H),
              "down": (H, I // tp), "lm_head": (shape["vocab_size"] // tp, H)}
    ours = "kvb_gemm_sk_bf16 (stream-K CTA pairs)"
    out = {}
    for name, (N, K) in shapes.items():
        if backend == "cublas" or (backend == "auto" and not auto_uses_stream_k(batch, N, K)):
            out[name] = "cuBLAS (F.linear)" + (" + kvb_silu_mul" if name == "gate_up" else "")
        elif backend == "tcgen05_pair":
            out[name] = "kvb_gemm_pair" + ("_silu_bf16" if name == "gate_up" else "_bf16")
        elif backend == "tcgen05" and batch > SK_MAX_TOKENS:
            out[name] = "kvb_gemm" + ("_silu_bf16" if name == "gate_up" else "_bf16")
        else:
            out[name] = ("kvb_gemm_sk_silu_bf16 (stream-K CTA pairs, SiLU fused)" if name == "gate_up"
                         and backend == "tcgen05" else ours)
    return out


def _config(args) -> dict:
    return {"workload": f"{args.model} decode step, batch {args.batch}, context {args.context}, TP={args.gpus}",
            "model": args.model, "global_batch": args.batch, "context": args.context, "block_size": 256,
            "parallelism": f"tp{args.gpus}", "gemm": args.gemm, "gemm_l2_prefetch": args.gemm_l2_prefetch,
            "pdl": args.pdl, "e2e_pipelined": args.e2e_pipelined, "decode_microbatches": args.microbatches,
            "l2": "inputs larger than L2 (per step: all weights + every sequence's KV pages)"}


# ----------------------------------------------------------------- our path
def step_bytes(shape: dict, tp: int, batch: int, context: int) -> int:
    """Algorithmic HBM bytes of one decode step per rank: every weight once,
    every context token's K/V once, the new K/V rows written, embedding rows."""
    H, I, L = shape["hidden_size"], shape["intermediate_size"], shape["num_hidden_layers"]
    hq, hkv, hd = shape["num_attention_heads"] // tp, shape["num_key_value_heads"] // tp, 128
    per_layer = H * (hq + 2 * hkv) * hd + hq * hd * H + 3 * H * (I // tp)
    weights = 2 * (L * per_layer + (shape["vocab_size"] // tp) * H)
    kv = L * batch * (context * 2 * hkv * hd * 2 + 2 * hkv * hd * 2)
    return weights + kv + 2 * batch * H


def allreduce_bus_bytes(shape: dict, tp: int, batch: int) -> float:
    """Bytes each rank must move over NVLink per decode step: 2L+1 all-reduces
    of [batch, hidden] bf16, each 2 (N-1)/N of the tensor (ring / two-shot)."""
    if tp <= 1:
        return 0.0
    L, H = shape["num_hidden_layers"], shape["hidden_size"]
    return (2 * L + 1) * 2 * (tp - 1) / tp * batch * H * 2


NVLINK_GBS = 900.0  # nominal per direction per GPU (the roofline's all-reduce term)
SWEEP_BATCHES = (1, 16, 64)  # BASELINE config 3's decode batches beside the headline 256


def attention_bytes(batch: int, context: int, hq: int, hkv: int) -> int:
    """Algorithmic bytes of one decode-attention launch: K and V of every
    context token once, q read and o written."""
    return batch * context * hkv * 128 * 2 * 2 + 2 * batch * hq * 128 * 2


def run_ours(args) -> int:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    else:
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", world_size=1, rank=0,
                                device_id=dev)

    from kavor_b200 import _kernels as K
    from kavor_b200 import _lib
    from kavor_b200.config import Config, write_model_dir
    from kavor_b200.engine.block_manager import BlockManager
    from kavor_b200.engine.model_runner import ModelRunner
    from kavor_b200.engine.sequence import Sequence
    from kavor_b200.sampling_params import SamplingParams

    shape = model_shape(args.model)
    B, ctx0 = args.batch, args.context
    extra = args.warmup + args.steps + 2
    max_len = ((ctx0 + 2 * extra + 255) // 256 + 1) * 256
    blocks_per_seq = (ctx0 + 2 * extra + 255) // 256
    tmp = tempfile.mkdtemp(prefix="kvb_bench_")
    model_dir = write_model_dir(os.path.join(tmp, f"r{rank}"), args.model)
    sweep = [b for b in SWEEP_BATCHES if b < B] if not args.no_sweep else []
    cfg = Config(model_dir, load_format="dummy", seed=0, tensor_parallel_size=world, max_model_len=max_len,
                 max_num_seqs=B, max_num_batched_tokens=4096, num_kvcache_blocks=B * blocks_per_seq + 8,
                 rdzv_port=1, graph_batch_sizes=tuple(sweep) + (B,), gemm_backend=args.gemm,
                 gemm_l2_prefetch=args.gemm_l2_prefetch, pdl=args.pdl, decode_microbatches=args.microbatches)
    runner = ModelRunner(cfg, rank, None)
    with torch.no_grad():
        runner.cache.pools.view(torch.bfloat16).normal_(0.0, 1.0)  # resident KV pages, N(0, 1)

    Sequence.block_size = 256
    bm = BlockManager(cfg.num_kvcache_blocks, 256, enable_prefix_cache=False)
    g = torch.Generator().manual_seed(0)
    seqs = []
    for _ in range(B):
        s = Sequence(torch.randint(0, 151936, (ctx0,), generator=g).tolist(),
                     SamplingParams(temperature=0.6, max_tokens=10 ** 6, ignore_eos=True))
        bm.allocate_prefill(s, 0)
        s.num_cached_tokens = ctx0 - 1  # KV of the first ctx0-1 tokens is resident
        s.is_prefill = False
        seqs.append(s)

    hq, hkv = shape["num_attention_heads"] // world, shape["num_key_value_heads"] // world
    bucket = next(b for b in runner.graph_bs if b >= B)
    graph = runner.graphs[bucket]

    # --- device-timed decode steps (metadata resident: every step repeats context ctx0)
    runner.run(seqs, False)  # fills the graph's static inputs for context ctx0
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("kvb_timed")
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    t_dev = max_over_ranks(start.elapsed_time(end) / 1e3)
    clk = clocks.stop()
    ms_per_step = t_dev / args.steps * 1e3
    value = B * args.steps / t_dev
    launches = runner.graph_launches.get(bucket, 0) * args.steps

    # --- the decode-scaling batch sizes below B: the first b
    # sequences, every one at context ctx0, each size's captured graph replayed
    batch_sweep = {}
    gb = None
    for b in sweep:
        runner.run(seqs[:b], False)  # static inputs of bucket b
        gb = runner.graphs[next(x for x in runner.graph_bs if x >= b)]
        for _ in range(args.warmup):
            gb.replay()
        torch.cuda.synchronize()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            gb.replay()
        s1.record()
        torch.cuda.synchronize()
        barrier()
        tb = max_over_ranks(s0.elapsed_time(s1) / 1e3)
        roof_b = max(step_bytes(shape, world, b, ctx0) / (measured_peaks()[0] * 1e9),
                     allreduce_bus_bytes(shape, world, b) / (NVLINK_GBS * 1e9))
        batch_sweep[str(b)] = {"tok_s": b * args.steps / tb, "ms_per_step": tb / args.steps * 1e3,
                               "step_roofline_frac": roof_b / (tb / args.steps)}
    # at TP > 1 a decode graph holds NCCL work (the vocab-shard sampling
    # all-gather): no reference may outlive the runner, or destroying the
    # process group waits for good
    gb = None
    runner.run(seqs, False)  # back to the full batch

    # --- decode attention alone, rotating over the layers' caches (no L2 reuse)
    attn = [m for m in runner.model.modules() if hasattr(m, "k_cache") and hasattr(m, "v_cache")]
    d = runner.decode_buffers.d
    q = torch.randn(B, hq, 128, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    bt, cl = d["block_tables"][:B], d["context_lens"][:B]

    def attn_launch(i):
        a = attn[i % len(attn)]
        K.paged_decode_attention(q, a.k_cache[0], a.v_cache[0], bt, cl, 128 ** -0.5, out=out)

    # launches captured in one CUDA graph and replayed, so the figure is device
    # time (eager launches of a ~20 us kernel would time the host instead)
    n_attn = 2 * len(attn)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for i in range(3):
            attn_launch(i)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    attn_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(attn_graph):
        for i in range(n_attn):
            attn_launch(i)
    attn_graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    attn_graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del attn_graph
    t_attn = max_over_ranks(e0.elapsed_time(e1) / 1e3 / n_attn)
    ctx_now = int(cl[0].item())
    a_bytes = attention_bytes(B, ctx_now, hq, hkv)
    peak, peak_src = measured_peaks()
    prof = ROOT / "profiles" / "decode_attention_traffic.json"
    traffic = None
    if prof.exists():  # ncu DRAM bytes of a captured small case, scaled by the units of this launch
        per_unit = json.loads(prof.read_text())["bytes_per_seq_kvhead_ctx1024"]
        traffic = per_unit * B * hkv * ctx_now / 1024
    achieved = a_bytes / t_attn / 1e9
    roofline = {"kernel": "decode_attn_kernel", "bound": "hbm", "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                "algorithmic_bytes": a_bytes, "avg_launch_us": t_attn * 1e6}
    s_bytes = step_bytes(shape, world, B, ctx0)
    t_roof = s_bytes / (peak * 1e9)
    ar_bytes = allreduce_bus_bytes(shape, world, B)
    t_ar = ar_bytes / (NVLINK_GBS * 1e9)
    t_step_roof = max(t_roof, t_ar)  # the slower of weight+KV bytes at HBM peak and all-reduce bytes over NVLink
    step_roof = {"bytes_per_rank": s_bytes, "t_hbm_us": t_roof * 1e6, "allreduce_bytes_per_rank": ar_bytes,
                 "t_nvlink_us": t_ar * 1e6, "nvlink_gbs": NVLINK_GBS, "t_roofline_us": t_step_roof * 1e6,
                 "frac": t_step_roof / (ms_per_step / 1e3), "peak_gbs": peak, "peak_source": peak_src}

    # --- end to end through ModelRunner.run (sequences advance one token per step)
    e2e = None
    if not args.no_e2e:
        from kavor_b200.engine.model_runner import advance_decode

        def run_e2e(n):
            advance_decode(runner, seqs, bm, n, pipelined=args.e2e_pipelined)

        run_e2e(args.warmup)
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        run_e2e(args.steps)
        f1.record()
        torch.cuda.synchronize()
        barrier()
        t_e2e = max_over_ranks(f0.elapsed_time(f1) / 1e3)
        e2e = {"value": B * args.steps / t_e2e, "unit": "tok/s", "ms_per_step": t_e2e / args.steps * 1e3,
               "h2d_bytes_per_step": runner.decode_buffers.nbytes, "d2h_bytes_per_step": 8 * B,
               "api": ("ModelRunner.run_async(seqs, chain=True), one step in flight" if args.e2e_pipelined
                       else "ModelRunner.run(seqs, is_prefill=False)")}

    # --- BASELINE config 5 at this TP size: the fused all-reduce + add+RMSNorm
    # against NCCL all_reduce + add+RMSNorm, on the model's communicator
    ar_micro = None
    if world > 1 and runner.tp_allreduce is not None and not args.no_sweep:
        from kavor_b200.profile_allreduce import fused_vs_nccl

        ar_micro = fused_vs_nccl(runner.tp_allreduce, [1, 16, 256, 4096])

    dev_err = _lib.device_error(clear=True)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sample = CpuDecodeSample(shape, B, ctx0, threads)
        t_step = statistics.median(sample.step_time() for _ in range(5))
        cpu = {"value": B / t_step, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"5 sampled decode steps (B={B}, ctx={ctx0}), median: each 1 timed decoder layer of "
                         f"{shape['num_hidden_layers']} + 1 timed LM-head GEMM on the CPU oracle, the layer's time "
                         f"extrapolated x{shape['num_hidden_layers']}; weights and KV pages are deterministic ramp "
                         f"fills (the CPU time does not depend on the values)",
               "ms_per_step": t_step * 1e3}

    # the pipelined e2e beside the synchronous one (one GPU, no collectives; a failure is reported, not raised)
    e2e_pipelined = None
    if world == 1 and not args.no_e2e and not args.e2e_pipelined:
        e2e_pipelined = _e2e_pipelined_probe(runner, seqs, bm, args)
    # the decode step with the package's GEMM in place of cuBLAS (re-captured graphs; same guard)
    gemm_probes = None
    if world == 1 and args.gemm == "auto" and not args.no_probes:
        graph = None  # the probes re-capture the decode graph
        gemm_probes = {f"{backend}_l2pf{pf}": _gemm_backend_probe(runner, seqs, B, args, backend, pf)
                       for backend, pf in (("tcgen05", 0), ("cublas", 0))}

    if rank == 0:
        line = {
            "metric": f"decode output tok/s ({args.model}, B={B}, ctx={ctx0})", "value": value, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init weights (reference checkpoint shapes), random token ids, KV pages N(0,1)",
            "config": dict(_config(args), gemm_dispatch=gemm_dispatch(shape, world, B, args.gemm)),
            "decode_step_us": ms_per_step * 1e3, "attn_hbm_gbs": achieved,
            "roofline": roofline, "step_roofline": step_roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": launches, "device_error_bits": dev_err,
        }
        if batch_sweep:
            line["batch_sweep"] = batch_sweep
        if ar_micro is not None:
            line["allreduce_add_rmsnorm_microbench"] = ar_micro
        if e2e_pipelined is not None:
            line["e2e_pipelined"] = e2e_pipelined
        if gemm_probes is not None:
            line["gemm_backend_probes"] = gemm_probes
        print(json.dumps(line), flush=True)
    # graphs hold NCCL work: every reference must be gone before the group is destroyed
    del graph, gb
    try:
        runner.exit()
        torch.cuda.synchronize()
        barrier()
        # past the last barrier nothing runs on any GPU; should destroying the group
        # still wait (a graph holding NCCL work outlived it), the line is printed:
        # say so and leave instead of holding every rank until the launcher's limit
        guard = _exit_if_stuck(TEARDOWN_LIMIT_S)
        dist.destroy_process_group()
        guard.cancel()
    except Exception:
        probes = [e2e_pipelined] + list((gemm_probes or {}).values())
        if not any(p is not None and "error" in p for p in probes):
            raise
        print(f"teardown after a failed probe: {sys.exc_info()[1]}", file=sys.stderr, flush=True)
    return 0


def _gemm_backend_probe(runner, seqs, B, args, backend: str, l2_prefetch: int) -> dict:
    """Device time of the decode step with every projection on the package's
    GEMM (Config.gemm_backend) instead of cuBLAS: the decode graph re-captured,
    the same resident batch, `steps` replays after `warmup`."""
    from kavor_b200 import _kernels as K
    from kavor_b200 import _lib
    from kavor_b200.layers.linear import set_gemm_backend

    try:
        set_gemm_backend(backend)
        K.gemm_set_l2_prefetch(l2_prefetch)
        runner.graphs.clear()
        runner.graph_pool = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        runner.capture_cudagraph()
        runner.run(seqs, False)  # the re-captured graph's static inputs
        graph = runner.graphs[next(b for b in runner.graph_bs if b >= B)]
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        return {"value": B * args.steps / t, "unit": "tok/s", "ms_per_step": t / args.steps * 1e3,
                "gemm_backend": backend, "l2_prefetch_ksteps": l2_prefetch,
                "device_error_bits": _lib.device_error(clear=True)}
    except Exception as exc:  # the probe of an option that is off by default must not cost the main line
        return {"error": f"{type(exc).__name__}: {exc}"[:400]}
    finally:
        set_gemm_backend(args.gemm)
        try:
            K.gemm_set_l2_prefetch(0)
        except Exception:
            pass


def _e2e_pipelined_probe(runner, seqs, bm, args) -> dict:
    """The e2e measurement again through ModelRunner.run_async with one step in
    flight (same per-step H2D / D2H), reported beside the synchronous e2e."""
    from kavor_b200 import _lib
    from kavor_b200.engine.model_runner import advance_decode

    try:
        advance_decode(runner, seqs, bm, args.warmup, pipelined=True)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        advance_decode(runner, seqs, bm, args.steps, pipelined=True)
        f1.record()
        torch.cuda.synchronize()
        t = f0.elapsed_time(f1) / 1e3
        return {"value": len(seqs) * args.steps / t, "unit": "tok/s", "ms_per_step": t / args.steps * 1e3,
                "api": "ModelRunner.run_async(seqs, chain=True), one step in flight",
                "device_error_bits": _lib.device_error(clear=True)}
    except Exception as exc:  # the probe of an option that is off by default must not cost the main line
        return {"error": f"{type(exc).__name__}: {exc}"[:400]}


TEARDOWN_LIMIT_S = 90.0


def _exit_if_stuck(seconds: float) -> threading.Timer:
    def fire():
        print(f"bench.py: the process group was not destroyed within {seconds:.0f} s of the final barrier "
              "(the result line is printed above); exiting", file=sys.stderr, flush=True)
        os._exit(0)

    t = threading.Timer(seconds, fire)
    t.daemon = True
    t.start()
    return t


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
