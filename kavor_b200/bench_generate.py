"""Offline generate throughput through the public API, on the workload of the
reference's own benchmark (benchs/bench.py:8-26).

    python -m kavor_b200.bench_generate [--model Qwen3-0.6B] [--tp 1] [--num-seqs 256] [--async-decode]
        [--gemm cublas|tcgen05] [--pdl]

256 sequences of uniform-random token ids in [0, 10000], prompt lengths
U[100, 1024], max_tokens U[100, 1024] (Python's `random` seeded with 0, drawn
in the reference's order), temperature 0.6, ignore_eos, prefix caching off,
random-init weights of the named checkpoint shape (load_format="dummy"; no
checkpoint or tokenizer is available offline). One short warm-up generate,
then the timed `LLM.generate` over all sequences (wall clock, as the reference
measures it). Prints one JSON line: total generated tokens, seconds,
tokens/s, and the reference's published figure for the same workload
(1434.13 tok/s, RTX 4070 Laptop, README.md:44-55) for context.
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time
from random import randint, seed

REFERENCE_PUBLISHED_TOK_S = 1434.13


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="Qwen3-0.6B")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--num-seqs", type=int, default=256)
    ap.add_argument("--max-input-len", type=int, default=1024)
    ap.add_argument("--max-output-len", type=int, default=1024)
    ap.add_argument("--async-decode", action="store_true", help="one decode step in flight (Config.async_decode)")
    ap.add_argument("--gemm", choices=["cublas", "tcgen05", "tcgen05_pair"], default="cublas")
    ap.add_argument("--pdl", action="store_true")
    ap.add_argument("--microbatches", type=int, choices=[1, 2], default=1,
                    help="TP > 1: decode as two halves on two streams (Config.decode_microbatches)")
    a = ap.parse_args(argv)

    from kavor_b200 import LLM, SamplingParams
    from kavor_b200.config import write_model_dir

    seed(0)
    prompts = [[randint(0, 10000) for _ in range(randint(100, a.max_input_len))] for _ in range(a.num_seqs)]
    params = [SamplingParams(temperature=0.6, ignore_eos=True, max_tokens=randint(100, a.max_output_len))
              for _ in range(a.num_seqs)]
    model_dir = write_model_dir(os.path.join(tempfile.mkdtemp(prefix="kvb_gen_"), "m"), a.model)
    llm = LLM(model_dir, load_format="dummy", tensor_parallel_size=a.tp, max_model_len=4096,
              enable_prefix_caching=False, async_decode=a.async_decode, gemm_backend=a.gemm, pdl=a.pdl,
              decode_microbatches=a.microbatches)
    try:
        llm.generate([[1, 2, 3, 4]], SamplingParams(max_tokens=8), use_tqdm=False)
        t0 = time.perf_counter()
        out = llm.generate(prompts, params, use_tqdm=False)
        dt = time.perf_counter() - t0
    finally:
        llm.exit()
    total = sum(sp.max_tokens for sp in params)
    generated = sum(len(o["token_ids"]) for o in out)
    print(json.dumps({"workload": f"offline generate, {a.model}, {a.num_seqs} seqs, prompt/output U[100,1024]",
                      "tp": a.tp, "async_decode": a.async_decode, "gemm": a.gemm, "pdl": a.pdl,
                      "decode_microbatches": a.microbatches,
                      "total_tokens": total, "generated_tokens": generated, "seconds": dt,
                      "tok_s": total / dt, "reference_published_tok_s": REFERENCE_PUBLISHED_TOK_S,
                      "reference_hardware": "RTX 4070 Laptop 8 GB (README.md:44-55)"}), flush=True)
    return 0 if generated == total else 1


if __name__ == "__main__":
    raise SystemExit(main())
