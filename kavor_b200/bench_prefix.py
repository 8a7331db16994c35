"""Prefill-heavy generate with a shared prefix, through the public API.

    python -m kavor_b200.bench_prefix [--model Qwen3-32B] [--tp 8] [--num-seqs 64] [--async-decode]
    (TP > 1 spawns its own worker processes: run it as one process)

Workload: `num_seqs` sequences, each a shared prefix of `prefix_len` random
token ids followed by a unique suffix of U[suffix_min, suffix_max] random ids
(ids in [0, 10000], Python's `random` seeded with 0), `max_tokens` output
tokens each, temperature 0.6, ignore_eos, prefix caching ON; random-init
weights of the named checkpoint shape (load_format="dummy"). The first
request is generated alone (it writes the shared prefix's blocks), then the
timed `LLM.generate` runs the rest, whose prompts find the prefix in the
cache: the paged prefill attention reads the cached prefix pages. Prints one
JSON line: prompt and output tokens, prefix-cache hit tokens, seconds, prompt
tokens/s and output tokens/s.
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time
from random import randint, seed


def workload(num_seqs: int, prefix_len: int, suffix_min: int, suffix_max: int) -> list[list[int]]:
    seed(0)
    prefix = [randint(0, 10000) for _ in range(prefix_len)]
    return [prefix + [randint(0, 10000) for _ in range(randint(suffix_min, suffix_max))] for _ in range(num_seqs)]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="Qwen3-32B")
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--num-seqs", type=int, default=64)
    ap.add_argument("--prefix-len", type=int, default=2048)
    ap.add_argument("--suffix-min", type=int, default=512)
    ap.add_argument("--suffix-max", type=int, default=6144)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--async-decode", action="store_true")
    ap.add_argument("--gemm", choices=["cublas", "tcgen05", "tcgen05_pair"], default="cublas")
    ap.add_argument("--pdl", action="store_true")
    ap.add_argument("--microbatches", type=int, choices=[1, 2], default=1,
                    help="TP > 1: decode as two halves on two streams (Config.decode_microbatches)")
    a = ap.parse_args(argv)

    from kavor_b200 import LLM, SamplingParams
    from kavor_b200.config import write_model_dir

    prompts = workload(a.num_seqs, a.prefix_len, a.suffix_min, a.suffix_max)
    params = SamplingParams(temperature=0.6, ignore_eos=True, max_tokens=a.max_tokens)
    max_len = a.prefix_len + a.suffix_max + a.max_tokens
    model_dir = write_model_dir(os.path.join(tempfile.mkdtemp(prefix="kvb_prefix_"), "m"), a.model)
    llm = LLM(model_dir, load_format="dummy", tensor_parallel_size=a.tp, max_model_len=max_len,
              enable_prefix_caching=True, async_decode=a.async_decode, gemm_backend=a.gemm, pdl=a.pdl,
              decode_microbatches=a.microbatches)
    try:
        llm.generate(prompts[:1], params, use_tqdm=False)  # the shared prefix's blocks enter the cache
        bm = llm.scheduler.block_manager
        hit0, prompt0 = bm.prefix_cache_hit_tokens, bm.prefix_cache_prompt_tokens
        t0 = time.perf_counter()
        out = llm.generate(prompts[1:], params, use_tqdm=False)
        dt = time.perf_counter() - t0
        hits, prompt_tokens = bm.prefix_cache_hit_tokens - hit0, bm.prefix_cache_prompt_tokens - prompt0
    finally:
        llm.exit()
    generated = sum(len(o["token_ids"]) for o in out)
    print(json.dumps({"workload": f"shared-prefix generate, {a.model}, TP={a.tp}, {a.num_seqs - 1} timed seqs, "
                                  f"prefix {a.prefix_len}, suffix U[{a.suffix_min},{a.suffix_max}], "
                                  f"{a.max_tokens} output tokens", "async_decode": a.async_decode, "gemm": a.gemm,
                      "pdl": a.pdl, "decode_microbatches": a.microbatches, "prompt_tokens": prompt_tokens, "prefix_cache_hit_tokens": hits,
                      "generated_tokens": generated, "seconds": dt, "prompt_tok_s": prompt_tokens / dt,
                      "output_tok_s": generated / dt}), flush=True)
    return 0 if generated == (a.num_seqs - 1) * a.max_tokens else 1


if __name__ == "__main__":
    raise SystemExit(main())
