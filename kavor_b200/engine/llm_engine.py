"""Offline engine (drop-in for kavor/engine/llm_engine.py, text prompts).

``LLMEngine(model, **config)`` spawns TP workers 1..N-1 (spawn context,
llm_engine.py:44-52), builds rank 0's ``ModelRunner`` and the ``Scheduler``;
``generate`` adds requests and steps until every sequence finished
(llm_engine.py:245-272). Prompts are strings (needs a tokenizer in the model
directory) or token-id lists. With ``async_decode=True`` decode steps run
with one step in flight (``DecodePipeline``). With ``profile=True`` every
step records {prefill, tokens, step_time, forward_time} in ``step_stats``
and finished requests land in ``request_stats`` (llm_engine.py:140-181).
"""
from __future__ import annotations

import atexit
import logging
import signal
from dataclasses import fields
from time import monotonic, perf_counter

import torch.multiprocessing as mp

from kavor_b200.config import Config
from kavor_b200.engine.model_runner import ModelRunner
from kavor_b200.engine.pipeline import DecodePipeline
from kavor_b200.engine.scheduler import Scheduler
from kavor_b200.engine.sequence import Sequence
from kavor_b200.sampling_params import SamplingParams

logger = logging.getLogger("kavor_b200")

WORKER_EXIT_TIMEOUT = 10.0   # after the exit message
WORKER_STOP_TIMEOUT = 330.0  # after a stop request (covers the process group's 300 s timeout)


def _stop_requested(signum, frame):
    raise SystemExit(f"TP worker stopped by signal {signum}")


def _worker_entry(config: Config, rank: int, event) -> None:
    # SIGTERM (LLMEngine._reap's stop request, or multiprocessing's exit
    # handling of daemonic children) becomes SystemExit in the worker's main
    # thread: ModelRunner.loop unwinds through abandon(), which closes the
    # all-reduce areas with the other ranks before the process ends
    signal.signal(signal.SIGTERM, _stop_requested)
    ModelRunner(config, rank, event)


def _load_tokenizer(path: str, trust_remote_code: bool):
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(path, use_fast=True, trust_remote_code=trust_remote_code)
    except Exception:  # a weight-less / tokenizer-less model directory: token-id prompts only
        return None


class LLMEngine:

    def __init__(self, model: str, **kwargs):
        names = {f.name for f in fields(Config)}
        config = Config(model, **{k: v for k, v in kwargs.items() if k in names})
        self.config = config
        Sequence.block_size = config.kvcache_block_size
        self.ps = []
        self.events = []
        self._exiting = False
        # whether a worker that ignores a stop request may be killed: only when
        # no rank holds memory that may be bound to an NVLink multicast object
        # (ending such a rank can fault the other ranks' GPUs); unknown until
        # rank 0's runner has chosen its all-reduce backend
        self._kill_ok = config.tensor_parallel_size == 1
        self.step_stats: list[dict] = []
        self.request_stats: list[dict] = []
        ctx = mp.get_context("spawn")
        for i in range(1, config.tensor_parallel_size):
            event = ctx.Event()
            p = ctx.Process(target=_worker_entry, args=(config, i, event), daemon=True)
            p.start()
            self.ps.append(p)
            self.events.append(event)
        atexit.register(self.exit)
        try:
            self.model_runner = ModelRunner(config, 0, self.events)
            tp = self.model_runner.tp_allreduce
            self._kill_ok = tp is None or tp.backend == "ipc"
            self.tokenizer = _load_tokenizer(config.model, config.trust_remote_code)
            if self.tokenizer is not None and self.tokenizer.eos_token_id is not None:
                config.eos = self.tokenizer.eos_token_id
            elif getattr(config.hf_config, "eos_token_id", None) is not None:
                eos = config.hf_config.eos_token_id
                config.eos = eos[0] if isinstance(eos, (list, tuple)) else eos
            self.scheduler = Scheduler(config)
            # one decode step in flight (Config.async_decode); profiling keeps the step-at-a-time loop
            self.pipeline = (DecodePipeline(self.scheduler, self.model_runner.call)
                             if config.async_decode and not config.profile else None)
        except BaseException:
            self.exit()
            raise

    def exit(self) -> None:
        if self._exiting:
            return
        self._exiting = True
        alive = all(p.is_alive() for p in self.ps)
        if getattr(self, "model_runner", None) is not None and alive:
            self.model_runner.call("exit")
            del self.model_runner
            self._reap(graceful=True)
        else:
            self._reap(graceful=False)

    def _reap(self, graceful: bool) -> None:
        """Wait for the workers; a worker still running gets SIGTERM, which
        its entry turns into an orderly exit (communicator closed with the
        other ranks). A worker that does not stop is killed only when no rank
        holds multicast-bound memory; otherwise it is logged and left alone."""
        if graceful:
            deadline = monotonic() + WORKER_EXIT_TIMEOUT
            for p in self.ps:
                p.join(timeout=max(0.0, deadline - monotonic()))
        for p in self.ps:
            if p.is_alive():
                logger.warning("TP worker %s did not exit, asking it to stop", p.name)
                p.terminate()
        deadline = monotonic() + WORKER_STOP_TIMEOUT
        for p in self.ps:
            p.join(timeout=max(0.0, deadline - monotonic()))
        for p in self.ps:
            if not p.is_alive():
                continue
            if self._kill_ok:
                logger.warning("TP worker %s ignored the stop request, killing it", p.name)
                p.kill()
                p.join(timeout=2.0)
            else:
                logger.error("TP worker %s ignored the stop request; left running: its all-reduce area may be "
                             "bound to an NVLink multicast object, and ending it could fault the other GPUs",
                             p.name)

    def add_request(self, prompt, sampling_params: SamplingParams, request_id: str | None = None) -> int:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise RuntimeError("this model directory has no tokenizer: pass token-id lists")
            prompt = self.tokenizer.encode(prompt)
        seq = Sequence(prompt, sampling_params)
        seq.request_id = request_id
        self.scheduler.add(seq)
        return seq.seq_id

    def step(self):
        if self.pipeline is not None:
            return [(s.seq_id, s.completion_token_ids) for s in self.pipeline.step()]
        seqs, is_prefill = self.scheduler.schedule()
        token_ids = self.model_runner.call("run", seqs, is_prefill)
        if is_prefill:
            now = perf_counter()
            for s in seqs:
                s.stats.first_token_time = now
        self.scheduler.postprocess(seqs, token_ids, is_prefill)
        return [(s.seq_id, s.completion_token_ids) for s in seqs if s.is_finished]

    def profile_step(self):
        start = perf_counter()
        seqs, is_prefill = self.scheduler.schedule()
        num_tokens = sum(s.num_scheduled_tokens for s in seqs)
        t0 = perf_counter()
        token_ids = self.model_runner.call("run", seqs, is_prefill)
        forward_time = perf_counter() - t0
        if is_prefill:
            now = perf_counter()
            for s in seqs:
                s.stats.first_token_time = now
        self.scheduler.postprocess(seqs, token_ids, is_prefill)
        now = perf_counter()
        self.step_stats.append({"ts": now, "prefill": is_prefill, "tokens": num_tokens,
                                "step_time": now - start, "forward_time": forward_time})
        for s in seqs:
            if s.is_finished:
                s.stats.finish_time = now
                self.request_stats.append({
                    "seq_id": s.seq_id, "request_id": s.request_id, "num_prompt_tokens": s.num_prompt_tokens,
                    "num_completion_tokens": s.num_completion_tokens, "arrival_time": s.stats.arrival_time,
                    "prefill_start_time": s.stats.prefill_start_time, "first_token_time": s.stats.first_token_time,
                    "finish_time": now, "prefix_cache_hit_tokens": s.stats.prefix_cache_hit_tokens})
        return [(s.seq_id, s.completion_token_ids) for s in seqs if s.is_finished]

    def is_finished(self) -> bool:
        if self.pipeline is not None:
            return self.pipeline.is_finished()
        return self.scheduler.is_finished()

    def generate(self, inputs, sampling_params: SamplingParams | list[SamplingParams], use_tqdm: bool = True):
        if self.config.profile:
            self.step_stats.clear()
            self.request_stats.clear()
        if not isinstance(sampling_params, list):
            sampling_params = [sampling_params] * len(inputs)
        for prompt, sp in zip(inputs, sampling_params):
            self.add_request(prompt, sp)
        outputs = {}
        step = self.profile_step if self.config.profile else self.step
        bar = None
        if use_tqdm:
            from tqdm.auto import tqdm

            bar = tqdm(total=len(inputs), desc="Generating", dynamic_ncols=True)
        while not self.is_finished():
            for seq_id, token_ids in step():
                outputs[seq_id] = token_ids
                if bar is not None:
                    bar.update(1)
        if bar is not None:
            bar.close()
        ordered = [outputs[k] for k in sorted(outputs)]
        decode = self.tokenizer.decode if self.tokenizer is not None else (lambda ids: None)
        return [{"text": decode(ids), "token_ids": ids} for ids in ordered]
