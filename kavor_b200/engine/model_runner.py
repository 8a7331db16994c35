"""Model runner (drop-in for kavor/engine/model_runner.py, Qwen3 text path).

Per step (model_runner.py:247-262): build the batch metadata on the host,
send it to the device in ONE pinned host->device copy, run the forward (a
captured CUDA graph for decode buckets, eager for prefill), sample on the
device and read the token ids back.

Tensor parallelism: one process per GPU over NCCL. Two launch modes:
* spawned by ``LLMEngine`` (rank 0 drives ranks > 0 through a shared-memory
  mailbox, model_runner.py:51-112);
* SPMD under an external launcher (torchrun): the process group already
  exists and every rank calls ``run`` itself with the same sequences.
Every rank computes the same sampled tokens (only (score, index) pairs cross
ranks, see ParallelLMHead.sample), so the LM head and the sampler stay inside
the decode graph at every TP size.
"""
from __future__ import annotations

import datetime
import itertools
import multiprocessing
import operator
import os
import pickle
import time
from multiprocessing.shared_memory import SharedMemory

import numpy as np
import torch
import torch.distributed as dist

from kavor_b200 import _kernels as K
from kavor_b200 import _lib
from kavor_b200.engine.cache_pool import CachePool
from kavor_b200.engine.sequence import Sequence
from kavor_b200.layers.allreduce import DecodeMicrobatches, TPAllReduce, set_decode_microbatches, set_tp_allreduce
from kavor_b200.layers.linear import set_gemm_backend
from kavor_b200.layers.sampler import Sampler
from kavor_b200.models import AutoModelForCausalLM
from kavor_b200.utils.context import reset_context, set_context

SHM_BYTES = 1 << 22
MAILBOX_WAIT_S = 60.0  # rank 0 waits at most this long for every worker to take the previous message
MAILBOX_POLL_S = 1.0   # a worker checks that rank 0's process is still alive this often while idle


# ----------------------------------------------------------------- host metadata
_NUM_TOKENS = operator.attrgetter("num_tokens")
_LAST_TOKEN = operator.attrgetter("last_token")
_BLOCK_TABLE = operator.attrgetter("block_table")
_TEMPERATURE = operator.attrgetter("temperature")


def block_table_matrix(seqs: list[Sequence], width: int | None = None) -> np.ndarray:
    """[B, max blocks] int32, rows padded with -1 (model_runner.py:469-473).
    One flat gather of every table and one masked scatter (no per-row numpy
    call: this runs on the host every decode step)."""
    lens = np.fromiter((len(s.block_table) for s in seqs), np.int64, len(seqs))
    w = int(lens.max(initial=0)) if width is None else width
    out = np.full((len(seqs), w), -1, dtype=np.int32)
    flat = np.fromiter(itertools.chain.from_iterable(s.block_table for s in seqs), np.int32, int(lens.sum()))
    out[np.arange(w) < lens[:, None]] = flat
    return out


def decode_metadata(seqs: list[Sequence], block_size: int) -> dict[str, np.ndarray]:
    """model_runner.py:448-467: the last token of every sequence at position len-1,
    written to slot block_table[-1]*block_size + last_block_num_tokens - 1.
    Attributes are pulled with C-level getters (no Python frame per sequence)
    and the last block id comes from the block-table matrix."""
    n = len(seqs)
    ctx = np.fromiter(map(_NUM_TOKENS, seqs), np.int64, n)
    tables = list(map(_BLOCK_TABLE, seqs))
    lens = np.fromiter(map(len, tables), np.int64, n)
    if n and int(lens.min()) == 0:
        raise ValueError("decode_metadata: every decoding sequence needs a block")
    w = int(lens.max(initial=0))
    bt = np.full((n, w), -1, dtype=np.int32)
    if w:
        bt[np.arange(w) < lens[:, None]] = np.fromiter(itertools.chain.from_iterable(tables), np.int32,
                                                       int(lens.sum()))
    pos = ctx - 1
    last_block = bt[np.arange(n), lens - 1].astype(np.int64)
    return {
        "input_ids": np.fromiter(map(_LAST_TOKEN, seqs), np.int64, n),
        "positions": pos,
        # last_block_num_tokens - 1 == (len - 1) % block_size
        "slot_mapping": (last_block * block_size + pos % block_size).astype(np.int32),
        "context_lens": ctx.astype(np.int32),
        "block_tables": bt,
    }


def prefill_metadata(seqs: list[Sequence], block_size: int) -> dict:
    """model_runner.py:385-446: tokens [num_cached, num_cached + num_scheduled) of
    every sequence, cumulative q/k lengths, slots through the block table, and
    the block tables only when some keys come from the cache (prefix hit or a
    later prefill chunk)."""
    ids, pos, slots = [], [], []
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    for s in seqs:
        start = s.num_cached_tokens
        end = start + s.num_scheduled_tokens
        ids.append(np.asarray(s.token_ids[start:end], dtype=np.int64))
        t = np.arange(start, end, dtype=np.int64)
        pos.append(t)
        cu_q.append(cu_q[-1] + end - start)
        cu_k.append(cu_k[-1] + end)
        max_q = max(max_q, end - start)
        max_k = max(max_k, end)
        if s.block_table:
            table = np.asarray(s.block_table, dtype=np.int64)
            slots.append((table[t // block_size] * block_size + t % block_size).astype(np.int32))
    meta = {
        "input_ids": np.concatenate(ids) if ids else np.zeros(0, np.int64),
        "positions": np.concatenate(pos) if pos else np.zeros(0, np.int64),
        "cu_seqlens_q": np.asarray(cu_q, dtype=np.int32),
        "cu_seqlens_k": np.asarray(cu_k, dtype=np.int32),
        "max_seqlen_q": max_q,
        "max_seqlen_k": max_k,
        "slot_mapping": np.concatenate(slots) if slots else np.zeros(0, np.int32),
        "block_tables": block_table_matrix(seqs) if cu_k[-1] > cu_q[-1] else None,
    }
    return meta


# ----------------------------------------------------------------- staging
class Staging:
    """Pinned host area + device area; the arrays of one step are packed at
    16-byte aligned offsets and cross PCIe in a single copy."""

    def __init__(self, device: torch.device, capacity: int = 1 << 20):
        self.device = device
        self._grow(capacity)

    def _grow(self, nbytes: int) -> None:
        self.host = torch.empty(nbytes, dtype=torch.uint8, device="cpu", pin_memory=True)
        self.dev = torch.empty(nbytes, dtype=torch.uint8, device=self.device)

    def upload(self, arrays: list[np.ndarray]) -> list[torch.Tensor]:
        offs, total = [], 0
        for a in arrays:
            offs.append(total)
            total += (a.nbytes + 15) & ~15
        if total > self.host.numel():
            torch.cuda.current_stream().synchronize()
            self._grow(max(total, 2 * self.host.numel()))
        hv = self.host.numpy()
        for a, o in zip(arrays, offs):
            hv[o:o + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
        self.dev[:total].copy_(self.host[:total], non_blocking=True)
        return [self.dev[o:o + a.nbytes].view(torch.from_numpy(a[:0]).dtype).view(a.shape)
                for a, o in zip(arrays, offs)]


class DecodeBuffers:
    """Static device inputs of the decode graphs (fixed addresses) with pinned
    host mirrors; one copy per step moves all of them. Mirror 0 serves the
    synchronous ``ModelRunner.run``; mirrors 1 and 2 alternate between the
    steps of ``run_async``, so a mirror is never rewritten while the copy of
    the step before is still queued. Sampled tokens come back through two
    alternating pinned buffers."""

    FIELDS = (("input_ids", np.int64), ("positions", np.int64), ("temperatures", np.float32),
              ("slot_mapping", np.int32), ("context_lens", np.int32))
    MIRRORS = 3

    def __init__(self, max_bs: int, max_blocks: int, device: torch.device):
        self.max_bs, self.max_blocks = max_bs, max_blocks
        layout, off = {}, 0
        for name, dt in self.FIELDS:
            layout[name] = (off, dt, (max_bs,))
            off += (max_bs * np.dtype(dt).itemsize + 15) & ~15
        layout["block_tables"] = (off, np.int32, (max_bs, max_blocks))
        off += max_bs * max_blocks * 4
        self.nbytes = off
        self.hosts = [torch.zeros(off, dtype=torch.uint8, device="cpu", pin_memory=True) for _ in range(self.MIRRORS)]
        self.host = self.hosts[0]
        self.dev = torch.zeros(off, dtype=torch.uint8, device=device)
        self.views: list[dict] = [{} for _ in range(self.MIRRORS)]
        self.d = {}
        for name, (o, dt, shape) in layout.items():
            n = int(np.prod(shape)) * np.dtype(dt).itemsize
            for m in range(self.MIRRORS):
                self.views[m][name] = self.hosts[m].numpy()[o:o + n].view(dt).reshape(shape)
            self.d[name] = self.dev[o:o + n].view(torch.from_numpy(np.zeros(0, dt)).dtype).view(shape)
        self.h = self.views[0]
        self.copied: list[torch.cuda.Event | None] = [None] * self.MIRRORS
        self.sampled = torch.zeros(max_bs, dtype=torch.int64, device=device)
        self.tokens_host = [torch.zeros(max_bs, dtype=torch.int64, device="cpu", pin_memory=True) for _ in range(2)]
        # a chained step's gather map: row i takes the previous step's sample chain[i]
        self.chain_host = [torch.zeros(max_bs, dtype=torch.int64, device="cpu", pin_memory=True) for _ in range(2)]
        self.chain_copied: list[torch.cuda.Event | None] = [None, None]
        self.chain_dev = torch.zeros(max_bs, dtype=torch.int64, device=device)

    def fill(self, meta: dict, temperatures: np.ndarray, bucket: int, mirror: int = 0) -> None:
        if self.copied[mirror] is not None:  # the previous copy out of this mirror has been read
            self.copied[mirror].synchronize()
        n = meta["input_ids"].shape[0]
        h = self.views[mirror]
        h["input_ids"][:n] = meta["input_ids"]
        h["input_ids"][n:bucket] = 0
        h["positions"][:n] = meta["positions"]
        h["positions"][n:bucket] = 0
        h["temperatures"][:n] = temperatures
        h["temperatures"][n:bucket] = 1.0
        h["slot_mapping"][:n] = meta["slot_mapping"]
        h["slot_mapping"][n:bucket] = -1
        h["context_lens"][:n] = meta["context_lens"]
        h["context_lens"][n:bucket] = 0
        bt = meta["block_tables"]
        h["block_tables"][:n, :bt.shape[1]] = bt
        h["block_tables"][:n, bt.shape[1]:] = -1
        self.dev.copy_(self.hosts[mirror], non_blocking=True)
        if mirror:
            self.copied[mirror] = torch.cuda.Event()
            self.copied[mirror].record()


class PendingDecode:
    """A decode step issued by ``ModelRunner.run_async``: ``result()`` waits for
    the step and returns its sampled token ids (read from pinned memory)."""

    def __init__(self, host: torch.Tensor, event: torch.cuda.Event, n: int):
        self.host, self.event, self.n = host, event, n
        self.done = False

    def result(self) -> list[int]:
        self.event.synchronize()
        self.done = True
        return self.host[:self.n].tolist()


def advance_decode(runner, seqs: list[Sequence], block_manager, steps: int, pipelined: bool = False) -> None:
    """Run `steps` decode steps of a fixed batch, growing every sequence by one
    token per step (blocks from `block_manager`). Synchronous: ``runner.run``
    per step. Pipelined: ``runner.run_async`` with one step in flight — step
    i+1 is issued, its input tokens chained on the device, before step i's
    tokens are read back; the host appends a placeholder (-1) per step and
    patches it when the tokens arrive, so the sequences end the same either
    way while the host's per-step work overlaps the GPU's."""
    if not pipelined:
        for _ in range(steps):
            block_manager.may_append_blocks(seqs)
            for s, t in zip(seqs, runner.run(seqs, False)):
                s.num_cached_tokens += 1
                s.append_token(t)
        return
    pending = None
    for _ in range(steps):
        block_manager.may_append_blocks(seqs)
        nxt = runner.run_async(seqs, chain=pending is not None)
        if pending is not None:
            for s, t in zip(seqs, pending.result()):
                s.token_ids[-1] = s.last_token = t
        for s in seqs:
            s.num_cached_tokens += 1
            s.append_token(-1)
        pending = nxt
    if pending is not None:
        for s, t in zip(seqs, pending.result()):
            s.token_ids[-1] = s.last_token = t


# ----------------------------------------------------------------- runner
class ModelRunner:

    def __init__(self, config, rank: int, event=None):
        self.config = config
        self.block_size = config.kvcache_block_size
        self.enforce_eager = config.enforce_eager
        self.world_size = config.tensor_parallel_size
        self.rank = rank
        self.event = event
        self.shm = None
        self._async_steps, self._async_bs = 0, 0
        self._pending: list[PendingDecode | None] = [None, None]
        self.owns_process_group = False
        if not dist.is_initialized():
            dist.init_process_group("nccl", f"tcp://127.0.0.1:{config.rdzv_port}", world_size=self.world_size,
                                    rank=rank, device_id=torch.device(f"cuda:{self._local_device(rank)}"),
                                    timeout=datetime.timedelta(seconds=300))
            self.owns_process_group = True
        if dist.get_world_size() != self.world_size:
            raise RuntimeError(f"process group has {dist.get_world_size()} ranks, config asks for {self.world_size}")
        self.device = torch.device("cuda", self._local_device(rank))
        torch.cuda.set_device(self.device)
        set_gemm_backend(config.gemm_backend)
        if config.gemm_backend == "tcgen05":
            K.gemm_set_l2_prefetch(config.gemm_l2_prefetch)
        if config.pdl:
            K.set_pdl(True)
        prev_dtype = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        torch.set_default_device(self.device)
        try:
            Sequence.block_size = config.kvcache_block_size
            self.model = AutoModelForCausalLM.from_pretrained(config.hf_config, load_format=config.load_format,
                                                              seed=config.seed)
            self.tp_allreduce = None
            self.decode_microbatches = None
            if self.world_size > 1 and config.fused_allreduce:
                max_tokens = max(config.max_num_batched_tokens, self._max_graph_bs())
                self.tp_allreduce = TPAllReduce(max_tokens, config.hf_config.hidden_size, self.device)
                set_tp_allreduce(self.tp_allreduce)
                if config.decode_microbatches == 2:  # two decode halves, a communicator each
                    half = (self._max_graph_bs() + 1) // 2
                    comms = tuple(TPAllReduce(half, config.hf_config.hidden_size, self.device,
                                              max_blocks=DecodeMicrobatches.MAX_BLOCKS) for _ in range(2))
                    self.decode_microbatches = DecodeMicrobatches(comms, config.decode_microbatch_min_bs,
                                                                  torch.cuda.Stream(self.device))
                    set_decode_microbatches(self.decode_microbatches)
            self.sampler = Sampler()
            self.staging = Staging(self.device)
            self.allocate_kv_cache()
            self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
            self.graph_pool = None
            if not self.enforce_eager:
                self.capture_cudagraph()
        finally:
            torch.set_default_device("cpu")
            torch.set_default_dtype(prev_dtype)
        if self.world_size > 1 and event is not None:
            self._open_mailbox()

    @staticmethod
    def _local_device(rank: int) -> int:
        if "LOCAL_RANK" in os.environ:
            return int(os.environ["LOCAL_RANK"])
        return rank % max(1, torch.cuda.device_count())

    # ------------------------------------------------------------ TP mailbox
    def _mailbox_name(self) -> str:
        return f"kavor_b200_{self.config.rdzv_port}"

    def _open_mailbox(self) -> None:
        name = self._mailbox_name()
        if self.rank == 0:
            try:
                stale = SharedMemory(name=name)
                stale.close()
                stale.unlink()
            except FileNotFoundError:
                pass
            self.shm = SharedMemory(name=name, create=True, size=SHM_BYTES)
            dist.barrier()
        else:
            dist.barrier()
            self.shm = SharedMemory(name=name)
            self.loop()

    def loop(self) -> None:
        try:
            while True:
                method, args = self.read_shm()
                self.call(method, *args)
                if method == "exit":
                    break
        except BaseException:
            # a stop request (SIGTERM turned into SystemExit by the engine's
            # worker entry), rank 0 gone, or a failed call: release this
            # rank's areas in order instead of leaving them to process exit
            self.abandon()
            raise

    def read_shm(self):
        parent = multiprocessing.parent_process()
        while not self.event.wait(MAILBOX_POLL_S):
            if parent is not None and not parent.is_alive():
                raise SystemExit(f"TP worker {self.rank}: rank 0's process exited without sending exit")
        n = int.from_bytes(self.shm.buf[0:4], "little")
        method, *args = pickle.loads(self.shm.buf[4:n + 4])
        self.event.clear()
        return method, args

    def write_shm(self, method: str, *args) -> None:
        data = pickle.dumps([method, *args])
        if len(data) + 4 > len(self.shm.buf):
            raise RuntimeError(f"TP message of {len(data)} bytes exceeds the {len(self.shm.buf)}-byte mailbox")
        # every worker has taken the previous message (a worker clears its event
        # after reading): calls that return before the step completes
        # (run_async) can otherwise come back before a worker has read
        deadline = time.monotonic() + MAILBOX_WAIT_S
        for ev in self.event:
            while ev.is_set():
                if time.monotonic() > deadline:
                    raise RuntimeError(f"a TP worker did not take the previous message within {MAILBOX_WAIT_S:.0f} s")
                time.sleep(0)
        self.shm.buf[0:4] = len(data).to_bytes(4, "little")
        self.shm.buf[4:len(data) + 4] = data
        for ev in self.event:
            ev.set()

    def call(self, method: str, *args):
        """Run `method` on every rank (model_runner.py:108-112). A model step
        ("run", "run_async") has its batch metadata built once, here on rank 0,
        and the workers receive those arrays (a few KB for a decode step)
        instead of the pickled sequences, so they neither unpickle the
        sequences nor rebuild the metadata."""
        if method in ("run", "run_async"):
            seqs, arg = args
            method, args = method + "_step", self._step_metadata(seqs, arg if method == "run" else False) + (arg,)
        if self.world_size > 1 and self.rank == 0 and self.shm is not None:
            self.write_shm(method, *args)
        return getattr(self, method)(*args)

    def exit(self) -> None:
        if self.shm is not None:
            self.shm.close()
            dist.barrier()
            if self.rank == 0:
                self.shm.unlink()
            self.shm = None
        self.graphs.clear()
        self.graph_pool = None
        torch.cuda.synchronize()
        if self.decode_microbatches is not None:
            set_decode_microbatches(None)
            self.decode_microbatches.close()
            self.decode_microbatches = None
        if self.tp_allreduce is not None:
            set_tp_allreduce(None)
            self.tp_allreduce.close()
            self.tp_allreduce = None
        if self.owns_process_group and dist.is_initialized():
            dist.destroy_process_group()

    def abandon(self) -> None:
        """Leave without the exit message (a worker that was asked to stop, or
        whose rank 0 is gone): no mailbox barrier; the device is drained and
        the all-reduce areas are closed (collectively: the other ranks' kernels
        may still read this rank's buffers, and the process-group timeout
        bounds the wait for a rank that is gone) before the process group is
        destroyed, so no area that may be bound to an NVLink multicast object
        disappears under a peer that is still using it."""
        if self.shm is not None:
            self.shm.close()
            self.shm = None
        self.graphs.clear()
        self.graph_pool = None
        try:
            torch.cuda.synchronize()
            for comm in (self.decode_microbatches, self.tp_allreduce):
                if comm is not None:
                    comm.close()
        except Exception:  # noqa: BLE001 - a peer is gone: the barrier timed out
            pass
        self.decode_microbatches = self.tp_allreduce = None
        set_decode_microbatches(None)
        set_tp_allreduce(None)
        if self.owns_process_group and dist.is_initialized():
            dist.destroy_process_group()

    # ------------------------------------------------------------ KV pool
    def _max_graph_bs(self) -> int:
        return min(self.config.max_num_seqs, 512)

    @property
    def max_blocks_per_seq(self) -> int:
        return (self.config.max_model_len + self.block_size - 1) // self.block_size

    @torch.inference_mode()
    def _profile_prefill(self) -> None:
        self._sync_ranks()
        seq_len = min(self.config.max_num_batched_tokens, self.config.max_model_len)
        num_seqs = max(1, min(self.config.max_num_batched_tokens // seq_len, self.config.max_num_seqs))
        total = seq_len * num_seqs
        ids = torch.zeros(total, dtype=torch.int64, device=self.device)
        pos = torch.arange(seq_len, device=self.device).repeat(num_seqs)
        cu = torch.arange(0, total + 1, seq_len, dtype=torch.int32, device=self.device)
        set_context(True, cu, cu, seq_len, seq_len, torch.zeros(total, dtype=torch.int32, device=self.device))
        try:
            hidden = self.model(ids, pos)
            temps = torch.ones(num_seqs, dtype=torch.float32, device=self.device)
            self.model.lm_head.sample(hidden, temps, self.sampler.seed)
        finally:
            reset_context()

    @torch.inference_mode()
    def _profile_decode(self, bs: int) -> None:
        self._sync_ranks()
        set_context(False, slot_mapping=torch.zeros(bs, dtype=torch.int32, device=self.device),
                    context_lens=torch.ones(bs, dtype=torch.int32, device=self.device),
                    block_tables=torch.zeros(bs, self.max_blocks_per_seq, dtype=torch.int32, device=self.device))
        try:
            K.WORKSPACE.reserve(self._decode_workspace_bytes(bs), self.device)
            hidden = self.model(torch.zeros(bs, dtype=torch.int64, device=self.device),
                                torch.zeros(bs, dtype=torch.int64, device=self.device))
            self.model.lm_head.sample(hidden, torch.ones(bs, dtype=torch.float32, device=self.device),
                                      self.sampler.seed)
        finally:
            reset_context()

    def _decode_workspace_bytes(self, bs: int) -> int:
        cfg = self.config.hf_config
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        return K.decode_workspace_bytes(bs, cfg.num_attention_heads // self.world_size,
                                        cfg.num_key_value_heads // self.world_size, hd, self.max_blocks_per_seq,
                                        self.block_size)

    def allocate_kv_cache(self) -> None:
        self.cache = CachePool(self.model, self.config, self.world_size)

        def peak(fn) -> int:
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats()
            base = torch.cuda.memory_allocated()
            fn()
            torch.cuda.synchronize()
            return torch.cuda.max_memory_allocated() - base

        prefill_peak = peak(self._profile_prefill)
        self.cache.allocate(num_blocks=2)
        decode_peak = peak(lambda: self._profile_decode(self._max_graph_bs()))
        reserve = (0 if self.enforce_eager else decode_peak) + max(prefill_peak, decode_peak)
        if self.config.num_kvcache_blocks > 0:
            layout = self.cache.allocate(num_blocks=self.config.num_kvcache_blocks)
        else:
            layout = self.cache.allocate(reserve=reserve)
        self.config.num_kvcache_blocks = layout.num_blocks

    # ------------------------------------------------------------ step
    def _decode_forward(self, bs: int) -> None:
        d = self.decode_buffers.d
        hidden = self.model(d["input_ids"][:bs], d["positions"][:bs])
        self.sampler.seed.add_(1)
        self.model.lm_head.sample(hidden, d["temperatures"][:bs], self.sampler.seed,
                                  out=self.decode_buffers.sampled[:bs])

    def _sync_ranks(self) -> None:
        """Before a forward that runs the fused all-reduce during set-up: the
        ranks' host work so far differs, and the kernel's peer wait is bounded."""
        if self.world_size > 1:
            torch.cuda.synchronize(self.device)
            dist.barrier()

    @torch.inference_mode()
    def capture_cudagraph(self) -> None:
        max_bs = self._max_graph_bs()
        self.decode_buffers = DecodeBuffers(max_bs, self.max_blocks_per_seq, self.device)
        if self.config.graph_batch_sizes:
            self.graph_bs = sorted(b for b in set(self.config.graph_batch_sizes) if 1 <= b <= max_bs)
        else:
            self.graph_bs = [b for b in (1, 2, 4, 8) if b <= max_bs] + list(range(16, max_bs + 1, 16))
        if not self.graph_bs or self.graph_bs[-1] != max_bs:
            self.graph_bs.append(max_bs)
        # scratch is allocated outside capture, sized for the largest need of any bucket
        K.WORKSPACE.reserve(max(self._decode_workspace_bytes(b) for b in self.graph_bs), self.device)
        d = self.decode_buffers.d
        seed0 = self.sampler.seed.clone()
        self.graph_launches: dict[int, int] = {}
        for bs in reversed(self.graph_bs):
            set_context(False, slot_mapping=d["slot_mapping"][:bs], context_lens=d["context_lens"][:bs],
                        block_tables=d["block_tables"][:bs])
            self._sync_ranks()
            self._decode_forward(bs)  # warm-up outside the graph
            graph = torch.cuda.CUDAGraph()
            calls0 = _lib.launch_count()
            with torch.cuda.graph(graph, self.graph_pool):
                self._decode_forward(bs)
            self.graph_launches[bs] = _lib.launch_count() - calls0
            if self.graph_pool is None:
                self.graph_pool = graph.pool()
            self.graphs[bs] = graph
            torch.cuda.synchronize()
            reset_context()
        self.sampler.seed.copy_(seed0)

    def _ensure_decode_buffers(self) -> None:
        if not hasattr(self, "decode_buffers"):
            self.decode_buffers = DecodeBuffers(self._max_graph_bs(), self.max_blocks_per_seq, self.device)

    # Every DEVICE_CHECK_EVERY steps the device-side error bits are read back
    # (a synchronising query): a bounded wait that gave up (a peer that did not
    # arrive within about a second), an index outside its buffer, ... raise
    # here instead of going unnoticed.
    DEVICE_CHECK_EVERY = 64

    def _check_device(self) -> None:
        self._steps = getattr(self, "_steps", 0) + 1
        if self._steps % self.DEVICE_CHECK_EVERY:
            return
        bits = _lib.device_error(clear=True)
        if bits:
            names = {1: "block table", 2: "slot mapping", 4: "wait timeout", 8: "token id", 16: "peer wait timeout",
                     32: "launch configuration"}
            what = ", ".join(n for b, n in names.items() if bits & b)
            raise RuntimeError(f"rank {self.rank}: device-side error bits {bits:#x} ({what}) within the last "
                               f"{self.DEVICE_CHECK_EVERY} steps")

    def _step_metadata(self, seqs: list[Sequence], is_prefill: bool) -> tuple[dict, np.ndarray]:
        """The host arrays of one model step: prefill_metadata / decode_metadata
        and the sampling temperatures."""
        temps = np.fromiter(map(_TEMPERATURE, seqs), np.float32, len(seqs))
        if is_prefill:
            return prefill_metadata(seqs, self.block_size), temps
        return decode_metadata(seqs, self.block_size), temps

    def run(self, seqs: list[Sequence], is_prefill: bool) -> list[int]:
        """One model step of `seqs` (model_runner.py:247-263): the sampled token
        of every sequence."""
        return self.run_step(*self._step_metadata(seqs, is_prefill), is_prefill)

    @torch.inference_mode()
    def run_step(self, meta: dict, temps: np.ndarray, is_prefill: bool) -> list[int]:
        """``run`` from the step's metadata arrays (what a TP worker receives)."""
        self._check_device()
        if is_prefill:
            arrays = [meta["input_ids"], meta["positions"], meta["cu_seqlens_q"], meta["cu_seqlens_k"],
                      meta["slot_mapping"], temps]
            if meta["block_tables"] is not None:
                arrays.append(meta["block_tables"])
            dev = self.staging.upload(arrays)
            ids, pos, cu_q, cu_k, slots, t_dev = dev[:6]
            set_context(True, cu_q, cu_k, meta["max_seqlen_q"], meta["max_seqlen_k"], slots, None,
                        dev[6] if len(dev) > 6 else None)
            try:
                hidden = self.model(ids, pos)
                self.sampler.seed.add_(1)
                tokens = self.model.lm_head.sample(hidden, t_dev, self.sampler.seed)
            finally:
                reset_context()
            return tokens.tolist()
        bs = self._decode_launch(meta, temps, mirror=0, chain=False)
        return self.decode_buffers.sampled[:bs].tolist()

    def _decode_launch(self, meta: dict, temps: np.ndarray, mirror: int, chain) -> int:
        """Upload one decode step's metadata (through pinned mirror `mirror`),
        optionally take the input tokens from the previous step's samples on
        the device (chain True: row i from row i; a list: row i from row
        chain[i]), and launch the step (graph replay, or eager)."""
        bs = len(temps)
        self._ensure_decode_buffers()
        buf = self.decode_buffers
        if bs > buf.max_bs or meta["block_tables"].shape[1] > buf.max_blocks:
            raise RuntimeError(f"decode batch {bs} x {meta['block_tables'].shape[1]} blocks exceeds the "
                               f"runner's {buf.max_bs} x {buf.max_blocks}")
        bucket = next((b for b in getattr(self, "graph_bs", []) if b >= bs), bs)
        buf.fill(meta, temps, bucket, mirror)
        if chain is True:
            buf.d["input_ids"][:bs].copy_(buf.sampled[:bs])
        elif chain:
            k = mirror - 1
            if buf.chain_copied[k] is not None:
                buf.chain_copied[k].synchronize()
            buf.chain_host[k][:bs] = torch.as_tensor(chain, dtype=torch.int64)
            buf.chain_dev[:bs].copy_(buf.chain_host[k][:bs], non_blocking=True)
            buf.chain_copied[k] = torch.cuda.Event()
            buf.chain_copied[k].record()
            torch.index_select(buf.sampled, 0, buf.chain_dev[:bs], out=buf.d["input_ids"][:bs])
        graph = self.graphs.get(bucket)
        if graph is not None:
            graph.replay()
        else:
            d = buf.d
            set_context(False, slot_mapping=d["slot_mapping"][:bs], context_lens=d["context_lens"][:bs],
                        block_tables=d["block_tables"][:bs])
            try:
                self._decode_forward(bs)
            finally:
                reset_context()
        return bs

    def run_async(self, seqs: list[Sequence], chain: bool | list[int] = False) -> PendingDecode | None:
        return self.run_async_step(*self._step_metadata(seqs, False), chain)

    @torch.inference_mode()
    def run_async_step(self, meta: dict, temps: np.ndarray, chain: bool | list[int] = False) -> PendingDecode | None:
        """One decode step, issued without waiting for it (no reference
        counterpart; ``run`` is the reference's synchronous call). With
        ``chain``, every sequence's input token is the token the previous
        ``run_async`` step sampled for it, copied on the device: True when the
        batch is the previous step's sequences in the same order, or a list
        giving each sequence's row in the previous step's batch; each sequence
        grew on the host since by one placeholder token (its value is not
        read). Returns a PendingDecode,
        whose ``result()`` must be read before the step after the next one is
        issued — except on a TP worker driven through the mailbox by rank 0,
        which returns None (every rank samples the same tokens; rank 0 reads
        them)."""
        self._check_device()
        k = self._async_steps % 2
        self._async_steps += 1
        mailbox_worker = self.rank > 0 and self.shm is not None
        prev = self._pending[k]
        if prev is not None and not prev.done and not mailbox_worker:
            raise RuntimeError("run_async: the result of the step issued two calls ago has not been read")
        n = len(temps)
        if chain is True and n != self._async_bs:
            raise RuntimeError(f"run_async: a chained step needs the previous step's {self._async_bs} sequences")
        if isinstance(chain, list) and (len(chain) != n or not all(0 <= i < self._async_bs for i in chain)):
            raise RuntimeError(f"run_async: the chain map must give every sequence a row of the previous "
                               f"{self._async_bs}-sequence step")
        bs = self._decode_launch(meta, temps, mirror=1 + k, chain=chain)
        self._async_bs = bs
        if mailbox_worker:
            return None
        buf = self.decode_buffers
        host = buf.tokens_host[k]
        host[:bs].copy_(buf.sampled[:bs], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._pending[k] = PendingDecode(host, ev, bs)
        return self._pending[k]
