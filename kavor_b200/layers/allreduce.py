"""Fused tensor-parallel all-reduce + residual add + RMSNorm over NVLink.

Replaces, for TP > 1, the NCCL all-reduce after every row-parallel projection
and the vocab-parallel embedding (linear.py:158-159, embed_head.py:39-41)
together with the add+RMSNorm that always follows it in Qwen3
(qwen3.py:155-160, 185). Each rank owns a symmetric area: mapped by torch
symmetric memory (peer pointers, and an NVLink multicast mapping where the
NVSwitch offers one, for sums reduced in the switch), or allocated by the
library with its CUDA IPC handles exchanged over the process group. Every call
is then a single kernel that reads the peers' partial sums over NVLink.

The producing kernel (row-parallel GEMM or embedding) writes its rank-local
result straight into one of three data buffers of the symmetric area
(``partial_buffer``); consecutive reductions must use different buffers, which
``next_buffer`` guarantees within a forward (the embedding uses buffer 2,
the layers alternate 0 and 1).
"""
from __future__ import annotations

import contextlib
import ctypes

import torch
import torch.distributed as dist

from kavor_b200 import _lib


class _CudaArray:
    """Zero-copy torch view of device memory owned by the library."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class TPAllReduce:
    """backend: "symmetric" maps the area with torch symmetric memory (peer
    pointers plus, where the NVSwitch supports it, an NVLink multicast mapping
    for the switch-reduced modes); "ipc" lets the library allocate it and
    exchanges CUDA IPC handles; "auto" tries symmetric first."""

    EMBED_BUFFER = 2

    def __init__(self, max_tokens: int, hidden: int, device: torch.device, group=None, backend: str = "auto",
                 mode: int = 0, max_blocks: int | None = None):
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.device = device
        self.mode = mode
        self.comm = ctypes.c_void_p()
        self._symm = None
        self.backend = None
        max_bytes = max_tokens * hidden * 2
        if backend in ("auto", "symmetric"):
            ok = 1
            try:
                self._attach_symmetric(max_bytes, group)
            except Exception as e:  # noqa: BLE001 - fall back to the library's own IPC mapping
                if backend == "symmetric":
                    raise
                self._symm_error = repr(e)
                ok = 0
            # every rank must take the same path
            flag = torch.tensor([ok], dtype=torch.int32, device=device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
            if not int(flag.item()) and self.comm:
                _lib.call("kvb_comm_destroy", self.comm)
                self.comm = ctypes.c_void_p()
                self._symm = None
        if not self.comm:
            self._create_ipc(max_bytes, group)
        self.multicast = bool(_lib.load().kvb_comm_has_multicast(self.comm))
        if max_blocks is not None:  # every rank passes the same value
            _lib.call("kvb_comm_set_max_blocks", self.comm, int(max_blocks))
        self.buffers = []
        for i in range(3):
            ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
            _lib.call("kvb_comm_data_buffer", self.comm, i, ctypes.byref(ptr), ctypes.byref(nbytes))
            raw = torch.as_tensor(_CudaArray(ptr.value, nbytes.value), device=device)
            self.buffers.append(raw.view(torch.bfloat16).view(max_tokens, hidden))
        po, pr = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.call("kvb_comm_result_rows", self.comm, ctypes.byref(po), ctypes.byref(pr))
        self.result_out, self.result_res = (
            torch.as_tensor(_CudaArray(p.value, max_bytes), device=device).view(torch.bfloat16).view(max_tokens, hidden)
            for p in (po, pr))
        dist.barrier(group=group)
        self._next = 0

    def _create_ipc(self, max_bytes: int, group) -> None:
        lib = _lib.load()
        hs = lib.kvb_comm_ipc_handle_size()
        handle = (ctypes.c_ubyte * hs)()
        _lib.call("kvb_comm_create", self.rank, self.world, max_bytes, ctypes.byref(self.comm), handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        _lib.call("kvb_comm_open_peers", self.comm, ctypes.c_char_p(b"".join(handles)))
        self.backend = "ipc"

    def _attach_symmetric(self, max_bytes: int, group) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        n = ctypes.c_size_t()
        _lib.call("kvb_comm_area_size", max_bytes, ctypes.byref(n))
        area = symm_mem.empty(int(n.value), dtype=torch.uint8, device=self.device)
        area.zero_()
        handle = symm_mem.rendezvous(area, group if group is not None else dist.group.WORLD)
        # the tensor may sit at an offset inside the symmetric allocation
        off = area.data_ptr() - int(handle.buffer_ptrs[self.rank])
        ptrs = [int(p) + off for p in handle.buffer_ptrs]
        mc = int(handle.multicast_ptr) if getattr(handle, "multicast_ptr", 0) else 0
        mc = mc + off if mc else 0
        arr = (ctypes.c_uint64 * self.world)(*ptrs)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        _lib.call("kvb_comm_attach", self.rank, self.world, arr, mc, int(n.value), max_bytes, ctypes.byref(self.comm))
        self._symm = (area, handle)
        self.backend = "symmetric+multicast" if mc else "symmetric"

    def start_forward(self) -> None:
        self._next = 0

    def next_buffer(self, tokens: int) -> tuple[int, torch.Tensor]:
        idx = self._next
        self._next ^= 1
        return idx, self.partial_buffer(idx, tokens)

    def partial_buffer(self, index: int, tokens: int) -> torch.Tensor:
        if tokens > self.max_tokens:
            raise RuntimeError(f"{tokens} tokens exceed the all-reduce buffers ({self.max_tokens})")
        return self.buffers[index][:tokens]

    def reduce_norm(self, index: int, tokens: int, residual: torch.Tensor | None, weight: torch.Tensor, eps: float,
                    mode: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        """(RMSNorm(sum + residual), sum + residual) with the residual updated in
        place. In the switch two-shot mode both come back as views of this
        rank's result rows (where the NVSwitch delivered them), valid until the
        next call."""
        mode = mode or self.mode
        if self.switch_two_shot(tokens, mode):
            out, res_out = self.result_out[:tokens], self.result_res[:tokens]
            mode = 4
        else:
            out = torch.empty(tokens, self.hidden, dtype=torch.bfloat16, device=self.device)
            res_out = residual if residual is not None else torch.empty_like(out)
            if res_out.data_ptr() == self.result_res.data_ptr():  # the residual stream leaves the result rows
                res_out = torch.empty_like(out)
        _lib.call("kvb_allreduce_add_rmsnorm", self.comm, index,
                  residual.data_ptr() if residual is not None else None, res_out.data_ptr(), out.data_ptr(),
                  weight.data_ptr(), tokens, self.hidden, float(eps), mode, torch.cuda.current_stream().cuda_stream)
        return out, res_out

    def switch_two_shot(self, tokens: int, mode: int = 0) -> bool:
        """Whether the library runs the switch two-shot for this call (its own
        choice in mode 0, asked through kvb_allreduce_plan)."""
        return self.multicast and allreduce_plan(self.world, True, tokens, self.hidden, mode)["switch"] == 2

    def close(self, group=None) -> None:
        """Collective: every rank's kernels that read this rank's buffers must
        be finished before the buffers are unmapped and freed."""
        if self.comm:
            torch.cuda.synchronize(self.device)
            if dist.is_initialized():
                dist.barrier(group=group)
                torch.cuda.synchronize(self.device)
            _lib.call("kvb_comm_destroy", self.comm)
            self.comm = ctypes.c_void_p()
            self.buffers = []
            self._symm = None


def allreduce_plan(world: int, multicast: bool, tokens: int, hidden: int, mode: int = 0) -> dict:
    """The exchange the fused kernel picks: {"peer_two_shot": 0/1, "switch": 0
    (peer modes), 1 (switch one-shot) or 2 (switch two-shot)}."""
    plan = (ctypes.c_int * 2)()
    _lib.call("kvb_allreduce_plan", world, 1 if multicast else 0, tokens, hidden, mode, plan)
    return {"peer_two_shot": plan[0], "switch": plan[1]}


class DecodeMicrobatches:
    """Plan of a TP > 1 decode step run as two micro-batches: rows [0, h) on
    the launching stream, rows [h, T) on a second stream, each half with its
    own communicator (its all-reduces are ordered on its stream, and two
    communicators never share flags, counters or buffers). The decode
    attention kernels of the two halves take turns (each waits for the
    previous one, whichever half ran it), so one half's attention, bound by
    HBM bandwidth, runs beside the other half's GEMMs and all-reduces, which
    are bound by latency at decode sizes.

    Every block of an all-reduce call spins, holding its SM slot, until the
    same block has arrived on every peer. With both halves' calls in flight,
    uncapped grids could hold a slot on every SM and leave no room for a
    kernel that needs a whole SM and that a peer's call waits behind; both
    communicators therefore cap their grids (``max_blocks``) so that SMs stay
    free for the other kernels.

    ``side_stream``: the second half's stream; None runs both halves on the
    current stream (no CUDA: the CPU tests of the wiring)."""

    MAX_BLOCKS = 64

    def __init__(self, comms: tuple, min_tokens: int, side_stream=None):
        if len(comms) != 2:
            raise ValueError("DecodeMicrobatches needs one communicator per half")
        self.comms = tuple(comms)
        self.min_tokens = max(2, int(min_tokens))
        self.side = side_stream
        self._last = None  # (half, event) of the latest attention

    def applies(self, tokens: int) -> bool:
        return tokens >= self.min_tokens and all(tokens - tokens // 2 <= c.max_tokens for c in self.comms)

    @staticmethod
    def spans(tokens: int) -> tuple[tuple[int, int], tuple[int, int]]:
        h = (tokens + 1) // 2
        return (0, h), (h, tokens)

    def fork(self) -> None:
        """Start of a step: the second stream waits for the work issued so far."""
        self._last = None
        if self.side is not None:
            self.side.wait_stream(torch.cuda.current_stream())

    def join(self) -> None:
        """End of a step: the launching stream waits for the second half."""
        self._last = None
        if self.side is not None:
            torch.cuda.current_stream().wait_stream(self.side)

    def on(self, half: int):
        """Issue the block's work for micro-batch `half` on its stream."""
        if half == 0 or self.side is None:
            return contextlib.nullcontext()
        return torch.cuda.stream(self.side)

    @contextlib.contextmanager
    def attention_turn(self, half: int):
        """Around one half's decode attention: wait until the previous
        attention (if the other half ran it) is complete, then mark this one."""
        if self.side is not None and self._last is not None and self._last[0] != half:
            torch.cuda.current_stream().wait_event(self._last[1])
        yield
        if self.side is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
            self._last = (half, ev)

    def close(self, group=None) -> None:
        for c in self.comms:
            c.close(group)


_TP: TPAllReduce | None = None
_MICROBATCH: DecodeMicrobatches | None = None


def set_decode_microbatches(plan: DecodeMicrobatches | None) -> None:
    global _MICROBATCH
    _MICROBATCH = plan


def get_decode_microbatches() -> DecodeMicrobatches | None:
    return _MICROBATCH


def set_tp_allreduce(comm: TPAllReduce | None) -> None:
    global _TP
    _TP = comm


def get_tp_allreduce() -> TPAllReduce | None:
    return _TP
