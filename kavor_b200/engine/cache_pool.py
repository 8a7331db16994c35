"""Paged KV pool (drop-in for the attention part of kavor/engine/cache_pool.py).

HBM layout (cache_pool.py:311-322): one uint8 pool per attention layer,
``pools[L, num_blocks, page_bytes]``; a page holds the K block
``[block_size, Hkv, head_dim]`` followed by the V block of the same shape, so
``k_cache = pools[l].view(bf16).as_strided([num_blocks, block_size, Hkv, hd],
[2 * block_elems, Hkv * hd, hd, 1])`` and ``v_cache`` is the same view offset
by ``block_elems``. The decode kernel's tensor map walks exactly these strides.

The number of blocks comes from the free device memory after the weights and a
measured activation reserve, agreed across TP ranks with a MIN all-reduce
(cache_pool.py:292-307).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class CacheLayout:
    num_layers: int
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    page_bytes: int

    @property
    def bytes_per_token(self) -> int:
        return self.page_bytes // self.block_size * self.num_layers


class CachePool:

    def __init__(self, model: torch.nn.Module, config, world_size: int):
        self.model = model
        self.config = config
        self.world_size = world_size
        self.layout: CacheLayout | None = None
        self.pools: torch.Tensor | None = None

    def attention_slots(self):
        slots = []
        for module in self.model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                slots.extend((module, i) for i in range(module.num_kv_slots))
        if not slots:
            raise RuntimeError("the model has no attention layers to bind a KV pool to")
        return slots

    def _all_reduce_min(self, value: int) -> int:
        if self.world_size == 1 or not dist.is_initialized():
            return value
        dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
        t = torch.tensor([value], dtype=torch.int64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    def plan(self, reserve: int = 0, num_blocks: int | None = None) -> CacheLayout:
        cfg = self.config.hf_config
        hkv = cfg.num_key_value_heads // self.world_size
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        dtype = torch.bfloat16
        block_size = self.config.kvcache_block_size
        page_bytes = 2 * hkv * hd * dtype.itemsize * block_size
        layers = len(self.attention_slots())
        if num_blocks is None:
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            free, total = torch.cuda.mem_get_info()
            budget = int(total * self.config.gpu_memory_utilization - (total - free)) - reserve
            num_blocks = budget // (layers * page_bytes)
        num_blocks = self._all_reduce_min(int(num_blocks))
        if num_blocks < 1:
            raise RuntimeError(
                f"the KV pool would hold {num_blocks} blocks after a {reserve / 2**20:.0f} MiB activation reserve;"
                " lower max_num_seqs / max_model_len or raise gpu_memory_utilization")
        self.layout = CacheLayout(layers, num_blocks, block_size, hkv, hd, dtype, page_bytes)
        return self.layout

    def allocate(self, reserve: int = 0, num_blocks: int | None = None) -> CacheLayout:
        self.unbind()
        layout = self.plan(reserve=reserve, num_blocks=num_blocks)
        self.pools = torch.empty(layout.num_layers, layout.num_blocks, layout.page_bytes, dtype=torch.uint8,
                                 device="cuda")
        block_elems = layout.block_size * layout.num_kv_heads * layout.head_dim
        shape = (layout.num_blocks, layout.block_size, layout.num_kv_heads, layout.head_dim)
        strides = (layout.page_bytes // layout.dtype.itemsize, layout.num_kv_heads * layout.head_dim,
                   layout.head_dim, 1)
        for pool, (module, slot) in enumerate(self.attention_slots()):
            flat = self.pools[pool].view(layout.dtype)
            base = flat.storage_offset()
            module.k_cache[slot] = flat.as_strided(shape, strides, base)
            module.v_cache[slot] = flat.as_strided(shape, strides, base + block_elems)
        return layout

    def unbind(self) -> None:
        if self.pools is None:
            return
        for module, slot in self.attention_slots():
            module.k_cache[slot] = torch.empty(0, device="cuda")
            module.v_cache[slot] = torch.empty(0, device="cuda")
        self.pools = None
        self.layout = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    @property
    def block_size(self) -> int:
        return self.layout.block_size

    @property
    def num_blocks(self) -> int:
        return self.layout.num_blocks
