"""Import-path alias of the reference module kavor/layers/attention/flash_attention_kvcache.py.

The implementation is ``paged_attention`` (sm_100a kernels, no flash_attn)."""
from kavor_b200.layers.attention.paged_attention import Attention, store_kvcache

__all__ = ["Attention", "store_kvcache"]
