from kavor_b200.layers.attention.paged_attention import Attention, store_kvcache

__all__ = ["Attention", "store_kvcache"]
