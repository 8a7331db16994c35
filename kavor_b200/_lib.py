"""ctypes binding of ``libkavor_b200.so`` (the C ABI in ``include/kavor_b200.h``).

The library is built in tree by ``python -m kavor_b200.build``. There is no
fallback: if it is missing or fails to load, every op raises. A non-zero
status returned by an entry point becomes a ``RuntimeError`` carrying the
library's own message (``kvb_last_error``), mirroring the assert/raise style
of the reference layers (e.g. flash_attention_kvcache.py:40-43).
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libkavor_b200.so")

P = c_void_p
I = c_int
L = c_int64
F = c_float

# name -> argument types (all entry points return int status)
SIGNATURES: dict[str, list] = {
    "kvb_version": [],
    "kvb_device_error": [POINTER(c_uint), I],
    "kvb_sm_count": [POINTER(c_int)],
    "kvb_store_kv": [P, L, P, L, P, P, L, L, I, I, I, P, I, P],
    "kvb_rmsnorm": [P, L, L, P, L, L, P, I, I, I, F, P],
    "kvb_add_rmsnorm": [P, P, P, P, I, I, F, P],
    "kvb_rope": [P, L, L, P, L, L, P, P, L, I, I, I, I, I, P],
    "kvb_qknorm_rope_store": [P, L, I, I, I, I, P, P, F, I, P, P, L, I, P, P, L, L, I, P, P],
    "kvb_silu_mul": [P, L, P, L, I, I, P],
    "kvb_embedding": [P, P, P, I, I, L, L, L, P],
    "kvb_paged_decode_attn_workspace_size": [I, I, I, I, I, I, I, POINTER(c_size_t)],
    "kvb_paged_decode_attn": [P, L, L, P, P, L, L, I, P, L, I, P, P, L, L, I, I, I, I, F, I, P, c_size_t, P],
    "kvb_paged_decode_attn_no_alloc": [P, L, L, P, P, L, L, I, P, L, I, P, P, L, L, I, I, I, I, F, I, P],
    "kvb_prefill_attn": [P, L, L, P, L, L, P, L, L, L, L, I, P, L, I, P, P, I, I, P, L, L, I, I, I, F, L, L, P],
    "kvb_sample": [P, L, P, P, P, I, I, P],
    "kvb_sample_partial": [P, L, P, P, P, P, I, I, L, L, P],
    "kvb_sample_combine": [P, P, I, P, I, P],
    "kvb_gemm_workspace_size": [I, I, I, I, POINTER(c_size_t)],
    "kvb_gemm_bf16": [P, L, P, L, P, L, I, I, I, I, P, c_size_t, P],
    "kvb_gemm_plan": [I, I, I, I, I, POINTER(c_int)],
    "kvb_gemm_set_l2_prefetch": [I],
    "kvb_gemm_pair_bf16": [P, L, P, L, P, L, I, I, I, I, P],
    "kvb_gemm_pair_silu_bf16": [P, L, P, L, P, L, I, I, I, I, P],
    "kvb_gemm_pair_plan": [I, I, I, I, I, POINTER(c_int)],
    "kvb_gemm_sk_workspace_size": [I, I, I, I, POINTER(c_size_t)],
    "kvb_gemm_sk_bf16": [P, L, P, L, P, L, I, I, I, P, c_size_t, P],
    "kvb_gemm_sk_silu_bf16": [P, L, P, L, P, L, I, I, I, P, c_size_t, P],
    "kvb_gemm_sk_plan": [I, I, I, I, POINTER(c_int)],
    "kvb_gemm_sk_set_plan": [I, I],
    "kvb_set_pdl": [I],
    "kvb_gemm_silu_workspace_size": [I, I, I, I, POINTER(c_size_t)],
    "kvb_gemm_silu_bf16": [P, L, P, L, P, L, I, I, I, I, P, c_size_t, P],
    "kvb_comm_ipc_handle_size": [],
    "kvb_comm_create": [I, I, c_size_t, POINTER(c_void_p), P],
    "kvb_comm_open_peers": [P, P],
    "kvb_comm_data_buffer": [P, I, POINTER(c_void_p), POINTER(c_size_t)],
    "kvb_comm_destroy": [P],
    "kvb_comm_area_size": [c_size_t, POINTER(c_size_t)],
    "kvb_comm_attach": [I, I, POINTER(ctypes.c_uint64), ctypes.c_uint64, c_size_t, c_size_t, POINTER(c_void_p)],
    "kvb_comm_has_multicast": [P],
    "kvb_comm_set_max_blocks": [P, I],
    "kvb_comm_result_rows": [P, POINTER(c_void_p), POINTER(c_void_p)],
    "kvb_allreduce_plan": [I, I, I, I, I, POINTER(c_int)],
    "kvb_allreduce_add_rmsnorm": [P, I, P, P, P, P, I, I, F, I, P],
}

_lib: ctypes.CDLL | None = None

# Entry points that only query or report (everything else launches kernels).
_QUERIES = {
    "kvb_version", "kvb_device_error", "kvb_sm_count", "kvb_paged_decode_attn_workspace_size",
    "kvb_gemm_workspace_size", "kvb_gemm_silu_workspace_size", "kvb_gemm_plan", "kvb_gemm_set_l2_prefetch",
    "kvb_set_pdl", "kvb_gemm_pair_plan", "kvb_comm_ipc_handle_size", "kvb_comm_area_size", "kvb_comm_attach",
    "kvb_comm_has_multicast", "kvb_comm_set_max_blocks", "kvb_comm_result_rows", "kvb_allreduce_plan", "kvb_comm_create", "kvb_comm_open_peers",
    "kvb_comm_data_buffer", "kvb_comm_destroy", "kvb_gemm_sk_workspace_size", "kvb_gemm_sk_plan",
    "kvb_gemm_sk_set_plan",
}
# Number of launching entry-point calls made so far (per name); used to count
# the kernels a captured CUDA graph contains.
CALLS: dict[str, int] = {}


def load() -> ctypes.CDLL:
    """Load (once) and declare the library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"kavor_b200 kernel library not found at {LIB_PATH}; build it with "
            "`python -m kavor_b200.build` (needs nvcc). There is no CPU or eager fallback.")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = c_int
    lib.kvb_last_error.argtypes = []
    lib.kvb_last_error.restype = ctypes.c_char_p
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return sorted([*SIGNATURES, "kvb_last_error"])


def check(status: int, name: str) -> None:
    if status != 0:
        msg = load().kvb_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed with status {status}: {msg}")


def call(name: str, *args) -> None:
    """Call entry point ``name`` and raise on a non-zero status."""
    rc = getattr(load(), name)(*args)
    if name == "kvb_comm_ipc_handle_size":
        return rc
    check(rc, name)
    if name not in _QUERIES:
        CALLS[name] = CALLS.get(name, 0) + 1


def launch_count() -> int:
    return sum(CALLS.values())


# Called with the bits when device_error(clear=True) reads and clears a
# non-zero word: state that a kernel which gave up may have left behind (the
# stream-K GEMM's hand-off flags) is reset there, so no later launch reads it.
_ON_CLEARED_ERROR: list = []


def on_cleared_device_error(fn) -> None:
    """Register ``fn(bits)``, run after device_error(clear=True) cleared non-zero bits."""
    if fn not in _ON_CLEARED_ERROR:
        _ON_CLEARED_ERROR.append(fn)


def device_error(clear: bool = True) -> int:
    """Device-side error bits of the current device (synchronises)."""
    bits = c_uint(0)
    call("kvb_device_error", ctypes.byref(bits), 1 if clear else 0)
    if clear and bits.value:
        for fn in _ON_CLEARED_ERROR:
            fn(int(bits.value))
    return int(bits.value)
