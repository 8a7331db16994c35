"""The C ABI's host-side argument checks (no GPU needed): every entry point
rejects bad sizes, NULL pointers, misalignment and unsupported shapes with a
negative status before any launch (-1 invalid, -2 unsupported), leaves a
message in kvb_last_error, and treats empty work as success. These are the
library's counterparts of the reference layers' asserts
(flash_attention_kvcache.py:40-43)."""
import ctypes

import pytest

from kavor_b200 import _lib

INVALID, UNSUPPORTED = -1, -2
NULL = None
FAKE = ctypes.c_void_p(0x1000)      # a 16-byte-aligned non-NULL value: never dereferenced on a rejected call
ODD = ctypes.c_void_p(0x1008)       # 8-byte aligned only


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def _status(lib, name, *args):
    return getattr(lib, name)(*args)


def _message(lib) -> str:
    return lib.kvb_last_error().decode()


CASES = [
    # name, args, expected status, fragment of the message
    ("kvb_store_kv", (NULL, 0, NULL, 0, NULL, NULL, 0, 0, 256, 8, 128, NULL, -1, NULL), INVALID, "bad sizes"),
    ("kvb_store_kv", (NULL, 0, NULL, 0, NULL, NULL, 0, 0, 256, 8, 128, NULL, 4, NULL), INVALID, "NULL"),
    ("kvb_rmsnorm", (FAKE, 128, 0, FAKE, 128, 0, FAKE, 4, 1, 0, 1e-6, NULL), INVALID, "bad sizes"),
    ("kvb_rmsnorm", (NULL, 128, 0, FAKE, 128, 0, FAKE, 4, 1, 128, 1e-6, NULL), INVALID, "NULL"),
    ("kvb_add_rmsnorm", (FAKE, FAKE, FAKE, FAKE, 4, 4100, 1e-6, NULL), INVALID, "aligned"),
    ("kvb_add_rmsnorm", (ODD, FAKE, FAKE, FAKE, 4, 4096, 1e-6, NULL), INVALID, "aligned"),
    ("kvb_rope", (FAKE, 0, 0, FAKE, 0, 0, FAKE, FAKE, 0, 4, 1, 1, 127, 1024, NULL), INVALID, "bad sizes"),
    ("kvb_silu_mul", (FAKE, 24, FAKE, 12, 4, 12, NULL), INVALID, "aligned"),
    ("kvb_silu_mul", (FAKE, 16, FAKE, 8, 4, 16, NULL), INVALID, "aligned"),  # x rows shorter than 2 x inter
    ("kvb_embedding", (FAKE, FAKE, FAKE, 4, 4096, 10, 5, 0, NULL), INVALID, "bad sizes"),
    ("kvb_paged_decode_attn", (FAKE, 1024, 128, FAKE, FAKE, 8, 2 * 256 * 8 * 128, 256, FAKE, 4, 4, FAKE, FAKE, 1024,
                               128, 4, 8, 8, 64, 0.125, 0, NULL, 0, NULL), UNSUPPORTED, "head_dim"),
    ("kvb_paged_decode_attn", (FAKE, 1024, 128, FAKE, FAKE, 8, 2 * 256 * 8 * 128, 256, FAKE, 4, 4, FAKE, FAKE, 1024,
                               128, 4, 12, 8, 128, 0.125, 0, NULL, 0, NULL), INVALID, "bad sizes"),  # 12 % 8
    ("kvb_paged_decode_attn", (FAKE, 1024, 128, FAKE, FAKE, 8, 2 * 256 * 8 * 128, 256, FAKE, 4, 4, FAKE, FAKE, 1024,
                               128, 4, 72, 8, 128, 0.125, 0, NULL, 0, NULL), UNSUPPORTED, "query heads per kv"),
    ("kvb_prefill_attn", (FAKE, 0, 0, FAKE, 0, 0, FAKE, 0, 0, 0, 0, 0, NULL, 0, 0, FAKE, FAKE, 2, 16, FAKE, 0, 0,
                          8, 8, 64, 0.125, 0, 0, NULL), UNSUPPORTED, "head_dim"),
    ("kvb_gemm_bf16", (FAKE, 64, FAKE, 64, FAKE, 64, -1, 64, 64, 0, NULL, 0, NULL), INVALID, "bad sizes"),
    ("kvb_gemm_bf16", (ODD, 64, FAKE, 64, FAKE, 64, 16, 64, 64, 0, NULL, 0, NULL), INVALID, "aligned"),
    ("kvb_gemm_bf16", (FAKE, 32, FAKE, 64, FAKE, 64, 16, 64, 64, 0, NULL, 0, NULL), INVALID, "leading"),  # ldx < K
    ("kvb_gemm_silu_bf16", (NULL, 64, FAKE, 64, FAKE, 64, 16, 64, 64, 0, NULL, 0, NULL), INVALID, "NULL"),
    ("kvb_sample", (FAKE, 10, FAKE, FAKE, FAKE, 4, 100, NULL), INVALID, "bad sizes"),  # row stride < vocab
    ("kvb_sample_combine", (FAKE, FAKE, 0, FAKE, 4, NULL), INVALID, "bad sizes"),
    ("kvb_comm_create", (0, 3, 1 << 20, ctypes.byref(ctypes.c_void_p()), ctypes.create_string_buffer(64)),
     UNSUPPORTED, "world size"),
    ("kvb_comm_create", (2, 2, 1 << 20, ctypes.byref(ctypes.c_void_p()), ctypes.create_string_buffer(64)),
     INVALID, "bad arguments"),
    ("kvb_allreduce_add_rmsnorm", (NULL, 0, NULL, FAKE, FAKE, FAKE, 4, 4096, 1e-6, 0, NULL), INVALID, "bad arguments"),
    ("kvb_comm_set_max_blocks", (NULL, 64), INVALID, "max_blocks"),
    ("kvb_comm_set_max_blocks", (FAKE, 0), INVALID, "max_blocks"),
    ("kvb_comm_set_max_blocks", (FAKE, 257), INVALID, "max_blocks"),
    ("kvb_allreduce_plan", (8, 1, 4, 4096, 9, ctypes.cast(ctypes.create_string_buffer(8), ctypes.POINTER(ctypes.c_int))),
     INVALID, "bad arguments"),
    ("kvb_gemm_plan", (0, 64, 64, 0, 0, ctypes.cast(ctypes.create_string_buffer(16), ctypes.POINTER(ctypes.c_int))),
     INVALID, "bad sizes"),
    ("kvb_gemm_set_l2_prefetch", (-1,), INVALID, "ksteps"),
    ("kvb_gemm_set_l2_prefetch", (65,), INVALID, "ksteps"),
    ("kvb_set_pdl", (2,), INVALID, "enable"),
    ("kvb_gemm_pair_bf16", (FAKE, 64, FAKE, 64, FAKE, 64, 16, 64, 64, 9, NULL), INVALID, "bad sizes"),  # splits > 8
    ("kvb_gemm_pair_bf16", (ODD, 64, FAKE, 64, FAKE, 64, 16, 64, 64, 0, NULL), INVALID, "aligned"),
    ("kvb_gemm_pair_plan", (0, 64, 64, 0, 0, ctypes.cast(ctypes.create_string_buffer(16), ctypes.POINTER(ctypes.c_int))),
     INVALID, "bad sizes"),
    ("kvb_gemm_pair_silu_bf16", (FAKE, 32, FAKE, 64, FAKE, 64, 16, 64, 64, 0, NULL), INVALID, "bad sizes"),  # ldx < K
]


@pytest.mark.parametrize("name,args,status,fragment", CASES, ids=[f"{c[0]}-{i}" for i, c in enumerate(CASES)])
def test_bad_arguments_are_rejected_on_the_host(lib, name, args, status, fragment):
    assert _status(lib, name, *args) == status
    assert fragment in _message(lib)


def test_tuning_knob_accepts_its_range(lib):
    assert lib.kvb_gemm_set_l2_prefetch(64) == 0
    assert lib.kvb_gemm_set_l2_prefetch(0) == 0


def test_empty_work_is_success(lib):
    assert lib.kvb_store_kv(NULL, 0, NULL, 0, NULL, NULL, 0, 0, 256, 8, 128, NULL, 0, NULL) == 0
    assert lib.kvb_add_rmsnorm(NULL, NULL, NULL, NULL, 0, 4096, 1e-6, NULL) == 0
    assert lib.kvb_silu_mul(NULL, 0, NULL, 0, 0, 128, NULL) == 0
    assert lib.kvb_gemm_bf16(NULL, 64, NULL, 64, NULL, 64, 0, 64, 64, 0, NULL, 0, NULL) == 0
    assert lib.kvb_sample(NULL, 100, NULL, NULL, NULL, 0, 100, NULL) == 0


def test_python_wrappers_raise_with_the_library_message(lib):
    with pytest.raises(RuntimeError, match="bad sizes"):
        _lib.call("kvb_gemm_bf16", FAKE, 64, FAKE, 64, FAKE, 64, -1, 64, 64, 0, NULL, 0, NULL)
