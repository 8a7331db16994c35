"""CPU oracle for Kavor's Qwen3 decode/prefill path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference computes on the hot
path, so the sm_100a kernels of ``kavor_b200`` can be checked against it:

* ``oracle.ops``   — per-kernel restatements (fp32 torch on CPU for the
  floating-point ops, plain index arithmetic for the KV write / metadata),
  each citing the reference file:line it follows;
* ``oracle.model`` — the Qwen3 (and Mistral, ERNIE 4.5) decoder layer / model
  forward composed from ``oracle.ops`` with the reference's residual wiring
  (qwen3.py:149-186);
* ``oracle.host``  — the reference's host-side batch metadata algorithm
  (model_runner.py:385-473) as straight Python loops.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own code
(imported from the reference tree in the build container, eager branches of
its layers) on seeded inputs and commits the results under ``tests/golden``;
``tests/test_oracle_golden.py`` checks this oracle against them. The two
third-party kernels the reference calls (flash-attn 2.8.3.post2 for
attention, NCCL for the all-reduce) are not in the reference tree and cannot
run on a CPU: attention is restated from flash-attn's documented semantics
(causal bottom-right alignment, fp32 softmax, scale head_dim**-0.5, GQA
head mapping). On the CPU that boundary is unpinned; on the GPU the same
flash-attn wheel runs beside the kernels on identical inputs
(tests/test_flash_attn_parity_gpu.py), which the kernels also match against
this oracle.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package. The product (``kavor_b200``) never does.
"""
