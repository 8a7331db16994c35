"""bench.py's arithmetic and its reference arm, on the CPU: the step's
algorithmic HBM bytes and all-reduce bus bytes (the roofline denominators),
the per-projection GEMM dispatch it reports, its argument rules, and the
reference arm's JSON line on a small case."""
import json

import pytest

import bench


def test_step_bytes_of_the_headline_workload():
    """Qwen3-8B, TP=1, B=256, context 1024: 192,937,984 parameters per layer,
    36 layers + the 151936 x 4096 LM head in bf16, every context token's K and
    V (147,456 B per token over the layers), the new rows, the embedding rows."""
    shape = bench.model_shape("Qwen3-8B")
    per_layer = 4096 * (32 + 16) * 128 + 32 * 128 * 4096 + 3 * 4096 * 12288
    assert per_layer == 192_937_984
    weights = 2 * (36 * per_layer + 151936 * 4096)
    kv = 36 * 256 * (1024 * 2 * 8 * 128 * 2 + 2 * 8 * 128 * 2)
    assert 36 * 2 * 8 * 128 * 2 == 147_456
    assert bench.step_bytes(shape, 1, 256, 1024) == weights + kv + 2 * 256 * 4096
    # TP shards the weights and the kv heads
    assert bench.step_bytes(shape, 8, 256, 1024) < bench.step_bytes(shape, 1, 256, 1024) / 7


def test_allreduce_bus_bytes():
    shape = bench.model_shape("Qwen3-8B")
    assert bench.allreduce_bus_bytes(shape, 1, 256) == 0
    # 2L + 1 reductions of [256, 4096] bf16, 2 (N - 1) / N of the tensor each (as in the TP=8 bench line)
    assert bench.allreduce_bus_bytes(shape, 8, 256) == 73 * 2 * 7 / 8 * 256 * 4096 * 2 == 267_911_168


def test_attention_bytes():
    assert bench.attention_bytes(256, 1024, 32, 8) == 256 * 1024 * 8 * 128 * 4 + 2 * 256 * 32 * 128 * 2


def test_gemm_dispatch_report():
    shape = bench.model_shape("Qwen3-8B")
    auto = bench.gemm_dispatch(shape, 1, 256, "auto")
    assert auto["lm_head"].startswith("kvb_gemm_sk_bf16")
    assert all(auto[k].startswith("cuBLAS") for k in ("qkv", "o", "gate_up", "down"))
    assert bench.gemm_dispatch(shape, 8, 256, "auto")["lm_head"].startswith("cuBLAS")  # the shard is small
    ours = bench.gemm_dispatch(shape, 1, 256, "tcgen05")
    assert ours["gate_up"].startswith("kvb_gemm_sk_silu_bf16") and ours["qkv"].startswith("kvb_gemm_sk_bf16")
    assert all(v.startswith("cuBLAS") for v in bench.gemm_dispatch(shape, 1, 256, "cublas").values())


def test_argument_rules():
    a = bench.parse_args([])
    assert (a.gpus, a.steps, a.warmup, a.gemm, a.impl) == (1, 30, 5, "auto", "ours")
    with pytest.raises(SystemExit):
        bench.main(["--warmup", "2"])


def test_reference_arm_on_other_ranks_does_nothing(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "3")
    assert bench.main(["--impl", "reference", "--gpus", "4"]) == 0
    assert capsys.readouterr().out == ""


def test_reference_arm_line(monkeypatch, capsys):
    """The reference arm's line carries the contract's keys: impl, the same
    metric/unit/higher_is_better as our arm, a cpu_baseline describing the
    run (value = the line's) and an e2e with no host-device bytes."""
    monkeypatch.setenv("RANK", "0")
    assert bench.main(["--impl", "reference", "--model", "Qwen3-0.6B", "--batch", "4", "--context", "64",
                       "--steps", "1", "--warmup", "3"]) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["value"] == line["value"] > 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "ramp fills" in line["cpu_baseline"]["sample"]
    # ms_per_step is the work each step ran (one layer + the LM head), so steps x ms_per_step
    # matches the run's clock; the value is the extrapolated whole step's throughput
    assert 0 < line["ms_per_step"] < line["ms_per_step_extrapolated"]
    assert line["value"] == pytest.approx(4 / (line["ms_per_step_extrapolated"] / 1e3))


def test_teardown_guard_is_cancelled_in_time():
    """The guard around destroying the process group fires only after its
    limit; cancelled before that, it does nothing."""
    import time

    t = bench._exit_if_stuck(5.0)
    time.sleep(0.05)
    t.cancel()
    assert not t.is_alive() or t.finished.is_set()
