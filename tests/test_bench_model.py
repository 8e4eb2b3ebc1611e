"""CPU: the work model bench.py divides by (algorithmic bytes and FLOPs).

The roofline fractions in the bench line are only as good as these counts, so
they are pinned here against the closed forms of the measurement definitions:
Qwen3-0.6B 596,042,752 parameters (440.4 M in the layers, 155.58 M in the tied
embedding), Stories110M 109,529,856; decode bytes per step = bf16 weights once
+ B x (K/V of T positions + the new K/V row); training = 3 x the forward's
FLOPs (2 x params + causal attention 2*L*Hq*hd*(S+1) per token).  Also the
host-side records of the line: the clock record (median SM clock, throttle
reasons) and the label of the gradient exchange.
"""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_parameter_counts(bench):
    import neural_engine_b200 as ne
    assert bench.PARAMS == 596_042_752
    assert bench.n_params(ne.QWEN3_06B) == bench.PARAMS
    assert bench.n_params(ne.STORIES110M) == 109_529_856
    layers = 28 * (2048 * 1024 + 2 * 1024 * 1024 + 1024 * 2048 + 3 * 3072 * 1024)
    assert layers == 440_401_920
    assert bench.PARAMS == layers + 28 * 2 * 1024 + 1024 + 151936 * 1024


def test_decode_bytes(bench):
    kv_per_pos = 28 * 2 * 8 * 128 * 2          # K and V, all layers, fp16
    assert kv_per_pos == 114_688
    for B, T in [(1, 512), (256, 640), (32, 767)]:
        want = 2 * 596_042_752 + B * (kv_per_pos * T + kv_per_pos)
        assert bench.decode_step_bytes(B, T) == want
    # one attention launch: one layer's K/V for T positions, q fp32 in, bf16 out
    assert bench.attention_bytes(64, 514) == 135_528_448
    assert 1.0 < bench.ATTN_TRAFFIC_RATIO < 1.05


def test_training_and_prefill_flops(bench):
    import neural_engine_b200 as ne
    attn = 2 * 28 * 16 * 128                   # per token per attended position
    assert attn == 114_688
    assert bench.train_flops_per_token(256) == 3 * (2 * 596_042_752 + attn * 257)
    assert bench.train_flops_per_token(256, ne.QWEN3_06B) == bench.train_flops_per_token(256)
    assert bench.train_flops_per_token(256, ne.STORIES110M) == \
        3 * (2 * 109_529_856 + 2 * 12 * 768 * 257)
    mats = 440_401_920
    for S in (256, 2048):
        assert bench.prefill_flops(16, S) == 16 * S * (2 * mats + attn * (S + 1)) + \
            16 * 2 * 151936 * 1024


def test_clock_record_reads_reasons_and_median(bench):
    """The clocks object of the bench line: median SM clock under load, the max
    clock, and which throttle reasons were active at any sample (the rejection
    rule reads hw_slowdown / hw_thermal_slowdown / sw_thermal_slowdown)."""
    cs = bench.ClockSampler(0)
    head = ["0"]
    cs.rows = [
        head + ["1965", "1965", "700.0", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
        head + ["1912", "1965", "990.1", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
        head + ["1927", "1965", "995.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
        head + ["[N/A]", "1965", "0", "0x0"],          # unreadable sample: skipped
        ["garbage"],
    ]
    rec = cs.stop()
    assert rec == {"sm_mhz": 1927.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    cs.rows = [head + ["1500", "1965", "900", "0x8", "Active", "Not Active", "Active", "Not Active"]]
    assert cs.stop()["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    cs.rows = []
    assert cs.stop() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_dp_label_names_the_exchange(bench, monkeypatch):
    monkeypatch.delenv("NE_COMM_PX", raising=False)
    monkeypatch.delenv("NE_PX_FUSED_DW", raising=False)
    assert bench.dp_label(1, "zero1").startswith("dp1 ")
    assert "peer memory" in bench.dp_label(4, "zero1") and "reduce-scatter kernels" in \
        bench.dp_label(4, "zero1")
    assert "all-reduce" in bench.dp_label(2, "allreduce")
    monkeypatch.setenv("NE_PX_FUSED_DW", "1")
    assert "dW GEMM epilogues" in bench.dp_label(8, "zero1")
    monkeypatch.setenv("NE_COMM_PX", "0")
    assert "NCCL reduce-scatter" in bench.dp_label(8, "zero1")
    assert bench.allmax(3.5, 1) == 3.5
