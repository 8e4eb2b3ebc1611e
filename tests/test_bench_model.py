"""CPU: the work model bench.py divides by (algorithmic bytes and FLOPs).

The roofline fractions in the bench line are only as good as these counts, so
they are pinned here against the closed forms of the measurement definitions:
Qwen3-0.6B 596,042,752 parameters (440.4 M in the layers, 155.58 M in the tied
embedding), Stories110M 109,529,856; decode bytes per step = bf16 weights once
+ B x (K/V of T positions + the new K/V row); training = 3 x the forward's
FLOPs (2 x params + causal attention 2*L*Hq*hd*(S+1) per token).
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
