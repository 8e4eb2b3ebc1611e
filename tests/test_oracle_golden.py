"""CPU: the oracle against the reference's own outputs (golden fixtures).

The ``ref_*`` fixtures were produced by the reference's tools/generate.py
(generate(), rmsnorm, softmax, silu, rope imported unchanged) by
tests/golden/make_golden.py.  The oracle restatement must reproduce the
reference's greedy tokens exactly and its logits to float32 rounding, both
feeding the prompt token by token (as generate.py:134 does) and in one
causal pass.
"""
import os

import numpy as np
import pytest

from oracle import decode as od
from oracle import model as om

REF_CASES = ["ref_tiny_gqa", "ref_tiny_mha", "ref_stories110m_c0"]


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, f"{name}.npz"))


def _cfg(g):
    c, cf = g["cfg"], g["cfg_f"]
    return om.ModelCfg(*[int(v) for v in c], eps=float(cf[0]), theta=float(cf[1]),
                       qk_norm=bool(cf[2]), qk_eps=float(cf[3]), res_alpha=float(cf[4]))


def _weights(g, cfg):
    layers, rf, emb, qk = om.init_weights(cfg, seed=int(g["wseed"]), std=float(g["std"]))
    if int(g["gains"]):
        layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    return layers, rf, emb, qk


@pytest.mark.parametrize("name", REF_CASES)
@pytest.mark.parametrize("token_by_token", [True, False])
def test_oracle_matches_reference_generate(golden_dir, name, token_by_token):
    g = _load(golden_dir, name)
    cfg = _cfg(g)
    layers, rf, emb, qk = _weights(g, cfg)
    from tests.golden.make_golden import weights_checksum
    np.testing.assert_allclose(weights_checksum(layers, rf, emb, qk), g["checksum"], rtol=0, atol=0)
    n = len(g["tokens"])
    toks, lg = od.greedy_generate(cfg, layers, rf, emb, g["prompt"][None], n,
                                  token_by_token=token_by_token, keep_logits=True)
    lg = np.stack([l[0] for l in lg])
    # identical greedy tokens for every step (the reference generated them)
    np.testing.assert_array_equal(toks[0], g["tokens"])
    # logits: float32 rounding only (summation order of BLAS vs numpy loops)
    st = g["full_steps"]
    scale = np.abs(g["full_logits"]).max()
    assert np.abs(lg[st] - g["full_logits"]).max() <= 2e-5 * max(1.0, scale)
    # the top-16 of every step agree in value
    np.testing.assert_allclose(np.take_along_axis(lg, g["top_idx"].astype(np.int64), -1),
                               g["top_val"], rtol=0, atol=2e-5 * max(1.0, scale))


@pytest.mark.parametrize("name", REF_CASES)
def test_oracle_functions_bit_exact(golden_dir, name):
    """rmsnorm / softmax / silu / rope equal generate.py's bit for bit."""
    g = _load(golden_dir, name)
    cfg = _cfg(g)
    x, w = g["fn_x"], g["fn_w"]
    np.testing.assert_array_equal(od.rmsnorm(x, w), g["fn_rmsnorm"])
    np.testing.assert_array_equal(od.softmax(x), g["fn_softmax"])
    np.testing.assert_array_equal(od.silu(x), g["fn_silu"])
    c, s = od.rope_tables(cfg.head_dim, [int(g["fn_rope_pos"])], cfg.theta)
    np.testing.assert_array_equal(od.rope(x[None], c, s, cfg.head_dim)[0], g["fn_rope"])


def test_qwen3_fixture_self_consistent(golden_dir):
    """The Qwen3 fixture (oracle-generated) regenerates from its seeds.

    Checks the weight generator (checksum) and the first 4 greedy steps, which
    pins the QK-norm / theta 1e6 / eps 1e-6 path of the restatement against
    accidental change.  Prompt shortened to keep the CPU test fast is not
    possible (the fixture is the 512-token config), so this runs the full
    prompt once (a few seconds of BLAS)."""
    g = _load(golden_dir, "qwen3_c1")
    cfg = om.QWEN3_06B
    layers, rf, emb, qk = om.init_weights(cfg, seed=0, bf16=True)
    from tests.golden.make_golden import weights_checksum
    np.testing.assert_allclose(weights_checksum(layers, rf, emb, qk), g["checksum"], rtol=1e-12)
    toks, lg = od.greedy_generate(cfg, layers, rf, emb, g["prompt"][None], 4, qk=qk,
                                  keep_logits=True)
    np.testing.assert_array_equal(toks[0], g["tokens"][:4])
    np.testing.assert_allclose(lg[0][0], g["full_logits"][0], rtol=0, atol=1e-4)


def test_defaults_reduce_to_reference():
    """QK-norm with unit gains and alpha 1 change nothing structural; theta and
    eps defaults are generate.py's (10000, 1e-5)."""
    c = om.ModelCfg(n_layers=1, dim=64, hidden=64, heads=2, kv_heads=1, head_dim=32, vocab=8)
    assert c.theta == 10000.0 and c.eps == 1e-5 and c.res_alpha == 1.0 and not c.qk_norm


def test_rope_interleaved_pairs():
    """RoPE rotates adjacent pairs (2i, 2i+1), not rotate_half halves (generate.py:106-109)."""
    hd = 8
    x = np.zeros((1, hd), np.float32)
    x[0, 0] = 1.0                                  # pair 0 -> (cos, sin) at frequency 1
    c, s = od.rope_tables(hd, [1], 10000.0)
    y = od.rope(x, c, s, hd)
    assert abs(y[0, 0] - np.cos(1.0)) < 1e-7 and abs(y[0, 1] - np.sin(1.0)) < 1e-7
    assert np.all(y[0, 2:] == 0)
