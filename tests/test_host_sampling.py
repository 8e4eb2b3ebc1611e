"""CPU: the token loop's sampling branch against the reference's own draws.

neural_engine_b200.generate pulls a sampled step's logits to the host and
applies generate.py:201-215 there: logits / temperature, softmax, the top-p
mask renormalised in float32, np.random.choice with numpy's global RNG.  The
``ref_tiny_gqa_topp`` / ``ref_tiny_gqa_temp`` fixtures (tests/golden/
make_golden.py) hold, for the reference's generate() run after
np.random.seed(seed), the tempered logits of every draw, the distribution it
passed to np.random.choice and the tokens it sampled.  From the same tempered
logits and seed the library must build the identical distribution, bit for
bit, and draw the identical tokens; the oracle's forward along the sampled
tokens must reproduce the tempered logits to float32 rounding.
"""
import os

import numpy as np
import pytest

from oracle import decode as od
from oracle import model as om

CASES = ["ref_tiny_gqa_topp", "ref_tiny_gqa_temp"]


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, f"{name}.npz"))


@pytest.mark.parametrize("name", CASES)
def test_sampling_rule_reproduces_the_reference_draws(golden_dir, name):
    from neural_engine_b200.generate import sample_probs, sample_token
    g = _load(golden_dir, name)
    vocab = int(g["cfg"][6])
    top_p = float(g["top_p"])
    tempered, probs_ref, toks = g["tempered"], g["probs"], g["tokens"]
    np.random.seed(int(g["seed"]))
    for i in range(len(toks)):
        p = sample_probs(tempered[i], top_p, vocab)
        assert p.dtype == probs_ref[i].dtype, (p.dtype, probs_ref[i].dtype)
        np.testing.assert_array_equal(p, probs_ref[i])
        # temperature 1 leaves the tempered logits unchanged (x / 1.0 == x)
        assert sample_token(tempered[i], 1.0, top_p, vocab) == int(toks[i]), i
    if top_p < 1.0:   # the mask really cut the distribution
        assert (probs_ref == 0).sum(axis=1).min() > 0


@pytest.mark.parametrize("name", CASES)
def test_recorded_logits_follow_the_forward(golden_dir, name):
    g = _load(golden_dir, name)
    cfg = om.ModelCfg(*[int(v) for v in g["cfg"]])
    layers, rf, emb, qk = om.init_weights(cfg, seed=int(g["wseed"]), std=float(g["std"]))
    if int(g["gains"]):
        layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    from tests.golden.make_golden import weights_checksum
    np.testing.assert_allclose(weights_checksum(layers, rf, emb, qk), g["checksum"], rtol=0, atol=0)
    prompt, toks, T = g["prompt"], g["tokens"], float(g["temperature"])
    dec = od.Decoder(cfg, layers, rf, emb, qk, batch=1, max_seq=len(prompt) + len(toks))
    lg = dec.forward(prompt[None].astype(np.int64), 0, last_only=True)[0]
    scale = np.abs(g["tempered"]).max()
    for i in range(len(toks)):
        assert np.abs(lg / T - g["tempered"][i]).max() <= 2e-5 * max(1.0, scale), i
        if i + 1 < len(toks):
            lg = dec.forward(np.array([[toks[i]]], np.int64), len(prompt) + i, last_only=True)[0]
