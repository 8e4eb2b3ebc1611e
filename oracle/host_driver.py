"""Host-side logic of the reference training driver (test infrastructure; see
oracle/__init__.py), restated for checking the ne_train command-line driver.

* ``Drand48``: the POSIX drand48 / srand48 generator the reference calls
  (train.m:236 ``srand48(42)``, train.m:389 ``srand48(42 + start_step)``,
  train.m:396 ``drand48()``): the 48-bit linear congruential generator
  x' = (0x5DEECE66D * x + 0xB) mod 2^48, seeded with x = (seed << 16) | 0x330E,
  returning x' / 2^48.  Pinned against the C library's own drand48 in
  tests/test_host_cli.py.
* ``scratch_init``: the reference's random initialisation (train.m:234-255):
  uniform scale * (2 * drand48() - 1) for Wq, Wk, Wv (1/sqrt(D)), Wo
  (1/sqrt(q_dim) * 1/sqrt(2L)), W1, W3 (1/sqrt(F)), W2 (1/sqrt(D) * 1/sqrt(2L)),
  layer by layer in that order; gains 1.0; embedding 0.02 * (2 * drand48() - 1).
  Float scales are promoted to double for the product and the result rounded
  to float, as the C expression does.
* ``sample_windows``: the data sampling of train.m:394-397: pos =
  (size_t)(drand48() * (n_tokens - SEQ - 1)) per sequence.
"""
from __future__ import annotations

import numpy as np

_A = 0x5DEECE66D
_C = 0xB
_MASK = (1 << 48) - 1


class Drand48:
    def __init__(self, seed: int):
        self.x = ((seed & 0xFFFFFFFF) << 16 | 0x330E) & _MASK

    def __call__(self) -> float:
        self.x = (_A * self.x + _C) & _MASK
        return self.x / float(1 << 48)


def scratch_init(n_layers, dim, hidden, heads, kv_heads, head_dim, vocab):
    """Returns (layers, rms_final, embed) exactly as train.m:234-255 computes them."""
    rng = Drand48(42)
    f32 = np.float32
    D, F = dim, hidden
    qd, kvd = heads * head_dim, kv_heads * head_dim
    scale_d = f32(1.0) / np.sqrt(f32(D))
    scale_qd = f32(1.0) / np.sqrt(f32(qd))
    scale_h = f32(1.0) / np.sqrt(f32(F))
    res_scale = f32(1.0) / np.sqrt(f32(2.0) * f32(n_layers))

    def fill(shape, scale):
        n = int(np.prod(shape))
        s = float(scale)
        return np.array([s * (2.0 * rng() - 1.0) for _ in range(n)], np.float64).astype(
            np.float32).reshape(shape)

    layers = []
    for _ in range(n_layers):
        lw = {}
        lw["Wq"] = fill((qd, D), scale_d)
        lw["Wk"] = fill((kvd, D), scale_d)
        lw["Wv"] = fill((kvd, D), scale_d)
        lw["Wo"] = fill((D, qd), f32(scale_qd * res_scale))
        lw["W1"] = fill((F, D), scale_h)
        lw["W2"] = fill((D, F), f32(scale_d * res_scale))
        lw["W3"] = fill((F, D), scale_h)
        lw["rms_att"] = np.ones(D, np.float32)
        lw["rms_ffn"] = np.ones(D, np.float32)
        layers.append(lw)
    rms_final = np.ones(D, np.float32)
    embed = fill((vocab, D), f32(0.02))
    return layers, rms_final, embed


def sample_windows(n_tokens: int, seq: int, count: int, seed: int = 42):
    """Start positions of `count` windows drawn as train.m:394-397 does."""
    rng = Drand48(seed)
    max_pos = n_tokens - seq - 1
    return [int(rng() * max_pos) for _ in range(count)]
