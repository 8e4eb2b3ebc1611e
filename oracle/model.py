"""Model presets and seeded synthetic inputs (test infrastructure).

Dimensions follow the reference's compile-time model headers
(ane-training/training/training_dynamic/models/stories110m.h:6-16,
models/qwen3_06b.h:6-16).  The numerics knobs that the reference hard-codes
(RoPE theta 10000 at tools/generate.py:103, RMSNorm eps 1e-5 at
tools/generate.py:81, no QK-norm, residual alpha 1 in generate.py but
1/sqrt(2L) in train.m:181) are explicit fields here so that the Qwen3
configurations (theta 1e6, eps 1e-6, per-head QK RMSNorm) can be expressed and
so that the defaults reduce exactly to generate.py.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from .ckpt_v4 import Checkpoint, CkptHeader


@dataclass(frozen=True)
class ModelCfg:
    n_layers: int
    dim: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-5
    theta: float = 10000.0
    qk_norm: bool = False
    qk_eps: float = 1e-6
    res_alpha: float = 1.0

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    def n_params(self) -> int:
        d = self.dim
        per = (self.q_dim * d + 2 * self.kv_dim * d + d * self.q_dim
               + 3 * self.hidden * d + 2 * d)
        return self.n_layers * per + d + self.vocab * d


STORIES110M = ModelCfg(n_layers=12, dim=768, hidden=2048, heads=12, kv_heads=12,
                       head_dim=64, vocab=32000)
QWEN3_06B = ModelCfg(n_layers=28, dim=1024, hidden=3072, heads=16, kv_heads=8,
                     head_dim=128, vocab=151936, eps=1e-6, theta=1e6, qk_norm=True)

PRESETS = {"stories110m": STORIES110M, "qwen3_06b": QWEN3_06B}


def tiny(**kw) -> ModelCfg:
    """A small GQA config for fast CPU tests."""
    base = ModelCfg(n_layers=2, dim=64, hidden=160, heads=4, kv_heads=2, head_dim=16,
                    vocab=256)
    return replace(base, **kw)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    u = ((u + rounding) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def init_weights(cfg: ModelCfg, seed: int = 0, std: float = 0.02, bf16: bool = False):
    """N(0, std) fp32 weights from ``np.random.default_rng(seed)``, gains 1.0.

    Tensors are drawn in v4 file order (per layer Wq, Wk, Wv, Wo, W1, W2, W3,
    then the embedding).  With ``bf16`` each value is rounded to bf16 so that
    a bf16 device copy holds exactly the values the fp32 oracle uses.
    Returns (layers, rms_final, embed, qk_gains or None).
    """
    rng = np.random.default_rng(seed)
    d = cfg.dim

    def draw(shape):
        a = rng.standard_normal(int(np.prod(shape)), dtype=np.float32).reshape(shape)
        a *= np.float32(std)
        return bf16_round(a) if bf16 else a

    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "Wq": draw((cfg.q_dim, d)), "Wk": draw((cfg.kv_dim, d)),
            "Wv": draw((cfg.kv_dim, d)), "Wo": draw((d, cfg.q_dim)),
            "W1": draw((cfg.hidden, d)), "W2": draw((d, cfg.hidden)),
            "W3": draw((cfg.hidden, d)),
            "rms_att": np.ones(d, np.float32), "rms_ffn": np.ones(d, np.float32),
        })
    embed = draw((cfg.vocab, d))
    rms_final = np.ones(d, np.float32)
    qk = None
    if cfg.qk_norm:
        qk = [(np.ones(cfg.head_dim, np.float32), np.ones(cfg.head_dim, np.float32))
              for _ in range(cfg.n_layers)]
    return layers, rms_final, embed, qk


def random_gains(cfg: ModelCfg, layers, rms_final, qk, seed: int = 7, spread: float = 0.25):
    """Perturb the RMSNorm / QK-norm gains away from 1.0 (exercises the gain path)."""
    rng = np.random.default_rng(seed)
    g = lambda n: (1.0 + spread * rng.standard_normal(n)).astype(np.float32)
    for lw in layers:
        lw["rms_att"] = g(cfg.dim)
        lw["rms_ffn"] = g(cfg.dim)
    rms_final = g(cfg.dim)
    if qk is not None:
        qk = [(g(cfg.head_dim), g(cfg.head_dim)) for _ in qk]
    return layers, rms_final, qk


def make_checkpoint(cfg: ModelCfg, layers, rms_final, embed, qk=None, seq_len=256) -> Checkpoint:
    h = CkptHeader(n_layers=cfg.n_layers, vocab=cfg.vocab, dim=cfg.dim, hidden=cfg.hidden,
                   heads=cfg.heads, seq_len=seq_len, kv_heads=cfg.kv_heads,
                   head_dim=cfg.head_dim, q_dim=cfg.q_dim)
    return Checkpoint(hdr=h, layers=layers, rms_final=rms_final, embed=embed, qk_norm=qk)


def prompt_tokens(vocab: int, n: int, seed: int, batch: int | None = None) -> np.ndarray:
    """Uniform token IDs in [0, vocab) from ``np.random.default_rng(seed)``."""
    rng = np.random.default_rng(seed)
    shape = (n,) if batch is None else (batch, n)
    return rng.integers(0, vocab, size=shape, dtype=np.int64).astype(np.int32)
