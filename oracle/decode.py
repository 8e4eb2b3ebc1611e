"""numpy restatement of the reference token loop (test infrastructure).

Follows ane-training/training/training_dynamic/tools/generate.py line by line
(function-level citations below), with four extensions that reduce to the
reference at their defaults:
  * ``theta`` (RoPE base; generate.py:103 hard-codes 10000.0),
  * ``eps`` (RMSNorm eps; generate.py:81 default 1e-5),
  * ``qk_norm`` (per-head RMSNorm of q and k after projection, before RoPE,
    with gains and ``qk_eps``; generate.py has no such step, while the
    Qwen3 models the reference converts carry q_norm / k_norm gains,
    tools/convert_hf.py:84-89 notes and skips them),
  * ``res_alpha`` (residual branch scale; 1.0 in generate.py:184,191, the
    training forward uses 1/sqrt(2L), train.m:181,441),
and two structural ones that do not change the arithmetic of a position:
  * a batch of independent sequences at the same position,
  * the prompt may be processed in one causal pass (``forward`` with S > 1)
    instead of one token at a time (generate.py:134 feeds it token by token).
Precision is fp32 throughout, as in generate.py (KV cache fp32,
generate.py:128-129).  RoPE angles and the rotation are evaluated in float64
and rounded to fp32 on store, exactly as generate.py:103-109 does when it
mixes Python floats with float32 elements.
"""
from __future__ import annotations

import numpy as np

from .model import ModelCfg

F32 = np.float32


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """generate.py:81-84, over the last axis."""
    rms = np.sqrt(np.mean(x ** 2, axis=-1, keepdims=True) + eps)
    return (x / rms) * w


def softmax(x: np.ndarray) -> np.ndarray:
    """generate.py:87-90, over the last axis."""
    x = x - np.max(x, axis=-1, keepdims=True)
    e = np.exp(x)
    return e / np.sum(e, axis=-1, keepdims=True)


def silu(x: np.ndarray) -> np.ndarray:
    """generate.py:93-94."""
    return x * (1.0 / (1.0 + np.exp(-x)))


def rope_tables(hd: int, positions, theta: float = 10000.0):
    """cos/sin of pos * theta^(-2i/hd) for i < hd/2, float64 [len(positions), hd/2].

    The frequency is formed exactly as generate.py:103 (Python float pow),
    the angle as generate.py:104 (pos * freq in float64).
    """
    freqs = [1.0 / (theta ** (2.0 * i / hd)) for i in range(hd // 2)]
    ang = np.array([[float(p) * f for f in freqs] for p in positions], dtype=np.float64)
    return np.cos(ang), np.sin(ang)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, hd: int) -> np.ndarray:
    """generate.py:97-110: rotate interleaved pairs (2i, 2i+1) of every head.

    x: [..., S, n_heads*hd] fp32; cos/sin: [S, hd/2] float64.
    """
    shp = x.shape
    xr = x.reshape(shp[:-1] + (shp[-1] // hd, hd // 2, 2)).astype(np.float64)
    c = cos[:, None, :]
    s = sin[:, None, :]
    v0, v1 = xr[..., 0], xr[..., 1]
    out = np.empty_like(xr)
    out[..., 0] = v0 * c - v1 * s
    out[..., 1] = v0 * s + v1 * c
    return out.astype(F32).reshape(shp)


def _lin(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """x[..., in] @ w[out, in]^T as one 2-D BLAS call (a batched 3-D matmul
    would re-read w once per leading index)."""
    return (x.reshape(-1, x.shape[-1]) @ w.T).reshape(x.shape[:-1] + (w.shape[0],))


class Decoder:
    """KV-cached batched forward (generate.py:113-195)."""

    def __init__(self, cfg: ModelCfg, layers, rms_final, embed, qk=None,
                 batch: int = 1, max_seq: int = 64):
        self.cfg = cfg
        self.layers = layers
        self.rms_final = rms_final
        self.embed = embed
        self.qk = qk
        self.B = batch
        self.max_seq = max_seq
        # generate.py:126-129: [n_layers][kv_heads, max_seq, hd] per sequence
        self.k_cache = np.zeros((cfg.n_layers, batch, cfg.kv_heads, max_seq, cfg.head_dim), F32)
        self.v_cache = np.zeros_like(self.k_cache)

    def forward(self, tokens: np.ndarray, pos0: int, last_only: bool = False) -> np.ndarray:
        """Run positions pos0 .. pos0+S-1 for all B sequences; return logits.

        tokens: int [B, S].  Returns fp32 [B, S, V] (or [B, V] if last_only).
        One position's arithmetic is generate.py:141-195.
        """
        cfg = self.cfg
        B, S = tokens.shape
        hd, H, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        grp = H // Hkv
        T = pos0 + S
        assert T <= self.max_seq
        cos, sin = rope_tables(hd, range(pos0, T), cfg.theta)
        scale = 1.0 / np.sqrt(hd)                                   # generate.py:166
        causal = np.arange(T)[None, :] <= (pos0 + np.arange(S))[:, None]   # [S, T]

        x = self.embed[tokens].astype(F32)                         # generate.py:142  [B,S,D]
        for L, lw in enumerate(self.layers):
            xn = rmsnorm(x, lw["rms_att"], cfg.eps)                  # :149
            q = _lin(xn, lw["Wq"])                                     # :151
            k = _lin(xn, lw["Wk"])                                     # :152
            v = _lin(xn, lw["Wv"])                                     # :153
            if cfg.qk_norm:
                qn, kn = self.qk[L]
                q = rmsnorm(q.reshape(B, S, H, hd), qn, cfg.qk_eps).reshape(B, S, H * hd)
                k = rmsnorm(k.reshape(B, S, Hkv, hd), kn, cfg.qk_eps).reshape(B, S, Hkv * hd)
            q = rope(q, cos, sin, hd)                                # :156
            k = rope(k, cos, sin, hd)                                # :157
            # :159-162 store KV
            self.k_cache[L, :, :, pos0:T] = k.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
            self.v_cache[L, :, :, pos0:T] = v.reshape(B, S, Hkv, hd).transpose(0, 2, 1, 3)
            # :164-181 GQA attention, q-head qh reads kv-head qh // grp
            qh = q.reshape(B, S, Hkv, grp, hd).transpose(0, 2, 3, 1, 4)      # [B,Hkv,grp,S,hd]
            kc = self.k_cache[L, :, :, :T]                                    # [B,Hkv,T,hd]
            vc = self.v_cache[L, :, :, :T]
            sc = (qh @ kc[:, :, None].swapaxes(-1, -2)) * scale              # [B,Hkv,grp,S,T]
            sc = sc.astype(F32)
            sc = np.where(causal, sc, -np.inf).astype(F32)
            p = softmax(sc)
            o = p @ vc[:, :, None]                                            # [B,Hkv,grp,S,hd]
            attn = o.transpose(0, 3, 1, 2, 4).reshape(B, S, H * hd).astype(F32)
            o_proj = _lin(attn, lw["Wo"])
            if cfg.res_alpha != 1.0:                                          # train.m:441
                o_proj = o_proj * F32(cfg.res_alpha)
            x = x + o_proj                                                    # :184
            xn = rmsnorm(x, lw["rms_ffn"], cfg.eps)                           # :187
            h1 = _lin(xn, lw["W1"])                                             # :188
            h3 = _lin(xn, lw["W3"])                                             # :189
            h1 = silu(h1) * h3                                                # :190
            f_proj = _lin(h1, lw["W2"])
            if cfg.res_alpha != 1.0:                                          # mil_dynamic.h:294-298
                f_proj = f_proj * F32(cfg.res_alpha)
            x = x + f_proj                                                    # :191
        if last_only:
            x = x[:, -1]
        x = rmsnorm(x, self.rms_final, cfg.eps)                               # :194
        return _lin(x, self.embed).astype(F32)                                # :195 tied


def greedy_generate(cfg: ModelCfg, layers, rms_final, embed, prompt: np.ndarray,
                    max_tokens: int, qk=None, token_by_token: bool = False,
                    keep_logits: bool = False):
    """Greedy decode (generate.py:134-200 with temperature 0).

    prompt: int [B, P].  Returns (tokens [B, max_tokens], logits list or None).
    ``logits[i]`` are the logits from which token i was chosen (the first from
    the last prompt position, generate.py:198).
    """
    prompt = np.asarray(prompt)
    if prompt.ndim == 1:
        prompt = prompt[None]
    B, P = prompt.shape
    dec = Decoder(cfg, layers, rms_final, embed, qk, batch=B, max_seq=P + max_tokens)
    if token_by_token:
        for p in range(P):
            lg = dec.forward(prompt[:, p:p + 1], p, last_only=True)
    else:
        lg = dec.forward(prompt, 0, last_only=True)
    out = np.zeros((B, max_tokens), np.int32)
    logits = [] if keep_logits else None
    for i in range(max_tokens):
        if keep_logits:
            logits.append(lg.copy())
        nxt = np.argmax(lg, axis=-1)                                          # :200
        out[:, i] = nxt
        if i + 1 < max_tokens:
            lg = dec.forward(nxt[:, None].astype(np.int64), P + i, last_only=True)
    return out, logits


def top2_margin(logits: np.ndarray) -> np.ndarray:
    """logit(top1) - logit(top2) per row."""
    part = np.partition(logits, -2, axis=-1)
    return part[..., -1] - part[..., -2]
