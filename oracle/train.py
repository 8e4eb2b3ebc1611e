"""Training-step oracle (test infrastructure; see oracle/__init__.py).

* ``loss_and_grads``: float64 torch autograd of the forward restated in
  oracle/decode.py (itself pinned to tools/generate.py), teacher-forced over
  S positions: inputs tokens[:, :S], targets tokens[:, 1:] (train.m:395-401),
  loss = mean over the B*S targets of -log softmax(logits)[target]
  (cpu_ops.h:348-382; the reference adds 1e-10 inside the log, which changes
  nothing visible at these magnitudes and nothing in the gradient).
* ``adamw``: cpu_ops.h:266-303 in float32, operation by operation.
* ``optimizer_step``: the reference's update block (train.m:782-897): scale by
  grad_scale, global L2 norm, clip to grad_clip, AdamW per tensor with weight
  decay on matrices and the embedding but not on the RMSNorm gains.
* ``lr_schedule``: train.m:851-858.
"""
from __future__ import annotations

import math

import numpy as np

from .model import ModelCfg

MATRICES = ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")
GAINS = ("rms_att", "rms_ffn")


def _torch():
    import torch
    return torch


def forward_loss(cfg: ModelCfg, params: dict, tokens: np.ndarray, compact=None):
    """params: torch float64 tensors {layers: [dict], rms_final, embed, qk: [(qn, kn)] or None}.
    compact: optional compact -> full vocabulary ids; the classifier then uses
    those embedding rows only and targets map to their compact index
    (vocab_map_build / vocab_compact_embed, cpu_ops.h:385-422)."""
    torch = _torch()
    tok = torch.as_tensor(np.asarray(tokens, np.int64))
    B, S1 = tok.shape
    S = S1 - 1
    inp, tgt = tok[:, :S], tok[:, 1:]
    hd, H, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    grp = H // Hkv

    def rms(x, w, eps):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w

    dt = params["embed"].dtype
    freqs = torch.tensor([1.0 / (cfg.theta ** (2.0 * i / hd)) for i in range(hd // 2)],
                         dtype=torch.float64)
    ang = torch.arange(S, dtype=torch.float64)[:, None] * freqs[None, :]
    cos, sin = torch.cos(ang).to(dt), torch.sin(ang).to(dt)

    def rope(x):  # x [B, S, nh, hd], interleaved pairs
        x0, x1 = x[..., 0::2], x[..., 1::2]
        c, s = cos[None, :, None, :], sin[None, :, None, :]
        y0 = x0 * c - x1 * s
        y1 = x0 * s + x1 * c
        return torch.stack([y0, y1], -1).reshape(x.shape)

    mask = torch.ones(S, S, dtype=torch.bool).tril()
    x = params["embed"][inp]
    alpha = cfg.res_alpha
    for L, lw in enumerate(params["layers"]):
        xn = rms(x, lw["rms_att"], cfg.eps)
        q = (xn @ lw["Wq"].T).reshape(B, S, H, hd)
        k = (xn @ lw["Wk"].T).reshape(B, S, Hkv, hd)
        v = (xn @ lw["Wv"].T).reshape(B, S, Hkv, hd)
        if cfg.qk_norm:
            qn, kn = params["qk"][L]
            q = rms(q, qn, cfg.qk_eps)
            k = rms(k, kn, cfg.qk_eps)
        q, k = rope(q), rope(k)
        k = k.repeat_interleave(grp, dim=2)
        v = v.repeat_interleave(grp, dim=2)
        sc = torch.einsum("bshd,bthd->bhst", q, k) / math.sqrt(hd)
        sc = sc.masked_fill(~mask, float("-inf"))
        p = torch.softmax(sc, -1)
        o = torch.einsum("bhst,bthd->bshd", p, v).reshape(B, S, H * hd)
        x = x + alpha * (o @ lw["Wo"].T)
        xn = rms(x, lw["rms_ffn"], cfg.eps)
        h1 = xn @ lw["W1"].T
        h3 = xn @ lw["W3"].T
        g = h1 * torch.sigmoid(h1) * h3
        x = x + alpha * (g @ lw["W2"].T)
    x = rms(x, params["rms_final"], cfg.eps)
    if compact is not None:
        c2f = torch.as_tensor(np.asarray(compact, np.int64))
        f2c = torch.full((params["embed"].shape[0],), -1, dtype=torch.int64)
        f2c[c2f] = torch.arange(len(c2f))
        logits = x @ params["embed"][c2f].T
        tgt = f2c[tgt]
        assert bool((tgt >= 0).all()), "target outside the compact vocabulary"
    else:
        logits = x @ params["embed"].T
    logp = torch.log_softmax(logits, -1)
    nll = -logp.gather(-1, tgt[..., None])[..., 0]
    return nll.mean()


def loss_and_grads(cfg: ModelCfg, layers, rms_final, embed, qk, tokens, dtype="float64",
                   compact=None):
    """Returns (loss, grads) with grads shaped like the inputs (numpy, `dtype`)."""
    torch = _torch()
    tdt = getattr(torch, dtype)
    t = lambda a: torch.tensor(np.asarray(a), dtype=tdt, requires_grad=True)
    P = {"layers": [{k: t(v) for k, v in lw.items()} for lw in layers],
         "rms_final": t(rms_final), "embed": t(embed),
         "qk": [(t(a), t(b)) for a, b in qk] if qk is not None else None}
    loss = forward_loss(cfg, P, tokens, compact)
    loss.backward()
    g = {"layers": [{k: v.grad.numpy() for k, v in lw.items()} for lw in P["layers"]],
         "rms_final": P["rms_final"].grad.numpy(), "embed": P["embed"].grad.numpy(),
         "qk": [(a.grad.numpy(), b.grad.numpy()) for a, b in P["qk"]] if qk is not None else None}
    return float(loss.item()), g


def adamw(w, g, m, v, t, lr, b1, b2, eps, wd):
    """cpu_ops.h:266-303, float32, same operation order (returns new w, m, v)."""
    f = np.float32
    w, g, m, v = (np.asarray(a, f).copy() for a in (w, g, m, v))
    bc1 = f(1.0) - f(b1) ** t
    bc2 = f(1.0) - f(b2) ** t
    ob1, ob2 = f(1.0) - f(b1), f(1.0) - f(b2)
    m = m * f(b1)
    m = g * ob1 + m
    v = v * f(b2)
    v = (g * g) * ob2 + v
    mh = m * (f(1.0) / bc1)
    vh = np.sqrt(v * (f(1.0) / bc2)) + f(eps)
    upd = mh / vh
    upd = w * f(wd) + upd
    w = upd * f(-lr) + w
    return w, m, v


def lr_schedule(step, max_lr, warmup, total, min_frac=0.1):
    """train.m:851-858."""
    if step < warmup:
        return max_lr * (step + 1) / warmup
    decay = (step - warmup) / (total - warmup)
    min_lr = max_lr * min_frac
    return min_lr + 0.5 * (1.0 + math.cos(math.pi * decay)) * (max_lr - min_lr)


def optimizer_step(params, grads, state, t, lr, b1=0.9, b2=0.95, eps=1e-8, wd=0.1,
                   grad_clip=1.0, grad_scale=1.0):
    """train.m:782-897.  params / grads: {"layers": [dict], "rms_final", "embed",
    "qk": [(qn, kn)] or None}; state: same structure holding (m, v) pairs
    (``init_state``).  Updates params in place; returns the pre-clip norm."""
    items = []   # (param container, key, grad, state container, decays)
    for L, lw in enumerate(params["layers"]):
        for k in lw:
            items.append((lw, k, grads["layers"][L][k], state["layers"][L], k in MATRICES))
    for k in ("rms_final", "embed"):
        items.append((params, k, grads[k], state, k == "embed"))
    if params.get("qk") is not None:
        for L in range(len(params["qk"])):
            pq = {"q": params["qk"][L][0], "k": params["qk"][L][1]}
            gq = {"q": grads["qk"][L][0], "k": grads["qk"][L][1]}
            for k in ("q", "k"):
                items.append((pq, k, gq[k], state["qk"][L], False))
            params["qk"][L] = pq  # replaced by the updated tuple below
    sq = sum(float(np.square(np.asarray(g, np.float64) * grad_scale).sum()) for _, _, g, _, _ in items)
    norm = math.sqrt(sq)
    scale = grad_scale
    if grad_clip > 0 and norm > grad_clip:
        scale *= grad_clip / norm
    for cont, k, g, st, decays in items:
        gg = (np.asarray(g, np.float64) * scale).astype(np.float32)
        m, v = st[k]
        w, m, v = adamw(cont[k], gg, m, v, t, lr, b1, b2, eps, wd if decays else 0.0)
        st[k] = (m, v)
        cont[k] = w
    if params.get("qk") is not None:
        params["qk"] = [(d["q"], d["k"]) for d in params["qk"]]
    return norm


def init_state(params):
    z = lambda a: (np.zeros_like(a, np.float32), np.zeros_like(a, np.float32))
    st = {"layers": [{k: z(v) for k, v in lw.items()} for lw in params["layers"]],
          "rms_final": z(params["rms_final"]), "embed": z(params["embed"])}
    if params.get("qk") is not None:
        st["qk"] = [{"q": z(a), "k": z(b)} for a, b in params["qk"]]
    return st
