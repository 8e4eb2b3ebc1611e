"""Generate the committed golden fixtures for the token loop.

Run in the build container, where the reference tree is mounted:

    python tests/golden/make_golden.py --ref <reference root> [--only name,...]

What it does
  * ``ref_*`` fixtures: runs the reference's OWN numpy token loop --
    ``generate()`` / ``rmsnorm`` / ``softmax`` / ``silu`` / ``rope`` imported
    unchanged from ane-training/training/training_dynamic/tools/generate.py --
    on seeded checkpoints, greedy (temperature 0), and records the generated
    tokens plus the logits the reference took each argmax of (captured by
    wrapping the module's ``np`` with a proxy whose ``argmax`` records its
    argument; the reference source is not modified).  ``read_checkpoint`` is
    NOT used: it reads the GQA header fields from the wrong slots
    (generate.py:28 vs config.h:89); the info dict is built from the correct
    header instead.
  * ``ref_tiny_gqa_topp`` / ``ref_tiny_gqa_temp``: the same generate() on the
    sampling branch (temperature 0.8 with top-p 0.9; temperature 1.3 without
    top-p) after ``np.random.seed``; records the tempered logits of every
    draw (the vocabulary-sized input of the module's ``softmax``, wrapped),
    the distribution passed to ``np.random.choice`` (through the ``np``
    proxy) and the sampled tokens.
  * ``qwen3_c1``: the Qwen3-0.6B decode configuration (QK-norm, theta 1e6,
    eps 1e-6 -- outside what generate.py can express) from the oracle's
    parameterised restatement, which the ``ref_*`` fixtures pin to
    generate.py at its defaults.

Fixtures are written to tests/golden/*.npz next to this script.  Weights are
not stored: they are regenerated from their seed by ``oracle.model`` and a
checksum of them is stored to detect generator drift.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import io
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import decode as odec            # noqa: E402
from oracle import model as om               # noqa: E402

GEN_REL = "ane-training/training/training_dynamic/tools/generate.py"


def load_reference_generate(ref_root: str):
    path = os.path.join(ref_root, GEN_REL)
    spec = importlib.util.spec_from_file_location("ref_generate", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _ArgmaxRecorder:
    """Forwards to numpy; records every array passed to ``argmax``."""

    def __init__(self):
        self.seen = []

    def __getattr__(self, name):
        return getattr(np, name)

    def argmax(self, a, *args, **kw):
        self.seen.append(np.array(a, dtype=np.float32, copy=True))
        return np.argmax(a, *args, **kw)


class _SampleRecorder:
    """Forwards to numpy; records the probabilities passed to
    ``np.random.choice`` (the reference's sampling draw, generate.py:215)."""

    def __init__(self):
        self.probs = []
        rec = self

        class _Random:
            def __getattr__(self, name):
                return getattr(np.random, name)

            def choice(self, a, *args, p=None, **kw):
                rec.probs.append(np.array(p, copy=True))
                return np.random.choice(a, *args, p=p, **kw)

        self.random = _Random()

    def __getattr__(self, name):
        return getattr(np, name)


class _StubTokenizer:
    eos_token_id = -1

    @staticmethod
    def decode(ids):
        return ""


def weights_checksum(layers, rms_final, embed, qk=None) -> np.ndarray:
    parts = []
    for lw in layers:
        for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3", "rms_att", "rms_ffn"):
            a = lw[k].astype(np.float64)
            parts += [a.sum(), np.abs(a).sum()]
    parts += [rms_final.astype(np.float64).sum(), embed.astype(np.float64).sum(),
              np.abs(embed.astype(np.float64)).sum()]
    if qk is not None:
        for qn, kn in qk:
            parts += [qn.astype(np.float64).sum(), kn.astype(np.float64).sum()]
    return np.array(parts, np.float64)


def run_reference(mod, cfg, layers, rms_final, embed, prompt, n_tokens):
    info = {"dim": cfg.dim, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
            "hd": cfg.head_dim, "q_dim": cfg.q_dim, "kv_dim": cfg.kv_dim,
            "gqa_ratio": cfg.heads // cfg.kv_heads, "hidden": cfg.hidden,
            "n_layers": cfg.n_layers, "vocab": cfg.vocab}
    rec = _ArgmaxRecorder()
    saved_np = mod.np
    mod.np = rec
    try:
        with contextlib.redirect_stdout(io.StringIO()):
            toks = mod.generate(info, layers, rms_final, embed, _StubTokenizer(),
                                [int(t) for t in prompt], n_tokens, 0.0, 1.0)
    finally:
        mod.np = saved_np
    return np.array(toks, np.int32), np.stack(rec.seen)


def topk(logits, k=16):
    idx = np.argsort(-logits, axis=-1, kind="stable")[..., :k]
    return idx.astype(np.int32), np.take_along_axis(logits, idx, -1)


def make_ref_case(mod, name, cfg, wseed, pseed, n_prompt, n_tokens, gains=False,
                  full_logit_steps=(0,), std=0.02):
    layers, rms_final, embed, qk = om.init_weights(cfg, seed=wseed, std=std)
    if gains:
        layers, rms_final, qk = om.random_gains(cfg, layers, rms_final, qk)
    prompt = om.prompt_tokens(cfg.vocab, n_prompt, pseed)
    t0 = time.time()
    toks, logits = run_reference(mod, cfg, layers, rms_final, embed, prompt, n_tokens)
    dt = time.time() - t0
    assert logits.shape == (n_tokens, cfg.vocab), logits.shape
    ti, tv = topk(logits)
    out = dict(cfg=np.array([cfg.n_layers, cfg.dim, cfg.hidden, cfg.heads, cfg.kv_heads,
                             cfg.head_dim, cfg.vocab]),
               cfg_f=np.array([cfg.eps, cfg.theta, float(cfg.qk_norm), cfg.qk_eps,
                               cfg.res_alpha]),
               wseed=wseed, pseed=pseed, gains=int(gains), std=std, prompt=prompt, tokens=toks,
               top_idx=ti, top_val=tv, margin=odec.top2_margin(logits),
               checksum=weights_checksum(layers, rms_final, embed, qk),
               full_steps=np.array(full_logit_steps, np.int32),
               full_logits=logits[list(full_logit_steps)],
               seconds=dt)
    # the library functions the restatement re-implements, on fixed inputs
    rng = np.random.default_rng(99)
    x = rng.standard_normal(cfg.q_dim).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(cfg.q_dim)).astype(np.float32)
    out["fn_x"] = x
    out["fn_w"] = w
    out["fn_rmsnorm"] = mod.rmsnorm(x, w)
    out["fn_softmax"] = mod.softmax(x)
    out["fn_silu"] = mod.silu(x)
    out["fn_rope_pos"] = 37
    out["fn_rope"] = mod.rope(x, 37, cfg.head_dim)
    np.savez(os.path.join(HERE, f"{name}.npz"), **out)
    print(f"{name}: {n_tokens} tokens in {dt:.1f}s; tokens[:8]={toks[:8]}")


def make_sampled_case(mod, name, cfg, wseed, pseed, n_prompt, n_tokens, temperature, top_p,
                      seed, gains=False, std=0.02):
    """The reference's own sampling branch (generate.py:201-215): generate()
    with temperature / top-p after ``np.random.seed(seed)``.  Records the
    tempered logits each draw was made from (the vocabulary-sized input of
    the module's ``softmax``), the distribution passed to np.random.choice
    and the sampled tokens."""
    layers, rms_final, embed, qk = om.init_weights(cfg, seed=wseed, std=std)
    if gains:
        layers, rms_final, qk = om.random_gains(cfg, layers, rms_final, qk)
    prompt = om.prompt_tokens(cfg.vocab, n_prompt, pseed)
    info = {"dim": cfg.dim, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
            "hd": cfg.head_dim, "q_dim": cfg.q_dim, "kv_dim": cfg.kv_dim,
            "gqa_ratio": cfg.heads // cfg.kv_heads, "hidden": cfg.hidden,
            "n_layers": cfg.n_layers, "vocab": cfg.vocab}
    tempered = []
    orig_softmax = mod.softmax

    def softmax_rec(x):
        if np.shape(x) == (cfg.vocab,):
            tempered.append(np.array(x, copy=True))
        return orig_softmax(x)

    rec = _SampleRecorder()
    saved_np = mod.np
    mod.np, mod.softmax = rec, softmax_rec
    try:
        np.random.seed(seed)
        with contextlib.redirect_stdout(io.StringIO()):
            toks = mod.generate(info, layers, rms_final, embed, _StubTokenizer(),
                                [int(t) for t in prompt], n_tokens, temperature, top_p)
    finally:
        mod.np, mod.softmax = saved_np, orig_softmax
    assert len(tempered) == len(rec.probs) == len(toks) == n_tokens
    np.savez(os.path.join(HERE, f"{name}.npz"),
             cfg=np.array([cfg.n_layers, cfg.dim, cfg.hidden, cfg.heads, cfg.kv_heads,
                           cfg.head_dim, cfg.vocab]),
             wseed=wseed, pseed=pseed, gains=int(gains), std=std, prompt=prompt,
             temperature=temperature, top_p=top_p, seed=seed, tokens=np.array(toks, np.int32),
             tempered=np.stack(tempered), probs=np.stack(rec.probs),
             checksum=weights_checksum(layers, rms_final, embed, qk))
    print(f"{name}: T {temperature} top-p {top_p}: tokens[:8]={toks[:8]}")


def make_qwen3_case(name, n_prompt, n_tokens, full_logit_steps=(0,)):
    cfg = om.QWEN3_06B
    layers, rms_final, embed, qk = om.init_weights(cfg, seed=0, bf16=True)
    prompt = om.prompt_tokens(cfg.vocab, n_prompt, 1)
    t0 = time.time()
    toks, logits = odec.greedy_generate(cfg, layers, rms_final, embed, prompt[None], n_tokens,
                                        qk=qk, keep_logits=True)
    dt = time.time() - t0
    logits = np.stack([l[0] for l in logits])
    ti, tv = topk(logits)
    np.savez(os.path.join(HERE, f"{name}.npz"),
             wseed=0, pseed=1, prompt=prompt, tokens=toks[0], top_idx=ti, top_val=tv,
             margin=odec.top2_margin(logits),
             checksum=weights_checksum(layers, rms_final, embed, qk),
             full_steps=np.array(full_logit_steps, np.int32),
             full_logits=logits[list(full_logit_steps)], seconds=dt)
    print(f"{name}: {n_tokens} tokens in {dt:.1f}s; tokens[:8]={toks[0, :8]}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference repository root")
    ap.add_argument("--skip-qwen3", action="store_true")
    ap.add_argument("--only", default="", help="comma-separated fixture names to write")
    args = ap.parse_args()
    mod = load_reference_generate(args.ref)
    cases = [
        # tiny GQA model with non-unit gains: exercises every branch quickly
        ("ref_tiny_gqa", lambda: make_ref_case(mod, "ref_tiny_gqa", om.tiny(), 3, 4, 8, 24,
                                               gains=True, full_logit_steps=tuple(range(24)),
                                               std=0.25)),
        # tiny MHA model (Stories-like head layout)
        ("ref_tiny_mha", lambda: make_ref_case(mod, "ref_tiny_mha", om.tiny(heads=4, kv_heads=4),
                                               5, 6, 6, 16, full_logit_steps=tuple(range(16)),
                                               std=0.25)),
        # the sampling branch: top-p masking, then plain temperature sampling
        ("ref_tiny_gqa_topp", lambda: make_sampled_case(mod, "ref_tiny_gqa_topp", om.tiny(), 3, 4,
                                                        8, 24, 0.8, 0.9, 1234, gains=True,
                                                        std=0.25)),
        ("ref_tiny_gqa_temp", lambda: make_sampled_case(mod, "ref_tiny_gqa_temp", om.tiny(), 3, 4,
                                                        8, 24, 1.3, 1.0, 77, gains=True,
                                                        std=0.25)),
        # Stories110M, seed-0 weights, 16-token prompt (seed 1), 64 tokens
        ("ref_stories110m_c0", lambda: make_ref_case(mod, "ref_stories110m_c0", om.STORIES110M,
                                                     0, 1, 16, 64, full_logit_steps=(0, 63))),
    ]
    if not args.skip_qwen3:
        # BASELINE config 1 (B = 1): 512-token prompt, first 32 greedy steps
        cases.append(("qwen3_c1", lambda: make_qwen3_case("qwen3_c1", 512, 32,
                                                          full_logit_steps=(0, 31))))
    only = set(filter(None, args.only.split(",")))
    for name, make in cases:
        if not only or name in only:
            make()


if __name__ == "__main__":
    main()
