"""GPU: the training step against float64 autograd and the restated AdamW.

Stated tolerances (bf16 GEMM operands and attention, fp32 accumulation and
masters, against float64 autograd of the numpy forward):
  * loss:      |gpu - ref| <= 2e-3 * ref
  * gradients: relative L2 error <= 3e-2 per tensor (every weight matrix,
               every RMSNorm / QK-norm gain, the tied embedding)
  * AdamW:     given the GPU's own gradients, the updated fp32 masters match
               cpu_ops.h:266-303 (restated in float32) to relative L2 1e-5,
               and the pre-clip global norm to 1e-4 relative.
"""
import numpy as np
import pytest

from oracle import model as om
from oracle import train as ot

pytestmark = pytest.mark.gpu

GRAD_REL = 3e-2
LOSS_REL = 2e-3


def _cfg(**kw):
    base = dict(n_layers=2, dim=128, hidden=256, heads=4, kv_heads=2, head_dim=64, vocab=512)
    base.update(kw)
    return om.ModelCfg(**base)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _engine(cfg, layers, rf, emb, qk, B, S):
    import neural_engine_b200 as ne
    e = ne.Engine(cfg)
    e.set_weights(layers, rf, emb, qk)
    e.train_alloc(B, S)
    e.train_set_masters(layers, emb)
    e.zero_grads()
    return e


def _compare_grads(cfg, g_gpu, g_ref):
    worst = ("", 0.0)
    for L in range(cfg.n_layers):
        for k, ref in g_ref["layers"][L].items():
            r = _rel(g_gpu["layers"][L][k], ref)
            worst = max(worst, (f"layer {L} {k}", r), key=lambda x: x[1])
            assert r <= GRAD_REL, f"layer {L} {k}: rel-L2 {r:.3e}"
        if cfg.qk_norm:
            for i, name in enumerate(("q_norm", "k_norm")):
                r = _rel(g_gpu["qk"][L][i], g_ref["qk"][L][i])
                assert r <= GRAD_REL, f"layer {L} {name}: rel-L2 {r:.3e}"
    for k in ("rms_final", "embed"):
        r = _rel(g_gpu[k], g_ref[k])
        assert r <= GRAD_REL, f"{k}: rel-L2 {r:.3e}"
    return worst


TINY = [dict(qk_norm=True, theta=1e6, eps=1e-6),
        dict(qk_norm=False, theta=1e4, eps=1e-5),
        dict(qk_norm=True, theta=1e6, eps=1e-6, res_alpha=0.5, heads=4, kv_heads=4)]


@pytest.mark.parametrize("kw", TINY)
@pytest.mark.parametrize("B,S", [(2, 32), (1, 128)])
def test_loss_and_grads_match_float64(kw, B, S):
    cfg = _cfg(**kw)
    layers, rf, emb, qk = om.init_weights(cfg, seed=61, std=0.08, bf16=True)
    layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    tok = om.prompt_tokens(cfg.vocab, S + 1, 62, batch=B)
    e = _engine(cfg, layers, rf, emb, qk, B, S)
    loss = e.train_fwd_bwd(tok)
    ref_loss, g_ref = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok)
    assert abs(loss - ref_loss) <= LOSS_REL * ref_loss, (loss, ref_loss)
    worst = _compare_grads(cfg, e.get_grads(), g_ref)
    print(f"loss {loss:.6f} ref {ref_loss:.6f}; worst grad rel-L2 {worst[1]:.3e} ({worst[0]})")
    e.close()


def test_gradients_accumulate_over_micro_steps():
    """Two fwd_bwd calls accumulate (train.m accumulates `accum` micro-steps)."""
    cfg = _cfg(qk_norm=True, theta=1e6, eps=1e-6)
    layers, rf, emb, qk = om.init_weights(cfg, seed=71, std=0.08, bf16=True)
    t1 = om.prompt_tokens(cfg.vocab, 33, 72, batch=2)
    t2 = om.prompt_tokens(cfg.vocab, 33, 73, batch=2)
    e = _engine(cfg, layers, rf, emb, qk, 2, 32)
    e.train_fwd_bwd(t1)
    e.train_fwd_bwd(t2)
    _, g1 = ot.loss_and_grads(cfg, layers, rf, emb, qk, t1)
    _, g2 = ot.loss_and_grads(cfg, layers, rf, emb, qk, t2)
    gg = e.get_grads()
    r = _rel(gg["layers"][1]["W2"], g1["layers"][1]["W2"] + g2["layers"][1]["W2"])
    assert r <= GRAD_REL
    r = _rel(gg["embed"], g1["embed"] + g2["embed"])
    assert r <= GRAD_REL
    e.close()


@pytest.mark.parametrize("clip", [1.0, 1e-3])
def test_adamw_step_matches_reference_update(clip):
    """One optimizer step (unscale 1/accum, norm, clip, AdamW with wd on
    matrices + embedding only) vs the float32 restatement, given identical
    gradients (the GPU's own, read back) and masters."""
    cfg = _cfg(qk_norm=True, theta=1e6, eps=1e-6)
    layers, rf, emb, qk = om.init_weights(cfg, seed=81, std=0.08, bf16=True)
    layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    tok = om.prompt_tokens(cfg.vocab, 33, 82, batch=2)
    e = _engine(cfg, layers, rf, emb, qk, 2, 32)
    e.train_fwd_bwd(tok)
    grads = e.get_grads()
    before = e.get_masters()
    lr = e.lr_schedule(3, 3e-4, 10, 100)
    # the schedule is evaluated in float32, as train.m:851-858 does
    assert abs(lr - ot.lr_schedule(3, 3e-4, 10, 100)) <= 1e-6 * lr
    norm = e.adamw_step(1, lr, grad_clip=clip, grad_scale=0.5)
    after = e.get_masters()
    state = ot.init_state(before)
    ref_norm = ot.optimizer_step(before, grads, state, 1, lr, grad_clip=clip, grad_scale=0.5)
    assert abs(norm - ref_norm) <= 1e-4 * ref_norm
    for L in range(cfg.n_layers):
        for k in after["layers"][L]:
            r = _rel(after["layers"][L][k], before["layers"][L][k])
            assert r <= 1e-5, f"layer {L} {k}: {r:.3e}"
        for i in range(2):
            assert _rel(after["qk"][L][i], before["qk"][L][i]) <= 1e-5
    assert _rel(after["rms_final"], before["rms_final"]) <= 1e-5
    assert _rel(after["embed"], before["embed"]) <= 1e-5
    # gradients are zeroed by the step
    assert np.abs(e.get_grads()["layers"][0]["Wq"]).max() == 0.0
    e.close()


def test_training_reduces_loss():
    """A few steps on one repeated batch drive the loss down (end-to-end sanity
    of forward, backward and optimizer together)."""
    cfg = _cfg(qk_norm=True, theta=1e6, eps=1e-6)
    layers, rf, emb, qk = om.init_weights(cfg, seed=91, std=0.08, bf16=True)
    tok = om.prompt_tokens(cfg.vocab, 65, 92, batch=2)
    e = _engine(cfg, layers, rf, emb, qk, 2, 64)
    losses = []
    for t in range(1, 9):
        losses.append(e.train_fwd_bwd(tok))
        e.adamw_step(t, 3e-3, weight_decay=0.0)
    assert losses[-1] < 0.8 * losses[0], losses
    e.close()


TC_ATTN = [dict(head_dim=128, heads=4, kv_heads=2, qk_norm=True, theta=1e6, eps=1e-6),
           dict(head_dim=128, heads=4, kv_heads=4, qk_norm=False, theta=1e4, eps=1e-5),
           dict(head_dim=64, heads=4, kv_heads=2, qk_norm=True, theta=1e6, eps=1e-6),
           dict(head_dim=64, heads=4, kv_heads=4, qk_norm=False, theta=1e4, eps=1e-5)]


@pytest.mark.parametrize("kw", TC_ATTN)
@pytest.mark.parametrize("B,S", [(2, 224), (1, 256), (4, 80), (1, 1088)])
def test_tensor_core_attention_backward(kw, B, S):
    """Head dim 128 takes the tcgen05 attention kernels (forward, dK / dV, and
    dQ from 256 positions on), head dim 64 the mma.sync ones by default:
    several 128-row query / key tiles, a ragged last tile, GQA groups of 2 and
    1, with and without QK-norm."""
    cfg = _cfg(**kw)
    layers, rf, emb, qk = om.init_weights(cfg, seed=71, std=0.08, bf16=True)
    layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    tok = om.prompt_tokens(cfg.vocab, S + 1, 72, batch=B)
    e = _engine(cfg, layers, rf, emb, qk, B, S)
    loss = e.train_fwd_bwd(tok)
    ref_loss, g_ref = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok)
    assert abs(loss - ref_loss) <= LOSS_REL * ref_loss, (loss, ref_loss)
    worst = _compare_grads(cfg, e.get_grads(), g_ref)
    print(f"loss {loss:.6f} ref {ref_loss:.6f}; worst grad rel-L2 {worst[1]:.3e} ({worst[0]})")
    e.close()


def _child_backward(kw, B, S, env, q):
    import os
    for k, v in env.items():
        os.environ[k] = v
    try:
        cfg = _cfg(**kw)
        layers, rf, emb, qk = om.init_weights(cfg, seed=71, std=0.08, bf16=True)
        layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
        tok = om.prompt_tokens(cfg.vocab, S + 1, 72, batch=B)
        e = _engine(cfg, layers, rf, emb, qk, B, S)
        loss = e.train_fwd_bwd(tok)
        ref_loss, g_ref = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok)
        assert abs(loss - ref_loss) <= LOSS_REL * ref_loss, (loss, ref_loss)
        worst = _compare_grads(cfg, e.get_grads(), g_ref)
        e.close()
        q.put(("ok", worst))
    except BaseException as ex:   # report to the parent
        q.put(("fail", repr(ex)))


def _in_child(kw, B, S, env):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child_backward, args=(kw, B, S, env, q))
    p.start()
    res = q.get(timeout=300)
    p.join(timeout=60)
    assert res[0] == "ok", res[1]


@pytest.mark.parametrize("kw", [TC_ATTN[0], TC_ATTN[3]])
@pytest.mark.parametrize("env", [{"NE_ATTN_BWD_TC": "1", "NE_ATTN_TC64": "1"},
                                 {"NE_ATTN_BWD_TC": "1", "NE_ATTN_TC64": "1",
                                  "NE_ATTN_BWD_MERGE": "0"},
                                 {"NE_ATTN_BWD_TC": "1", "NE_ATTN_TC64": "1", "NE_DQ_TP": "0",
                                  "NE_DKDV_TP": "0"}])
def test_tensor_core_dq_at_short_sequences(kw, env):
    """The tcgen05 dQ kernels at 256 positions: pipelined (dQ and dK/dV in one
    launch, or with NE_ATTN_BWD_MERGE=0 in two) and, with NE_DQ_TP=0 /
    NE_DKDV_TP=0, the serial ones; run in a fresh process so the switches are
    read there."""
    _in_child(kw, 2, 256, env)


@pytest.mark.parametrize("B,S", [(2, 224), (1, 1088)])
def test_one_tile_forward_kernel_for_even_groups(B, S):
    """GQA groups of 2 take the two-tile forward by default; NE_ATTN_FWD2=0
    runs the one-tile kernel for them too."""
    _in_child(TC_ATTN[0], B, S, {"NE_ATTN_FWD2": "0"})


@pytest.mark.parametrize("kw", [TC_ATTN[2], TC_ATTN[3]])
@pytest.mark.parametrize("B,S", [(2, 224), (1, 1088)])
def test_head_dim_64_tensor_core_attention(kw, B, S):
    """Head dim 64 on the tcgen05 forward, dQ and dK/dV kernels
    (NE_ATTN_TC64=1; the default keeps the mma.sync ones there)."""
    _in_child(kw, B, S, {"NE_ATTN_TC64": "1"})


@pytest.mark.parametrize("name", ["stories110m", "qwen3_06b"])
def test_full_width_two_layers(name):
    """Full-width Stories110M / Qwen3-0.6B layers (2 of them, full vocabulary,
    B=1, S=64) against float64 autograd."""
    base = om.PRESETS[name]
    from dataclasses import replace
    cfg = replace(base, n_layers=2)
    layers, rf, emb, qk = om.init_weights(cfg, seed=0, std=0.02, bf16=True)
    tok = om.prompt_tokens(cfg.vocab, 65, 3, batch=1)
    e = _engine(cfg, layers, rf, emb, qk, 1, 64)
    loss = e.train_fwd_bwd(tok)
    ref_loss, g_ref = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok)
    assert abs(loss - ref_loss) <= LOSS_REL * ref_loss, (loss, ref_loss)
    worst = _compare_grads(cfg, e.get_grads(), g_ref)
    print(f"{name}: loss {loss:.6f} ref {ref_loss:.6f}; worst grad rel-L2 {worst[1]:.3e} ({worst[0]})")
    e.close()


@pytest.mark.parametrize("CV", [97, 128])
def test_compact_vocabulary_classifier(CV):
    """The reference's vocabulary compaction: softmax over the embedding rows of
    the tokens in use only; gradients (including the tied embedding's, added
    back into the used rows) vs float64 autograd of the compacted forward."""
    cfg = _cfg(qk_norm=True, theta=1e6, eps=1e-6)
    layers, rf, emb, qk = om.init_weights(cfg, seed=101, std=0.08, bf16=True)
    rng = np.random.default_rng(CV)
    c2f = np.sort(rng.choice(cfg.vocab, CV, replace=False)).astype(np.int32)
    B, S = 2, 32
    tok = c2f[rng.integers(0, CV, (B, S + 1))]
    e = _engine(cfg, layers, rf, emb, qk, B, S)
    e.train_set_vocab_map(c2f)
    loss = e.train_fwd_bwd(tok)
    ref_loss, g_ref = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok, compact=c2f)
    assert abs(loss - ref_loss) <= LOSS_REL * ref_loss, (loss, ref_loss)
    _compare_grads(cfg, e.get_grads(), g_ref)
    # back to the full vocabulary: the same batch gives the uncompacted loss
    e.zero_grads()
    e.train_set_vocab_map(None)
    full = e.train_fwd_bwd(tok)
    ref_full, _ = ot.loss_and_grads(cfg, layers, rf, emb, qk, tok)
    assert abs(full - ref_full) <= LOSS_REL * ref_full
    e.close()
