"""GPU: the training boundary -- per-layer entry points, v4 checkpoint save /
resume with the full optimizer state (train.m:97-165), and the token-major
RMSNorm entry points.

Tolerances: the per-layer composition and the resumed run repeat the same
kernels in the same order, so they agree with the monolithic step / the
uninterrupted run up to the order of floating-point atomics (gain and
embedding gradients): relative L2 <= 1e-5.  Checkpoint tensors are copied,
not computed: exact.
"""
import numpy as np
import pytest

from oracle import ckpt_v4
from oracle import model as om
from oracle import train as ot

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _cfg(**kw):
    base = dict(n_layers=2, dim=128, hidden=256, heads=4, kv_heads=2, head_dim=64, vocab=512,
                qk_norm=True, theta=1e6, eps=1e-6)
    base.update(kw)
    return om.ModelCfg(**base)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _engine(cfg, seed, B, S):
    import neural_engine_b200 as ne
    layers, rf, emb, qk = om.init_weights(cfg, seed=seed, std=0.08, bf16=True)
    layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    e = ne.Engine(cfg)
    e.set_weights(layers, rf, emb, qk)
    e.train_alloc(B, S)
    e.train_set_masters(layers, emb)
    e.zero_grads()
    return e, (layers, rf, emb, qk)


def _all_close(a, b, tol, path=""):
    if isinstance(a, dict):
        for k in a:
            _all_close(a[k], b[k], tol, f"{path}/{k}")
    elif isinstance(a, (list, tuple)):
        for i, (x, y) in enumerate(zip(a, b)):
            _all_close(x, y, tol, f"{path}[{i}]")
    elif a is None:
        assert b is None
    else:
        if tol == 0:
            assert np.array_equal(a, b), path
        else:
            r = _rel(a, b)
            assert r <= tol, f"{path}: rel-L2 {r:.3e}"


def test_per_layer_entry_points_compose_to_the_training_step():
    cfg = _cfg()
    B, S = 2, 64
    tok = om.prompt_tokens(cfg.vocab, S + 1, 5, batch=B)
    ea, _ = _engine(cfg, 3, B, S)
    eb, _ = _engine(cfg, 3, B, S)
    la = ea.train_fwd_bwd(tok)
    d_tok = torch.tensor(tok, dtype=torch.int32, device="cuda")
    d_loss = torch.zeros(1, device="cuda")
    eb.embed_fwd(d_tok.data_ptr())
    for l in range(cfg.n_layers):
        eb.attn_fwd(l)
        eb.ffn_fwd(l)
    eb.lmhead_ce_fwd_bwd(d_loss.data_ptr())
    for l in reversed(range(cfg.n_layers)):
        eb.ffn_bwd(l)
        eb.attn_bwd(l)
    eb.embed_bwd()
    eb.sync()
    assert abs(float(d_loss.item()) - la) <= 1e-6 * la
    _all_close(eb.get_grads(), ea.get_grads(), 1e-5)
    with pytest.raises(Exception):
        eb.attn_fwd(cfg.n_layers)          # layer out of range is an error, not a fault
    ea.close()
    eb.close()


def test_checkpoint_save_matches_device_state_and_reference_layout(tmp_path):
    cfg = _cfg()
    B, S = 2, 32
    e, _ = _engine(cfg, 7, B, S)
    for t in range(1, 3):
        e.train_fwd_bwd(om.prompt_tokens(cfg.vocab, S + 1, 10 + t, batch=B))
        e.adamw_step(t, 1e-3)
    path = str(tmp_path / "ane_qwen3_dyn_ckpt.bin")
    e.save_checkpoint(path, step=2, total_steps=100, lr=1e-3, loss=3.5, adam_t=2, cum_steps=2)
    ck = ckpt_v4.read_v4(path, with_adam=True)
    h = ck.hdr
    assert (h.step, h.total_steps, h.adam_t, h.seq_len, h.n_layers, h.vocab, h.q_dim) == \
        (2, 100, 2, S, cfg.n_layers, cfg.vocab, cfg.heads * cfg.head_dim)
    w, m, v = e.get_masters(), e.get_adam("m"), e.get_adam("v")
    for L in range(cfg.n_layers):
        for k in ckpt_v4.LAYER_KEYS:
            assert np.array_equal(ck.layers[L][k], w["layers"][L][k]), (L, k)
            assert np.array_equal(ck.adam["layers"][L][k][0], m["layers"][L][k]), (L, k)
            assert np.array_equal(ck.adam["layers"][L][k][1], v["layers"][L][k]), (L, k)
        assert np.array_equal(ck.qk_norm[L][0], w["qk"][L][0])
        assert np.array_equal(ck.qk_adam[L][1][1], v["qk"][L][1])
    assert np.array_equal(ck.embed, w["embed"])
    assert np.array_equal(ck.adam["embed"][1], v["embed"])
    assert np.array_equal(ck.rms_final, w["rms_final"])
    # the Adam moments are non-trivial after two steps
    assert np.abs(ck.adam["layers"][1]["W3"][1]).max() > 0
    e.close()


def test_resume_continues_the_same_trajectory(tmp_path):
    """Train 2 steps, save, resume in a fresh context, take step 3 on both:
    the resumed masters equal the uninterrupted ones."""
    import neural_engine_b200 as ne
    cfg = _cfg()
    B, S = 2, 32
    e, _ = _engine(cfg, 9, B, S)
    toks = [om.prompt_tokens(cfg.vocab, S + 1, 20 + t, batch=B) for t in range(3)]
    for t in range(2):
        e.train_fwd_bwd(toks[t])
        e.adamw_step(t + 1, 2e-3)
    path = str(tmp_path / "ck.bin")
    e.save_checkpoint(path, step=2, adam_t=2)
    r = ne.Engine(cfg)
    info = r.load_checkpoint(path)           # weights only (no training state yet)
    r.train_alloc(B, S)
    info = r.load_checkpoint(path)           # full state: masters, gains, Adam moments
    assert info["adam_t"] == 2 and info["has_qk_norm"] == 1
    _all_close(r.get_masters(), e.get_masters(), 0)
    _all_close(r.get_adam("v"), e.get_adam("v"), 0)
    l1 = e.train_fwd_bwd(toks[2])
    l2 = r.train_fwd_bwd(toks[2])
    assert abs(l1 - l2) <= 1e-6 * l1
    e.adamw_step(3, 2e-3)
    r.adamw_step(3, 2e-3)
    _all_close(r.get_masters(), e.get_masters(), 1e-5)
    e.close()
    r.close()


def test_reference_checkpoint_without_qk_block_resumes_with_unit_gains(tmp_path):
    """A file in the reference's exact layout (no QKN1 block) loads into the
    training state with its Adam moments and unit QK-norm gains."""
    import neural_engine_b200 as ne
    cfg = _cfg()
    layers, rf, emb, _ = om.init_weights(cfg, seed=13, std=0.05, bf16=True)
    ck = om.make_checkpoint(cfg, layers, rf, emb)
    rng = np.random.default_rng(0)
    ck.adam = {"layers": [{k: (rng.standard_normal(a.shape).astype(np.float32),
                               rng.random(a.shape).astype(np.float32)) for k, a in lw.items()}
                          for lw in layers],
               "rms_final": (np.zeros(cfg.dim, np.float32), np.ones(cfg.dim, np.float32)),
               "embed": (np.full(emb.shape, 0.5, np.float32), np.full(emb.shape, 2.0, np.float32))}
    ck.hdr.adam_t = 5
    path = str(tmp_path / "ref.bin")
    ckpt_v4.write_v4(path, ck)
    e = ne.Engine(cfg)
    e.load_checkpoint(path)
    e.train_alloc(1, 64)
    info = e.load_checkpoint(path)
    assert info["adam_t"] == 5 and info["has_qk_norm"] == 0
    w, m = e.get_masters(), e.get_adam("m")
    assert np.array_equal(w["layers"][1]["W1"], layers[1]["W1"].astype(np.float32))
    assert np.array_equal(m["layers"][0]["W3"], ck.adam["layers"][0]["W3"][0])
    assert np.array_equal(m["embed"], ck.adam["embed"][0])
    assert np.all(w["qk"][0][0] == 1.0) and np.all(w["qk"][1][1] == 1.0)
    e.close()


def test_rmsnorm_entry_points_match_float64():
    import neural_engine_b200 as ne
    cfg = _cfg(dim=1024, hidden=256, heads=16, kv_heads=8, head_dim=128)
    e = ne.Engine(cfg)
    rows = 48
    g = torch.Generator().manual_seed(1)
    x = torch.randn(rows, cfg.dim, generator=g)
    w = 1 + 0.1 * torch.randn(cfg.dim, generator=g)
    dy = torch.randn(rows, cfg.dim, generator=g)
    res = torch.randn(rows, cfg.dim, generator=g)
    dx_, x_, w_, dy_, res_ = (t.cuda() for t in (torch.zeros_like(x), x, w, dy, res))
    out = torch.zeros(rows, cfg.dim, dtype=torch.bfloat16, device="cuda")
    dw = torch.zeros(cfg.dim, device="cuda")
    e.lib.ne_rmsnorm_fwd(e._ctx, x_.data_ptr(), w_.data_ptr(), rows, out.data_ptr())
    e._check(e.lib.ne_rmsnorm_bwd_add(e._ctx, dy_.data_ptr(), x_.data_ptr(), w_.data_ptr(), rows,
                                      res_.data_ptr(), dx_.data_ptr(), dw.data_ptr()))
    e.sync()
    xd, wd = x.double().requires_grad_(), w.double().requires_grad_()
    y = xd / torch.sqrt((xd * xd).mean(-1, keepdim=True) + cfg.eps) * wd
    y.backward(dy.double())
    assert (out.cpu().double() - y.detach()).abs().max().item() <= 2 ** -7 * y.abs().max().item()
    assert _rel(dx_.cpu(), xd.grad + res.double()) <= 1e-5
    assert _rel(dw.cpu(), wd.grad) <= 1e-5
    e.close()


@pytest.mark.parametrize("hd,Hq,Hkv,B,S", [(128, 4, 2, 2, 256), (128, 2, 2, 1, 200),
                                           (128, 4, 2, 1, 384), (128, 2, 1, 3, 64),
                                           (64, 4, 2, 2, 160), (64, 12, 12, 2, 256),
                                           (64, 2, 1, 1, 300), (64, 4, 2, 1, 1024)])
def test_sdpa_forward_matches_float64(hd, Hq, Hkv, B, S):
    """Causal GQA attention (tcgen05 kernel at head_dim 128, the mma.sync one at
    64 unless NE_ATTN_TC64=1) vs float64 softmax;
    ragged and multi-tile sequence lengths; the row LSE (log2 domain) too.
    Tolerance: bf16 output, max-abs <= 2^-7 * max|O| + 1e-3; LSE <= 1e-3."""
    import neural_engine_b200 as ne
    cfg = ne.ModelConfig(1, 256, 256, Hq, Hkv, hd, 512)
    e = ne.Engine(cfg)
    g = torch.Generator().manual_seed(S + hd)
    q = torch.randn(B * S, Hq * hd, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, hd, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, hd, generator=g).to(torch.bfloat16)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    out = torch.zeros(B * S, Hq * hd, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(B, Hq, S, device="cuda")
    e.sdpa_fwd_device(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, out.data_ptr(),
                      lse.data_ptr())
    e.sync()
    qd = q.double().reshape(B, S, Hq, hd).permute(0, 2, 1, 3)
    kd = k.double().repeat_interleave(Hq // Hkv, 1)
    vd = v.double().repeat_interleave(Hq // Hkv, 1)
    sc = qd @ kd.transpose(-1, -2) / hd ** 0.5
    sc = sc.masked_fill(~torch.ones(S, S, dtype=torch.bool).tril(), float("-inf"))
    ref = (torch.softmax(sc, -1) @ vd).permute(0, 2, 1, 3).reshape(B * S, Hq * hd)
    got = out.cpu().double()
    assert (got - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item() + 1e-3
    ref_lse = torch.logsumexp(sc, -1) / np.log(2.0)
    assert (lse.cpu().double() - ref_lse).abs().max().item() <= 1e-3
    e.close()


@pytest.mark.parametrize("hd", [128, 64])
@pytest.mark.parametrize("S", [1024, 640])
def test_sdpa_forward_rows_rescale_at_different_tiles(S, hd):
    """Scores that grow along the keys at a rate that alternates between
    neighbouring query rows: odd rows' running maximum moves at every key tile
    (their accumulated output is rescaled), even rows' never does after the
    first, so the rows of one warp take different paths.  The output must
    still match float64 (same tolerance as above)."""
    import neural_engine_b200 as ne
    Hq, Hkv, B = 2, 1, 1
    cfg = ne.ModelConfig(1, 256, 256, Hq, Hkv, hd, 512)
    e = ne.Engine(cfg)
    g = torch.Generator().manual_seed(S)
    u = torch.randn(hd, generator=g)
    c = torch.where(torch.arange(S) % 2 == 1, torch.tensor(1.0), torch.tensor(0.05))
    q = (c[:, None, None] * u[None, None, :]).expand(S, Hq, hd).reshape(S, Hq * hd)
    q = q.to(torch.bfloat16)
    t = torch.arange(S, dtype=torch.float32) / 128.0
    k = (t[:, None] * u[None, :]).reshape(1, 1, S, hd).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, hd, generator=g).to(torch.bfloat16)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    out = torch.zeros(B * S, Hq * hd, dtype=torch.bfloat16, device="cuda")
    e.sdpa_fwd_device(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, out.data_ptr(), 0)
    e.sync()
    qd = q.double().reshape(B, S, Hq, hd).permute(0, 2, 1, 3)
    kd = k.double().repeat_interleave(Hq // Hkv, 1)
    vd = v.double().repeat_interleave(Hq // Hkv, 1)
    sc = qd @ kd.transpose(-1, -2) / hd ** 0.5
    sc = sc.masked_fill(~torch.ones(S, S, dtype=torch.bool).tril(), float("-inf"))
    ref = (torch.softmax(sc, -1) @ vd).permute(0, 2, 1, 3).reshape(B * S, Hq * hd)
    got = out.cpu().double()
    assert (got - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item() + 1e-3
    e.close()
