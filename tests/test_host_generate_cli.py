"""CPU: the command line of neural_engine_b200.generate (generate.py:231-274).

The library's forward runs on a GPU; here the Engine is replaced by a stand-in
that runs the oracle's numpy forward (the CUDA forward has its own GPU parity
tests), so what is checked is the host side a user of the reference's
``tools/generate.py`` meets: the arguments, the checkpoint reader, the seed,
the greedy and sampled loops (generate.py:134-215) and the printed lines.
"""
import contextlib
import io
import os
import subprocess

import numpy as np
import pytest

from oracle import decode as od
from oracle import model as om

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_train")
SHAPE = ["--model", "custom", "--layers", "2", "--dim", "64", "--hidden", "128", "--heads", "4",
         "--kv-heads", "2", "--head-dim", "16", "--vocab", "96"]


class OracleEngine:
    """The Engine calls generate() makes, answered by the oracle forward."""

    def __init__(self, cfg, device=0):
        self.cfg = cfg
        self.max_batch = self.max_seq = 0

    def set_weights(self, layers, rms_final, embed, qk=None):
        self.w = (layers, rms_final, embed, qk)

    def kv_alloc(self, max_batch, max_seq):
        c = self.cfg
        ocfg = om.ModelCfg(c.n_layers, c.dim, c.hidden, c.heads, c.kv_heads, c.head_dim, c.vocab,
                           eps=c.eps, theta=c.theta, qk_norm=c.qk_norm, qk_eps=c.qk_eps,
                           res_alpha=c.res_alpha)
        self.dec = od.Decoder(ocfg, *self.w, batch=max_batch, max_seq=max_seq)
        self.max_batch, self.max_seq = max_batch, max_seq

    def _step(self, toks, pos, return_logits):
        lg = self.dec.forward(np.asarray(toks, np.int64), pos, last_only=True)
        nxt = np.argmax(lg, -1).astype(np.int32)
        return (nxt, lg) if return_logits else nxt

    def prefill(self, tokens, pos0=0, return_logits=False):
        return self._step(np.atleast_2d(tokens), pos0, return_logits)

    def decode_step(self, tok, pos, return_logits=False):
        return self._step(np.atleast_1d(tok)[:, None], pos, return_logits)


@pytest.fixture()
def ckpt(tmp_path):
    if not os.path.exists(BIN):
        from neural_engine_b200 import build
        build.build(verbose=False)
    path = str(tmp_path / "init.bin")
    subprocess.run([BIN, *SHAPE, "--seq", "32", "--dump-init", path], check=True, timeout=60)
    return path


def _run(monkeypatch, argv):
    from neural_engine_b200 import generate as gen
    monkeypatch.setattr(gen, "Engine", OracleEngine)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        toks = gen.main(argv)
    return toks, out.getvalue()


def _direct(ckpt, prompt, n, temperature, top_p, seed):
    """generate.py's loop written out over the oracle's logits."""
    from neural_engine_b200.generate import read_checkpoint, sample_token
    info, layers, rf, emb = read_checkpoint(ckpt)
    cfg = om.ModelCfg(info["n_layers"], info["dim"], info["hidden"], info["heads"],
                      info["kv_heads"], info["hd"], info["vocab"])
    dec = od.Decoder(cfg, layers, rf, emb, None, batch=1, max_seq=len(prompt) + n)
    np.random.seed(seed)
    lg = dec.forward(np.array([prompt], np.int64), 0, last_only=True)[0]
    out = []
    for i in range(n):
        tok = int(np.argmax(lg)) if temperature < 1e-6 else \
            sample_token(lg, temperature, top_p, cfg.vocab)
        out.append(tok)
        if i + 1 < n:
            lg = dec.forward(np.array([[tok]], np.int64), len(prompt) + i, last_only=True)[0]
    return out


def test_greedy_command_line(monkeypatch, ckpt):
    toks, text = _run(monkeypatch, [ckpt, "--prompt-ids", "5,17,3,88", "-n", "7", "-t", "0"])
    assert toks == _direct(ckpt, [5, 17, 3, 88], 7, 0.0, 0.9, 0)
    lines = text.splitlines()
    assert lines[0] == "Prompt (4 tokens): 5,17,3,88"
    assert lines[1] == "Generating 7 tokens (temp=0.0, top_p=0.9)..."
    assert lines[2] == "---"
    assert lines[3].split() == [str(t) for t in toks]
    assert lines[-2:] == ["---", "Generated 7 tokens"]


@pytest.mark.parametrize("temp,top_p", [(0.8, 0.9), (1.3, 1.0)])
def test_sampled_command_line_follows_the_seed(monkeypatch, ckpt, temp, top_p):
    argv = [ckpt, "--prompt-ids", "1,2,3", "-n", "10", "-t", str(temp), "--top-p", str(top_p),
            "--seed", "11"]
    toks, _ = _run(monkeypatch, argv)
    assert toks == _direct(ckpt, [1, 2, 3], 10, temp, top_p, 11)
    again, _ = _run(monkeypatch, argv)
    assert again == toks


def test_command_line_refuses_bad_prompts(monkeypatch, ckpt):
    from neural_engine_b200 import generate as gen
    monkeypatch.setattr(gen, "Engine", OracleEngine)
    with contextlib.redirect_stderr(io.StringIO()):
        with pytest.raises(SystemExit):
            gen.main([ckpt, "--prompt", "hello"])              # text prompt needs --model
        with pytest.raises(SystemExit):
            gen.main([ckpt, "--prompt-ids", "1,96", "-n", "2"])  # id outside the vocabulary
