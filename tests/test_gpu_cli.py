"""GPU: the ne_train command-line driver end to end on a small model -- scratch
initialisation, windows from a uint16 token file, micro-steps with gradient
accumulation, the scheduled AdamW step, best-loss checkpoints and --resume --
against the same run driven step by step through the Python bindings
(same kernels in the same order: masters agree to relative L2 1e-5, the
tolerance covering the order of the gain gradients' float atomics)."""
import math
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import ckpt_v4
from oracle import host_driver as hd

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_train")
L, D, F, H, HKV, HD, V, S = 2, 128, 256, 4, 2, 64, 512, 64
SHAPE = ["--model", "custom", "--layers", str(L), "--dim", str(D), "--hidden", str(F),
         "--heads", str(H), "--kv-heads", str(HKV), "--head-dim", str(HD), "--vocab", str(V),
         "--seq", str(S)]


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def _replay(data, steps, accum, lr, warmup):
    """The driver's loop through the Python bindings; masters after each update."""
    import neural_engine_b200 as ne
    cfg = ne.ModelConfig(L, D, F, H, HKV, HD, V, eps=1e-5, theta=1e4, qk_norm=False,
                         res_alpha=1.0 / math.sqrt(2.0 * L))
    layers, rf, emb = hd.scratch_init(L, D, F, H, HKV, HD, V)
    e = ne.Engine(cfg)
    e.set_weights(layers, rf, emb, None)
    e.train_alloc(1, S)
    e.train_set_masters(layers, emb)
    rng = hd.Drand48(42)
    out, losses, t = {}, [], 0
    for step in range(steps):
        pos = int(rng() * (len(data) - S - 1))
        losses.append(e.train_fwd_bwd(data[pos:pos + S + 1].astype(np.int32)[None]))
        if (step + 1) % accum == 0 or step == steps - 1:
            t += 1
            e.adamw_step(t, e.lr_schedule(step, lr, warmup, steps), grad_clip=1.0,
                         grad_scale=1.0 / accum)
            out[step + 1] = e.get_masters()
    e.close()
    return out, losses


def test_cli_training_run_matches_the_binding_driven_loop(tmp_path):
    rs = np.random.default_rng(5)
    data = rs.integers(0, V, 20_000).astype(np.uint16)
    dpath = tmp_path / "tok.bin"
    data.tofile(dpath)
    ck = str(tmp_path / "ck.bin")
    args = [BIN, *SHAPE, "--data", str(dpath), "--ckpt", ck, "--lr", "2e-3", "--accum", "2",
            "--warmup", "2", "--save-every", "2"]
    r = subprocess.run(args + ["--scratch", "--steps", "6"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    steps = [(int(m.group(1)), float(m.group(2)))
             for m in re.finditer(r"step\s+(\d+)\s+loss=([\d.]+)", r.stdout)]
    assert steps and steps[0][0] == 0
    assert "[ckpt saved, best_loss=" in r.stdout
    # the lines the reference's dashboard parses (training/dashboard.py:338-357)
    for pat in (r"ANE Dynamic Training: (.+?) \((\d+) layers",
                r"dim=(\d+) q_dim=(\d+) kv_dim=(\d+) hd=(\d+) hidden=(\d+) seq=(\d+) vocab=(\d+)",
                r"Params: ([\d.]+)M \(transformer ([\d.]+)M \+ embed ([\d.]+)M\)",
                r"Accum (\d+).*LR=([\d.e+-]+)",
                r"step\s+(\d+)\s+loss=([\d.]+)(?:\s+lr=([\d.e+-]+))?(?:\s+([\d.]+)ms/step)?",
                r"\[ckpt saved, best_loss=([\d.]+)\]",
                # the web dashboard's step, timing and io_bwd lines
                # (training/dashboard-web/app.py:40-53), printed as train.m:766-776 does
                r"step\s+(\d+)\s+loss=([\d.]+)\s+lr=([\d.e+-]+)\s+([\d.]+)ms/step\s+"
                r"x\[([-\d.]+),([-\d.]+)\]\s+dy\[([-\d.e+-]+),([-\d.e+-]+)\]",
                r"timing: ane_fwd=([\d.]+) io_fwd=([\d.]+) rms=([\d.]+) "
                r"ane_bwd=([\d.]+) io_bwd=([\d.]+) rms_bwd=([\d.]+) "
                r"cls=([\d.]+) dw=([\d.]+) dwait=([\d.]+) resid=([\d.]+) "
                r"gqa=([\d.]+) rope=([\d.]+) \[gap=([\d.]+)\]",
                r"io_bwd: ffn_w=([\d.]+) ffn_r=([\d.]+) wot_w=([\d.]+) "
                r"s1=([\d.]+) s2=([\d.]+) s2r=([\d.]+) qkv_w=([\d.]+) qkv_r=([\d.]+)"):
        assert re.search(pat, r.stdout), pat
    t = re.search(r"timing: ane_fwd=([\d.]+) .* ane_bwd=([\d.]+) .* cls=([\d.]+)", r.stdout)
    assert float(t.group(1)) > 0 and float(t.group(2)) > 0 and float(t.group(3)) > 0
    xr = re.search(r"x\[([-\d.]+),([-\d.]+)\]\s+dy\[([-\d.e+-]+),([-\d.e+-]+)\]", r.stdout)
    assert float(xr.group(1)) < float(xr.group(2)) and float(xr.group(3)) < float(xr.group(4))
    m = re.search(r"step\s+(\d+)\s+loss=([\d.]+)(?:\s+lr=([\d.e+-]+))?(?:\s+([\d.]+)ms/step)?",
                  r.stdout)
    assert m.group(3) is not None and m.group(4) is not None   # lr and ms/step parsed too
    ref, losses = _replay(data, 6, 2, 2e-3, 2)
    assert abs(steps[0][1] - losses[0]) <= 1e-4
    got = ckpt_v4.read_v4(ck)
    saved = got.hdr.step
    assert saved in ref and got.hdr.adam_t == saved // 2
    for Lr in range(L):
        for k in ckpt_v4.LAYER_KEYS:
            assert _rel(got.layers[Lr][k], ref[saved]["layers"][Lr][k]) <= 1e-5, (Lr, k)
    assert _rel(got.embed, ref[saved]["embed"]) <= 1e-5


def test_cli_resume_continues_from_the_checkpoint(tmp_path):
    rs = np.random.default_rng(6)
    data = rs.integers(0, V, 20_000).astype(np.uint16)
    dpath = tmp_path / "tok.bin"
    data.tofile(dpath)
    ck = str(tmp_path / "ck.bin")
    base = [BIN, *SHAPE, "--data", str(dpath), "--ckpt", ck, "--lr", "1e-3", "--accum", "1",
            "--warmup", "1", "--save-every", "2"]
    r = subprocess.run(base + ["--scratch", "--steps", "2"], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    first = ckpt_v4.read_v4(ck, with_adam=True)
    assert first.hdr.step == 2 and first.hdr.adam_t == 2
    # the resumed run takes total_steps from the checkpoint (train.m:216-219)
    r = subprocess.run(base + ["--resume"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "[RESUMED step 2" in r.stdout
    assert "Total steps:  0" in r.stdout          # 2 of 2 steps were already done
