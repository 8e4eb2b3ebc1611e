"""CPU: the ne_train command-line driver's host logic against the restated
reference driver (oracle/host_driver.py): the drand48 generator (pinned to the
C library's own), the scratch initialisation written as a v4 checkpoint
(--dump-init), and the data windows (--print-windows).  None of these touch a
GPU."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from oracle import ckpt_v4
from oracle import host_driver as hd

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_train")


def _bin():
    if not os.path.exists(BIN):
        from neural_engine_b200 import build
        build.build(verbose=False)
    return BIN


def test_drand48_restatement_matches_the_c_library():
    libc = ctypes.CDLL(None)
    libc.drand48.restype = ctypes.c_double
    libc.srand48.argtypes = [ctypes.c_long]
    for seed in (42, 43, 1042, 0):
        libc.srand48(seed)
        r = hd.Drand48(seed)
        for _ in range(1000):
            assert libc.drand48() == r()


SHAPE = ["--model", "custom", "--layers", "2", "--dim", "64", "--hidden", "128", "--heads", "4",
         "--kv-heads", "2", "--head-dim", "64", "--vocab", "96"]


def test_scratch_init_is_the_reference_initialisation(tmp_path):
    path = str(tmp_path / "init.bin")
    subprocess.run([_bin(), *SHAPE, "--seq", "32", "--dump-init", path], check=True, timeout=60)
    ck = ckpt_v4.read_v4(path, with_adam=True)
    layers, rf, emb = hd.scratch_init(2, 64, 128, 4, 2, 64, 96)
    assert ck.hdr.n_layers == 2 and ck.hdr.q_dim == 256 and ck.hdr.seq_len == 32
    for L in range(2):
        for k in ckpt_v4.LAYER_KEYS:
            assert np.array_equal(ck.layers[L][k], layers[L][k]), (L, k)
            assert not ck.adam["layers"][L][k][0].any()
    assert np.array_equal(ck.rms_final, rf)
    assert np.array_equal(ck.embed, emb)


def test_data_windows_follow_the_reference_sampling(tmp_path):
    n = 100_000
    data = (np.arange(n) % 50_000).astype(np.uint16)
    path = tmp_path / "tok.bin"
    data.tofile(path)
    out = subprocess.run([_bin(), *SHAPE, "--seq", "256", "--data", str(path),
                          "--print-windows", "20"], check=True, capture_output=True, text=True,
                         timeout=60).stdout.split()
    assert [int(x) for x in out] == hd.sample_windows(n, 256, 20, seed=42)


def test_cli_rejects_unknown_flags():
    r = subprocess.run([_bin(), "--bogus"], capture_output=True, text=True, timeout=30)
    assert r.returncode == 2
    r = subprocess.run([_bin(), "--help"], capture_output=True, text=True, timeout=30)
    assert r.returncode == 0 and "--scratch" in r.stdout


def test_vocab_compaction_map_is_the_reference_map(tmp_path):
    """vocab_map_build (cpu_ops.h:391-414): ids present in the data, ascending."""
    rs = np.random.default_rng(3)
    data = rs.choice([5, 17, 3, 90, 41, 95], size=5000).astype(np.uint16)
    path = tmp_path / "tok.bin"
    data.tofile(path)
    out = subprocess.run([_bin(), *SHAPE, "--data", str(path), "--print-vocab"], check=True,
                         capture_output=True, text=True, timeout=60).stdout.split()
    assert int(out[0]) == 6 and [int(x) for x in out[1:]] == sorted(set(data.tolist()))
    out = subprocess.run([_bin(), *SHAPE, "--data", str(path), "--print-vocab",
                          "--no-compact-vocab"], check=True, capture_output=True, text=True,
                         timeout=60).stdout.split()
    assert out == ["0"]


def test_uint32_token_file_reads_ids_beyond_uint16(tmp_path):
    """--data-u32: the same windows and compaction map over uint32 ids, so a
    Qwen3-vocabulary token file (ids up to 151,935) can be fed."""
    shape = [*SHAPE[:-2], "--vocab", "151936"]
    ids = [5, 70_000, 151_935, 65_536, 17]
    data = np.random.default_rng(4).choice(ids, size=6000).astype(np.uint32)
    path = tmp_path / "tok32.bin"
    data.tofile(path)
    out = subprocess.run([_bin(), *shape, "--data", str(path), "--data-u32", "--print-vocab"],
                         check=True, capture_output=True, text=True, timeout=60).stdout.split()
    assert int(out[0]) == len(ids) and [int(x) for x in out[1:]] == sorted(ids)
    out = subprocess.run([_bin(), *shape, "--seq", "256", "--data", str(path), "--data-u32",
                          "--print-windows", "10"], check=True, capture_output=True, text=True,
                         timeout=60).stdout.split()
    assert [int(x) for x in out] == hd.sample_windows(len(data), 256, 10, seed=42)


def test_lr_schedule_follows_train_m():
    """ne_lr_schedule (a host function of libne.so, no GPU) against train.m:851-858
    restated in float32 (numpy's float32 cos stands in for libm's cosf: one ulp)."""
    from neural_engine_b200 import runtime
    from oracle import train as ot
    lib = runtime.load_library()
    f32 = np.float32
    for max_lr, warmup, total, frac in [(3e-4, 100, 1000, 0.1), (1e-3, 0, 50, 0.0),
                                         (2e-4, 10, 11, 0.5)]:
        for step in range(total):
            got = lib.ne_lr_schedule(step, max_lr, warmup, total, frac)
            mx, mn = f32(max_lr), f32(max_lr) * f32(frac)
            if step < warmup:
                want = mx * f32(step + 1) / f32(warmup)
            else:
                ratio = f32(step - warmup) / f32(total - warmup)
                arg = f32(np.pi * np.float64(ratio))           # cosf(M_PI * decay_ratio)
                want = mn + f32(0.5) * (f32(1.0) + np.cos(arg)) * (mx - mn)
            assert abs(got - float(want)) <= 2.5e-7 * max_lr, (step, got, want)
            assert abs(got - ot.lr_schedule(step, max_lr, warmup, total, frac)) <= 1e-6 * max_lr
