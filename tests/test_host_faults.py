"""CPU: failure paths made on the host, with no GPU and no GPU fault.

* ne_ckpt_probe (and the same checks inside ne_load_ckpt_v4) rejects a
  corrupt header and a truncated file before anything is loaded; the
  reference's own loader (train.m:133-165) reads fixed sizes and would take
  a short file's garbage;
* ne_train refuses a checkpoint that fails those checks, and a token file cut
  inside a token, before it initialises a GPU;
* a data-parallel rank whose rank 0 never starts gives up at the deadline
  instead of waiting for good;
* NE_FAULT_INJECT fails the n-th call of a named entry point with the chosen
  status, before the call does any work.
"""
import os
import struct
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_train")
SHAPE = ["--model", "custom", "--layers", "2", "--dim", "64", "--hidden", "128", "--heads", "4",
         "--kv-heads", "2", "--head-dim", "64", "--vocab", "96"]
IO, FORMAT = 4, 5


def _bin():
    if not os.path.exists(BIN):
        from neural_engine_b200 import build
        build.build(verbose=False)
    return BIN


def _dump(tmp_path, name="init.bin"):
    path = str(tmp_path / name)
    subprocess.run([_bin(), *SHAPE, "--seq", "32", "--dump-init", path], check=True, timeout=60)
    return path


def _status(path):
    from neural_engine_b200 import runtime
    try:
        runtime.ckpt_probe(path)
        return 0
    except runtime.NeError as e:
        return e.status


def _patch(path, out, offset, fmt, value):
    raw = bytearray(open(path, "rb").read())
    struct.pack_into(fmt, raw, offset, value)
    open(out, "wb").write(bytes(raw))
    return out


def test_probe_reads_the_shape_of_a_written_checkpoint(tmp_path):
    from neural_engine_b200 import runtime
    shape, hdr = runtime.ckpt_probe(_dump(tmp_path))
    assert shape == {"n_layers": 2, "dim": 64, "hidden": 128, "n_heads": 4, "kv_heads": 2,
                     "head_dim": 64, "vocab": 96, "qk_norm": 0}
    assert hdr["seq_len"] == 32 and hdr["has_qk_norm"] == 0


def test_probe_rejects_corrupt_headers(tmp_path):
    good = _dump(tmp_path)
    assert _status(good) == 0
    bad = str(tmp_path / "bad.bin")
    # magic, version, n_layers, vocab, n_heads vs q_dim, kv_heads not dividing n_heads
    for off, fmt, val in [(0, "<i", 0x11111111), (4, "<i", 5), (16, "<i", -2), (20, "<i", 0),
                          (32, "<i", 3), (84, "<i", 3)]:
        assert _status(_patch(good, bad, off, fmt, val)) == FORMAT, (off, val)
    # a header claiming more layers than the body holds reads as truncated
    assert _status(_patch(good, bad, 16, "<i", 3)) == FORMAT
    assert _status(str(tmp_path / "missing.bin")) == IO


def test_probe_rejects_truncated_files(tmp_path):
    good = _dump(tmp_path)
    raw = open(good, "rb").read()
    cut = str(tmp_path / "cut.bin")
    for n in (len(raw) - 4, len(raw) - 1, len(raw) // 2, 96, 50, 0):
        open(cut, "wb").write(raw[:n])
        assert _status(cut) == FORMAT, n
    # the optional QK-norm block: whole, then cut
    qk = str(tmp_path / "qk.bin")
    block = b"QKN1" + struct.pack("<ii", 2, 64) + bytes(4 * 6 * 2 * 64)
    open(qk, "wb").write(raw + block)
    from neural_engine_b200 import runtime
    shape, hdr = runtime.ckpt_probe(qk)
    assert shape["qk_norm"] == 1 and hdr["has_qk_norm"] == 1
    open(qk, "wb").write(raw + block[:-8])
    assert _status(qk) == FORMAT
    # a block for another layer count
    open(qk, "wb").write(raw + b"QKN1" + struct.pack("<ii", 3, 64) + bytes(4 * 6 * 3 * 64))
    assert _status(qk) == FORMAT


def test_resume_from_a_corrupt_checkpoint_stops_before_the_gpu(tmp_path):
    good = _dump(tmp_path)
    raw = open(good, "rb").read()
    cut = str(tmp_path / "cut.bin")
    open(cut, "wb").write(raw[:-100])
    r = subprocess.run([_bin(), *SHAPE, "--seq", "32", "--synthetic", "--resume", "--ckpt", cut],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1
    assert "[RESUME FAILED]" in r.stdout and "truncated" in r.stdout
    r = subprocess.run([_bin(), *SHAPE, "--seq", "16", "--synthetic", "--resume", "--ckpt",
                        _patch(good, str(tmp_path / "other.bin"), 24, "<i", 128)],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "[RESUME FAILED]" in r.stdout


def test_truncated_token_file_is_refused(tmp_path):
    data = str(tmp_path / "tok.bin")
    open(data, "wb").write(bytes(2 * 1000 + 1))
    r = subprocess.run([_bin(), *SHAPE, "--seq", "32", "--data", data, "--print-windows", "1"],
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "truncated" in r.stdout
    open(data, "wb").write(bytes(4 * 1000 + 2))
    r = subprocess.run([_bin(), *SHAPE, "--seq", "32", "--data", data, "--data-u32",
                        "--print-windows", "1"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "truncated" in r.stdout


def test_rank_whose_rank0_never_starts_gives_up(tmp_path):
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="0",
               NE_COMM_ID_FILE=str(tmp_path / "never_written.bin"), NE_COMM_TIMEOUT_MS="1500")
    t0 = time.time()
    r = subprocess.run([_bin(), *SHAPE, "--seq", "32", "--synthetic", "--scratch"], env=env,
                       capture_output=True, text=True, timeout=60)
    took = time.time() - t0
    assert r.returncode == 1 and "did not start" in r.stderr, (r.stdout, r.stderr)
    assert 1.4 < took < 30, took


_INJECT = r"""
import sys
sys.path.insert(0, sys.argv[1])
from neural_engine_b200 import runtime
lib = runtime.load_library()
out = []
for _ in range(4):
    try:
        runtime.shard_range(1000, 4, 1, lib)
        out.append(0)
    except runtime.NeError as e:
        out.append(e.status)
out.append(runtime.fault_calls("ne_shard_range", lib))
for _ in range(2):
    try:
        runtime.ckpt_probe(sys.argv[2], lib)
        out.append(0)
    except runtime.NeError as e:
        out.append(e.status)
out.append(runtime.fault_calls("ne_prefill", lib))
print(out)
"""


def test_fault_injection_fails_the_chosen_call(tmp_path):
    good = _dump(tmp_path)
    env = dict(os.environ, NE_FAULT_INJECT="ne_shard_range:2:timeout,ne_shard_range:4,"
                                           "ne_ckpt_probe:1:io,bogus,ne_prefill:x")
    r = subprocess.run([sys.executable, "-c", _INJECT, ROOT, good], env=env, capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    # calls 2 (timeout) and 4 (default cuda) fail; the probe's first call fails
    # with io, its second reads the good file; malformed items are ignored
    assert r.stdout.strip().splitlines()[-1] == "[0, 6, 0, 2, 4, 4, 0, 0]"


def test_ne_train_reports_an_injected_failure(tmp_path):
    good = _dump(tmp_path)
    env = dict(os.environ, NE_FAULT_INJECT="ne_ckpt_probe:1:io")
    r = subprocess.run([_bin(), *SHAPE, "--seq", "32", "--synthetic", "--resume", "--ckpt", good],
                       env=env, capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "[RESUME FAILED]" in r.stdout, (r.stdout, r.stderr)
