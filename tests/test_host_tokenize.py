"""CPU: neural_engine_b200.tokenize_data (tools/tokenize_data.py's command line).

The HF tokenizer needs the network, so ``AutoTokenizer.from_pretrained`` is
replaced by a stand-in whose ids are a fixed function of the text.  Checked:
the inputs joined with blank lines and encoded once, ``--max-tokens``, missing
files skipped, stdin, the uint16 file of the reference and its refusal of ids
beyond 65,535, and the ``--u32`` extension, whose file ``ne_train --data-u32``
reads back (its vocabulary map lists exactly the ids written).
"""
import contextlib
import io
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_train")


class FakeTokenizer:
    vocab_size = 151936

    def __init__(self, scale):
        self.scale = scale
        self.seen = []

    def encode(self, text):
        self.seen.append(text)
        return [(ord(c) * self.scale) % self.vocab_size for c in text]


@pytest.fixture()
def tok(monkeypatch):
    transformers = pytest.importorskip("transformers")
    holder = {}

    def from_pretrained(name, trust_remote_code=False):
        holder["tok"] = FakeTokenizer(holder.get("scale", 1))
        return holder["tok"]

    monkeypatch.setattr(transformers.AutoTokenizer, "from_pretrained", from_pretrained)
    return holder


def _main(argv, stdin=None):
    from neural_engine_b200 import tokenize_data as td
    out = io.StringIO()
    old = sys.stdin
    if stdin is not None:
        sys.stdin = io.StringIO(stdin)
    try:
        with contextlib.redirect_stdout(out):
            arr = td.main(argv)
    finally:
        sys.stdin = old
    return arr, out.getvalue()


def test_uint16_file_as_the_reference_writes_it(tmp_path, tok):
    a, b = tmp_path / "a.txt", tmp_path / "b.txt"
    a.write_text("Once upon a time")
    b.write_text("there was a cat")
    out = tmp_path / "data.bin"
    arr, text = _main([str(a), str(tmp_path / "missing.txt"), str(b), "-m", "x", "-o", str(out)])
    assert tok["tok"].seen == ["Once upon a time\n\nthere was a cat"]
    want = np.array([ord(c) for c in "Once upon a time\n\nthere was a cat"], np.uint16)
    assert np.array_equal(np.fromfile(out, np.uint16), want) and arr.dtype == np.uint16
    assert "Warning: " + str(tmp_path / "missing.txt") + " not found, skipping" in text
    assert "--data-u32" not in text.splitlines()[-1]
    _, _ = _main([str(a), "-m", "x", "-o", str(out), "--max-tokens", "4"])
    assert np.fromfile(out, np.uint16).tolist() == [ord(c) for c in "Once"]
    _, _ = _main(["-", "-m", "x", "-o", str(out)], stdin="hi")
    assert np.fromfile(out, np.uint16).tolist() == [ord("h"), ord("i")]


def test_ids_beyond_uint16_need_u32(tmp_path, tok):
    tok["scale"] = 1500                       # ord('z') * 1500 = 183,000 -> mod 151,936
    src = tmp_path / "a.txt"
    src.write_text("zebra" * 200)        # more than one 256-token window
    out = tmp_path / "data.bin"
    with pytest.raises(SystemExit):
        _main([str(src), "-m", "x", "-o", str(out)])
    arr, text = _main([str(src), "-m", "x", "-o", str(out), "--u32"])
    ids = np.fromfile(out, np.uint32)
    assert arr.dtype == np.uint32 and ids.max() > 65535
    assert ids.tolist() == [(ord(c) * 1500) % 151936 for c in "zebra" * 200]
    assert text.splitlines()[-1].endswith("--data-u32")
    if not os.path.exists(BIN):
        from neural_engine_b200 import build
        build.build(verbose=False)
    shape = ["--model", "custom", "--layers", "2", "--dim", "64", "--hidden", "128", "--heads",
             "4", "--kv-heads", "2", "--head-dim", "16", "--vocab", "151936"]
    got = subprocess.run([BIN, *shape, "--data", str(out), "--data-u32", "--print-vocab"],
                         check=True, capture_output=True, text=True, timeout=60).stdout.split()
    assert int(got[0]) == len(set(ids.tolist()))
    assert [int(x) for x in got[1:]] == sorted(set(ids.tolist()))
