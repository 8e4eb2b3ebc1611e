"""Golden checksums of the reference's HF -> v4 converter.

Run in the build container, where the reference tree is mounted:

    python tests/golden/make_convert_golden.py --ref <reference root>

Imports ``write_checkpoint`` from the reference's own
``ane-training/training/training_dynamic/tools/convert_hf.py`` unchanged (its
HF-hub loader is not called: the state dict comes from the seeded synthetic
model of ``oracle/hf_fixture.py``), writes the checkpoint for each fixture
variant into a temporary directory and records its SHA-256 and size in
``convert_hf_ref.json``.  tests/test_host_convert.py converts the same
synthetic model with ne_convert and compares the bytes' checksum.
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import importlib.util
import io
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import hf_fixture  # noqa: E402

VARIANTS = {
    "qwen3_tied": dict(seed=5, qk_norm=True, lm_head=False),
    "llama_lm_head": dict(seed=6, qk_norm=False, lm_head=True, kv_heads=4),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference repository root")
    args = ap.parse_args()
    path = os.path.join(args.ref, "ane-training", "training", "training_dynamic", "tools",
                        "convert_hf.py")
    spec = importlib.util.spec_from_file_location("ref_convert_hf", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    with tempfile.TemporaryDirectory() as td:
        for name, kw in VARIANTS.items():
            t, cfg = hf_fixture.make_hf_model(**kw)
            ck = os.path.join(td, name + ".bin")
            with contextlib.redirect_stdout(io.StringIO()):
                mod.write_checkpoint(ck, t, cfg)
            data = open(ck, "rb").read()
            out[name] = {"params": kw, "sha256": hashlib.sha256(data).hexdigest(),
                         "bytes": len(data)}
    with open(os.path.join(HERE, "convert_hf_ref.json"), "w") as f:
        json.dump(out, f, indent=2)
    print(json.dumps(out, indent=2))


if __name__ == "__main__":
    main()
