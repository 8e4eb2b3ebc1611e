"""CPU: ne_convert, the HF safetensors <-> v4 checkpoint tool.

* from-hf without options writes the bytes of the reference's own converter
  (tools/convert_hf.py write_checkpoint; checksums in tests/golden/
  convert_hf_ref.json, made by tests/golden/make_convert_golden.py from the
  same synthetic model), whatever the shard split and the source dtype.
* --hf-exact (QK-norm block + RoPE row permutation) makes the checkpoint
  compute what the HF model computes: the oracle's interleaved-pair forward on
  the converted weights equals the HF rotate_half forward on the originals.
* to-hf inverts it exactly.
"""
import dataclasses
import hashlib
import json
import os
import subprocess

import numpy as np
import pytest

from oracle import ckpt_v4
from oracle import decode as od
from oracle import hf_fixture as hf
from oracle import model as om

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "neural_engine_b200", "ne_convert")
GOLD = json.load(open(os.path.join(ROOT, "tests", "golden", "convert_hf_ref.json")))


def _bin():
    if not os.path.exists(BIN):
        import importlib.util
        spec = importlib.util.spec_from_file_location(
            "ne_build", os.path.join(ROOT, "neural_engine_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build_convert(verbose=False)
    return BIN


def _model_dir(tmp_path, name, tensors, config, shards=2, dtype="BF16"):
    d = tmp_path / name
    d.mkdir()
    (d / "config.json").write_text(json.dumps(config))
    keys = list(tensors)
    for i in range(shards):
        part = {k: tensors[k] for k in keys[i::shards]}
        hf.write_safetensors(str(d / f"model-{i + 1:05d}-of-{shards:05d}.safetensors"), part, dtype)
    return d


@pytest.mark.parametrize("variant", sorted(GOLD))
@pytest.mark.parametrize("shards,dtype", [(1, "F32"), (3, "BF16")])
def test_from_hf_writes_the_reference_bytes(tmp_path, variant, shards, dtype):
    t, cfg = hf.make_hf_model(**GOLD[variant]["params"])
    d = _model_dir(tmp_path, variant, t, cfg, shards, dtype)
    out = tmp_path / "ck.bin"
    subprocess.run([_bin(), "from-hf", str(d), "-o", str(out)], check=True,
                   capture_output=True, timeout=60)
    data = out.read_bytes()
    assert len(data) == GOLD[variant]["bytes"]
    assert hashlib.sha256(data).hexdigest() == GOLD[variant]["sha256"]


def _oracle_from_ckpt(path, cfg):
    ck = ckpt_v4.read_v4(str(path))
    h = ck.hdr
    mc = om.ModelCfg(n_layers=h.n_layers, dim=h.dim, hidden=h.hidden, heads=h.heads,
                     kv_heads=h.kv_heads, head_dim=h.head_dim, vocab=h.vocab,
                     eps=cfg["rms_norm_eps"], theta=cfg["rope_theta"],
                     qk_norm=ck.qk_norm is not None, qk_eps=cfg["rms_norm_eps"])
    return mc, ck


@pytest.mark.parametrize("kv_heads", [2, 4])
def test_hf_exact_computes_the_hf_model(tmp_path, kv_heads):
    t, cfg = hf.make_hf_model(seed=11, qk_norm=True, kv_heads=kv_heads)
    d = _model_dir(tmp_path, "m", t, cfg)
    tok = np.random.default_rng(12).integers(0, cfg["vocab_size"], 19)
    want = hf.hf_forward(t, cfg, tok)
    scale = np.abs(want).max()
    errs = {}
    for flags in ([], ["--hf-exact"]):
        out = tmp_path / f"ck{len(flags)}.bin"
        subprocess.run([_bin(), "from-hf", str(d), "-o", str(out), *flags], check=True,
                       capture_output=True, timeout=60)
        mc, ck = _oracle_from_ckpt(out, cfg)
        if not flags:
            assert ck.qk_norm is None      # the reference drops the gains
            mc = dataclasses.replace(mc, qk_norm=True)   # and would need them: give them back
            qk = [(t[f"model.layers.{L}.self_attn.q_norm.weight"],
                   t[f"model.layers.{L}.self_attn.k_norm.weight"]) for L in range(mc.n_layers)]
        else:
            qk = ck.qk_norm
        dec = od.Decoder(mc, ck.layers, ck.rms_final, ck.embed, qk, batch=1, max_seq=32)
        got = dec.forward(tok[None, :], 0)[0]
        errs[len(flags)] = np.abs(got - want).max() / scale
    assert errs[1] < 2e-5, errs          # permuted rows: the HF model, to fp32 rounding
    assert errs[0] > 1e-2, errs          # HF row order under interleaved RoPE: a different model


def test_to_hf_inverts_from_hf(tmp_path):
    t, cfg = hf.make_hf_model(seed=13, qk_norm=True)
    d = _model_dir(tmp_path, "m", t, cfg)
    ck = tmp_path / "ck.bin"
    subprocess.run([_bin(), "from-hf", str(d), "-o", str(ck), "--hf-exact"], check=True,
                   capture_output=True, timeout=60)
    out = tmp_path / "hf_out"
    subprocess.run([_bin(), "to-hf", str(ck), "-o", str(out), "--hf-exact",
                    "--config", str(d / "config.json")], check=True, capture_output=True,
                   timeout=60)
    back = hf.read_safetensors(str(out / "model.safetensors"))
    assert set(back) == set(t)
    for k, a in t.items():
        assert back[k].dtype == np.float32 and np.array_equal(back[k], a), k
    assert json.loads((out / "config.json").read_text()) == cfg
    # without --config: the minimal config export_hf.py writes, from the header
    out2 = tmp_path / "hf_min"
    subprocess.run([_bin(), "to-hf", str(ck), "-o", str(out2)], check=True,
                   capture_output=True, timeout=60)
    c2 = json.loads((out2 / "config.json").read_text())
    for k in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads",
              "head_dim", "num_hidden_layers", "vocab_size"):
        assert c2[k] == cfg[k], k
    assert c2["tie_word_embeddings"] is True


def test_cli_errors(tmp_path):
    assert subprocess.run([_bin()], capture_output=True, timeout=30).returncode == 2
    assert subprocess.run([_bin(), "sideways", "x"], capture_output=True, timeout=30).returncode == 2
    r = subprocess.run([_bin(), "from-hf", str(tmp_path)], capture_output=True, text=True,
                       timeout=30)
    assert r.returncode == 1 and "config.json" in r.stderr
    t, cfg = hf.make_hf_model(seed=1)
    del t["model.layers.1.mlp.up_proj.weight"]
    d = _model_dir(tmp_path, "broken", t, cfg)
    r = subprocess.run([_bin(), "from-hf", str(d), "-o", str(tmp_path / "x.bin")],
                       capture_output=True, text=True, timeout=30)
    assert r.returncode == 1 and "model.layers.1.mlp.up_proj.weight" in r.stderr
