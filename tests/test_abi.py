"""CPU: the C ABI library loads and exports what include/ne.h declares; host
logic that needs no GPU (v4 checkpoint layout, argument validation)."""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    txt = open(os.path.join(ROOT, "include", "ne.h")).read()
    return sorted(set(re.findall(r"NE_API\s+[\w\s\*]+?\b(ne_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    syms = _declared_symbols()
    assert "ne_init" in syms and "ne_decode_step" in syms and "ne_gemm_device" in syms
    assert len(syms) >= 15


def test_library_exports_every_declared_symbol():
    import neural_engine_b200 as ne
    lib = ctypes.CDLL(ne.LIB_PATH)
    for s in _declared_symbols():
        assert hasattr(lib, s), f"libne.so does not export {s}"
    assert set(_declared_symbols()) == set(ne.EXPORTED)


def test_version_and_status_strings():
    import neural_engine_b200 as ne
    lib = ne.load_library()
    assert b"sm_100a" in lib.ne_version()
    assert lib.ne_status_str(0) == b"ok"
    assert lib.ne_status_str(6) == b"device wait timed out"


def test_init_rejects_bad_configs_without_touching_a_gpu():
    """Shape validation happens before any CUDA call."""
    import neural_engine_b200 as ne
    from neural_engine_b200.runtime import ModelCfgC
    lib = ne.load_library()
    ctx = ctypes.c_void_p()
    bad_hd = ModelCfgC(2, 128, 256, 4, 2, 32, 512, 1e-5, 1e4, 0, 1e-6, 1.0)   # head_dim 32
    assert lib.ne_init(ctypes.byref(ctx), ctypes.byref(bad_hd), 0) == 7       # UNSUPPORTED
    bad_gqa = ModelCfgC(2, 128, 256, 6, 4, 64, 512, 1e-5, 1e4, 0, 1e-6, 1.0)  # 6 % 4 != 0
    assert lib.ne_init(ctypes.byref(ctx), ctypes.byref(bad_gqa), 0) == 1      # INVALID
    assert lib.ne_init(None, ctypes.byref(bad_gqa), 0) == 1


def test_v4_roundtrip_and_product_reader(tmp_path):
    """Oracle writer -> product reader (neural_engine_b200.generate.read_checkpoint)."""
    from oracle import ckpt_v4, model as om
    from neural_engine_b200.generate import read_checkpoint
    cfg = om.tiny(head_dim=16)
    layers, rf, emb, qk = om.init_weights(cfg, seed=11)
    ck = om.make_checkpoint(cfg, layers, rf, emb)
    p = str(tmp_path / "a.bin")
    ckpt_v4.write_v4(p, ck)
    nparams = cfg.n_params()
    # 96-byte header + weights + Adam m, v (3x params, fp32)
    assert os.path.getsize(p) == 96 + 12 * nparams
    info, L2, rf2, emb2 = read_checkpoint(p)
    assert info["kv_heads"] == cfg.kv_heads and info["hd"] == cfg.head_dim
    for a, b in zip(layers, L2):
        for k in a:
            np.testing.assert_array_equal(a[k], b[k])
    np.testing.assert_array_equal(emb, emb2)
    back = ckpt_v4.read_v4(p, with_adam=True)
    assert back.hdr.q_dim == cfg.q_dim and back.qk_norm is None


def test_v4_qk_extension_block(tmp_path):
    from oracle import ckpt_v4, model as om
    from neural_engine_b200.generate import read_checkpoint
    cfg = om.tiny(head_dim=16, qk_norm=True)
    layers, rf, emb, qk = om.init_weights(cfg, seed=12)
    layers, rf, qk = om.random_gains(cfg, layers, rf, qk)
    ck = om.make_checkpoint(cfg, layers, rf, emb, qk=qk)
    p = str(tmp_path / "b.bin")
    ckpt_v4.write_v4(p, ck)
    info, _, _, _ = read_checkpoint(p)
    assert info["qk_norm"]
    for (q1, k1), q2, k2 in zip(qk, info["q_norm"], info["k_norm"]):
        np.testing.assert_array_equal(q1, q2)
        np.testing.assert_array_equal(k1, k2)


def test_reference_reader_header_slots():
    """The reference's generate.py:28 reads kv_heads/hd/q_dim from header
    fields 15..17 (cum_steps, cum_batches, adam_t); config.h:89 puts them at
    18..20.  The product reader uses 18..20."""
    from oracle.ckpt_v4 import CkptHeader, HDR_FMT
    h = CkptHeader(n_layers=1, vocab=8, dim=64, hidden=64, heads=2, kv_heads=1, head_dim=32,
                   q_dim=64, cum_steps=5, cum_batches=6, adam_t=7)
    v = struct.unpack(HDR_FMT, h.pack())
    assert v[15:18] == (5, 6, 7) and v[18:21] == (1, 32, 64)
