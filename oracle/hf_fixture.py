"""Synthetic Hugging Face checkpoints and the HF forward (test infrastructure;
see oracle/__init__.py).

* ``make_hf_model`` draws a seeded Qwen3/Llama-style state dict under the HF
  tensor names that tools/convert_hf.py reads (convert_hf.py:77-131), every
  value exactly representable in bf16.
* ``write_safetensors`` / ``read_safetensors`` implement the safetensors file
  layout (8-byte little-endian header length, JSON header of
  {name: {dtype, shape, data_offsets}}, data block) for F32 and BF16.
* ``hf_forward`` is the HF modelling arithmetic of a Qwen3 decoder in
  float64: RMSNorm, q/k/v projections, per-head QK RMSNorm, RoPE in the
  rotate_half convention (dimension i pairs with i + hd/2, frequency
  theta^(-2i/hd)), causal GQA attention, SwiGLU MLP, tied LM head.  The
  reference's kernels rotate interleaved pairs (2i, 2i+1) instead
  (tools/generate.py:97-110), which is why a converted HF model needs its
  q/k rows permuted.
"""
from __future__ import annotations

import json
import struct

import numpy as np

F32 = np.float32


def _bf16_values(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(a, F32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(F32)


def make_hf_model(seed=0, n_layers=2, dim=64, hidden=96, heads=4, kv_heads=2, head_dim=32,
                  vocab=80, qk_norm=True, lm_head=False, std=0.08):
    rs = np.random.default_rng(seed)

    def w(*shape, s=std):
        return _bf16_values(rs.normal(0.0, s, size=shape).astype(F32))

    def gain(n):
        return _bf16_values((1.0 + rs.uniform(-0.3, 0.3, size=n)).astype(F32))

    q_dim, kv_dim = heads * head_dim, kv_heads * head_dim
    t = {"model.embed_tokens.weight": w(vocab, dim, s=0.5), "model.norm.weight": gain(dim)}
    if lm_head:
        t["lm_head.weight"] = w(vocab, dim, s=0.5)
    for L in range(n_layers):
        p = f"model.layers.{L}."
        t[p + "self_attn.q_proj.weight"] = w(q_dim, dim)
        t[p + "self_attn.k_proj.weight"] = w(kv_dim, dim)
        t[p + "self_attn.v_proj.weight"] = w(kv_dim, dim)
        t[p + "self_attn.o_proj.weight"] = w(dim, q_dim)
        t[p + "mlp.gate_proj.weight"] = w(hidden, dim)
        t[p + "mlp.up_proj.weight"] = w(hidden, dim)
        t[p + "mlp.down_proj.weight"] = w(dim, hidden)
        t[p + "input_layernorm.weight"] = gain(dim)
        t[p + "post_attention_layernorm.weight"] = gain(dim)
        if qk_norm:
            t[p + "self_attn.q_norm.weight"] = gain(head_dim)
            t[p + "self_attn.k_norm.weight"] = gain(head_dim)
    config = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3",
              "hidden_size": dim, "intermediate_size": hidden, "num_attention_heads": heads,
              "num_key_value_heads": kv_heads, "head_dim": head_dim,
              "num_hidden_layers": n_layers, "vocab_size": vocab, "rms_norm_eps": 1e-6,
              "rope_theta": 1000000.0, "tie_word_embeddings": not lm_head,
              "torch_dtype": "bfloat16"}
    return t, config


def write_safetensors(path: str, tensors: dict, dtype: str = "BF16") -> None:
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, F32)
        if dtype == "BF16":
            raw = (a.view(np.uint32) >> 16).astype(np.uint16).tobytes()
        else:
            raw = a.tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - (8 + len(h)) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        buf = f.read()
    (n,) = struct.unpack("<Q", buf[:8])
    header = json.loads(buf[8:8 + n])
    base = 8 + n
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        b0, b1 = e["data_offsets"]
        raw = buf[base + b0: base + b1]
        if e["dtype"] == "F32":
            a = np.frombuffer(raw, F32)
        elif e["dtype"] == "BF16":
            a = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(F32)
        else:
            raise ValueError(e["dtype"])
        out[name] = a.reshape(e["shape"]).copy()
    return out


def _rms(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def hf_forward(t: dict, config: dict, tokens: np.ndarray) -> np.ndarray:
    """float64 logits [S, V] of one sequence, HF conventions (see module doc)."""
    D = config["hidden_size"]
    H, Hkv, hd = config["num_attention_heads"], config["num_key_value_heads"], config["head_dim"]
    eps, theta = config["rms_norm_eps"], config["rope_theta"]
    S = len(tokens)
    g = lambda k: t[k].astype(np.float64)
    inv = 1.0 / theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd)
    ang = np.arange(S, dtype=np.float64)[:, None] * inv[None, :]          # [S, hd/2]
    cos = np.concatenate([np.cos(ang), np.cos(ang)], -1)[:, None, :]
    sin = np.concatenate([np.sin(ang), np.sin(ang)], -1)[:, None, :]

    def rot_half(x):
        return np.concatenate([-x[..., hd // 2:], x[..., :hd // 2]], -1)

    x = g("model.embed_tokens.weight")[tokens]
    mask = np.tril(np.ones((S, S), bool))
    for L in range(config["num_hidden_layers"]):
        p = f"model.layers.{L}."
        xn = _rms(x, g(p + "input_layernorm.weight"), eps)
        q = (xn @ g(p + "self_attn.q_proj.weight").T).reshape(S, H, hd)
        k = (xn @ g(p + "self_attn.k_proj.weight").T).reshape(S, Hkv, hd)
        v = (xn @ g(p + "self_attn.v_proj.weight").T).reshape(S, Hkv, hd)
        if p + "self_attn.q_norm.weight" in t:
            q = _rms(q, g(p + "self_attn.q_norm.weight"), eps)
            k = _rms(k, g(p + "self_attn.k_norm.weight"), eps)
        q = q * cos + rot_half(q) * sin
        k = k * cos + rot_half(k) * sin
        o = np.empty((S, H, hd))
        for h in range(H):
            kh = h // (H // Hkv)
            s = q[:, h] @ k[:, kh].T / np.sqrt(hd)
            s = np.where(mask, s, -np.inf)
            s = np.exp(s - s.max(-1, keepdims=True))
            o[:, h] = (s / s.sum(-1, keepdims=True)) @ v[:, kh]
        x = x + o.reshape(S, H * hd) @ g(p + "self_attn.o_proj.weight").T
        xn = _rms(x, g(p + "post_attention_layernorm.weight"), eps)
        a = xn @ g(p + "mlp.gate_proj.weight").T
        u = xn @ g(p + "mlp.up_proj.weight").T
        x = x + (a / (1.0 + np.exp(-a)) * u) @ g(p + "mlp.down_proj.weight").T
    x = _rms(x, g("model.norm.weight"), eps)
    head = "lm_head.weight" if "lm_head.weight" in t else "model.embed_tokens.weight"
    return x @ g(head).T
