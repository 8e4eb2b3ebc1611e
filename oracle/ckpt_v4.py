"""v4 checkpoint reader/writer (test infrastructure; see oracle/__init__.py).

Layout restated from the reference:
  * header ``CkptHdr`` -- ane-training/training/training_dynamic/config.h:83-91:
        int magic=0x424C5A54, version=4, step, total_steps
        int n_layers, vocab_size, dim, hidden_dim, n_heads, seq_len
        float lr, loss
        double cum_compile, cum_train, cum_wall
        int cum_steps, cum_batches, adam_t
        int kv_heads, head_dim, q_dim
    96 bytes, no padding (struct "iiiiiiiiiiffdddiiiiii").
  * body -- train.m:110-130 (save_checkpoint):
        for each layer: Wq, Wk, Wv, Wo, W1, W2, W3, rms_att, rms_ffn (fp32),
                        then (m, v) for each of those nine tensors, in order;
        rms_final, its m, v;  embed [V*D], its m, v.
  * optional trailing extension block (this build only; v4 readers stop
    before it, generate.py:73-76 and train.m:159-162 read fixed sizes):
        char magic[4] = "QKN1"; int n_layers, head_dim;
        for each layer: q_norm[hd], k_norm[hd], then m, v of each.

Note the reference's own ``generate.py:28`` reads kv_heads/hd/q_dim from the
cum_steps/cum_batches/adam_t slots (``hdr_data[15:18]``); this reader uses the
correct slots ``[18:21]`` (config.h:89).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = 0x424C5A54
VERSION = 4
HDR_FMT = "<iiiiiiiiiiffdddiiiiii"
HDR_SIZE = struct.calcsize(HDR_FMT)
assert HDR_SIZE == 96
EXT_MAGIC = b"QKN1"

LAYER_KEYS = ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3", "rms_att", "rms_ffn")


@dataclass
class CkptHeader:
    step: int = 0
    total_steps: int = 10000
    n_layers: int = 0
    vocab: int = 0
    dim: int = 0
    hidden: int = 0
    heads: int = 0
    seq_len: int = 256
    lr: float = 3e-4
    loss: float = 0.0
    cum_compile: float = 0.0
    cum_train: float = 0.0
    cum_wall: float = 0.0
    cum_steps: int = 0
    cum_batches: int = 0
    adam_t: int = 0
    kv_heads: int = 0
    head_dim: int = 0
    q_dim: int = 0

    def pack(self) -> bytes:
        return struct.pack(
            HDR_FMT, MAGIC, VERSION, self.step, self.total_steps,
            self.n_layers, self.vocab, self.dim, self.hidden, self.heads, self.seq_len,
            self.lr, self.loss, self.cum_compile, self.cum_train, self.cum_wall,
            self.cum_steps, self.cum_batches, self.adam_t,
            self.kv_heads, self.head_dim, self.q_dim)

    @classmethod
    def unpack(cls, raw: bytes) -> "CkptHeader":
        v = struct.unpack(HDR_FMT, raw[:HDR_SIZE])
        if v[0] != MAGIC:
            raise ValueError(f"bad magic {v[0]:#x}")
        if v[1] != VERSION:
            raise ValueError(f"unsupported version {v[1]}")
        return cls(step=v[2], total_steps=v[3], n_layers=v[4], vocab=v[5], dim=v[6],
                   hidden=v[7], heads=v[8], seq_len=v[9], lr=v[10], loss=v[11],
                   cum_compile=v[12], cum_train=v[13], cum_wall=v[14], cum_steps=v[15],
                   cum_batches=v[16], adam_t=v[17], kv_heads=v[18], head_dim=v[19],
                   q_dim=v[20])


def layer_shapes(h: CkptHeader) -> dict:
    """Per-layer tensor shapes, config.h:26-32 (row-major [out, in])."""
    kv_dim = h.kv_heads * h.head_dim
    return {"Wq": (h.q_dim, h.dim), "Wk": (kv_dim, h.dim), "Wv": (kv_dim, h.dim),
            "Wo": (h.dim, h.q_dim), "W1": (h.hidden, h.dim), "W2": (h.dim, h.hidden),
            "W3": (h.hidden, h.dim), "rms_att": (h.dim,), "rms_ffn": (h.dim,)}


@dataclass
class Checkpoint:
    hdr: CkptHeader
    layers: list                      # list of dict name -> fp32 array
    rms_final: np.ndarray
    embed: np.ndarray                 # [V, D]
    adam: dict | None = None          # optional: "layers": [dict name -> (m, v)], "rms_final": (m, v), "embed": (m, v)
    qk_norm: list | None = None       # optional: per layer (q_norm[hd], k_norm[hd])
    qk_adam: list | None = field(default=None)


def write_v4(path: str, ck: Checkpoint) -> None:
    h = ck.hdr
    shapes = layer_shapes(h)
    with open(path, "wb") as f:
        f.write(h.pack())
        for L, lw in enumerate(ck.layers):
            for k in LAYER_KEYS:
                a = np.ascontiguousarray(lw[k], dtype=np.float32)
                assert a.shape == shapes[k], (k, a.shape, shapes[k])
                f.write(a.tobytes())
            for k in LAYER_KEYS:
                if ck.adam is not None:
                    m, v = ck.adam["layers"][L][k]
                    f.write(np.ascontiguousarray(m, np.float32).tobytes())
                    f.write(np.ascontiguousarray(v, np.float32).tobytes())
                else:
                    z = np.zeros(int(np.prod(shapes[k])), np.float32).tobytes()
                    f.write(z)
                    f.write(z)
        f.write(np.ascontiguousarray(ck.rms_final, np.float32).tobytes())
        if ck.adam is not None:
            for a in ck.adam["rms_final"]:
                f.write(np.ascontiguousarray(a, np.float32).tobytes())
        else:
            f.write(np.zeros(2 * h.dim, np.float32).tobytes())
        f.write(np.ascontiguousarray(ck.embed, np.float32).tobytes())
        if ck.adam is not None:
            for a in ck.adam["embed"]:
                f.write(np.ascontiguousarray(a, np.float32).tobytes())
        else:
            z = np.zeros(h.vocab * h.dim, np.float32).tobytes()
            f.write(z)
            f.write(z)
        if ck.qk_norm is not None:
            f.write(EXT_MAGIC)
            f.write(struct.pack("<ii", h.n_layers, h.head_dim))
            for L, (qn, kn) in enumerate(ck.qk_norm):
                f.write(np.ascontiguousarray(qn, np.float32).tobytes())
                f.write(np.ascontiguousarray(kn, np.float32).tobytes())
                for i in range(2):
                    if ck.qk_adam is not None:
                        m, v = ck.qk_adam[L][i]
                    else:
                        m = v = np.zeros(h.head_dim, np.float32)
                    f.write(np.ascontiguousarray(m, np.float32).tobytes())
                    f.write(np.ascontiguousarray(v, np.float32).tobytes())


def read_v4(path: str, with_adam: bool = False) -> Checkpoint:
    with open(path, "rb") as f:
        h = CkptHeader.unpack(f.read(HDR_SIZE))
        shapes = layer_shapes(h)

        def rd(shape):
            n = int(np.prod(shape))
            buf = f.read(4 * n)
            if len(buf) != 4 * n:
                raise ValueError("truncated checkpoint")
            return np.frombuffer(buf, np.float32).reshape(shape).copy()

        layers, ladam = [], []
        for _ in range(h.n_layers):
            lw = {k: rd(shapes[k]) for k in LAYER_KEYS}
            la = {}
            for k in LAYER_KEYS:
                if with_adam:
                    la[k] = (rd(shapes[k]), rd(shapes[k]))
                else:
                    f.seek(8 * int(np.prod(shapes[k])), 1)
            layers.append(lw)
            ladam.append(la)
        rms_final = rd((h.dim,))
        rf_adam = (rd((h.dim,)), rd((h.dim,))) if with_adam else None
        if not with_adam:
            f.seek(8 * h.dim, 1)
        embed = rd((h.vocab, h.dim))
        emb_adam = (rd((h.vocab, h.dim)), rd((h.vocab, h.dim))) if with_adam else None
        if not with_adam:
            f.seek(8 * h.vocab * h.dim, 1)
        qk, qk_adam = None, None
        tail = f.read(4)
        if tail == EXT_MAGIC:
            nl, hd = struct.unpack("<ii", f.read(8))
            if nl != h.n_layers or hd != h.head_dim:
                raise ValueError("QKN1 block does not match header")
            qk, qk_adam = [], []
            for _ in range(nl):
                qn, kn = rd((hd,)), rd((hd,))
                st = [(rd((hd,)), rd((hd,))), (rd((hd,)), rd((hd,)))]
                qk.append((qn, kn))
                qk_adam.append(st)
    adam = None
    if with_adam:
        adam = {"layers": ladam, "rms_final": rf_adam, "embed": emb_adam}
    return Checkpoint(hdr=h, layers=layers, rms_final=rms_final, embed=embed,
                      adam=adam, qk_norm=qk, qk_adam=qk_adam if with_adam else None)
