"""ctypes binding of libne.so (the C ABI declared in include/ne.h).

The library is the product: every computation below happens in its sm_100a
kernels.  There is no CPU fallback -- if libne.so is missing or cannot be
loaded, importing the runtime raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libne.so")

# ne_status values (include/ne.h)
NE_OK = 0
STATUS_NAMES = {0: "NE_OK", 1: "NE_ERR_INVALID", 2: "NE_ERR_CUDA", 3: "NE_ERR_OOM",
                4: "NE_ERR_IO", 5: "NE_ERR_FORMAT", 6: "NE_ERR_TIMEOUT",
                7: "NE_ERR_UNSUPPORTED", 8: "NE_ERR_STATE", 9: "NE_ERR_BOUNDS"}

# every entry point include/ne.h declares
EXPORTED = ("ne_init", "ne_free", "ne_last_error", "ne_status_str", "ne_sync", "ne_get_cfg",
            "ne_version", "ne_set_layer_weights", "ne_set_global_weights", "ne_load_ckpt_v4",
            "ne_kv_alloc", "ne_kv_reset", "ne_prefill", "ne_decode_step", "ne_generate", "ne_prefill_device",
            "ne_decode_loop_device", "ne_gemm_device", "ne_gemm_device_ex",
            "ne_decode_kernels_per_step", "ne_get_stream", "ne_profile_decode_step",
            "ne_gemm_splitk_noalloc", "ne_train_alloc", "ne_train_set_masters",
            "ne_train_sync_weights", "ne_train_zero_grads", "ne_train_fwd_bwd_device",
            "ne_train_fwd_bwd", "ne_train_grad_norm", "ne_adamw_step", "ne_lr_schedule",
            "ne_train_get_layer", "ne_gemm", "ne_train_grad_pool", "ne_save_ckpt_v4",
            "ne_embed_fwd", "ne_attn_fwd", "ne_ffn_fwd", "ne_lmhead_ce_fwd_bwd", "ne_ffn_bwd",
            "ne_attn_bwd", "ne_embed_bwd", "ne_rmsnorm_fwd", "ne_rmsnorm_bwd_add",
            "ne_comm_unique_id", "ne_comm_init", "ne_comm_set_reduce", "ne_grad_allreduce_async",
            "ne_sdpa_fwd_device", "ne_train_set_vocab_map", "ne_stream_read",
            "ne_comm_set_sharding", "ne_train_gather_state", "ne_train_fwd_bwd_timed",
            "ne_train_value_ranges", "ne_comm_set_timeout", "ne_shard_range",
            "ne_gemm_dw_owned", "ne_ckpt_probe", "ne_fault_calls")

def shard_range(n: int, world: int, rank: int, lib=None):
    """(offset, length) of the part of an n-element tensor that `rank` owns
    under ZeRO-1 over peer memory (ne_shard_range; host arithmetic)."""
    lib = lib or load_library()
    off, ln = C.c_longlong(0), C.c_longlong(0)
    st = lib.ne_shard_range(int(n), int(world), int(rank), C.byref(off), C.byref(ln))
    if st != 0:
        raise NeError(st, "ne_shard_range")
    return off.value, ln.value


def ckpt_probe(path: str, lib=None) -> tuple:
    """Check a v4 checkpoint on the host (ne_ckpt_probe): returns (model shape
    dict, header dict); raises NeError (io / format) for a missing, corrupt or
    truncated file."""
    lib = lib or load_library()
    cfg, info = ModelCfgC(), CkptInfoC()
    st = lib.ne_ckpt_probe(os.fsencode(path), C.byref(cfg), C.byref(info))
    if st != 0:
        raise NeError(st, f"ne_ckpt_probe {path}")
    shape = {k: getattr(cfg, k) for k in ("n_layers", "dim", "hidden", "n_heads", "kv_heads",
                                          "head_dim", "vocab", "qk_norm")}
    hdr = {k: getattr(info, k) for k, _ in CkptInfoC._fields_}
    return shape, hdr


def fault_calls(entry: str, lib=None) -> int:
    """Calls of `entry` counted by the NE_FAULT_INJECT hooks of this process."""
    lib = lib or load_library()
    return int(lib.ne_fault_calls(entry.encode()))


PROF_GROUPS = ("gemm_qkv", "qkv_post", "decode_attention", "gemm_wo", "resid_rmsnorm",
               "gemm_w13", "swiglu", "gemm_w2", "gemm_lm_head", "embed_argmax")


class NeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class ModelCfgC(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("dim", C.c_int), ("hidden", C.c_int),
                ("n_heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("vocab", C.c_int), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("qk_norm", C.c_int), ("qk_eps", C.c_float), ("res_alpha", C.c_float)]


class CkptInfoC(C.Structure):
    _fields_ = [("step", C.c_int), ("total_steps", C.c_int), ("seq_len", C.c_int),
                ("adam_t", C.c_int), ("lr", C.c_float), ("loss", C.c_float),
                ("cum_compile", C.c_double), ("cum_train", C.c_double),
                ("cum_wall", C.c_double), ("cum_steps", C.c_int), ("cum_batches", C.c_int),
                ("has_qk_norm", C.c_int)]


class GemmDescC(C.Structure):
    _fields_ = [("a", C.c_void_p), ("lda", C.c_longlong), ("a_mn", C.c_int),
                ("b", C.c_void_p), ("ldb", C.c_longlong), ("b_mn", C.c_int),
                ("M", C.c_int), ("N", C.c_int), ("K", C.c_int), ("epi", C.c_int),
                ("out", C.c_void_p), ("ld", C.c_longlong), ("alpha", C.c_float),
                ("aux0", C.c_void_p), ("aux1", C.c_void_p), ("aux_ld", C.c_longlong),
                ("bn", C.c_int), ("half_out", C.c_int)]


class AdamCfgC(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float),
                ("weight_decay", C.c_float), ("grad_clip", C.c_float), ("grad_scale", C.c_float)]


@dataclass(frozen=True)
class ModelConfig:
    """Run-time model description (the reference fixes it at compile time in
    ane-training/training/training_dynamic/models/*.h)."""
    n_layers: int
    dim: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-5
    theta: float = 10000.0
    qk_norm: bool = False
    qk_eps: float = 1e-6
    res_alpha: float = 1.0

    @property
    def q_dim(self):
        return self.heads * self.head_dim

    @property
    def kv_dim(self):
        return self.kv_heads * self.head_dim

    def to_c(self) -> ModelCfgC:
        return ModelCfgC(self.n_layers, self.dim, self.hidden, self.heads, self.kv_heads,
                         self.head_dim, self.vocab, self.eps, self.theta, int(self.qk_norm),
                         self.qk_eps, self.res_alpha)

    @classmethod
    def from_any(cls, c) -> "ModelConfig":
        names = ("n_layers", "dim", "hidden", "heads", "kv_heads", "head_dim", "vocab", "eps",
                 "theta", "qk_norm", "qk_eps", "res_alpha")
        return cls(**{n: getattr(c, n) for n in names})


STORIES110M = ModelConfig(12, 768, 2048, 12, 12, 64, 32000)
QWEN3_06B = ModelConfig(28, 1024, 3072, 16, 8, 128, 151936, eps=1e-6, theta=1e6, qk_norm=True)

_lib = None


def load_library(path: str = LIB_PATH) -> C.CDLL:
    """Load libne.so; raises if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} not built; run `python neural_engine_b200/build.py`")
    lib = C.CDLL(path)
    P, I, LL, F = C.c_void_p, C.c_int, C.c_longlong, C.c_float
    lib.ne_init.argtypes = [C.POINTER(P), C.POINTER(ModelCfgC), I]
    lib.ne_free.argtypes = [P]
    lib.ne_free.restype = None
    lib.ne_last_error.argtypes = [P]
    lib.ne_last_error.restype = C.c_char_p
    lib.ne_status_str.argtypes = [I]
    lib.ne_status_str.restype = C.c_char_p
    lib.ne_version.restype = C.c_char_p
    lib.ne_sync.argtypes = [P]
    lib.ne_get_cfg.argtypes = [P, C.POINTER(ModelCfgC)]
    lib.ne_set_layer_weights.argtypes = [P, I] + [P] * 11
    lib.ne_set_global_weights.argtypes = [P, P, P]
    lib.ne_load_ckpt_v4.argtypes = [P, C.c_char_p, C.POINTER(CkptInfoC)]
    lib.ne_save_ckpt_v4.argtypes = [P, C.c_char_p, C.POINTER(CkptInfoC)]
    lib.ne_embed_fwd.argtypes = [P, P]
    for n in ("ne_attn_fwd", "ne_ffn_fwd", "ne_ffn_bwd", "ne_attn_bwd"):
        getattr(lib, n).argtypes = [P, I]
    lib.ne_lmhead_ce_fwd_bwd.argtypes = [P, P]
    lib.ne_embed_bwd.argtypes = [P]
    lib.ne_rmsnorm_fwd.argtypes = [P, P, P, I, P]
    lib.ne_rmsnorm_bwd_add.argtypes = [P, P, P, P, I, P, P, P]
    lib.ne_comm_unique_id.argtypes = [P]
    lib.ne_comm_init.argtypes = [P, P, I, I]
    lib.ne_comm_set_reduce.argtypes = [P, I]
    lib.ne_comm_set_timeout.argtypes = [P, I]
    lib.ne_shard_range.argtypes = [C.c_longlong, I, I, C.POINTER(C.c_longlong),
                                   C.POINTER(C.c_longlong)]
    lib.ne_comm_set_sharding.argtypes = [P, I]
    lib.ne_train_gather_state.argtypes = [P, I]
    lib.ne_grad_allreduce_async.argtypes = [P]
    lib.ne_sdpa_fwd_device.argtypes = [P, P, P, P, I, I, P, P]
    lib.ne_train_set_vocab_map.argtypes = [P, P, I]
    lib.ne_kv_alloc.argtypes = [P, I, I]
    lib.ne_kv_reset.argtypes = [P]
    lib.ne_prefill.argtypes = [P, P, I, I, I, P, P]
    lib.ne_decode_step.argtypes = [P, P, I, I, P, P]
    lib.ne_generate.argtypes = [P, P, I, I, I, P]
    lib.ne_prefill_device.argtypes = [P, P, I, I, I, P]
    lib.ne_decode_loop_device.argtypes = [P, P, I, I, I, P]
    lib.ne_gemm_device.argtypes = [P, P, LL, I, P, LL, I, I, I, P, LL, F]
    lib.ne_gemm_device_ex.argtypes = [P, P, LL, I, P, LL, I, I, I, P, LL, F, I, I, LL,
                                      C.POINTER(C.c_int)]
    lib.ne_gemm_dw_owned.argtypes = [P, P, LL, I, P, LL, I, I, F, C.POINTER(P),
                                     C.POINTER(LL), I, I, LL]
    lib.ne_ckpt_probe.argtypes = [C.c_char_p, C.POINTER(ModelCfgC), C.POINTER(CkptInfoC)]
    lib.ne_fault_calls.argtypes = [C.c_char_p]
    lib.ne_fault_calls.restype = I
    lib.ne_decode_kernels_per_step.argtypes = [P, I]
    lib.ne_get_stream.argtypes = [P]
    lib.ne_get_stream.restype = P
    lib.ne_profile_decode_step.argtypes = [P, I, I, C.POINTER(C.c_float)]
    lib.ne_gemm.argtypes = [P, C.POINTER(GemmDescC)]
    lib.ne_train_grad_pool.argtypes = [P, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    lib.ne_train_alloc.argtypes = [P, I, I]
    lib.ne_train_set_masters.argtypes = [P, I] + [P] * 7
    lib.ne_train_sync_weights.argtypes = [P]
    lib.ne_train_zero_grads.argtypes = [P]
    lib.ne_train_fwd_bwd_device.argtypes = [P, P, P]
    lib.ne_train_fwd_bwd.argtypes = [P, P, C.POINTER(C.c_float)]
    lib.ne_train_fwd_bwd_timed.argtypes = [P, P, C.POINTER(C.c_float), C.POINTER(C.c_float)]
    lib.ne_train_value_ranges.argtypes = [P, C.POINTER(C.c_float)]
    lib.ne_train_grad_norm.argtypes = [P, F, C.POINTER(C.c_float)]
    lib.ne_adamw_step.argtypes = [P, C.POINTER(AdamCfgC), I, C.POINTER(C.c_float)]
    lib.ne_lr_schedule.argtypes = [I, F, I, I, F]
    lib.ne_lr_schedule.restype = F
    lib.ne_train_get_layer.argtypes = [P, I, I] + [P] * 11
    lib.ne_stream_read.argtypes = [P, C.c_longlong, P, P]
    _lib = lib
    return lib


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


class Engine:
    """One GPU context of libne.so (one model, its weights and KV cache)."""

    def __init__(self, cfg, device: int = 0):
        self.lib = load_library()
        self.cfg = ModelConfig.from_any(cfg)
        self._ctx = C.c_void_p()
        c = self.cfg.to_c()
        st = self.lib.ne_init(C.byref(self._ctx), C.byref(c), int(device))
        if st != NE_OK:
            raise NeError(st, f"ne_init failed ({self.lib.ne_status_str(st).decode()})")
        self.max_batch = 0
        self.max_seq = 0

    # -- plumbing
    def _check(self, st: int):
        if st != NE_OK:
            raise NeError(st, self.lib.ne_last_error(self._ctx).decode())

    def close(self):
        if self._ctx:
            self.lib.ne_free(self._ctx)
            self._ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._ctx

    def sync(self):
        self._check(self.lib.ne_sync(self._ctx))

    # -- weights
    def set_weights(self, layers, rms_final, embed, qk=None):
        f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
        for l, lw in enumerate(layers):
            t = [f32(lw[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3", "rms_att", "rms_ffn")]
            qn = kn = None
            if qk is not None:
                qn, kn = f32(qk[l][0]), f32(qk[l][1])
            self._check(self.lib.ne_set_layer_weights(self._ctx, l, *[_ptr(a) for a in t],
                                                      _ptr(qn), _ptr(kn)))
        self._check(self.lib.ne_set_global_weights(self._ctx, _ptr(f32(rms_final)), _ptr(f32(embed))))

    def load_checkpoint(self, path: str) -> dict:
        """Weights only; after train_alloc the full training state (resume)."""
        info = CkptInfoC()
        self._check(self.lib.ne_load_ckpt_v4(self._ctx, path.encode(), C.byref(info)))
        return {f: getattr(info, f) for f, _ in CkptInfoC._fields_}

    def save_checkpoint(self, path: str, **info):
        """Full training state in the v4 layout; info: CkptInfoC field values."""
        ci = CkptInfoC()
        for k, v in info.items():
            setattr(ci, k, v)
        self._check(self.lib.ne_save_ckpt_v4(self._ctx, path.encode(), C.byref(ci)))

    # -- per-layer entry points (one micro-step = embed_fwd, attn/ffn fwd per
    #    layer, lmhead_ce, ffn/attn bwd per layer in reverse, embed_bwd)
    def embed_fwd(self, d_tokens: int):
        self._check(self.lib.ne_embed_fwd(self._ctx, C.c_void_p(d_tokens)))

    def attn_fwd(self, layer: int):
        self._check(self.lib.ne_attn_fwd(self._ctx, int(layer)))

    def ffn_fwd(self, layer: int):
        self._check(self.lib.ne_ffn_fwd(self._ctx, int(layer)))

    def lmhead_ce_fwd_bwd(self, d_loss: int | None = None):
        self._check(self.lib.ne_lmhead_ce_fwd_bwd(self._ctx, C.c_void_p(d_loss) if d_loss else None))

    def ffn_bwd(self, layer: int):
        self._check(self.lib.ne_ffn_bwd(self._ctx, int(layer)))

    def attn_bwd(self, layer: int):
        self._check(self.lib.ne_attn_bwd(self._ctx, int(layer)))

    def embed_bwd(self):
        self._check(self.lib.ne_embed_bwd(self._ctx))

    def sdpa_fwd_device(self, d_q: int, d_k: int, d_v: int, B: int, S: int, d_out: int,
                        d_lse: int | None = None):
        self._check(self.lib.ne_sdpa_fwd_device(self._ctx, C.c_void_p(d_q), C.c_void_p(d_k),
                                                C.c_void_p(d_v), int(B), int(S), C.c_void_p(d_out),
                                                C.c_void_p(d_lse) if d_lse else None))

    # -- data-parallel gradient exchange (NCCL)
    @staticmethod
    def comm_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        st = load_library().ne_comm_unique_id(buf)
        if st != NE_OK:
            raise NeError(st, "ne_comm_unique_id")
        return buf.raw

    def comm_init(self, uid: bytes, rank: int, world: int):
        buf = C.create_string_buffer(bytes(uid), 128)
        self._check(self.lib.ne_comm_init(self._ctx, buf, int(rank), int(world)))

    def comm_set_timeout(self, timeout_ms: int):
        """Deadline of every wait on the gradient exchange (0 = default)."""
        self._check(self.lib.ne_comm_set_timeout(self._ctx, int(timeout_ms)))

    def comm_set_reduce(self, on: bool):
        self._check(self.lib.ne_comm_set_reduce(self._ctx, int(bool(on))))

    def comm_set_sharding(self, on: bool):
        """ZeRO-1: reduce-scatter, sharded AdamW, all-gathered compute copies."""
        self._check(self.lib.ne_comm_set_sharding(self._ctx, int(bool(on))))

    def gather_state(self, grads: bool = False):
        """Collective: whole masters and moments (or reduced gradients) on every rank."""
        self._check(self.lib.ne_train_gather_state(self._ctx, int(bool(grads))))

    def grad_allreduce(self):
        self._check(self.lib.ne_grad_allreduce_async(self._ctx))

    # -- token loop
    def kv_alloc(self, max_batch: int, max_seq: int):
        self._check(self.lib.ne_kv_alloc(self._ctx, int(max_batch), int(max_seq)))
        self.max_batch, self.max_seq = int(max_batch), int(max_seq)

    def kv_reset(self):
        """Clear the KV cache and decode state for a new set of sequences."""
        self._check(self.lib.ne_kv_reset(self._ctx))

    def prefill(self, tokens: np.ndarray, pos0: int = 0, return_logits: bool = False):
        tokens = np.ascontiguousarray(np.atleast_2d(tokens), dtype=np.int32)
        B, S = tokens.shape
        nxt = np.zeros(B, np.int32)
        lg = np.zeros((B, self.cfg.vocab), np.float32) if return_logits else None
        self._check(self.lib.ne_prefill(self._ctx, _ptr(tokens), B, S, int(pos0), _ptr(nxt), _ptr(lg)))
        return (nxt, lg) if return_logits else nxt

    def decode_step(self, tok: np.ndarray, pos: int, return_logits: bool = False):
        tok = np.ascontiguousarray(np.atleast_1d(tok), dtype=np.int32)
        B = tok.shape[0]
        nxt = np.zeros(B, np.int32)
        lg = np.zeros((B, self.cfg.vocab), np.float32) if return_logits else None
        self._check(self.lib.ne_decode_step(self._ctx, _ptr(tok), B, int(pos), _ptr(nxt), _ptr(lg)))
        return (nxt, lg) if return_logits else nxt

    def generate_greedy(self, prompt: np.ndarray, n_new: int) -> np.ndarray:
        prompt = np.ascontiguousarray(np.atleast_2d(prompt), dtype=np.int32)
        B, P = prompt.shape
        out = np.zeros((B, n_new), np.int32)
        self._check(self.lib.ne_generate(self._ctx, _ptr(prompt), B, P, int(n_new), _ptr(out)))
        return out

    # -- device-resident (pointers are device addresses, e.g. torch .data_ptr())
    def prefill_device(self, d_tokens: int, B: int, S: int, pos0: int, d_next: int):
        self._check(self.lib.ne_prefill_device(self._ctx, C.c_void_p(d_tokens), B, S, pos0,
                                               C.c_void_p(d_next)))

    def decode_loop_device(self, d_tok: int, B: int, pos0: int, n_steps: int, d_out: int | None):
        self._check(self.lib.ne_decode_loop_device(self._ctx, C.c_void_p(d_tok), B, pos0, n_steps,
                                                   C.c_void_p(d_out) if d_out else None))

    def gemm_device_ex(self, d_a: int, lda: int, M: int, d_b: int, ldb: int, N: int, K: int,
                       epi: int, d_out: int, ld: int, alpha: float = 1.0, bn: int = 0,
                       splits: int = 1, split_stride: int = 0) -> int:
        used = C.c_int(0)
        self._check(self.lib.ne_gemm_device_ex(self._ctx, C.c_void_p(d_a), lda, M, C.c_void_p(d_b),
                                               ldb, N, K, epi, C.c_void_p(d_out), ld, alpha, bn,
                                               splits, split_stride, C.byref(used)))
        return used.value

    def gemm_dw_owned(self, d_a: int, lda: int, M: int, d_b: int, ldb: int, N: int, K: int,
                      alpha: float, dst: list, bounds: list, rank: int, ld: int):
        """acc = A^T . B (both MN-major bf16), element m*ld + n added (x alpha) into
        dst[q] for the q whose [bounds[q], bounds[q+1]) holds it."""
        world = len(dst)
        d = (C.c_void_p * world)(*[C.c_void_p(x) for x in dst])
        b = (C.c_longlong * (world + 1))(*bounds)
        self._check(self.lib.ne_gemm_dw_owned(self._ctx, C.c_void_p(d_a), lda, M, C.c_void_p(d_b),
                                              ldb, N, K, alpha, d, b, world, rank, ld))

    def gemm(self, a: int, lda: int, M: int, b: int, ldb: int, N: int, K: int, epi: int, out: int,
             ld: int, alpha: float = 1.0, a_mn: int = 0, b_mn: int = 0, aux0: int = 0,
             aux1: int = 0, aux_ld: int = 0, bn: int = 0, half_out: int = 0):
        d = GemmDescC(a, lda, a_mn, b, ldb, b_mn, M, N, K, epi, out, ld, alpha, aux0 or None,
                      aux1 or None, aux_ld, bn, half_out)
        self._check(self.lib.ne_gemm(self._ctx, C.byref(d)))

    # -- training (train.m step loop)
    def train_alloc(self, B: int, S: int):
        self._check(self.lib.ne_train_alloc(self._ctx, int(B), int(S)))
        self.train_B, self.train_S = int(B), int(S)

    def train_set_masters(self, layers, embed):
        """Exact fp32 masters (the weights set earlier were stored as bf16)."""
        f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
        for l, lw in enumerate(layers):
            t = [f32(lw[k]) for k in ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3")]
            self._check(self.lib.ne_train_set_masters(self._ctx, l, *[_ptr(a) for a in t]))
        e = f32(embed)
        self._check(self.lib.ne_train_set_masters(self._ctx, -1, _ptr(e), *([None] * 6)))
        self._check(self.lib.ne_train_sync_weights(self._ctx))

    def train_fwd_bwd(self, tokens: np.ndarray) -> float:
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        assert tokens.shape == (self.train_B, self.train_S + 1), tokens.shape
        loss = C.c_float(0)
        self._check(self.lib.ne_train_fwd_bwd(self._ctx, _ptr(tokens), C.byref(loss)))
        return float(loss.value)

    TRAIN_PHASES = ("embed_fwd", "attn_fwd", "ffn_fwd", "classifier", "ffn_bwd", "attn_bwd",
                    "embed_bwd", "step")

    def train_fwd_bwd_timed(self, tokens: np.ndarray):
        """One micro-step (as train_fwd_bwd) with per-stage device times in ms;
        returns (loss, {phase: ms})."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        loss = C.c_float(0.0)
        ms = (C.c_float * 8)()
        self._check(self.lib.ne_train_fwd_bwd_timed(self._ctx, _ptr(tok), C.byref(loss), ms))
        return float(loss.value), dict(zip(self.TRAIN_PHASES, [float(v) for v in ms]))

    def value_ranges(self):
        """(x_min, x_max, dy_min, dy_max) of the last micro-step."""
        out = (C.c_float * 4)()
        self._check(self.lib.ne_train_value_ranges(self._ctx, out))
        return tuple(float(v) for v in out)

    def train_fwd_bwd_device(self, d_tokens: int, d_loss: int | None = None):
        self._check(self.lib.ne_train_fwd_bwd_device(self._ctx, C.c_void_p(d_tokens),
                                                     C.c_void_p(d_loss) if d_loss else None))

    def train_set_vocab_map(self, compact_to_full=None):
        """Classifier over the given vocabulary rows only (None: all rows)."""
        if compact_to_full is None:
            self._check(self.lib.ne_train_set_vocab_map(self._ctx, None, 0))
            return
        a = np.ascontiguousarray(compact_to_full, dtype=np.int32)
        self._check(self.lib.ne_train_set_vocab_map(self._ctx, _ptr(a), int(a.size)))

    def zero_grads(self):
        self._check(self.lib.ne_train_zero_grads(self._ctx))

    def grad_norm(self, grad_scale: float = 1.0) -> float:
        out = C.c_float(0)
        self._check(self.lib.ne_train_grad_norm(self._ctx, grad_scale, C.byref(out)))
        return float(out.value)

    def adamw_step(self, t: int, lr: float, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1,
                   grad_clip=1.0, grad_scale=1.0, return_norm: bool = True):
        """One optimizer step; returns the pre-clip gradient norm (waits for the
        step) or, with return_norm=False, None without waiting."""
        cfg = AdamCfgC(lr, beta1, beta2, eps, weight_decay, grad_clip, grad_scale)
        if not return_norm:
            self._check(self.lib.ne_adamw_step(self._ctx, C.byref(cfg), int(t), None))
            return None
        norm = C.c_float(0)
        self._check(self.lib.ne_adamw_step(self._ctx, C.byref(cfg), int(t), C.byref(norm)))
        return float(norm.value)

    def lr_schedule(self, step, max_lr, warmup, total, min_frac=0.1) -> float:
        return float(self.lib.ne_lr_schedule(step, max_lr, warmup, total, min_frac))

    def _train_tensors(self, which: int):
        c = self.cfg
        D, F, qd, kvd = c.dim, c.hidden, c.q_dim, c.kv_dim
        layers, qk = [], []
        for l in range(c.n_layers):
            t = {"Wq": np.zeros((qd, D), np.float32), "Wk": np.zeros((kvd, D), np.float32),
                 "Wv": np.zeros((kvd, D), np.float32), "Wo": np.zeros((D, qd), np.float32),
                 "W1": np.zeros((F, D), np.float32), "W2": np.zeros((D, F), np.float32),
                 "W3": np.zeros((F, D), np.float32), "rms_att": np.zeros(D, np.float32),
                 "rms_ffn": np.zeros(D, np.float32)}
            qn, kn = np.zeros(c.head_dim, np.float32), np.zeros(c.head_dim, np.float32)
            order = ("Wq", "Wk", "Wv", "Wo", "W1", "W2", "W3", "rms_att", "rms_ffn")
            self._check(self.lib.ne_train_get_layer(self._ctx, l, which, *[_ptr(t[k]) for k in order],
                                                    _ptr(qn), _ptr(kn)))
            layers.append(t)
            qk.append((qn, kn))
        rf = np.zeros(D, np.float32)
        emb = np.zeros((c.vocab, D), np.float32)
        self._check(self.lib.ne_train_get_layer(self._ctx, -1, which, _ptr(emb), None, None, None,
                                                None, None, None, _ptr(rf), None, None, None))
        return {"layers": layers, "rms_final": rf, "embed": emb,
                "qk": qk if c.qk_norm else None}

    def grad_pool(self):
        """(device pointer, float count) of the contiguous fp32 gradient pool."""
        p, n = C.c_void_p(), C.c_size_t()
        self._check(self.lib.ne_train_grad_pool(self._ctx, C.byref(p), C.byref(n)))
        return int(p.value), int(n.value)

    def grad_pool_tensor(self):
        """The gradient pool as a torch CUDA tensor view (no copy)."""
        import torch
        ptr, n = self.grad_pool()

        class _View:
            __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                        "version": 3, "strides": None}
        return torch.as_tensor(_View(), device=f"cuda:{torch.cuda.current_device()}")

    def get_grads(self) -> dict:
        return self._train_tensors(0)

    def get_adam(self, moment: str) -> dict:
        """Adam first ("m") or second ("v") moments, same structure as get_grads."""
        return self._train_tensors({"m": 2, "v": 3}[moment])

    def get_masters(self) -> dict:
        return self._train_tensors(1)

    @property
    def stream_ptr(self) -> int:
        """cudaStream_t of the context (wrap with torch.cuda.ExternalStream)."""
        return int(self.lib.ne_get_stream(self._ctx) or 0)

    def profile_decode_step(self, B: int, pos: int) -> dict:
        """Device ms per kernel group of one un-graphed decode step."""
        arr = (C.c_float * len(PROF_GROUPS))()
        self._check(self.lib.ne_profile_decode_step(self._ctx, B, pos, arr))
        return {g: float(arr[i]) for i, g in enumerate(PROF_GROUPS)}

    def kernels_per_step(self, B: int) -> int:
        return int(self.lib.ne_decode_kernels_per_step(self._ctx, B))

    def gemm_device(self, d_a: int, lda: int, M: int, d_b: int, ldb: int, N: int, K: int,
                    epi: int, d_out: int, ld: int, alpha: float = 1.0):
        self._check(self.lib.ne_gemm_device(self._ctx, C.c_void_p(d_a), lda, M, C.c_void_p(d_b), ldb,
                                            N, K, epi, C.c_void_p(d_out), ld, alpha))
