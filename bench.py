#!/usr/bin/env python3
"""Headline benchmark: Qwen3-0.6B KV-cached greedy decode on B200.

Workload: Qwen3-0.6B (28 layers, hidden 1024, GQA 16/8 x
128, per-head QK RMSNorm, SwiGLU 3072, vocab 151936 tied, theta 1e6, eps
1e-6), bf16 N(0, 0.02) weights, fp16 KV cache, 512-token uniform-random
prompts, 256 greedy tokens per sequence, 256 independent sequences per GPU.

  step   = one pass of 256 greedy decode steps over the batch, starting from
           the prefilled 512-token cache (each step is a CUDA-graph replay of
           the whole 28-layer forward + LM head + argmax; the argmax feeds the
           next step on the device).
  value  = generated tokens per second over all GPUs (device time, CUDA events
           on the library's stream, max over ranks).
  e2e    = the same metric through the public call a user makes
           (ne_generate: host prompt in, prefill, decode, host tokens out).

Multi-GPU: one process per GPU (torchrun); sequences are independent, so each
rank decodes its own 256 sequences with no collective on the data path
(weak scaling).  `--impl reference` times the CPU restatement of the
reference's numpy token loop on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-0.6B decode tokens/sec (greedy, 512-token prompt, 256 new tokens)"
TRAIN_METRIC = "Qwen3-0.6B training tokens/sec (fwd + bwd + AdamW, seq 256, batch 16 per GPU)"
UNIT = "tokens/s"

# Qwen3-0.6B sizes (models/qwen3_06b.h:6-16 of the reference) for the byte and
# FLOP models below: algorithmic counts, i.e. what the step must read, write or
# multiply at least once, independent of how the kernels tile it
L, D, F, HQ, HKV, HD, V = 28, 1024, 3072, 16, 8, 128, 151936
PARAMS = L * ((HQ * HD) * D + 2 * (HKV * HD) * D + D * (HQ * HD) + 3 * F * D + 2 * D) + D + V * D


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=256, help="sequences per GPU")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-train", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the prefill measurement (config 2)")
    ap.add_argument("--no-stories", action="store_true",
                    help="skip the Stories110M training measurement (config 3)")
    ap.add_argument("--gemm-square", type=int, default=0,
                    help="time one n x n x n bf16 product on the tcgen05 GEMM and exit "
                         "(profiling aid; not a bench number)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="skip everything but the prefill measurement (profiling runs)")
    ap.add_argument("--prefill-seqs", default="256,2048",
                    help="comma-separated prompt lengths of the prefill measurement")
    ap.add_argument("--prefill-batch", type=int, default=16,
                    help="sequences per GPU of the prefill measurement")
    ap.add_argument("--train-only", action="store_true",
                    help="skip the decode headline; print the training object alone "
                         "(profiling runs)")
    ap.add_argument("--profile-layers", type=int, default=0,
                    help="with --train-only: a Qwen3-0.6B-width model of this many layers "
                         "(per-launch kernel shapes unchanged, a few GB on the device) for "
                         "ncu captures of the layer kernels; not a bench number")
    ap.add_argument("--profile-vocab", type=int, default=0,
                    help="with --profile-layers: vocabulary of the profiling model")
    ap.add_argument("--train-model", choices=("qwen3_06b", "stories110m"), default="qwen3_06b",
                    help="with --train-only: which training leg (config 4 or config 3)")
    ap.add_argument("--train-batch", type=int, default=16, help="training sequences per GPU")
    ap.add_argument("--train-seq", type=int, default=256)
    ap.add_argument("--train-seqs", default="256,1024",
                    help="Qwen3 training sequence lengths measured after the decode (config 4)")
    ap.add_argument("--dp-mode", choices=("zero1", "allreduce"), default="zero1",
                    help="training with N > 1: ZeRO-1 (reduce-scatter, sharded AdamW, "
                         "all-gathered bf16 weights) or all-reduce with replicated AdamW")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def log(msg: str):
    """Progress on stderr (the JSON line stays the only stdout)."""
    rank = int(os.environ.get("RANK", 0))
    print(f"[bench rank {rank} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def allmax(x: float, world: int) -> float:
    """Max over ranks of a host float (the coordination group is gloo, CPU)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Sustained dense bf16 TFLOP/s (a kernel timed inside a long step)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def n_params(cfg) -> int:
    """Parameters of a model config (matrices, gains, embedding)."""
    d = cfg.dim
    per = cfg.q_dim * d + 2 * cfg.kv_dim * d + d * cfg.q_dim + 3 * cfg.hidden * d + 2 * d
    return cfg.n_layers * per + d + cfg.vocab * d


def train_flops_per_token(S: int, cfg=None) -> float:
    """3 x forward: 2 x params (596.0 M for Qwen3-0.6B, 109.5 M for Stories110M)
    + causal attention 2*L*Hq*hd*(S+1)."""
    if cfg is None:
        return 3.0 * (2.0 * PARAMS + 2.0 * L * HQ * HD * (S + 1))
    return 3.0 * (2.0 * n_params(cfg) + 2.0 * cfg.n_layers * cfg.q_dim * (S + 1))


def prefill_flops(B: int, S: int) -> float:
    """FLOPs one Qwen3-0.6B prefill of B x S tokens executes: the layer
    matrices for every token (2 x 440.4 M), causal attention counted once
    (2*L*Hq*hd*(S+1) per token) and the tied LM head for the last position of
    each sequence only (the token loop needs no other logits)."""
    mats = L * ((HQ * HD) * D + 2 * (HKV * HD) * D + D * (HQ * HD) + 3 * F * D)
    return B * S * (2.0 * mats + 2.0 * L * HQ * HD * (S + 1)) + B * 2.0 * V * D


# ----------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None
        self.th = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.th = threading.Thread(target=self._read, daemon=True)
        self.th.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            if self.th:
                self.th.join(timeout=5)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except (ValueError, IndexError):
                continue
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- byte model
def decode_step_bytes(B: int, T: int) -> float:
    """Algorithmic HBM bytes of one decode step for B sequences at context T:
    bf16 weights once (tied LM head reads the whole embedding) plus per
    sequence: K and V of T positions x 28 layers x 8 heads x 128 (fp16) and
    the new K/V row written.  The greedy loop's LM head keeps only each row's
    best (logit, id), so no logits reach HBM and none are counted."""
    weights = 2.0 * PARAMS
    kv_read = L * 2 * HKV * HD * 2 * T
    kv_write = L * 2 * HKV * HD * 2
    return weights + B * (kv_read + kv_write)


def attention_bytes(B: int, T: int) -> float:
    """Decode attention, one launch (one layer): K+V read for T positions,
    q (fp32) read, output (bf16) written."""
    return B * (HKV * T * HD * 2 * 2 + HQ * HD * 4 + HQ * HD * 2)


# DRAM bytes (read + write) per algorithmic byte of the decode attention: one
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of a launch at
# B 64, context 514 -- 139,092,736 B against 135,528,448 algorithmic bytes.
# Both grow in proportion to B x T, so the full launch's traffic is this ratio
# times its algorithmic bytes.
ATTN_TRAFFIC_RATIO = 139092736 / 135528448


def gemm_bytes(group: str, B: int) -> float:
    n_out, k = {"gemm_qkv": ((HQ + 2 * HKV) * HD, D), "gemm_wo": (D, HQ * HD),
                "gemm_w13": (2 * F, D), "gemm_w2": (D, F), "gemm_lm_head": (V, D)}[group]
    return n_out * k * 2 + B * k * 2 + B * n_out * 4


# ----------------------------------------------------------------- CPU baseline
def read_ceiling(nbytes: int, iters: int = 10) -> float:
    """Median time (ms) of ne_stream_read over nbytes: the read-only floor of
    the decode attention's data path for that many bytes in one launch."""
    import torch
    from neural_engine_b200 import runtime as rt
    lib = rt.load_library()
    nbytes = nbytes // 16 * 16
    buf = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    buf.fill_(1)
    sink = torch.zeros(2, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    ts = []
    for i in range(iters + 3):
        flush.fill_(i & 0xFF)   # larger than L2: every timed read comes from HBM
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        st = lib.ne_stream_read(buf.data_ptr(), nbytes, sink.data_ptr(), stream)
        b.record()
        if st != 0:
            raise RuntimeError(f"ne_stream_read failed ({st})")
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(a.elapsed_time(b))
    if int(sink[1].item()):
        raise RuntimeError("ne_stream_read: a bounded wait ran out")
    ts.sort()
    del buf, flush
    return ts[len(ts) // 2]


def cpu_decode_sample(layers, rms_final, embed, qk, B=256, steps=4, prompt=512, seed=5):
    """Time the oracle's numpy token loop (restated from the reference's
    tools/generate.py) on every host core: B sequences, KV cache pre-filled
    with `prompt` positions, `steps` greedy decode steps after one untimed
    step.  Returns (tokens/s, seconds, BLAS threads)."""
    from oracle import decode as od
    from oracle import model as om
    threads = host_threads()
    cfg = om.QWEN3_06B
    dec = od.Decoder(cfg, layers, rms_final, embed, qk, batch=B, max_seq=prompt + steps + 1)
    rng = np.random.default_rng(seed)
    # the attention's cost does not depend on the cached values: one random
    # [prompt, head_dim] block broadcast over layers, sequences and heads
    blk = rng.standard_normal((prompt, cfg.head_dim), dtype=np.float32)
    dec.k_cache[:, :, :, :prompt] = blk
    dec.v_cache[:, :, :, :prompt] = blk
    tok = rng.integers(0, cfg.vocab, size=(B, 1))
    dec.forward(tok, prompt, last_only=True)          # warm caches / BLAS threads
    t0 = time.perf_counter()
    for i in range(steps):
        lg = dec.forward(tok, prompt + 1 + i, last_only=True)
        tok = np.argmax(lg, -1)[:, None]
    dt = time.perf_counter() - t0
    return B * steps / dt, dt, threads


def host_weights(seed=0, cfg=None):
    """bf16-valued N(0, 0.02) weights generated on the GPU, returned as host
    fp32 (Qwen3-0.6B unless another model config is given)."""
    import torch
    import neural_engine_b200 as ne
    cfg = cfg or ne.QWEN3_06B
    g = torch.Generator(device="cuda").manual_seed(seed)
    d, f, qd, kd = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim

    def t(*shape):
        return (torch.randn(*shape, generator=g, device="cuda") * 0.02).to(torch.bfloat16) \
            .float().cpu().numpy()

    layers = []
    for _ in range(cfg.n_layers):
        layers.append({"Wq": t(qd, d), "Wk": t(kd, d), "Wv": t(kd, d),
                       "Wo": t(d, qd), "W1": t(f, d), "W2": t(d, f), "W3": t(f, d),
                       "rms_att": np.ones(d, np.float32), "rms_ffn": np.ones(d, np.float32)})
    embed = t(cfg.vocab, d)
    qk = ([(np.ones(cfg.head_dim, np.float32), np.ones(cfg.head_dim, np.float32))
           for _ in range(cfg.n_layers)] if cfg.qk_norm else None)
    return layers, np.ones(d, np.float32), embed, qk


# ----------------------------------------------------------------- reference arm
_THREAD_LIMITS = []


def host_threads() -> int:
    """Give the host's BLAS and torch every core, whatever OMP_NUM_THREADS the
    launcher set (torchrun sets 1 per process for nproc > 1), and return the
    BLAS thread count now in effect."""
    import threadpoolctl
    n = os.cpu_count() or 1
    _THREAD_LIMITS.append(threadpoolctl.threadpool_limits(limits=n))
    try:
        import torch
        torch.set_num_threads(n)
    except Exception:
        pass
    info = [i.get("num_threads", 0) for i in threadpoolctl.threadpool_info()
            if i.get("user_api") == "blas"]
    return max(info) if info else n


def run_reference(args):
    """The reference's CPU token loop (the oracle's numpy restatement of
    tools/generate.py:113-228) on the host cores, on this arm's workload: each
    step is one greedy decode step of all `--batch` sequences over a KV cache
    pre-filled with `--prompt` positions.  Rank 0 alone runs it."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    threads = host_threads()
    from oracle import decode as od
    from oracle import model as om
    cfg = om.QWEN3_06B
    layers, rf, emb, qk = om.init_weights(cfg, seed=0, bf16=True)
    B, P = args.batch, args.prompt
    dec = od.Decoder(cfg, layers, rf, emb, qk, batch=B, max_seq=P + 2)
    rng = np.random.default_rng(5)
    # the attention's cost does not depend on the cached values: one random
    # [P, head_dim] block broadcast over layers, sequences and heads
    blk = rng.standard_normal((P, cfg.head_dim), dtype=np.float32)
    dec.k_cache[:, :, :, :P] = blk
    dec.v_cache[:, :, :, :P] = blk
    tok = rng.integers(0, cfg.vocab, size=(B, 1))
    ts = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        lg = dec.forward(tok, P, last_only=True)
        tok = np.argmax(lg, -1)[:, None]
        if i >= args.warmup:
            ts.append(time.perf_counter() - t0)
    sec = statistics.mean(ts)
    value = B / sec
    sample = (f"oracle numpy port of tools/generate.py, Qwen3-0.6B, {B} sequences, one greedy "
              f"decode step per timed step at context {P} ({threads} BLAS threads)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sec,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "qwen3_06b_decode", "model": "Qwen3-0.6B",
                       "batch_per_gpu": B, "prompt_len": P, "gen_tokens": args.gen,
                       "kv_cache": "fp32 (generate.py:128-129)"},
            "extrapolated_from": (f"B={B} x 1 greedy step per timed step at context {P}; the "
                                  f"GPU arm decodes {args.gen} steps at contexts {P}-"
                                  f"{P + args.gen - 1}"),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- training
def profile_cfg(args):
    """Qwen3-0.6B layer width with fewer layers / a smaller vocabulary (ncu
    captures of the per-layer training kernels on a small case)."""
    import dataclasses
    import neural_engine_b200 as ne
    return dataclasses.replace(ne.QWEN3_06B, n_layers=args.profile_layers,
                               vocab=args.profile_vocab or ne.QWEN3_06B.vocab)


def cpu_train_sample(layers, rf, emb, qk, S=256, reps=3, model="qwen3_06b"):
    """torch-CPU float32 fwd + bwd of one sequence of S tokens (the oracle's
    restatement of the training forward), all host cores.  Returns tokens/s."""
    import torch
    from oracle import model as om
    from oracle import train as ot
    threads = host_threads()
    cfg = om.PRESETS[model]
    tok = np.random.default_rng(7).integers(0, cfg.vocab, size=(1, S + 1))
    t0 = time.perf_counter()
    for _ in range(reps):
        ot.loss_and_grads(cfg, layers, rf, emb, qk, tok, dtype="float32")
    dt = time.perf_counter() - t0
    return reps * S / dt, dt, threads


def dp_label(world, mode):
    """How the training step's gradients are exchanged at this world size."""
    if world == 1:
        return "dp1 (one GPU: no gradient exchange)"
    if mode != "zero1":
        return f"dp{world} (per-layer NCCL all-reduce buckets overlapped with the backward)"
    if os.environ.get("NE_COMM_PX", "1") == "0":
        return (f"dp{world} ZeRO-1 (per-layer NCCL reduce-scatter buckets overlapped with the "
                "backward, sharded AdamW, bf16 weight all-gather)")
    if os.environ.get("NE_PX_FUSED_DW", "0") != "1":
        return (f"dp{world} ZeRO-1 over NVLink peer memory (the library's per-layer "
                "reduce-scatter kernels overlapped with the backward, sharded AdamW, bf16 "
                "weight all-gather overlapped with the next forward; no NCCL on the step)")
    return (f"dp{world} ZeRO-1 over NVLink peer memory (the dW GEMM epilogues add into the "
            "owning ranks' gradients, the gains are reduce-scattered per layer, sharded AdamW, "
            "bf16 weight all-gather overlapped with the next forward; no NCCL on the step)")


def run_train(args, rank, local, world, layers, rf, emb, qk, barrier, model="qwen3_06b",
              B=None, S=None):
    """Data-parallel training steps: BASELINE config 4 (Qwen3-0.6B, S 256, B 16
    per GPU; token ids from seed 3) or config 3 (Stories110M, S 256, B 32 per
    GPU; seed 2)."""
    import torch
    import torch.distributed as dist
    import neural_engine_b200 as ne
    stories = model == "stories110m"
    cfg = ne.STORIES110M if stories else ne.QWEN3_06B
    if not stories and args.profile_layers > 0:
        cfg = profile_cfg(args)
    B = B or args.train_batch
    S = S or args.train_seq
    eng = ne.Engine(cfg, device=local)
    eng.set_weights(layers, rf, emb, qk)
    eng.train_alloc(B, S)
    log(f"train {model} S={S}: allocated")
    stream = torch.cuda.ExternalStream(eng.stream_ptr)
    gen = torch.Generator(device="cuda").manual_seed((2000 if stories else 3000) + rank)
    tok = torch.randint(0, cfg.vocab, (B, S + 1), generator=gen, device="cuda", dtype=torch.int32)
    if world > 1:
        # the library's own exchange: one NCCL bucket per layer, issued as the
        # backward finishes the layer, on its comm stream
        uid = [ne.Engine.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        eng.comm_init(uid[0], rank, world)
        if args.dp_mode == "zero1":
            eng.comm_set_sharding(True)
    tstep = [0]

    def step():
        eng.train_fwd_bwd_device(tok.data_ptr())
        tstep[0] += 1
        eng.adamw_step(tstep[0], 3e-4, grad_scale=1.0 / world, return_norm=False)

    for _ in range(args.warmup):
        step()
    eng.sync()        # bounded by the exchange's deadline: a stuck exchange raises
    log(f"train {model} S={S}: warm")
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    eng.sync()
    ev1.synchronize()
    clk = clocks.stop()
    t_ms = allmax(ev0.elapsed_time(ev1), world)
    ms_step = t_ms / args.steps
    log(f"train {model} S={S}: {ms_step:.3f} ms/step")
    value = world * B * S * args.steps / (t_ms / 1000.0)
    peak, kind = tensor_peak()
    fpt = train_flops_per_token(S, cfg)
    ach = fpt * B * S / (ms_step / 1000.0) / 1e12
    # e2e through the host-buffer call: tokens H2D, fwd+bwd, loss D2H, AdamW
    h_tok = tok.cpu().numpy()
    barrier()
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        eng.train_fwd_bwd(h_tok)
        tstep[0] += 1
        eng.adamw_step(tstep[0], 3e-4, grad_scale=1.0 / world, return_norm=False)
    eng.sync()   # the last AdamW is asynchronous: the timed region ends when it has run
    te = allmax((time.perf_counter() - t0) / reps, world)
    eng.close()
    log(f"train {model} S={S}: e2e done")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and cfg.n_layers in (12, 28):
        v, dt, thr = cpu_train_sample(layers, rf, emb, qk, S=S, model=model,
                                      reps=3 if S <= 256 else 1)
        cpu = {"value": round(v, 3), "unit": UNIT, "cores": thr, "kind": "port",
               "sample": f"torch-CPU float32 fwd+bwd of the oracle's "
                         f"{'Stories110M' if stories else 'Qwen3-0.6B'} forward, "
                         f"{3 if S <= 256 else 1} x 1 x {S} tokens ({dt:.1f} s)"}
    metric = (f"Stories110M training tokens/sec (fwd + bwd + AdamW, seq {S}, batch {B} per GPU)"
              if stories else
              f"Qwen3-0.6B training tokens/sec (fwd + bwd + AdamW, seq {S}, batch {B} per GPU)")
    return {"metric": metric, "value": round(value, 1), "unit": UNIT,
            "ms_per_step": round(ms_step, 3), "steps": args.steps, "warmup": args.warmup,
            "scaling": "weak", "dtype": "bf16",
            "config": {"workload": (f"{model}_train" if cfg.n_layers in (12, 28) else
                                    f"profiling case: {cfg.n_layers} layers, vocab {cfg.vocab}"),
                       "batch_per_gpu": B, "seq_len": S,
                       "global_batch": B * world, "optimizer": "AdamW lr 3e-4 b 0.9/0.95 "
                       "eps 1e-8 wd 0.1 clip 1.0", "masters": "fp32",
                       "parallelism": dp_label(world, args.dp_mode)},
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(ach / peak, 4), "peak_kind": kind,
                         "flops_per_token": fpt, "scope": "whole step"},
            "clocks": clk,
            "e2e": {"value": round(world * B * S / te, 1), "unit": UNIT,
                    "h2d_bytes_per_step": B * (S + 1) * 4, "d2h_bytes_per_step": 8},
            "cpu_baseline": cpu}


# ----------------------------------------------------------------- prefill
def run_prefill(args, rank, local, world, layers, rf, emb, qk):
    """Qwen3-0.6B prefill -- the token loop's causal pass
    over the prompt that fills the fp16 KV cache (ne_prefill_device) -- at B 16
    per GPU, S 256 and 2048, uniform-random token ids.  Device time of whole
    calls on the library's stream (CUDA events, max over ranks); the KV cache
    and activations (>= 470 MB per call) exceed L2."""
    import torch
    import torch.distributed as dist
    import neural_engine_b200 as ne
    cfg = ne.QWEN3_06B
    B, reps = args.prefill_batch, 5
    seqs = tuple(int(x) for x in args.prefill_seqs.split(","))
    peak, kind = tensor_peak()
    runs = {}
    eng = ne.Engine(cfg, device=local)
    try:
        eng.set_weights(layers, rf, emb, qk)
        eng.kv_alloc(B, max(seqs))
        stream = torch.cuda.ExternalStream(eng.stream_ptr)
        nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
        for S in seqs:
            gen = torch.Generator(device="cuda").manual_seed(4000 + 7 * rank + S)
            tok = torch.randint(0, cfg.vocab, (B, S), generator=gen, device="cuda",
                                dtype=torch.int32)
            torch.cuda.synchronize()
            for _ in range(3):
                eng.prefill_device(tok.data_ptr(), B, S, 0, nxt.data_ptr())
            eng.sync()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            for _ in range(reps):
                eng.prefill_device(tok.data_ptr(), B, S, 0, nxt.data_ptr())
            ev1.record(stream)
            eng.sync()
            ev1.synchronize()
            ms = allmax(ev0.elapsed_time(ev1) / reps, world)
            fl = prefill_flops(B, S)
            ach = fl / (ms / 1000.0) / 1e12
            runs[f"seq{S}"] = {"seq_len": S, "ms_per_call": round(ms, 3),
                               "tokens_per_s": round(world * B * S / (ms / 1000.0), 1),
                               "flops_per_call": fl, "achieved_tflops": round(ach, 1),
                               "frac": round(ach / peak, 4)}
    finally:
        eng.close()
    return {"metric": "Qwen3-0.6B prefill tokens/sec (causal pass filling the fp16 KV cache)",
            "unit": UNIT, "workload": "qwen3_06b_prefill", "batch_per_gpu": B,
            "global_batch": B * world, "calls_timed": reps,
            "roofline": {"bound": "tensor", "peak": peak, "unit": "TFLOP/s", "peak_kind": kind,
                         "flops": "layer matrices for every token + causal attention once + "
                                  "LM head on the last position"},
            "runs": runs}


# ----------------------------------------------------------------- decode legs
def run_decode(args, eng, prompt, B, P, G, rank, world, barrier, with_clocks=True):
    """Timed greedy decode of B sequences (config 1): `--steps` passes of G
    CUDA-graph decode steps from the prefilled P-position cache, after
    `--warmup` passes; device time on the library's stream, max over ranks.
    Returns the measurements and the per-kernel-group times of one step at the
    mean context length."""
    import torch
    first = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros(G * B, dtype=torch.int32, device="cuda")
    eng.prefill_device(prompt.data_ptr(), B, P, 0, first.data_ptr())
    eng.sync()
    stream = torch.cuda.ExternalStream(eng.stream_ptr)
    for _ in range(args.warmup):
        eng.decode_loop_device(first.data_ptr(), B, P, G, out.data_ptr())
    eng.sync()
    barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", 0))) if with_clocks else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        eng.decode_loop_device(first.data_ptr(), B, P, G, out.data_ptr())
    ev1.record(stream)
    eng.sync()
    ev1.synchronize()
    clk = clocks.stop() if clocks else None
    barrier()
    t_ms = allmax(ev0.elapsed_time(ev1), world)
    ms_step = t_ms / args.steps
    value = world * B * G * args.steps / (t_ms / 1000.0)
    T_mid = P + G // 2
    groups = {}
    for _ in range(3):
        for k, v in eng.profile_decode_step(B, T_mid).items():
            groups[k] = groups.get(k, 0.0) + v / 3
    peak, _ = peaks()
    step_bytes = sum(decode_step_bytes(B, P + i) for i in range(G)) / G
    whole = {"bytes_per_decode_step": step_bytes,
             "achieved_gbs": round(step_bytes / (ms_step / G / 1000.0) / 1e9, 1),
             "frac_of_peak": round(step_bytes / (ms_step / G / 1000.0) / 1e9 / peak, 4)}
    return {"value": value, "ms_per_step": ms_step, "ms_per_decode_step": ms_step / G,
            "groups": groups, "whole": whole, "clocks": clk, "first": first, "T_mid": T_mid}


# ----------------------------------------------------------------- our arm
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist
    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        # coordination only (barriers, max over ranks, the NCCL id): a CPU
        # group with a timeout, so no collective of this script can hold a GPU;
        # the gradient exchange is the library's own communicator
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier()

    import neural_engine_b200 as ne
    cfg = ne.QWEN3_06B
    B, P, G = args.batch, args.prompt, args.gen
    if args.profile_layers > 0 and not args.train_only:
        raise SystemExit("--profile-layers needs --train-only")
    layers, rf, emb, qk = host_weights(seed=0, cfg=profile_cfg(args) if args.profile_layers > 0
                                       else None)
    if args.gemm_square > 0:
        n = args.gemm_square
        eng = ne.Engine(ne.ModelConfig(1, 128, 256, 2, 2, 64, 256), device=local)
        g = torch.Generator(device="cuda").manual_seed(9)
        a = (torch.randn(n, n, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        b = (torch.randn(n, n, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        c = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
        stream = torch.cuda.ExternalStream(eng.stream_ptr)
        ts = []
        for i in range(8):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            eng.gemm_device(a.data_ptr(), n, n, b.data_ptr(), n, n, n, 2, c.data_ptr(), n)
            e1.record(stream)
            eng.sync()
            if i >= 3:
                ts.append(e0.elapsed_time(e1))
        ms = statistics.median(ts)
        eng.close()
        print(json.dumps({"gemm": f"{n}x{n}x{n} bf16 -> bf16", "ms": round(ms, 4),
                          "tflops": round(2.0 * n ** 3 / (ms / 1000.0) / 1e12, 1)}), flush=True)
        return
    if args.prefill_only:
        pf = run_prefill(args, rank, local, world, layers, rf, emb, qk)
        if rank == 0:
            print(json.dumps(dict(pf, n_gpus=world, data="synthetic")), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.train_only:
        if args.train_model == "stories110m":
            s_w = host_weights(seed=0, cfg=ne.STORIES110M)
            train = run_train(args, rank, local, world, *s_w, barrier, model="stories110m",
                              B=32, S=256)
        else:
            train = run_train(args, rank, local, world, layers, rf, emb, qk, barrier)
        if rank == 0:
            print(json.dumps(dict(train, n_gpus=world, higher_is_better=True, vs_baseline=None,
                                  data="synthetic")), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    log("decode: weights ready")
    eng = ne.Engine(cfg, device=local)
    eng.set_weights(layers, rf, emb, qk)
    eng.kv_alloc(B, P + G)
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    prompt = torch.randint(0, cfg.vocab, (B, P), generator=gen, device="cuda", dtype=torch.int32)
    torch.cuda.synchronize()
    d = run_decode(args, eng, prompt, B, P, G, rank, world, barrier)
    ms_step, value, groups, whole, clk = (d["ms_per_step"], d["value"], d["groups"], d["whole"],
                                          d["clocks"])
    log(f"decode B={B}: {value:.0f} tokens/s")
    T_mid = d["T_mid"]
    dom = max(groups, key=groups.get)
    dom_ms = groups[dom] / (L if dom in ("gemm_qkv", "qkv_post", "decode_attention", "gemm_wo",
                                         "gemm_w13", "swiglu", "gemm_w2") else 1)
    if dom == "decode_attention":
        dom_bytes = attention_bytes(B, T_mid + 1)
    elif dom.startswith("gemm"):
        dom_bytes = gemm_bytes(dom, B)
    else:
        dom_bytes = None
    peak, peak_kind = peaks()
    roof = None
    if dom_bytes is not None:
        ach = dom_bytes / (dom_ms / 1000.0) / 1e9
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": None,
                "peak_kind": peak_kind, "bytes_per_launch": dom_bytes,
                "ms_per_launch": round(dom_ms, 4)}
    if roof is not None and dom == "decode_attention":
        roof["traffic"] = round(ATTN_TRAFFIC_RATIO * dom_bytes)
        roof["traffic_source"] = ("ncu DRAM read + write bytes of one launch at B 64, context "
                                  "514, scaled by the algorithmic bytes (B x T)")
    if roof is not None and dom == "decode_attention" and rank == 0:
        # the same bytes through the same data path with no arithmetic
        rc_ms = read_ceiling(int(dom_bytes))
        rc_gbs = dom_bytes / (rc_ms / 1000.0) / 1e9
        roof["read_floor"] = {"kernel": "ne_stream_read", "ms": round(rc_ms, 4),
                              "gbs": round(rc_gbs, 1), "frac_of_peak": round(rc_gbs / peak, 4)}
        roof["frac_of_read_floor"] = round(rc_ms / dom_ms, 4)

    # end to end through the public API: host prompt -> ne_generate -> host tokens
    e2e = None
    if not args.no_e2e:
        h_prompt = prompt.cpu().numpy()
        eng.generate_greedy(h_prompt, G)        # warm (graph already captured)
        barrier()
        reps = 2
        t0 = time.perf_counter()
        for _ in range(reps):
            eng.generate_greedy(h_prompt, G)
        te = allmax((time.perf_counter() - t0) / reps, world)
        e2e = {"value": world * B * G / te, "unit": UNIT, "h2d_bytes_per_step": B * P * 4,
               "d2h_bytes_per_step": B * G * 4, "s_per_call": round(te, 4),
               "includes": "H2D prompt, prefill of 512 positions, 255 decode steps, D2H tokens"}

    # the other batch sizes of config 1 (B = 1 runs as one replica per GPU)
    decode_batches = {}
    for Bx in (1, 32):
        if Bx >= B:
            continue
        dx = run_decode(args, eng, prompt[:Bx], Bx, P, G, rank, world, barrier,
                        with_clocks=False)
        decode_batches[f"b{Bx}"] = {
            "batch_per_gpu": Bx, "global_batch": Bx * world,
            "value": round(dx["value"], 1), "unit": UNIT,
            "ms_per_step": round(dx["ms_per_step"], 3),
            "ms_per_decode_step": round(dx["ms_per_decode_step"], 4),
            "roofline_whole_step": dx["whole"],
            "kernel_groups_ms_per_step": {k: round(v, 4) for k, v in dx["groups"].items()},
            "parallelism": ("replicas (one sequence per GPU)" if Bx == 1 else
                            f"sequence-sharded x{world} (no collective)")}
        log(f"decode B={Bx}: {dx['value']:.1f} tokens/s")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        steps_c = 4
        v, dt, thr = cpu_decode_sample(layers, rf, emb, qk, B=B, steps=steps_c, prompt=P)
        cpu = {"value": round(v, 3), "unit": UNIT, "cores": thr, "kind": "port",
               "sample": (f"oracle numpy port of tools/generate.py on all host cores, Qwen3-0.6B,"
                          f" {B} sequences, KV pre-filled with {P} positions, {steps_c} greedy "
                          f"steps ({dt:.1f} s)")}

    kps = eng.kernels_per_step(B)
    eng.close()

    # the other legs: a failure is recorded in the line instead of ending the
    # run; after one, legs with collectives are skipped (ranks may disagree on
    # where they stopped)
    errors = {}

    def leg(name, fn):
        if errors and world > 1:
            return {"skipped": "an earlier leg failed on this rank"}
        log(f"{name}: start")
        try:
            r = fn()
            log(f"{name}: done")
            return r
        except Exception as ex:          # noqa: BLE001 -- recorded in the JSON line
            errors[name] = f"{type(ex).__name__}: {ex}"
            log(f"{name}: FAILED {errors[name]}")
            return {"error": errors[name]}

    prefill = None
    if not args.no_prefill:
        prefill = leg("prefill", lambda: run_prefill(args, rank, local, world, layers, rf, emb,
                                                     qk))
    train = train_s1024 = train_stories = None
    if not args.no_train:
        tseqs = [int(x) for x in args.train_seqs.split(",") if x]
        if 256 in tseqs:
            train = leg("train", lambda: run_train(args, rank, local, world, layers, rf, emb, qk,
                                                   barrier))
        if 1024 in tseqs:
            train_s1024 = leg("train_s1024", lambda: run_train(args, rank, local, world, layers,
                                                               rf, emb, qk, barrier, S=1024))
        if not args.no_stories:
            import neural_engine_b200 as ne_mod
            s_w = host_weights(seed=0, cfg=ne_mod.STORIES110M)
            train_stories = leg("train_stories110m",
                                lambda: run_train(args, rank, local, world, *s_w, barrier,
                                                  model="stories110m", B=32, S=256))
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "qwen3_06b_decode", "model": "Qwen3-0.6B",
                           "batch_per_gpu": B, "global_batch": B * world, "prompt_len": P,
                           "gen_tokens": G, "kv_cache": "fp16", "weights": "bf16 N(0,0.02)",
                           "parallelism": f"sequence-sharded x{world} (no collective)",
                           "l2": "inputs larger than L2: 1.19 GB weights + KV cache re-read "
                                 "every decode step"},
                "ms_per_decode_step": round(ms_step / G, 4),
                "roofline": roof, "roofline_whole_step": whole,
                "kernel_groups_ms_per_step": {k: round(v, 4) for k, v in groups.items()},
                "clocks": clk, "e2e": e2e, "cpu_baseline": cpu,
                "gpu_launches": kps * G * args.steps, "kernels_per_decode_step": kps,
                "decode_batches": decode_batches,
                "prefill": prefill, "train": train, "train_s1024": train_s1024,
                "train_stories110m": train_stories}
        if errors:
            line["errors"] = errors
        print(json.dumps(line), flush=True)
    if world > 1:
        try:
            dist.destroy_process_group()
        except Exception:                # noqa: BLE001 -- teardown after a failed leg
            pass


if __name__ == "__main__":
    main()
