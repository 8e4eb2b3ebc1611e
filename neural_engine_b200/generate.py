"""Drop-in for the reference's numpy token loop, running on libne.so.

Mirrors ane-training/training/training_dynamic/tools/generate.py:
  * ``read_checkpoint(path)`` -> (info, layers, rms_final, embed) like
    generate.py:18-78, but reading the GQA fields from their real header
    slots (config.h:89; generate.py:28 reads cum_steps/cum_batches/adam_t);
  * ``generate(info, layers, rms_final, embed, tokenizer, prompt_tokens,
    max_tokens, temperature, top_p)`` with the same arguments and return value
    as generate.py:113-228.  The forward pass runs in the CUDA kernels;
    greedy decoding (temperature < 1e-6) stays entirely on the device, and
    sampling pulls the step's logits to the host and applies generate.py's
    temperature / top-p rule (generate.py:201-215) with numpy's global RNG;
  * ``main()``: the command line of generate.py:231-274
    (``python -m neural_engine_b200.generate ckpt.bin -m <tokenizer> -p ...``).
Extra ``info`` keys select the Qwen3 numerics the reference cannot express:
``eps``, ``theta``, ``qk_norm`` (with ``q_norm`` / ``k_norm`` gains lists),
``qk_eps``, ``res_alpha``.
"""
from __future__ import annotations

import argparse
import struct
import sys

import numpy as np

from .runtime import Engine, ModelConfig

_HDR = "<iiiiiiiiiiffdddiiiiii"


def read_checkpoint(path: str):
    with open(path, "rb") as f:
        h = struct.unpack(_HDR, f.read(struct.calcsize(_HDR)))
        magic, version, step = h[0], h[1], h[2]
        n_layers, vocab, dim, hidden, heads, seq = h[4:10]
        loss = h[11]
        kv_heads, hd, q_dim = h[18:21]
        if magic != 0x424C5A54:
            raise ValueError(f"Bad magic: {magic:#x}")
        if version != 4:
            raise ValueError(f"Unsupported version: {version}")
        kv_dim = kv_heads * hd
        info = {"step": step, "loss": loss, "dim": dim, "hidden": hidden, "heads": heads,
                "kv_heads": kv_heads, "hd": hd, "q_dim": q_dim, "kv_dim": kv_dim,
                "gqa_ratio": heads // kv_heads, "n_layers": n_layers, "vocab": vocab}
        shapes = [("Wq", (q_dim, dim)), ("Wk", (kv_dim, dim)), ("Wv", (kv_dim, dim)),
                  ("Wo", (dim, q_dim)), ("W1", (hidden, dim)), ("W2", (dim, hidden)),
                  ("W3", (hidden, dim)), ("rms_att", (dim,)), ("rms_ffn", (dim,))]
        layers = []
        for _ in range(n_layers):
            lw = {}
            for name, shp in shapes:
                n = int(np.prod(shp))
                lw[name] = np.frombuffer(f.read(4 * n), np.float32).reshape(shp).copy()
            for _, shp in shapes:                       # Adam m, v
                f.seek(8 * int(np.prod(shp)), 1)
            layers.append(lw)
        rms_final = np.frombuffer(f.read(4 * dim), np.float32).copy()
        f.seek(8 * dim, 1)
        embed = np.frombuffer(f.read(4 * vocab * dim), np.float32).reshape(vocab, dim).copy()
        f.seek(8 * vocab * dim, 1)
        tail = f.read(4)
        if tail == b"QKN1":
            nl, hd2 = struct.unpack("<ii", f.read(8))
            qn, kn = [], []
            for _ in range(nl):
                qn.append(np.frombuffer(f.read(4 * hd2), np.float32).copy())
                kn.append(np.frombuffer(f.read(4 * hd2), np.float32).copy())
                f.seek(16 * hd2, 1)
            info["qk_norm"] = True
            info["q_norm"], info["k_norm"] = qn, kn
    return info, layers, rms_final, embed


def config_from_info(info: dict) -> ModelConfig:
    return ModelConfig(n_layers=info["n_layers"], dim=info["dim"], hidden=info["hidden"],
                       heads=info["heads"], kv_heads=info["kv_heads"], head_dim=info["hd"],
                       vocab=info["vocab"], eps=info.get("eps", 1e-5),
                       theta=info.get("theta", 10000.0), qk_norm=bool(info.get("qk_norm", False)),
                       qk_eps=info.get("qk_eps", 1e-6), res_alpha=info.get("res_alpha", 1.0))


def _softmax(x):
    x = x - np.max(x)
    e = np.exp(x)
    return e / np.sum(e)


def sample_probs(lg, top_p: float, vocab: int):
    """The sampling distribution of generate.py:203-213 from tempered logits
    ``lg`` (logits / temperature): softmax, then, for top_p < 1, the smallest
    set of most probable tokens whose cumulative probability reaches top_p,
    renormalised in float32."""
    probs = _softmax(lg)
    if top_p < 1.0:
        sorted_idx = np.argsort(-probs)
        cum = np.cumsum(probs[sorted_idx])
        cutoff = np.searchsorted(cum, top_p) + 1
        mask = np.zeros(vocab, dtype=np.float32)
        mask[sorted_idx[:cutoff]] = probs[sorted_idx[:cutoff]]
        mask /= mask.sum()
        probs = mask
    return probs


def sample_token(logits, temperature: float, top_p: float, vocab: int) -> int:
    """One sampled token (generate.py:202-215) drawn with numpy's global RNG."""
    return int(np.random.choice(vocab, p=sample_probs(logits / temperature, top_p, vocab)))


def generate(info, layers, rms_final, embed, tokenizer, prompt_tokens, max_tokens, temperature,
             top_p, engine: Engine | None = None):
    """Autoregressive generation with KV cache (generate.py:113-228)."""
    cfg = config_from_info(info)
    prompt = np.asarray(list(prompt_tokens), np.int32)
    if engine is None:
        engine = Engine(cfg)
        qk = None
        if cfg.qk_norm:
            qk = list(zip(info["q_norm"], info["k_norm"]))
        engine.set_weights(layers, rms_final, embed, qk)
    max_seq = len(prompt) + max_tokens
    if engine.max_batch < 1 or engine.max_seq < max_seq:
        engine.kv_alloc(1, max_seq)
    generated = []
    greedy = temperature < 1e-6
    if greedy:
        nxt, logits = engine.prefill(prompt[None], 0), None
    else:
        nxt, logits = engine.prefill(prompt[None], 0, return_logits=True)
    pos = len(prompt)
    for i in range(max_tokens):
        if greedy:
            tok = int(nxt[0])                                         # generate.py:200
        else:
            tok = sample_token(logits[0], temperature, top_p, cfg.vocab)  # :202-215
        generated.append(tok)
        print(tokenizer.decode([tok]), end="", flush=True)            # :220-221
        if tok == tokenizer.eos_token_id or i == max_tokens - 1:      # :224
            break
        if greedy:
            nxt = engine.decode_step(np.array([tok], np.int32), pos)
        else:
            nxt, logits = engine.decode_step(np.array([tok], np.int32), pos, return_logits=True)
        pos += 1
    print()
    return generated


class _IdTokenizer:
    """Stand-in tokenizer for ``--prompt-ids``: prints token ids, no EOS."""
    eos_token_id = None

    @staticmethod
    def decode(ids):
        return "".join(f"{int(i)} " for i in ids)


def main(argv=None):
    """Command line of generate.py:231-274 (same arguments and output), on
    libne.so.  ``--prompt-ids`` (comma-separated token ids) stands in for a
    text prompt where no tokenizer is at hand; ``--model`` is then not needed."""
    parser = argparse.ArgumentParser(description="Generate text from a v4 checkpoint (libne.so)")
    parser.add_argument("checkpoint", help="Path to the v4 checkpoint (.bin)")
    parser.add_argument("--model", "-m", default=None,
                        help="HF model ID for tokenizer (e.g. Qwen/Qwen3-0.6B)")
    parser.add_argument("--prompt", "-p", default="Once upon a time",
                        help="Text prompt (default: 'Once upon a time')")
    parser.add_argument("--prompt-ids", default=None,
                        help="comma-separated prompt token ids instead of --prompt")
    parser.add_argument("--tokens", "-n", type=int, default=100,
                        help="Max tokens to generate (default: 100)")
    parser.add_argument("--temp", "-t", type=float, default=0.8,
                        help="Sampling temperature (default: 0.8, 0=greedy)")
    parser.add_argument("--top-p", type=float, default=0.9,
                        help="Top-p nucleus sampling (default: 0.9)")
    parser.add_argument("--seed", type=int, default=None,
                        help="Random seed for reproducibility")
    args = parser.parse_args(argv)
    if args.prompt_ids is None and args.model is None:
        parser.error("--model is required for a text prompt (or give --prompt-ids)")

    if args.seed is not None:
        np.random.seed(args.seed)

    info, layers, rms_final, embed = read_checkpoint(args.checkpoint)
    if args.prompt_ids is not None:
        tokenizer = _IdTokenizer()
        prompt_tokens = [int(t) for t in args.prompt_ids.split(",") if t.strip()]
        shown = args.prompt_ids
    else:
        try:
            from transformers import AutoTokenizer
        except ImportError:
            print("Install dependencies: pip install transformers")
            sys.exit(1)
        print(f"Loading tokenizer: {args.model}")
        tokenizer = AutoTokenizer.from_pretrained(args.model, trust_remote_code=True)
        prompt_tokens = tokenizer.encode(args.prompt)
        shown = args.prompt
    if not prompt_tokens or min(prompt_tokens) < 0 or max(prompt_tokens) >= info["vocab"]:
        parser.error(f"prompt token ids must lie in [0, {info['vocab']})")
    print(f"Prompt ({len(prompt_tokens)} tokens): {shown}")
    print(f"Generating {args.tokens} tokens (temp={args.temp}, top_p={args.top_p})...")
    print("---")

    generated = generate(info, layers, rms_final, embed, tokenizer, prompt_tokens, args.tokens,
                         args.temp, args.top_p)

    print("---")
    print(f"Generated {len(generated)} tokens")
    return generated


if __name__ == "__main__":
    main()
