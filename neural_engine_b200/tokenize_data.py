"""Text files -> flat token-id file for ``ne_train --data``.

Mirrors ane-training/training/training_dynamic/tools/tokenize_data.py: the
same arguments (inputs, ``-`` for stdin, ``--model``, ``--output``,
``--max-tokens``), the same joining of the inputs with blank lines, one
``tokenizer.encode`` of the whole text, the same printed lines, and a flat
uint16 file (tokenize_data.py:67-76).  Extension: ``--u32`` writes uint32 ids
(read by ``ne_train --data-u32``) for vocabularies beyond 65,536, such as
Qwen3's 151,936, where the reference stops with an error.

    python -m neural_engine_b200.tokenize_data data/*.txt --model Qwen/Qwen3-0.6B --u32
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np


def main(argv=None):
    parser = argparse.ArgumentParser(description="Tokenize text for ne_train")
    parser.add_argument("inputs", nargs="+", help="Text files to tokenize (use - for stdin)")
    parser.add_argument("--model", "-m", required=True,
                        help="HF model ID for tokenizer (e.g. Qwen/Qwen3-0.6B)")
    parser.add_argument("--output", "-o", default="train_data.bin",
                        help="Output binary file (default: train_data.bin)")
    parser.add_argument("--max-tokens", type=int, default=None,
                        help="Maximum number of tokens to output")
    parser.add_argument("--u32", action="store_true",
                        help="write uint32 ids (ne_train --data-u32) instead of uint16")
    args = parser.parse_args(argv)

    try:
        from transformers import AutoTokenizer
    except ImportError:
        print("Install dependencies: pip install transformers")
        sys.exit(1)

    print(f"Loading tokenizer: {args.model}")
    tokenizer = AutoTokenizer.from_pretrained(args.model, trust_remote_code=True)
    print(f"Vocab size: {tokenizer.vocab_size}")

    all_text = []
    for inp in args.inputs:
        if inp == "-":
            print("Reading from stdin...")
            all_text.append(sys.stdin.read())
        else:
            path = Path(inp)
            if not path.exists():
                print(f"Warning: {inp} not found, skipping")
                continue
            print(f"Reading {inp} ({path.stat().st_size / 1e6:.1f} MB)")
            all_text.append(path.read_text(encoding="utf-8", errors="ignore"))
    if not all_text:
        print("No input text found")
        sys.exit(1)

    combined = "\n\n".join(all_text)
    print(f"Total text: {len(combined):,} characters")
    print("Tokenizing...")
    tokens = tokenizer.encode(combined)
    print(f"Total tokens: {len(tokens):,}")
    if args.max_tokens and len(tokens) > args.max_tokens:
        tokens = tokens[:args.max_tokens]
        print(f"Truncated to {len(tokens):,} tokens")
    if not tokens:
        print("No tokens produced")
        sys.exit(1)

    max_tok = max(tokens)
    limit = 0xFFFFFFFF if args.u32 else 0xFFFF
    if max_tok > limit:
        hint = "" if args.u32 else " Write uint32 ids with --u32 (ne_train --data-u32)."
        print(f"ERROR: Token ID {max_tok} exceeds {'uint32' if args.u32 else 'uint16'} range.{hint}")
        sys.exit(1)

    arr = np.array(tokens, dtype=np.uint32 if args.u32 else np.uint16)
    arr.tofile(args.output)
    size_mb = Path(args.output).stat().st_size / 1e6
    print(f"\nSaved: {args.output} ({len(tokens):,} tokens, {size_mb:.1f} MB)")
    flag = " --data-u32" if args.u32 else ""
    print(f"Train with: neural_engine_b200/ne_train --resume --data {args.output}{flag}")
    return arr


if __name__ == "__main__":
    main()
