"""CPU oracle for the transformer hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference's
``training_dynamic`` pipeline so that the CUDA product path can be checked
against it.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it, and only as the
checker or the timed CPU baseline.  The product (``neural_engine_b200`` and
``libne.so``) never imports, links or calls anything here.

Modules
  ckpt_v4   -- byte-exact v4 checkpoint reader/writer
               (ane-training/training/training_dynamic/config.h:83-91,
                train.m:97-165)
  model     -- model presets and the seeded synthetic weight/token generators
  decode    -- numpy token loop restated from tools/generate.py:81-228,
               parameterised (RoPE theta, eps, QK-norm, residual alpha,
               batched sequences, prompt processed in one causal pass)
  hf_fixture -- seeded synthetic Hugging Face checkpoints (safetensors I/O)
               and the HF Qwen3 forward (rotate_half RoPE) in float64, for the
               converter tests
  train     -- float64 torch autograd of the same forward (teacher-forced,
               full-vocab mean cross-entropy) and the AdamW step restated from
               cpu_ops.h:266-303 with the schedule / clip of train.m:782-858

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``tools/generate.py`` functions (imported from the reference tree in the
build container) on seeded checkpoints and commits the resulting tokens and
logits as fixtures; ``tests/test_oracle_golden.py`` checks this restatement
against them.  The reference ships no golden vectors of its own for this path.
"""
