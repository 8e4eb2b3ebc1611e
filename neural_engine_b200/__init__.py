"""neural_engine_b200 -- B200 (sm_100a) implementation of the reference's
per-layer transformer step (ane-training/training/training_dynamic) behind a
C ABI (include/ne.h, libne.so), with Python host bindings.

The package name uses underscores because a hyphenated directory cannot be
imported.  Importing it loads libne.so and raises if the library is missing:
there is no CPU fallback.
"""
from .runtime import (EXPORTED, LIB_PATH, QWEN3_06B, STORIES110M, Engine, ModelConfig, NeError,
                      load_library)

load_library()

__all__ = ["Engine", "ModelConfig", "NeError", "load_library", "LIB_PATH", "EXPORTED",
           "QWEN3_06B", "STORIES110M"]
