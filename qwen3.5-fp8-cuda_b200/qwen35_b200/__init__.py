"""B200-native (sm_100a) batch-1 decode hot path of the Qwen3.5 hybrid decoder.

The compute lives in two shared libraries built from ``../csrc`` (``lib/``),
exporting the reference engine's ctypes C-ABI plus new entry points; this
package binds them (``_lib``), wraps them for torch tensors (``ops``) and
drives a whole decode step from a CUDA graph (``engine``).
"""

from . import config, weights  # noqa: F401

__all__ = ["config", "weights", "ops", "engine", "_lib"]
