"""CPU oracle for the batch-1 decode hot path of francisown/qwen3.5-fp8-cuda.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU with PyTorch
tensors, the arithmetic of the reference's decode path so the CUDA library in
``qwen3.5-fp8-cuda_b200/`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py`` may import it, and only as the checker or as the timed CPU
baseline; the product path never routes through it.

Every function cites the reference file:line it follows.  Paths are relative
to the reference project root (``main.py``, ``qwen3_infer/csrc/*.cu``).

Parity pins (see ``tests/golden/``):
  * fixtures made by importing the reference's own ``main.py`` on the CPU
    (``tests/golden/make_golden_cpu.py``): RMSNorm, gates, gated norm, the
    decode delta rule and HF's conv1d / recurrent delta-rule helpers that the
    reference calls;
  * fixtures made by running the reference's CUDA kernels, compiled for
    sm_100a from their own sources by ``oracle/Makefile`` into ``oracle/_ref``
    (``tests/golden/make_golden_gpu.py``): the block-scaled GEMV family, the
    fused gate/up/SiLU MLP, RMSNorm and the delta-rule decode kernel.
"""

from . import model, ops, synth  # noqa: F401
