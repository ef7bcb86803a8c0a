"""Seeded synthetic inputs with the shapes and distributions of the benchmark
configs (test infrastructure; the reference ships no data or checkpoint).

* ``fp8_weight``: W = clip(N(0,1)*64, +-448) cast to E4M3; block scales
  ``[ceil(N/128), ceil(K/128)]`` FP32 = 10**U(-4,-2) (log-uniform).
* ``bf16_vector``: x ~ N(0,1) BF16.

Generation runs on the CPU with ``torch.Generator`` so the same seed gives the
same tensors everywhere; tensors are then moved to whatever device needs them.
"""

from __future__ import annotations

import torch

BLOCK = 128


def gen(seed: int, device: str = "cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def fp8_weight(n: int, k: int, g: torch.Generator, device: str = "cpu", std: float = 64.0):
    """E4M3 bytes ``[n, k]`` uint8 and FP32 block scales ``[ceil(n/128), ceil(k/128)]``."""
    w = torch.randn(n, k, generator=g, device=device) * std
    w = w.clamp_(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    nb, kb = (n + BLOCK - 1) // BLOCK, (k + BLOCK - 1) // BLOCK
    s = torch.pow(10.0, torch.rand(nb, kb, generator=g, device=device) * 2.0 - 4.0)
    return w.contiguous(), s.to(torch.float32).contiguous()


def bf16_vector(n: int, g: torch.Generator, device: str = "cpu", std: float = 1.0):
    return (torch.randn(n, generator=g, device=device) * std).to(torch.bfloat16)


def config0(seed: int = 0):
    """Single GEMV 9216x2560."""
    g = gen(seed)
    x = bf16_vector(2560, g)
    w, s = fp8_weight(9216, 2560, g)
    return x, w, s


# (name, N, K) of one decoder layer's GEMV set.
LAYER_GEMVS = [
    ("full.q", 8192, 2560), ("full.k", 1024, 2560), ("full.v", 1024, 2560),
    ("full.o", 2560, 4096),
    ("gdn.qkv", 8192, 2560), ("gdn.z", 4096, 2560), ("gdn.a", 32, 2560), ("gdn.b", 32, 2560),
    ("gdn.out", 2560, 4096),
    ("mlp.gate", 9216, 2560), ("mlp.up", 9216, 2560), ("mlp.down", 2560, 9216),
]


def gemv_bytes(n: int, k: int, scale_bytes: int = 2) -> int:
    """Algorithmic bytes of one GEMV: weights + scales + x + y."""
    nb, kb = (n + BLOCK - 1) // BLOCK, (k + BLOCK - 1) // BLOCK
    return n * k + scale_bytes * nb * kb + 2 * k + 2 * n
