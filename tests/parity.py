"""Tolerance checks shared by the GPU parity tests.

Floating-point outputs are compared with the oracle's FP32 value *before* its
final BF16 rounding, with the bars of the hot-path contract:

* max relative error  max|y - y_ref| / max|y_ref|  <= 2e-3
  (a BF16 output rounded once is within 2^-9 = 1.95e-3 of its FP32 value);
* cosine similarity  >= 0.99999.

Integer / index results (greedy token ids) must be equal.
"""

import torch

MAX_REL = 2e-3
MIN_COS = 0.99999


def max_rel(y, ref) -> float:
    y, ref = y.float().reshape(-1).cpu(), ref.float().reshape(-1).cpu()
    return float((y - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def cosine(y, ref) -> float:
    y, ref = y.double().reshape(-1).cpu(), ref.double().reshape(-1).cpu()
    return float((y @ ref) / (y.norm() * ref.norm()).clamp_min(1e-300))


def assert_close(y, ref, max_rel_err=MAX_REL, min_cos=MIN_COS, what=""):
    r, c = max_rel(y, ref), cosine(y, ref)
    assert r <= max_rel_err and c >= min_cos, f"{what}: max_rel={r:.3e} (<= {max_rel_err}) cos={c:.8f} (>= {min_cos})"
    return r, c


def bf16_ulp_diff(y, ref_bf16):
    """Elementwise |y - ref| in units of ref's BF16 ulp."""
    y, ref = y.float().reshape(-1).cpu(), ref_bf16.float().reshape(-1).cpu()
    ulp = torch.pow(2.0, torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 7)
    return (y - ref).abs() / ulp
