"""Prefill GEMM (fp8_gemm_batch, fp8_kernels.cu:23-89) on the tcgen05 path.

y[M, N] = bf16(x[M, K] @ dequant(W, scale)^T) with BF16 block scales, checked
against the CPU oracle's explicit block dequant + FP32 matmul (main.py:497-501)
at config-4 shapes, ragged token counts and N = 32, and against the reference's
own fp8_gemm_batch built for sm_100a when it is present.
"""

import ctypes
import os

import pytest
import torch

from conftest import REF_LIB
from oracle import ops, synth
from parity import assert_close

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p
BF16 = torch.bfloat16


def _p(t):
    return P(t.data_ptr())


def _gemm(x, w, s):
    from qwen35_b200 import _lib
    lib = _lib.fp8()
    m, k = x.shape
    n = w.shape[0]
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    y = torch.full((m, n), float("nan"), dtype=BF16, device="cuda")
    lib.fp8_gemm_batch(_p(xd), _p(wd), _p(sd), _p(y), m, n, k, k // 128, P(0))
    torch.cuda.synchronize()
    assert lib.qwen_fp8_last_error() == 0
    from qwen35_b200 import _lib as L
    assert L.device_error() == 0
    return y.cpu()


@pytest.mark.parametrize("m,n,k", [(3, 1024, 2560), (100, 2560, 4096), (512, 9216, 2560), (65, 32, 2560),
                                   (256, 2560, 9216), (2048, 1024, 2560)])
def test_gemm_matches_oracle(m, n, k):
    g = synth.gen(1000 + m + n)
    w, s32 = synth.fp8_weight(n, k, g)
    s = s32.to(BF16)
    x = torch.randn(m, k, generator=g).to(BF16)
    y = _gemm(x, w, s)
    assert not torch.isnan(y.float()).any()
    ref = x.float() @ ops.dequant(w, s).T
    assert_close(y, ref, what=f"gemm {m}x{n}x{k}")


def test_gemm_heavy_tailed_rows():
    """Rows with a few large entries and many tiny ones (the down projection's input)."""
    g = synth.gen(77)
    m, n, k = 130, 2560, 9216
    w, s32 = synth.fp8_weight(n, k, g)
    s = s32.to(BF16)
    x = torch.randn(m, k, generator=g) * 0.01
    x[:, ::97] *= 3000.0
    x = x.to(BF16)
    y = _gemm(x, w, s)
    ref = x.float() @ ops.dequant(w, s).T
    assert_close(y, ref, what="gemm heavy tails")


def test_gemm_matches_reference_kernel():
    path = os.path.join(REF_LIB, "libref_fp8.so")
    if not os.path.exists(path):
        pytest.skip("reference kernels not built (oracle/Makefile)")
    ref = ctypes.CDLL(path)
    ref.fp8_gemm_batch.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
    g = synth.gen(5)
    m, n, k = 128, 2560, 2560
    w, s32 = synth.fp8_weight(n, k, g)
    s = s32.to(BF16)
    x = torch.randn(m, k, generator=g).to(BF16)
    xd, wd, sd = x.cuda(), w.cuda(), s.cuda()
    yr = torch.empty(m, n, dtype=BF16, device="cuda")
    ref.fp8_gemm_batch(_p(xd), _p(wd), _p(sd), _p(yr), m, n, k, k // 128, P(0))
    torch.cuda.synchronize()
    y = _gemm(x, w, s)
    assert_close(y, yr.cpu().float(), what="gemm vs reference kernel")


def test_gemm_repeatable():
    g = synth.gen(9)
    m, n, k = 96, 1024, 2560
    w, s32 = synth.fp8_weight(n, k, g)
    s = s32.to(BF16)
    x = torch.randn(m, k, generator=g).to(BF16)
    assert torch.equal(_gemm(x, w, s), _gemm(x, w, s))
