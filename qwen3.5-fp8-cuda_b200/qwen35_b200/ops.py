"""Torch-facing wrappers over the C-ABI, mirroring the reference's op layer.

``fp8_linear``, ``maybe_fp8_linear``, ``fused_qkv`` and ``fused_gate_up``
keep the names, arguments and dispatch of main.py:242-317 (decode GEMV for
M == 1, batched GEMM otherwise; the scale-mode encoding of main.py:249-251).
The others wrap the new entry points.  PyTorch provides buffers and the
current stream only; every computation is a kernel of libqwen_*.so.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

P = ctypes.c_void_p


def _p(t) -> P:
    return P(0) if t is None else P(t.data_ptr())


def _stream():
    return P(torch.cuda.current_stream().cuda_stream)


def scale_mode(n_rows: int, scale: torch.Tensor) -> int:
    """Reference K_blk encoding (main.py:249-251): >1 block, 1 per-row, <0 per-row-block."""
    kb = scale.shape[1]
    return -kb if scale.shape[0] == n_rows and kb > 1 else kb


def fp8_linear(input_bf16: torch.Tensor, w_bytes: torch.Tensor, w_scale_inv: torch.Tensor) -> torch.Tensor:
    """output = input @ W^T (main.py:242-270): GEMV for M == 1, GEMM otherwise."""
    orig_shape = input_bf16.shape
    in_dim = orig_shape[-1]
    out_dim = w_bytes.shape[0]
    x_2d = input_bf16.reshape(-1, in_dim).contiguous()
    m = x_2d.shape[0]
    kblk = scale_mode(out_dim, w_scale_inv)
    y = torch.empty(m, out_dim, dtype=torch.bfloat16, device=input_bf16.device)
    if m == 1:
        _lib.fused().launch_gemv_v4_extern(_p(x_2d), _p(w_bytes), _p(w_scale_inv), _p(y), out_dim, in_dim, kblk,
                                           _stream())
        _lib.check_last("launch_gemv_v4_extern")
    else:
        _lib.fp8().fp8_gemm_batch(_p(x_2d), _p(w_bytes), _p(w_scale_inv), _p(y), m, out_dim, in_dim, kblk,
                                  _stream())
        e = _lib.fp8().qwen_fp8_last_error()
        if e:
            raise RuntimeError(f"fp8_gemm_batch failed with CUDA error {e}")
    return y.reshape(*orig_shape[:-1], out_dim)


def maybe_fp8_linear(input_bf16: torch.Tensor, weight) -> torch.Tensor:
    """FP8 tuple -> fp8_linear; a BF16 tensor is not a supported weight (main.py:273-278)."""
    if isinstance(weight, tuple):
        return fp8_linear(input_bf16, *weight)
    raise TypeError("BF16 linear weights are outside this library's decode path")


def fused_qkv(x_bf16, w_q, s_q, w_k, s_k, w_v, s_v):
    """Fused q/k/v GEMVs (main.py:281-298)."""
    k = x_bf16.shape[-1]
    n_q, n_k, n_v = w_q.shape[0], w_k.shape[0], w_v.shape[0]
    kblk = s_q.shape[1]
    dev = x_bf16.device
    q_out = torch.empty(n_q, dtype=torch.bfloat16, device=dev)
    k_out = torch.empty(n_k, dtype=torch.bfloat16, device=dev)
    v_out = torch.empty(n_v, dtype=torch.bfloat16, device=dev)
    _lib.fused().launch_fused_qkv(_p(x_bf16), _p(w_q), _p(w_k), _p(w_v), _p(s_q), _p(s_k), _p(s_v), _p(q_out),
                                  _p(k_out), _p(v_out), k, n_q, n_k, n_v, kblk, s_q.shape[0], s_k.shape[0],
                                  s_v.shape[0], _stream())
    _lib.check_last("launch_fused_qkv")
    return q_out, k_out, v_out


def fused_gate_up(x_bf16, w_g, s_g, w_u, s_u):
    """Fused gate and up GEMVs (main.py:301-317)."""
    k = x_bf16.shape[-1]
    n_g, n_u = w_g.shape[0], w_u.shape[0]
    kblk = scale_mode(n_g, s_g)
    dev = x_bf16.device
    gate_out = torch.empty(n_g, dtype=torch.bfloat16, device=dev)
    up_out = torch.empty(n_u, dtype=torch.bfloat16, device=dev)
    _lib.fused().launch_fused_gate_up(_p(x_bf16), _p(w_g), _p(w_u), _p(s_g), _p(s_u), _p(gate_out), _p(up_out), k,
                                      n_g, n_u, kblk, s_g.shape[0], s_u.shape[0], _stream())
    _lib.check_last("launch_fused_gate_up")
    return gate_out, up_out


def rmsnorm_(x: torch.Tensor, weight_f32: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """In-place RMSNorm(1+w) over the last dim (main.py:926-933 decode branch)."""
    x2 = x.reshape(-1, x.shape[-1])
    _lib.fused().launch_rmsnorm_ip(_p(x2), _p(weight_f32), x2.shape[0], x2.shape[1], eps, _stream())
    _lib.check_last("launch_rmsnorm_ip")
    return x


def gemv_f32s(x, w, s_f32, kblk=None):
    """GEMV with FP32 block scales (no BF16 rounding of the scale)."""
    n, k = w.shape
    kblk = scale_mode(n, s_f32) if kblk is None else kblk
    y = torch.empty(n, dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.fused().launch_gemv_f32s(_p(x), _p(w), _p(s_f32), _p(y), n, k, kblk, _stream()),
               "launch_gemv_f32s")
    return y


def lm_head_argmax(x, w, s, norm_w=None, eps=1e-6, row_offset=0, ws=None, want_logits=False):
    """Fused (RMSNorm) + LM-head GEMV + greedy argmax.  Returns (token, key, logits|None)."""
    n, k = w.shape
    dev = x.device
    if ws is None:
        ws = torch.zeros(2, dtype=torch.int64, device=dev)
    key = torch.zeros(1, dtype=torch.int64, device=dev)
    tok = torch.zeros(1, dtype=torch.int64, device=dev)
    logits = torch.empty(n, dtype=torch.bfloat16, device=dev) if want_logits else None
    _lib.check(_lib.fused().launch_lm_head_argmax(_p(x), _p(norm_w), eps, _p(w), _p(s), n, k, scale_mode(n, s),
                                                  row_offset, _p(ws), _p(key), _p(tok), _p(logits), P(0),
                                                  _stream()), "launch_lm_head_argmax")
    return tok, key, logits
