"""CPU restatement of the reference decode-path arithmetic (test oracle only).

Every function names the reference lines it restates.  Inputs are CPU torch
tensors; BF16 values are rounded exactly where the reference rounds them
(round-to-nearest-even, as ``__float2bfloat16`` and ``Tensor.to(bfloat16)``
both do).  Summation order is whatever torch's CPU kernels use: parity with the
CUDA path is judged with the tolerances written in ``tests/``.
"""

from __future__ import annotations

import math

import torch

F32 = torch.float32
BF16 = torch.bfloat16
BLOCK = 128  # main.py:32, fused_kernels.cu:102 (row / 128)


# ---------------------------------------------------------------------------
# FP8 E4M3 block-scaled linear algebra
# ---------------------------------------------------------------------------

def e4m3_to_f32(w_u8: torch.Tensor) -> torch.Tensor:
    """Decode E4M3 bytes exactly (main.py:497-501: ``w.view(float8_e4m3fn)``)."""
    assert w_u8.dtype == torch.uint8
    return w_u8.view(torch.float8_e4m3fn).to(F32)


def scale_mode(n_rows: int, scale: torch.Tensor) -> int:
    """The reference's int ``K_blk`` encoding of the scale layout.

    main.py:249-251 (and 305, 1243-1244, 1380-1381):
      * ``>1``  block scales ``[ceil(N/128), K_blk]``;
      * ``==1`` one scale per output row ``[N, 1]``;
      * ``<0``  per-row-per-128-K-block scales ``[N, -K_blk]``.
    """
    kb = scale.shape[1]
    return -kb if scale.shape[0] == n_rows and kb > 1 else kb


def expand_scales(n_rows: int, k: int, scale: torch.Tensor, kblk: int) -> torch.Tensor:
    """Per-element FP32 scale grid ``[N, K]``.

    Index rule of gemv_v4_kernel (fused_kernels.cu:99-114): per-row-block mode
    uses ``row*K_blk + k/128``; per-row mode uses ``row``; block mode uses
    ``(row/128)*K_blk + k/128``.
    """
    s = scale.to(F32)
    kcols = torch.arange(k, device=s.device) // BLOCK
    rows = torch.arange(n_rows, device=s.device)
    if kblk < 0:
        grid = s.reshape(n_rows, -kblk)[:, kcols]
    elif kblk == 1:
        grid = s.reshape(-1)[:n_rows].unsqueeze(1).expand(n_rows, k)
    else:
        grid = s.reshape(-1, kblk)[rows // BLOCK][:, kcols]
    return grid


def dequant(w_u8: torch.Tensor, scale: torch.Tensor, kblk: int | None = None) -> torch.Tensor:
    """Explicit FP8 -> FP32 block dequant (main.py:497-501 semantics).

    ``scale`` is used exactly as the kernel consumes it: BF16 on the ABI path
    (main.py:597 rounds every ``weight_scale_inv`` to BF16) or FP32 on the
    ``*_f32s`` entry points.
    """
    n, k = w_u8.shape
    if kblk is None:
        kblk = scale_mode(n, scale)
    if kblk > 1 and n % BLOCK == 0 and k % BLOCK == 0 and scale.shape == (n // BLOCK, k // BLOCK):
        # same values as the index form below, by broadcasting over 128x128 blocks
        w = e4m3_to_f32(w_u8).view(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
        return (w * scale.to(F32).view(n // BLOCK, 1, k // BLOCK, 1)).view(n, k)
    return e4m3_to_f32(w_u8) * expand_scales(n, k, scale, kblk)


def gemv(x: torch.Tensor, w_u8: torch.Tensor, scale: torch.Tensor, kblk: int | None = None) -> torch.Tensor:
    """y = bf16(x . (W*scale)^T) with FP32 accumulation.

    Restates gemv_v4_kernel (fused_kernels.cu:91-151) as explicit dequant +
    FP32 matmul; the output is rounded to BF16 once (fused_kernels.cu:150).
    """
    xf = x.reshape(-1).to(F32)
    return (dequant(w_u8, scale, kblk) @ xf).to(BF16)


def gemm(x: torch.Tensor, w_u8: torch.Tensor, scale: torch.Tensor, kblk: int | None = None) -> torch.Tensor:
    """Y[M,N] = bf16(X . Wdq^T): fp8_gemm_batch_kernel (fp8_kernels.cu:23-64)."""
    return (x.to(F32) @ dequant(w_u8, scale, kblk).T).to(BF16)


def linear_bf16(x: torch.Tensor, w_bf16: torch.Tensor) -> torch.Tensor:
    """BF16-weight LM head: ``F.linear`` (main.py:1600-1601), FP32 accumulate."""
    return (w_bf16.to(F32) @ x.reshape(-1).to(F32)).to(BF16)


# ---------------------------------------------------------------------------
# Normalisation
# ---------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w_f32: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm(1+w) per row: rmsnorm_ip_kernel / rmsnorm_out_kernel.

    fused_kernels.cu:489-547: ``rms = rsqrt(sum(x^2)/D + eps)``;
    ``out = bf16(x * rms * (1 + w))`` with FP32 weights.
    """
    d = x.shape[-1]
    xf = x.to(F32).reshape(-1, d)
    ss = (xf * xf).sum(-1, keepdim=True)
    rms = torch.rsqrt(ss / d + eps)
    out = (xf * rms) * (1.0 + w_f32.to(F32))
    return out.to(BF16).reshape(x.shape)


def rmsnorm_gated(core: torch.Tensor, z: torch.Tensor, w_bf16: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNormGated of the default decode path, main.py:1152-1159.

    ``normed = bf16(core * rsqrt(mean(core^2) + eps))``; ``normed = bf16(normed*w)``;
    ``out = bf16(normed * bf16(silu(z)))`` -- each product rounds to BF16
    because every operand is a BF16 tensor.
    """
    d = core.shape[-1]
    cf = core.to(F32).reshape(-1, d)
    var = (cf * cf).mean(-1, keepdim=True)
    normed = (cf * torch.rsqrt(var + eps)).to(BF16)
    normed = (normed.to(F32) * w_bf16.to(F32)).to(BF16)
    zs = silu_bf16(z.reshape(-1, d))
    return (normed.to(F32) * zs.to(F32)).to(BF16).reshape(core.shape)


def silu_f32(x: torch.Tensor) -> torch.Tensor:
    """x / (1 + exp(-x)) in FP32 (fused_kernels.cu:476)."""
    return x / (1.0 + torch.exp(-x))


def silu_bf16(x: torch.Tensor) -> torch.Tensor:
    """``F.silu`` on a BF16 tensor: FP32 math, one BF16 rounding."""
    return silu_f32(x.to(F32)).to(BF16)


def sigmoid_bf16(x: torch.Tensor) -> torch.Tensor:
    """``Tensor.sigmoid()`` on BF16: FP32 math, one BF16 rounding."""
    return torch.sigmoid(x.to(F32)).to(BF16)


# ---------------------------------------------------------------------------
# MLP
# ---------------------------------------------------------------------------

def gate_up_silu(x, wg, sg, wu, su, kblk=None):
    """fused_gate_up_silu_v4_kernel (fused_kernels.cu:398-479).

    Gate and up stay FP32 accumulators; ``silu = bf16(silu(g) * u)`` uses the
    FP32 values (fused_kernels.cu:476).  Returns (gate_bf16, up_bf16, silu_bf16).
    """
    xf = x.reshape(-1).to(F32)
    g = dequant(wg, sg, kblk) @ xf
    u = dequant(wu, su, kblk) @ xf
    return g.to(BF16), u.to(BF16), (silu_f32(g) * u).to(BF16)


def add_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """elem_add_kernel (fused_kernels.cu:553-559): bf16(float(a)+float(b))."""
    return (a.to(F32) + b.to(F32)).to(BF16)


def mlp_post(hidden, o_out, norm_w, wg, sg, wu, su, wd, sd, eps=1e-6):
    """layer_post_o_fp8_mlp (fused_kernels.cu:1156-1195).

    h2 = bf16(hidden + o); n = RMSNorm(1+w)(h2); s = bf16(silu(g)*u);
    d = bf16(down(s)); out = bf16(h2 + d).  Returns a dict of every buffer
    the reference leaves written.
    """
    h2 = add_bf16(hidden, o_out)
    n = rmsnorm(h2, norm_w, eps)
    gate, up, s = gate_up_silu(n, wg, sg, wu, su)
    d = gemv(s, wd, sd)
    out = add_bf16(h2, d)
    return {"output": out, "h2": h2, "normed": n, "gate": gate, "up": up, "silu": s, "down": d}


def layer_post_attn(hidden, attn_out, wo, so, norm_w, wg, sg, wu, su, wd, sd, eps=1e-6):
    """layer_post_attn (fused_kernels.cu:1102-1150): o_proj then the MLP."""
    o = gemv(attn_out, wo, so)
    r = mlp_post(hidden, o, norm_w, wg, sg, wu, su, wd, sd, eps)
    r["o"] = o
    return r


# ---------------------------------------------------------------------------
# GatedDeltaNet decode
# ---------------------------------------------------------------------------

def conv1d_update(x_new: torch.Tensor, conv_state: torch.Tensor, conv_w: torch.Tensor):
    """Depthwise causal conv1d decode update + SiLU.

    Restates HF ``torch_causal_conv1d_update`` as called at main.py:1097 /
    1423: the state ``[C, W]`` holds the last W inputs; the new input is
    appended, the last W entries become the new state and the output is
    ``silu(bf16(sum_t w[c,t] * window[c,t]))`` over the last W entries
    (state[1:], x), rounded to BF16 after the conv and again after SiLU.
    Returns (out_bf16 [C], new_state_bf16 [C, W]).
    """
    c, wlen = conv_state.shape
    window = torch.cat([conv_state[:, 1:], x_new.reshape(c, 1).to(BF16)], dim=1)
    acc = (window.to(F32) * conv_w.reshape(c, wlen).to(F32)).sum(-1)
    out = silu_bf16(acc.to(BF16))
    return out, window.clone()


def softplus_f32(x: torch.Tensor) -> torch.Tensor:
    """torch ``F.softplus`` (beta=1, threshold=20) in FP32, main.py:1122."""
    return torch.where(x > 20.0, x, torch.log1p(torch.exp(x)))


def linear_gates(a_bf16, b_bf16, a_log_f32, dt_bias_f32):
    """main.py:1120-1122: beta = sigmoid(b) (BF16); g = -exp(A_log)*softplus(a+dt)."""
    beta = sigmoid_bf16(b_bf16)
    g = -torch.exp(a_log_f32.to(F32)) * softplus_f32(a_bf16.to(F32) + dt_bias_f32.to(F32))
    return g.to(F32), beta


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """x * rsqrt(sum(x^2) + eps) (main.py:320-323; fused_kernels.cu:658-659)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def delta_rule_decode(q, k, v, g, beta, state):
    """One gated delta-rule decode step, delta_rule_decode_kernel (fused_kernels.cu:623-684).

    q, k, v: BF16 ``[H, D]`` (value heads; q/k already repeated 16->32);
    g: FP32 ``[H]``; beta: BF16 ``[H]``; state: FP32 ``[H, Dk, Dv]``.
    q_hat = l2n(q)/sqrt(D), k_hat = l2n(k); S' = e^g S; delta = (v - S'^T k_hat)*beta;
    S'' = S' + k_hat delta^T; out = bf16(S''^T q_hat).  Returns (out, new_state).
    """
    d = q.shape[-1]
    qf = l2norm(q.to(F32)) * (1.0 / math.sqrt(d))
    kf = l2norm(k.to(F32))
    vf = v.to(F32)
    decay = torch.exp(g.to(F32)).reshape(-1, 1, 1)
    s = state.to(F32) * decay
    pred = (s * kf.unsqueeze(-1)).sum(-2)
    delta = (vf - pred) * beta.to(F32).reshape(-1, 1)
    s = s + kf.unsqueeze(-1) * delta.unsqueeze(-2)
    out = (s * qf.unsqueeze(-1)).sum(-2)
    return out.to(BF16), s


# ---------------------------------------------------------------------------
# Full attention decode (not graded as a kernel target; needed end to end)
# ---------------------------------------------------------------------------

def rope_tables(max_pos: int, rotary_dim: int, theta: float):
    """Partial-RoPE cos/sin tables ``[max_pos, rotary_dim]`` FP32 (main.py:525-533)."""
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim))
    pos = torch.arange(max_pos).float()
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


def rope_apply(x: torch.Tensor, cos_row: torch.Tensor, sin_row: torch.Tensor, rotary_dim: int) -> torch.Tensor:
    """rope_decode_kernel (fused_kernels.cu:872-903) on BF16 heads ``[h, D]``."""
    half = rotary_dim // 2
    xf = x.to(F32).clone()
    x0 = xf[:, :half].clone()
    x1 = xf[:, half:rotary_dim].clone()
    out = x.clone()
    out[:, :half] = (x0 * cos_row[:half] - x1 * sin_row[:half]).to(BF16)
    out[:, half:rotary_dim] = (x1 * cos_row[half:rotary_dim] + x0 * sin_row[half:rotary_dim]).to(BF16)
    return out


def attention_decode(q_all, k_new, v_new, q_norm, k_norm, cos, sin, k_cache, v_cache, pos,
                     n_heads, n_kv, head_dim, rotary_dim, eps=1e-6):
    """Full-attention decode of the default path (main.py:1000-1059 with
    layer_mid_attn, fused_kernels.cu:1224-1297, and fused_attn_v2_kernel 787-867).

    q_all: BF16 ``[n_heads*2*head_dim]`` laid out per head as [q | gate]
    (main.py:1001); k_new/v_new BF16 ``[n_kv*head_dim]``; caches BF16
    ``[n_kv, max_seq, head_dim]`` updated in place at ``pos``.
    Returns the gated attention output BF16 ``[n_heads*head_dim]``
    (``out * bf16(sigmoid(gate))``, main.py:1059).
    """
    qh = q_all.reshape(n_heads, 2 * head_dim)
    q = qh[:, :head_dim]
    gate = qh[:, head_dim:]
    q = rmsnorm(q, q_norm, eps)
    k = rmsnorm(k_new.reshape(n_kv, head_dim), k_norm, eps)
    q = rope_apply(q, cos[pos], sin[pos], rotary_dim)
    k = rope_apply(k, cos[pos], sin[pos], rotary_dim)
    k_cache[:, pos] = k
    v_cache[:, pos] = v_new.reshape(n_kv, head_dim)
    total = pos + 1
    grp = n_heads // n_kv
    kc = k_cache[:, :total].to(F32).repeat_interleave(grp, dim=0)
    vc = v_cache[:, :total].to(F32).repeat_interleave(grp, dim=0)
    qs = q.to(F32) * (1.0 / math.sqrt(head_dim))
    scores = torch.einsum("hd,htd->ht", qs, kc)
    p = torch.softmax(scores, dim=-1)
    out = torch.einsum("ht,htd->hd", p, vc).to(BF16)
    gated = (out.to(F32) * sigmoid_bf16(gate).to(F32)).to(BF16)
    return gated.reshape(-1)


# ---------------------------------------------------------------------------
# Greedy argmax
# ---------------------------------------------------------------------------

def argmax_first(logits_bf16: torch.Tensor) -> int:
    """torch ``argmax`` over BF16 logits: the first maximal index (N8)."""
    v = logits_bf16.reshape(-1).to(F32)
    m = v.max()
    return int(torch.nonzero(v == m)[0, 0])


def bf16_orderable(bits16: int) -> int:
    """Map BF16 bits to an unsigned key that sorts like the value (+0 == -0)."""
    bits16 &= 0xFFFF
    if bits16 & 0x7FFF == 0:
        bits16 = 0
    return (~bits16) & 0xFFFF if bits16 & 0x8000 else bits16 | 0x8000


def packed_key(logit_bf16_bits: int, index: int) -> int:
    """Cross-shard argmax key: orderable(bf16) << 32 | (0xFFFFFFFF - index).

    The max key is the largest BF16 logit with the lowest index on ties, i.e.
    the torch argmax of the concatenated logits.
    """
    return (bf16_orderable(logit_bf16_bits) << 32) | (0xFFFFFFFF - index)


def key_to_index(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


def top2_gap(logits_bf16: torch.Tensor) -> float:
    """Gap between the largest and the second largest distinct-index logit."""
    v = logits_bf16.reshape(-1).to(F32)
    t = torch.topk(v, 2).values
    return float(t[0] - t[1])
