"""Random-initialised weights for the Qwen3.5 hybrid decoder.

There is no checkpoint or network here, so every benchmark and parity run uses
seeded random weights with the reference's on-device layout
(``QwenEngineFP8Opt._load_weights_fp8``, main.py:573-720):

* block-FP8 linear weights as ``(uint8 [N, K] E4M3 bytes, scale [ceil(N/128), K/128])``
  with the scale rounded to BF16 as the reference does at load (main.py:597);
  values: ``clip(N(0,1)*64, +-448)`` cast to E4M3, scales ``10**U(-4,-2)``;
* RMSNorm(1+w) weights FP32 ~ N(0, 0.02) (main.py:659-669 load them as FP32);
* ``A_log = log U(1,16)``, ``dt_bias = 1`` FP32 (main.py:606-610 keep the stored dtype);
* ``conv1d`` BF16 ~ N(0, 0.1) stored ``[C, W]`` (main.py:694 squeezes ``[C,1,W]``);
* gated-norm weight BF16 ``1 + N(0, 0.02)`` (main.py:695-698; Qwen3_5RMSNormGated
  multiplies by the weight itself, initialised to ones);
* embedding BF16 ~ N(0, 0.02); LM head block-FP8 (or BF16 ~ N(0, 0.02)).

Per-layer dict keys are the reference's (main.py:652-715).
"""

from __future__ import annotations

import torch

BLOCK = 128


def _fp8(n, k, g, device):
    w = torch.randn(n, k, generator=g, device=device).mul_(64.0)
    w = w.clamp_(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)
    nb, kb = (n + BLOCK - 1) // BLOCK, (k + BLOCK - 1) // BLOCK
    s = torch.pow(10.0, torch.rand(nb, kb, generator=g, device=device) * 2.0 - 4.0)
    return w.contiguous(), s.to(torch.bfloat16).contiguous()


def _normal(shape, std, g, device, dtype=torch.float32, mean=0.0):
    return (torch.randn(*shape, generator=g, device=device) * std + mean).to(dtype).contiguous()


def random_weights(cfg, seed: int = 0, device: str = "cpu") -> dict:
    """Seeded random weights for ``cfg`` (a ``Qwen35Config``) on ``device``."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, I = cfg.hidden_size, cfg.intermediate_size
    w = {
        "embed": _normal((cfg.vocab_size, H), 0.02, g, device, torch.bfloat16),
        "norm_f": _normal((H,), 0.02, g, device),
        "layers": [],
    }
    for lt in cfg.layer_types:
        ly = {"layer_type": lt,
              "input_layernorm": _normal((H,), 0.02, g, device),
              "post_attention_layernorm": _normal((H,), 0.02, g, device)}
        if lt == "full_attention":
            qd = cfg.num_attention_heads * cfg.head_dim
            kvd = cfg.num_key_value_heads * cfg.head_dim
            ly["q_proj"] = _fp8(2 * qd, H, g, device)
            ly["k_proj"] = _fp8(kvd, H, g, device)
            ly["v_proj"] = _fp8(kvd, H, g, device)
            ly["o_proj"] = _fp8(H, qd, g, device)
            ly["q_norm"] = _normal((cfg.head_dim,), 0.02, g, device)
            ly["k_norm"] = _normal((cfg.head_dim,), 0.02, g, device)
        else:
            nv = cfg.linear_num_value_heads
            ly["in_proj_qkv"] = _fp8(cfg.conv_dim, H, g, device)
            ly["in_proj_a"] = _fp8(nv, H, g, device)
            ly["in_proj_b"] = _fp8(nv, H, g, device)
            ly["in_proj_z"] = _fp8(cfg.linear_value_dim, H, g, device)
            ly["out_proj"] = _fp8(H, cfg.linear_value_dim, g, device)
            ly["A_log"] = torch.log(torch.rand(nv, generator=g, device=device) * 15.0 + 1.0).float()
            ly["dt_bias"] = torch.ones(nv, device=device, dtype=torch.float32)
            ly["conv1d_w"] = _normal((cfg.conv_dim, cfg.linear_conv_kernel_dim), 0.1, g, device,
                                     torch.bfloat16)
            ly["norm_w"] = _normal((cfg.linear_value_head_dim,), 0.02, g, device, torch.bfloat16,
                                   mean=1.0)
        ly["gate_proj"] = _fp8(I, H, g, device)
        ly["up_proj"] = _fp8(I, H, g, device)
        ly["down_proj"] = _fp8(H, I, g, device)
        w["layers"].append(ly)
    if cfg.fp8_lm_head:
        w["lm_head"] = _fp8(cfg.vocab_size, H, g, device)
    else:
        w["lm_head"] = _normal((cfg.vocab_size, H), 0.02, g, device, torch.bfloat16)
    return w


def to_device(w, device):
    """Copy a weights dict (nested tuples/lists/dicts of tensors) to ``device``."""
    if isinstance(w, torch.Tensor):
        return w.to(device).contiguous()
    if isinstance(w, tuple):
        return tuple(to_device(t, device) for t in w)
    if isinstance(w, list):
        return [to_device(t, device) for t in w]
    if isinstance(w, dict):
        return {k: to_device(v, device) for k, v in w.items()}
    return w


def linear_bytes(w) -> int:
    """Bytes a decode step streams for one linear weight entry."""
    if isinstance(w, tuple):
        return sum(t.numel() * t.element_size() for t in w)
    return w.numel() * w.element_size()
