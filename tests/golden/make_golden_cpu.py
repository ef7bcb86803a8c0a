"""Generate CPU golden fixtures by running the reference's own Python code.

Run in a container that has the reference checkout (default /root/reference)
and the reference kernels built by ``oracle/Makefile`` (``oracle/_ref``); the
reference's ``main.py`` opens those libraries at import time but nothing here
launches a GPU kernel: every call below is a CPU torch path of the reference.

    python tests/golden/make_golden_cpu.py [--ref /root/reference]

Writes ``tests/golden/cpu_golden.safetensors``.  Cases:

* ``rmsnorm_*``   QwenEngineFP8Opt.qwen_rmsnorm (main.py:949-956), FP32 formulation
* ``gdn_*``       QwenEngineFP8Opt.linear_attention_forward decode branch
                  (main.py:1064-1163), BF16 weights equal to E4M3 x 2^e block
                  dequantisation, the fused delta-rule call replaced by the
                  oracle's restatement of delta_rule_decode_kernel
* ``attn_*``      QwenEngineFP8Opt.full_attention_forward decode (main.py:981-1062)
                  on its torch path (_HAS_MID_ATTN off), the CUDA RMSNorm call
                  replaced by the oracle's restatement of rmsnorm_ip_kernel
* ``conv_*``      HF torch_causal_conv1d_update as called at main.py:1097
* ``delta_*``     HF torch_recurrent_gated_delta_rule on FP32 inputs
                  (use_qk_l2norm_in_kernel=True), the math of fused_kernels.cu:623-684
"""

from __future__ import annotations

import argparse
import os
import sys
import types

import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import ops  # noqa: E402

BF16, F32 = torch.bfloat16, torch.float32


def fp8_pow2(n, k, g):
    """E4M3 bytes and power-of-two BF16 block scales: W*scale is exact in BF16."""
    w = (torch.randn(n, k, generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    e = torch.randint(-12, -6, ((n + 127) // 128, (k + 127) // 128), generator=g)
    s = torch.pow(2.0, e.float()).to(BF16)
    return w.contiguous(), s.contiguous()


def as_bf16_weight(w, s):
    wd = ops.dequant(w, s)
    assert torch.equal(wd.to(BF16).float(), wd), "power-of-two dequant must be exact in BF16"
    return wd.to(BF16)


def load_reference(ref_dir):
    ref_lib = os.path.join(REPO, "oracle", "_ref")
    os.environ.setdefault("QWEN_FP8_DLL", os.path.join(ref_lib, "libref_fp8.so"))
    os.environ.setdefault("QWEN_FUSED_DLL", os.path.join(ref_lib, "libref_fused.so"))
    sys.path.insert(0, ref_dir)
    import main as ref  # the reference engine module
    ref.DEV = "cpu"
    return ref


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--out", default=os.path.join(HERE, "cpu_golden.safetensors"))
    args = ap.parse_args()
    ref = load_reference(args.ref)
    Eng = ref.QwenEngineFP8Opt
    g = torch.Generator().manual_seed(1234)
    out = {}

    # ---- RMSNorm(1+w), FP32 formulation ----
    x = (torch.randn(3, 2560, generator=g) * 2).to(BF16)
    w = torch.randn(2560, generator=g) * 0.02
    out["rmsnorm_x"], out["rmsnorm_w"] = x, w
    out["rmsnorm_y"] = Eng.qwen_rmsnorm(None, x, w, 1e-6)

    # ---- GatedDeltaNet layer, decode step ----
    H, Hk, Hv, D, cw = 256, 1, 2, 128, 4  # K = 256: two 128-wide K blocks (K_blk == 1 means per-row)
    kd, vd = Hk * D, Hv * D
    conv_dim = 2 * kd + vd
    lw = {}
    for name, (n, k) in {"in_proj_qkv": (conv_dim, H), "in_proj_a": (Hv, H), "in_proj_b": (Hv, H),
                         "in_proj_z": (vd, H), "out_proj": (H, vd)}.items():
        wq, sq = fp8_pow2(n, k, g)
        out[f"gdn_{name}_w"], out[f"gdn_{name}_s"] = wq, sq
        lw[name] = as_bf16_weight(wq, sq)
    lw["A_log"] = torch.log(torch.rand(Hv, generator=g) * 15 + 1)
    lw["dt_bias"] = torch.ones(Hv)
    lw["conv1d_w"] = (torch.randn(conv_dim, 1, cw, generator=g) * 0.1).to(BF16)
    lw["norm_w"] = (1 + torch.randn(D, generator=g) * 0.02).to(BF16)
    for k_ in ("A_log", "dt_bias", "norm_w"):
        out[f"gdn_{k_}"] = lw[k_]
    out["gdn_conv1d_w"] = lw["conv1d_w"].reshape(conv_dim, cw).contiguous()
    conv_state = (torch.randn(1, conv_dim, cw, generator=g)).to(BF16)
    rec_state = torch.randn(1, Hv, D, D, generator=g) * 0.05
    hid = (torch.randn(1, 1, H, generator=g)).to(BF16)
    out["gdn_conv_state_in"] = conv_state[0].clone()
    out["gdn_state_in"] = rec_state[0].clone()
    out["gdn_x"] = hid.reshape(-1).clone()

    def delta_rule_decode(self_, q, k, v, g_, beta, initial_state):
        o, s = ops.delta_rule_decode(q.reshape(Hv, D), k.reshape(Hv, D), v.reshape(Hv, D),
                                     g_.reshape(Hv), beta.reshape(Hv), initial_state.reshape(Hv, D, D))
        initial_state.copy_(s.reshape(initial_state.shape))
        return o.reshape(1, 1, Hv, D), None

    fake = types.SimpleNamespace(
        linear_num_k_heads=Hk, linear_k_head_dim=D, linear_num_v_heads=Hv, linear_v_head_dim=D,
        linear_conv_kernel=cw, conv_states=[conv_state], recurrent_states=[rec_state])
    fake.delta_rule_decode = types.MethodType(delta_rule_decode, fake)
    y = Eng.linear_attention_forward(fake, hid, lw, 0, past_len=7)
    out["gdn_y"] = y.reshape(-1).contiguous()
    out["gdn_conv_state_out"] = conv_state[0].clone()
    out["gdn_state_out"] = rec_state[0].clone()

    # ---- Full attention layer, decode step ----
    nh, nkv, hd, rot, max_seq, pos = 2, 1, 256, 64, 16, 5
    aw = {}
    for name, (n, k) in {"q_proj": (2 * nh * hd, H), "k_proj": (nkv * hd, H), "v_proj": (nkv * hd, H),
                         "o_proj": (H, nh * hd)}.items():
        wq, sq = fp8_pow2(n, k, g)
        out[f"attn_{name}_w"], out[f"attn_{name}_s"] = wq, sq
        aw[name] = as_bf16_weight(wq, sq)
    aw["q_norm"] = torch.randn(hd, generator=g) * 0.02
    aw["k_norm"] = torch.randn(hd, generator=g) * 0.02
    out["attn_q_norm"], out["attn_k_norm"] = aw["q_norm"], aw["k_norm"]
    kc = (torch.randn(1, nkv, max_seq, hd, generator=g)).to(BF16)
    vc = (torch.randn(1, nkv, max_seq, hd, generator=g)).to(BF16)
    out["attn_k_cache_in"], out["attn_v_cache_in"] = kc[0].clone(), vc[0].clone()
    hid = (torch.randn(1, 1, H, generator=g)).to(BF16)
    out["attn_x"] = hid.reshape(-1).clone()
    theta = 10_000_000.0
    cos, sin = ops.rope_tables(max_seq, rot, theta)

    def rmsnorm_cpu(self_, x_, weight, eps=1e-6):
        return ops.rmsnorm(x_, weight, eps)

    afake = types.SimpleNamespace(
        n_heads=nh, n_kv_heads=nkv, head_dim=hd, partial_rotary_factor=rot / hd,
        k_cache=[kc], v_cache=[vc], _rope_cos=cos, _rope_sin=sin)
    afake.rmsnorm = types.MethodType(rmsnorm_cpu, afake)
    afake.apply_partial_rope = types.MethodType(Eng.apply_partial_rope, afake)
    afake.rotate_half = Eng.rotate_half
    ref._HAS_MID_ATTN = False
    y = Eng.full_attention_forward(afake, hid, aw, 0, torch.tensor([pos]), pos)
    out["attn_y"] = y.reshape(-1).contiguous()
    out["attn_k_cache_out"], out["attn_v_cache_out"] = kc[0].clone(), vc[0].clone()
    out["attn_meta"] = torch.tensor([nh, nkv, hd, rot, max_seq, pos], dtype=torch.int32)

    # ---- HF conv1d update and recurrent delta rule (reference dependencies) ----
    from transformers.models.qwen3_5.modeling_qwen3_5 import (
        torch_causal_conv1d_update, torch_recurrent_gated_delta_rule)
    C = 640
    cx = (torch.randn(1, C, 1, generator=g)).to(BF16)
    cst = (torch.randn(1, C, cw, generator=g)).to(BF16)
    cwt = (torch.randn(C, cw, generator=g) * 0.3).to(BF16)
    out["conv_x"], out["conv_state_in"], out["conv_w"] = cx.reshape(-1).clone(), cst[0].clone(), cwt
    co = torch_causal_conv1d_update(cx, cst, cwt, None, "silu")
    out["conv_y"], out["conv_state_out"] = co.reshape(-1).contiguous(), cst[0].clone()

    Hd = 4
    q = torch.randn(1, 1, Hd, D, generator=g)
    k = torch.randn(1, 1, Hd, D, generator=g)
    v = torch.randn(1, 1, Hd, D, generator=g)
    gg = -torch.rand(1, 1, Hd, generator=g) * 3
    bb = torch.rand(1, 1, Hd, generator=g)
    s0 = torch.randn(1, Hd, D, D, generator=g) * 0.1
    o, s1 = torch_recurrent_gated_delta_rule(q, k, v, gg, bb, initial_state=s0.clone(), output_final_state=True,
                                             use_qk_l2norm_in_kernel=True)
    for name, t in {"q": q, "k": k, "v": v, "g": gg, "beta": bb, "state_in": s0, "out": o,
                    "state_out": s1}.items():
        out[f"delta_{name}"] = t.contiguous()

    out = {k_: v_.contiguous() for k_, v_ in out.items()}
    save_file(out, args.out)
    print(f"wrote {args.out}: {len(out)} tensors, {sum(t.numel() * t.element_size() for t in out.values())} bytes")


if __name__ == "__main__":
    main()
