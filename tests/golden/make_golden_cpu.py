"""Generate CPU golden fixtures by running the reference's own Python code.

Run in a container that has the reference checkout (the --ref argument)
and the reference kernels built by ``oracle/Makefile`` (``oracle/_ref``); the
reference's ``main.py`` opens those libraries at import time but nothing here
launches a GPU kernel: every call below is a CPU torch path of the reference.

    python tests/golden/make_golden_cpu.py [--ref REFERENCE_CHECKOUT]

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
* ``quant_*``     QwenEngineFP8Opt._quantize_bf16_to_fp8 (main.py:834-848) on a
                  ragged 300 x 200 BF16 matrix with an all-zero block
* ``load_*``      QwenEngineFP8Opt._load_weights_fp8 (main.py:573-720) on the
                  micro checkpoint this script also writes to
                  ``tests/golden/micro_ckpt/`` (config.json + model.safetensors)
"""

from __future__ import annotations

import argparse
import json
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


MICRO = {  # a 2-layer member of the family, small enough to commit
    "hidden_size": 128, "intermediate_size": 256, "num_hidden_layers": 2, "vocab_size": 320,
    "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 64,
    "linear_num_key_heads": 1, "linear_num_value_heads": 2, "linear_key_head_dim": 64,
    "linear_value_head_dim": 64, "linear_conv_kernel_dim": 4,
    "layer_types": ["linear_attention", "full_attention"],
    "rope_parameters": {"rope_theta": 10000000, "partial_rotary_factor": 0.25},
}


def make_micro_checkpoint(ckpt_dir, g):
    """A block-FP8 checkpoint exercising every branch of the reference loader:
    FP8 linears with FP32 scales that BF16 does not represent, an FP8 linear
    without a scale tensor, a BF16 linear, norms stored BF16 and FP32, a BF16
    dt_bias, conv1d as [C, 1, W], an FP8 LM head, and vision / MTP tensors the
    decoder does not read."""
    c = MICRO
    H, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    qd, kvd = c["num_attention_heads"] * c["head_dim"], c["num_key_value_heads"] * c["head_dim"]
    nv, vd = c["linear_num_value_heads"], c["linear_num_value_heads"] * c["linear_value_head_dim"]
    conv = 2 * c["linear_num_key_heads"] * c["linear_key_head_dim"] + vd
    t = {}

    def fp8(key, n, k, scaled=True):
        t[key] = (torch.randn(n, k, generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
        if scaled:
            nb, kb = (n + 127) // 128, (k + 127) // 128
            t[key + "_scale_inv"] = torch.pow(10.0, torch.rand(nb, kb, generator=g) * 2 - 4)

    def vec(key, n, dtype, mean=0.0, std=0.02):
        t[key] = (torch.randn(n, generator=g) * std + mean).to(dtype)

    p = "model.language_model."
    t[p + "embed_tokens.weight"] = (torch.randn(V, H, generator=g) * 0.02).to(BF16)
    vec(p + "norm.weight", H, BF16)
    fp8("lm_head.weight", V, H)
    for i, lt in enumerate(c["layer_types"]):
        b = f"{p}layers.{i}."
        vec(b + "input_layernorm.weight", H, BF16)
        vec(b + "post_attention_layernorm.weight", H, F32)
        if lt == "linear_attention":
            fp8(b + "linear_attn.in_proj_qkv.weight", conv, H)
            t[b + "linear_attn.in_proj_a.weight"] = (torch.randn(nv, H, generator=g) * 0.05).to(BF16)
            fp8(b + "linear_attn.in_proj_b.weight", nv, H, scaled=False)
            fp8(b + "linear_attn.in_proj_z.weight", vd, H)
            fp8(b + "linear_attn.out_proj.weight", H, vd)
            t[b + "linear_attn.A_log"] = torch.log(torch.rand(nv, generator=g) * 15 + 1)
            t[b + "linear_attn.dt_bias"] = (torch.rand(nv, generator=g) + 0.5).to(BF16)
            t[b + "linear_attn.conv1d.weight"] = (torch.randn(conv, 1, 4, generator=g) * 0.1).to(BF16)
            vec(b + "linear_attn.norm.weight", c["linear_value_head_dim"], F32, mean=1.0)
        else:
            fp8(b + "self_attn.q_proj.weight", 2 * qd, H)
            fp8(b + "self_attn.k_proj.weight", kvd, H)
            fp8(b + "self_attn.v_proj.weight", kvd, H)
            fp8(b + "self_attn.o_proj.weight", H, qd)
            vec(b + "self_attn.q_norm.weight", c["head_dim"], BF16)
            vec(b + "self_attn.k_norm.weight", c["head_dim"], F32)
        fp8(b + "mlp.gate_proj.weight", I, H)
        fp8(b + "mlp.up_proj.weight", I, H)
        fp8(b + "mlp.down_proj.weight", H, I)
    t["model.visual.patch_embed.proj.weight"] = torch.randn(8, 8, generator=g).to(BF16)
    t["mtp.fc.weight"] = torch.randn(8, 8, generator=g).to(BF16)
    os.makedirs(ckpt_dir, exist_ok=True)
    with open(os.path.join(ckpt_dir, "config.json"), "w") as f:
        json.dump({"text_config": MICRO, "tie_word_embeddings": False}, f, indent=1)
    save_file({k: v.contiguous() for k, v in t.items()}, os.path.join(ckpt_dir, "model.safetensors"),
              metadata={"format": "pt"})


def load_with_reference(Eng, ckpt_dir):
    """QwenEngineFP8Opt._load_weights_fp8 (main.py:573-720) run on a stub with
    the attributes it reads; its closing CUDA synchronize and memory report
    are replaced by no-ops (no GPU here).  Returns its tensors, flattened."""
    with open(os.path.join(ckpt_dir, "config.json")) as f:
        tc = json.load(f)["text_config"]
    stub = types.SimpleNamespace(n_layers=tc["num_hidden_layers"], layer_types=tc["layer_types"],
                                 _quantize_bf16_to_fp8=Eng._quantize_bf16_to_fp8)
    sync, mem = torch.cuda.synchronize, torch.cuda.memory_allocated
    torch.cuda.synchronize, torch.cuda.memory_allocated = (lambda *a, **k: None), (lambda *a, **k: 0)
    try:
        Eng._load_weights_fp8(stub, ckpt_dir)
    finally:
        torch.cuda.synchronize, torch.cuda.memory_allocated = sync, mem
    res = {"embed": stub.embed, "norm_f": stub.norm_f,
           "lm_head_w": stub.lm_head_fp8, "lm_head_s": stub.lm_head_scale}
    for i, ly in enumerate(stub.layers):
        for name, v in ly.items():
            if isinstance(v, tuple):
                res[f"L{i}_{name}_w"], res[f"L{i}_{name}_s"] = v
            elif isinstance(v, torch.Tensor):
                res[f"L{i}_{name}"] = v
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("QWEN_REFERENCE_ROOT")
                    or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"),
                    help="reference checkout (default: $QWEN_REFERENCE_ROOT, else 'reference' beside the repository)")
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

    # ---- checkpoint loading and BF16 -> block-FP8 quantization ----
    # own generator: the cases above keep their random streams
    gq = torch.Generator().manual_seed(4321)
    wq_in = (torch.randn(300, 200, generator=gq) * torch.rand(300, 1, generator=gq) * 4).to(BF16)
    wq_in[128:256, 0:128] = 0  # an all-zero block: the scale's 1e-12 floor
    qw, qs = Eng._quantize_bf16_to_fp8(wq_in)
    out["quant_w_in"], out["quant_w"], out["quant_s"] = wq_in, qw.view(torch.uint8), qs
    ckpt_dir = os.path.join(HERE, "micro_ckpt")
    make_micro_checkpoint(ckpt_dir, gq)
    for k_, v_ in load_with_reference(Eng, ckpt_dir).items():
        out["load_" + k_] = v_

    out = {k_: v_.contiguous() for k_, v_ in out.items()}
    save_file(out, args.out)
    print(f"wrote {args.out}: {len(out)} tensors, {sum(t.numel() * t.element_size() for t in out.values())} bytes")


if __name__ == "__main__":
    main()
