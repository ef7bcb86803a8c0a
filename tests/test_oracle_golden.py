"""The CPU oracle against golden vectors made by the reference itself (CPU).

Fixtures: tests/golden/cpu_golden.safetensors, produced by
tests/golden/make_golden_cpu.py from the reference's own main.py and the HF
helpers it calls.  Tolerances: BF16 outputs may differ by one BF16 rounding
(relative 2^-8) where torch's CPU kernels sum in a different order.
"""

import os

import pytest
import torch
from safetensors.torch import load_file

from conftest import GOLDEN
from oracle import ops

BF16, F32 = torch.bfloat16, torch.float32


@pytest.fixture(scope="module")
def gold():
    return load_file(os.path.join(GOLDEN, "cpu_golden.safetensors"))


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def close_bf16(a, b, ulps=1, frac=0.02):
    """At most `frac` of elements differ, each by at most `ulps` BF16 ulps."""
    a, b = a.float().reshape(-1), b.float().reshape(-1)
    ulp = torch.pow(2.0, torch.floor(torch.log2(b.abs().clamp_min(1e-30))) - 7)
    d = (a - b).abs()
    assert bool((d <= ulps * ulp + 1e-30).all()), f"max ulp diff {float((d / ulp).max())}"
    assert float((d > 0).float().mean()) <= frac


def test_rmsnorm_matches_reference_fp32_formulation(gold):
    y = ops.rmsnorm(gold["rmsnorm_x"], gold["rmsnorm_w"])
    close_bf16(y, gold["rmsnorm_y"])


def test_conv1d_update_matches_hf(gold):
    out, st = ops.conv1d_update(gold["conv_x"], gold["conv_state_in"], gold["conv_w"])
    assert torch.equal(st, gold["conv_state_out"])
    close_bf16(out, gold["conv_y"])


def test_delta_rule_matches_hf_recurrent(gold):
    q, k, v = gold["delta_q"][0, 0], gold["delta_k"][0, 0], gold["delta_v"][0, 0]
    g, b = gold["delta_g"][0, 0], gold["delta_beta"][0, 0]
    # the oracle takes BF16 q/k/v/beta as the kernel does; feed FP32 through a
    # BF16-exact path by comparing on FP32 math directly
    d = q.shape[-1]
    qf = ops.l2norm(q) / d ** 0.5
    kf = ops.l2norm(k)
    s = gold["delta_state_in"][0] * torch.exp(g).reshape(-1, 1, 1)
    pred = (s * kf.unsqueeze(-1)).sum(-2)
    delta = (v - pred) * b.reshape(-1, 1)
    s = s + kf.unsqueeze(-1) * delta.unsqueeze(-2)
    o = (s * qf.unsqueeze(-1)).sum(-2)
    assert rel_err(s, gold["delta_state_out"][0]) < 1e-5
    assert rel_err(o, gold["delta_out"][0, 0]) < 1e-5
    # and the oracle function itself on BF16-rounded inputs stays close
    o2, s2 = ops.delta_rule_decode(q.to(BF16), k.to(BF16), v.to(BF16), g, b.to(BF16), gold["delta_state_in"][0])
    assert rel_err(s2, gold["delta_state_out"][0]) < 2e-2


def test_gdn_layer_matches_reference_linear_attention_forward(gold):
    """oracle.model layer math == main.py linear_attention_forward (decode)."""
    from oracle.model import OracleModel  # noqa: F401  (layer helper below mirrors OracleModel._linear)
    g = gold
    Hv, D, Hk = 2, 128, 1
    kd, vd = Hk * D, Hv * D
    x = g["gdn_x"]
    mixed = ops.gemv(x, g["gdn_in_proj_qkv_w"], g["gdn_in_proj_qkv_s"])
    a = ops.gemv(x, g["gdn_in_proj_a_w"], g["gdn_in_proj_a_s"])
    b = ops.gemv(x, g["gdn_in_proj_b_w"], g["gdn_in_proj_b_s"])
    z = ops.gemv(x, g["gdn_in_proj_z_w"], g["gdn_in_proj_z_s"])
    conv_out, conv_state = ops.conv1d_update(mixed, g["gdn_conv_state_in"], g["gdn_conv1d_w"])
    assert torch.equal(conv_state, g["gdn_conv_state_out"])
    q, k, v = torch.split(conv_out, [kd, kd, vd])
    gg, beta = ops.linear_gates(a, b, g["gdn_A_log"], g["gdn_dt_bias"])
    q = q.reshape(Hk, D).repeat_interleave(Hv // Hk, 0)
    k = k.reshape(Hk, D).repeat_interleave(Hv // Hk, 0)
    core, state = ops.delta_rule_decode(q, k, v.reshape(Hv, D), gg, beta, g["gdn_state_in"])
    assert rel_err(state, g["gdn_state_out"]) < 1e-6
    gated = ops.rmsnorm_gated(core, z.reshape(Hv, D), g["gdn_norm_w"])
    y = ops.gemv(gated.reshape(-1), g["gdn_out_proj_w"], g["gdn_out_proj_s"])
    assert rel_err(y, g["gdn_y"]) < 4e-3  # measured: bit-exact


def test_attention_layer_matches_reference_full_attention_forward(gold):
    g = gold
    nh, nkv, hd, rot, max_seq, pos = [int(v) for v in g["attn_meta"]]
    x = g["attn_x"]
    q_all = ops.gemv(x, g["attn_q_proj_w"], g["attn_q_proj_s"])
    k = ops.gemv(x, g["attn_k_proj_w"], g["attn_k_proj_s"])
    v = ops.gemv(x, g["attn_v_proj_w"], g["attn_v_proj_s"])
    kc, vc = g["attn_k_cache_in"].clone(), g["attn_v_cache_in"].clone()
    cos, sin = ops.rope_tables(max_seq, rot, 10_000_000.0)
    out = ops.attention_decode(q_all, k, v, g["attn_q_norm"], g["attn_k_norm"], cos, sin, kc, vc, pos,
                               nh, nkv, hd, rot)
    # the reference's torch path keeps the roped q in FP32; the CUDA path rounds it to BF16
    assert torch.equal(kc, g["attn_k_cache_out"])
    assert torch.equal(vc, g["attn_v_cache_out"])
    y = ops.gemv(out, g["attn_o_proj_w"], g["attn_o_proj_s"])
    assert rel_err(y, g["attn_y"]) < 2e-2


def test_packed_argmax_key_order():
    vals = torch.tensor([1.0, -2.0, 3.0, 3.0, -0.0, 0.0], dtype=BF16)
    bits = vals.view(torch.int16).to(torch.int32) & 0xFFFF
    keys = [ops.packed_key(int(b), i) for i, b in enumerate(bits)]
    assert ops.key_to_index(max(keys)) == ops.argmax_first(vals) == 2
    # -0 and +0 tie: the lower index wins
    assert ops.packed_key(int(bits[4]), 4) > ops.packed_key(int(bits[5]), 5)


def test_scale_modes_expand():
    w = torch.randint(0, 120, (256, 384), dtype=torch.uint8)
    blk = torch.rand(2, 3)
    per_row = torch.rand(256, 1)
    per_row_blk = torch.rand(256, 3)
    assert ops.scale_mode(256, blk) == 3
    assert ops.scale_mode(256, per_row) == 1
    assert ops.scale_mode(256, per_row_blk) == -3
    d = ops.dequant(w, blk)
    assert torch.equal(d[130, 260], ops.e4m3_to_f32(w)[130, 260] * blk[1, 2])
    d = ops.dequant(w, per_row_blk)
    assert torch.equal(d[7, 200], ops.e4m3_to_f32(w)[7, 200] * per_row_blk[7, 1])
