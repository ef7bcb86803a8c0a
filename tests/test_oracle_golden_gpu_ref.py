"""The CPU oracle against golden vectors produced by the reference's own CUDA
kernels (compiled unmodified for sm_100a into oracle/_ref and run on a B200 by
tests/golden/make_golden_gpu.py).  Pins the oracle's restatement of
gemv_v4_kernel (three scale modes), fp8_gemm_batch, rmsnorm_ip_kernel,
layer_post_o_fp8_mlp, delta_rule_decode_kernel, prepare_linear_gates_kernel,
rmsnorm_gated_decode_kernel and layer_mid_attn to the reference's outputs.

Tolerances: FP32 oracle values vs the reference's BF16 outputs use the GEMV
bar (max relative error 2e-3, cosine 0.99999); BF16 elementwise results may
differ by one BF16 rounding.
"""

import math
import os

import pytest
import torch
from safetensors.torch import load_file

from conftest import GOLDEN
from oracle import ops
from parity import assert_close, bf16_ulp_diff, max_rel, rel_l2

BF16 = torch.bfloat16
PATH = os.path.join(GOLDEN, "gpu_golden.safetensors")

pytestmark = pytest.mark.skipif(not os.path.exists(PATH), reason="reference-kernel fixture not generated yet")


@pytest.fixture(scope="module")
def gold():
    return load_file(PATH)


@pytest.mark.parametrize("mode", ["blk", "row", "rb"])
def test_gemv_scale_modes(gold, mode):
    s = gold[f"gemv_s_{mode}"]
    y32 = ops.dequant(gold["gemv_w"], s) @ gold["gemv_x"].float()
    assert_close(gold[f"gemv_y_{mode}"], y32, what=f"gemv {mode}")


def test_gemm_batch(gold):
    y32 = gold["gemm_x"].float() @ ops.dequant(gold["gemv_w"], gold["gemv_s_blk"]).T
    assert_close(gold["gemm_y"], y32, what="fp8_gemm_batch")


def test_rmsnorm(gold):
    y = ops.rmsnorm(gold["rms_x"], gold["rms_w"])
    assert float(bf16_ulp_diff(y, gold["rms_y"]).max()) <= 1.0


def test_mlp_composite(gold):
    g = gold
    r = ops.mlp_post(g["mlp_hidden"], g["mlp_o"], g["mlp_nw"], g["mlp_wg"], g["mlp_sg"], g["mlp_wu"], g["mlp_su"],
                     g["mlp_wd"], g["mlp_sd"])
    n = r["normed"].float()
    g32 = ops.dequant(g["mlp_wg"], g["mlp_sg"]) @ n
    u32 = ops.dequant(g["mlp_wu"], g["mlp_su"]) @ n
    assert_close(g["mlp_gate"], g32, what="gate")
    assert_close(g["mlp_up"], u32, what="up")
    assert_close(g["mlp_silu"], ops.silu_f32(g32) * u32, what="silu")
    d32 = ops.dequant(g["mlp_wd"], g["mlp_sd"]) @ g["mlp_silu"].float()
    assert_close(g["mlp_ws"], d32, what="down")
    assert float((bf16_ulp_diff(r["output"], g["mlp_output"]) > 1).float().mean()) < 0.01


def test_delta_rule(gold):
    g = gold
    o, s = ops.delta_rule_decode(g["delta_q"], g["delta_k"], g["delta_v"], g["delta_g"], g["delta_beta"],
                                 g["delta_state_in"])
    assert max_rel(s, g["delta_state_out"]) < 1e-5
    assert rel_l2(o, g["delta_out"]) < 4e-3


def test_gates_and_gated_norm(gold):
    g = gold
    gg, beta = ops.linear_gates(g["gates_a"], g["gates_b"], g["gates_alog"], g["gates_dt"])
    assert max_rel(gg, g["gates_g"]) < 1e-5
    assert torch.equal(beta, g["gates_beta"])
    cf = g["gn_core"].float()
    ref32 = cf * torch.rsqrt((cf * cf).mean(-1, keepdim=True) + 1e-6) * g["gn_w"].float() * ops.silu_f32(
        g["gn_z"].float())
    assert_close(g["gn_out"], ref32, what="gated norm")


def test_layer_mid_attn(gold):
    g = gold
    nh, nkv, hd, rot, max_seq, pos = [int(v) for v in g["attn_meta"]]
    qr = ops.rope_apply(ops.rmsnorm(g["attn_q"], g["attn_qn"]), g["attn_cos"][pos], g["attn_sin"][pos], rot)
    kr = ops.rope_apply(ops.rmsnorm(g["attn_k"], g["attn_kn"]), g["attn_cos"][pos], g["attn_sin"][pos], rot)
    assert float(bf16_ulp_diff(qr, g["attn_q_out"]).max()) <= 1.0
    kc, vc = g["attn_kc_in"].clone(), g["attn_vc_in"].clone()
    kc[:, pos], vc[:, pos] = kr, g["attn_v"]
    assert rel_l2(kc, g["attn_kc_out"]) < 4e-3
    assert torch.equal(vc, g["attn_vc_out"])
    grp = nh // nkv
    k = g["attn_kc_out"][:, :pos + 1].float().repeat_interleave(grp, 0)
    v = g["attn_vc_out"][:, :pos + 1].float().repeat_interleave(grp, 0)
    sc = torch.einsum("hd,htd->ht", g["attn_q_out"].float() / math.sqrt(hd), k)
    ref32 = torch.einsum("ht,htd->hd", torch.softmax(sc, -1), v)
    assert_close(g["attn_out"], ref32, what="attention")
