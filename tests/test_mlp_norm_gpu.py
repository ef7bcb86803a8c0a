"""GPU parity of RMSNorm(1+w) and the fused MLP composites (layer_pre_attn,
layer_post_attn, layer_post_o_fp8_mlp, and the engine's gate/up + down)."""

import ctypes

import pytest
import torch

from oracle import ops, synth
from parity import assert_close, bf16_ulp_diff

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
BF16 = torch.bfloat16
H, I = 2560, 9216


def _p(t):
    return P(0) if t is None else P(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from qwen35_b200 import _lib
    return _lib.fused()


@pytest.mark.parametrize("rows,d", [(1, 2560), (16, 256), (4, 256), (3, 5000), (2, 100)])
def test_rmsnorm_inplace_and_out(lib, rows, d):
    g = synth.gen(rows * 31 + d)
    x = (torch.randn(rows, d, generator=g) * 3).to(BF16)
    w = torch.randn(d, generator=g) * 0.02
    ref = ops.rmsnorm(x, w)
    xd, wd = x.cuda(), w.cuda()
    out = torch.empty_like(xd)
    lib.launch_rmsnorm_out(_p(xd), _p(wd), _p(out), rows, d, 1e-6, P(0))
    lib.launch_rmsnorm_ip(_p(xd), _p(wd), rows, d, 1e-6, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), xd.cpu())
    assert float(bf16_ulp_diff(out, ref).max()) <= 1.0
    xf = x.float()
    ref32 = xf * torch.rsqrt((xf * xf).sum(-1, keepdim=True) / d + 1e-6) * (1 + w)
    assert_close(out.cpu(), ref32, what="rmsnorm")


def _mlp_weights(seed):
    g = synth.gen(seed)
    wg, sg = synth.fp8_weight(I, H, g)
    wu, su = synth.fp8_weight(I, H, g)
    wd, sd = synth.fp8_weight(H, I, g)
    return g, [(wg, sg.to(BF16)), (wu, su.to(BF16)), (wd, sd.to(BF16))]


def test_layer_post_o_fp8_mlp(lib):
    g, ((wg, sg), (wu, su), (wd, sd)) = _mlp_weights(5)
    hidden = (torch.randn(H, generator=g) * 4).to(BF16)
    o = (torch.randn(H, generator=g) * 2).to(BF16)
    nw = torch.randn(H, generator=g) * 0.02
    ref = ops.mlp_post(hidden, o, nw, wg, sg, wu, su, wd, sd)
    d = {k: v.cuda() for k, v in dict(hidden=hidden, o=o, nw=nw, wg=wg, sg=sg, wu=wu, su=su, wd=wd, sd=sd).items()}
    out = torch.empty(H, dtype=BF16, device="cuda")
    ws = torch.empty(I, dtype=BF16, device="cuda")
    gate = torch.empty(I, dtype=BF16, device="cuda")
    up = torch.empty(I, dtype=BF16, device="cuda")
    silu = torch.empty(I, dtype=BF16, device="cuda")
    lib.layer_post_o_fp8_mlp(_p(d["hidden"]), _p(d["o"]), _p(d["nw"]), _p(d["wg"]), _p(d["sg"]), I, _p(d["wu"]),
                             _p(d["su"]), I, _p(d["wd"]), _p(d["sd"]), H, _p(out), _p(ws), _p(gate), _p(up),
                             _p(silu), H, 20, 72, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    n = ref["normed"]
    g32 = ops.dequant(wg, sg) @ n.float()
    u32 = ops.dequant(wu, su) @ n.float()
    assert_close(gate.cpu(), g32, what="gate")
    assert_close(up.cpu(), u32, what="up")
    assert_close(silu.cpu(), ops.silu_f32(g32) * u32, what="silu*up")
    d32 = ops.dequant(wd, sd) @ silu.cpu().float()  # down of our own SiLU output
    assert_close(ws.cpu()[:H], d32, what="down")
    assert_close(out.cpu(), ref["h2"].float() + ws.cpu()[:H].float(), what="output")
    assert float((bf16_ulp_diff(out, ref["output"]) > 1).float().mean()) < 0.01


def test_layer_post_attn_and_pre_attn(lib):
    g, ((wg, sg), (wu, su), (wd, sd)) = _mlp_weights(6)
    wo, so = synth.fp8_weight(H, 4096, g)
    so = so.to(BF16)
    hidden = (torch.randn(H, generator=g) * 4).to(BF16)
    attn = (torch.randn(4096, generator=g)).to(BF16)
    nw = torch.randn(H, generator=g) * 0.02
    ref = ops.layer_post_attn(hidden, attn, wo, so, nw, wg, sg, wu, su, wd, sd)
    c = lambda t: t.cuda()  # noqa: E731
    out = torch.empty(H, dtype=BF16, device="cuda")
    ws = torch.empty(I, dtype=BF16, device="cuda")
    bufs = [torch.empty(I, dtype=BF16, device="cuda") for _ in range(3)]
    dh, da, dn = c(hidden), c(attn), c(nw)
    dwo, dso, dwg, dsg, dwu, dsu, dwd, dsd = map(c, (wo, so, wg, sg, wu, su, wd, sd))
    lib.layer_post_attn(_p(dh), _p(da), _p(dwo), _p(dso), H, 20, _p(dn), _p(dwg), _p(dsg), I, 72, _p(dwu), _p(dsu),
                        I, 72, _p(dwd), _p(dsd), H, 20, _p(out), _p(ws), _p(bufs[0]), _p(bufs[1]), _p(bufs[2]), H,
                        4096, 32, 20, 72, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    o32 = ops.dequant(wo, so) @ attn.float()
    h2 = (hidden.float() + o32.to(BF16).float())
    d32 = ops.dequant(wd, sd) @ bufs[2].cpu().float()
    assert_close(ws.cpu()[:H], d32, what="down")
    assert float((bf16_ulp_diff(out, ref["output"]) > 1).float().mean()) < 0.01
    assert_close(out.cpu(), h2.to(BF16).float() + ws.cpu()[:H].float(), what="output")

    # layer_pre_attn: norm_ws = RMSNorm(hidden), then q/k/v GEMVs
    wq, sq = synth.fp8_weight(8192, H, g)
    wk, sk = synth.fp8_weight(1024, H, g)
    sq, sk = sq.to(BF16), sk.to(BF16)
    q = torch.empty(8192, dtype=BF16, device="cuda")
    k = torch.empty(1024, dtype=BF16, device="cuda")
    v = torch.empty(1024, dtype=BF16, device="cuda")
    nws = torch.empty(H, dtype=BF16, device="cuda")
    dwq, dsq, dwk, dsk = map(c, (wq, sq, wk, sk))
    lib.layer_pre_attn(_p(dh), _p(dn), _p(dwq), _p(dsq), 8192, 64, _p(dwk), _p(dsk), 1024, 8, _p(dwk), _p(dsk),
                       1024, 8, _p(q), _p(k), _p(v), _p(nws), H, 20, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    xn = ops.rmsnorm(hidden, nw)
    assert float(bf16_ulp_diff(nws, xn).max()) <= 1.0
    assert_close(q.cpu(), ops.dequant(wq, sq) @ nws.cpu().float(), what="q")
    assert_close(k.cpu(), ops.dequant(wk, sk) @ nws.cpu().float(), what="k")
    assert torch.equal(k.cpu(), v.cpu())


def test_engine_mlp_entry_points(lib):
    """qwen_mlp_gate_up + qwen_linear_resid (the engine's MLP pair)."""
    g, ((wg, sg), (wu, su), (wd, sd)) = _mlp_weights(9)
    h2 = (torch.randn(H, generator=g) * 4).to(BF16)
    nw = torch.randn(H, generator=g) * 0.02
    c = lambda t: t.cuda()  # noqa: E731
    silu = torch.empty(I, dtype=BF16, device="cuda")
    out = torch.empty(H, dtype=BF16, device="cuda")
    dh2, dnw, dwg, dsg, dwu, dsu, dwd, dsd = map(c, (h2, nw, wg, sg, wu, su, wd, sd))
    assert lib.qwen_mlp_gate_up(_p(dh2), _p(dnw), 1e-6, _p(dwg), _p(dsg), _p(dwu), _p(dsu), I, H, 20, _p(silu),
                                P(0)) == 0
    assert lib.qwen_linear_resid(_p(silu), _p(dwd), _p(dsd), H, I, 72, _p(dh2), _p(out), P(0)) == 0
    torch.cuda.synchronize()
    n = ops.rmsnorm(h2, nw).float()
    g32, u32 = ops.dequant(wg, sg) @ n, ops.dequant(wu, su) @ n
    assert_close(silu.cpu(), ops.silu_f32(g32) * u32, what="silu")
    d = (ops.dequant(wd, sd) @ silu.cpu().float()).to(BF16).float()
    assert_close(out.cpu(), h2.float() + d, what="resid")
