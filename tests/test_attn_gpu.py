"""GPU parity of the full-attention decode kernels: the reference-named
launch_fused_attn_v2 / layer_mid_attn and the engine's split-KV qwen_attn_decode
(norm + RoPE + KV write + attention + sigmoid gate)."""

import ctypes
import math

import pytest
import torch

from oracle import ops, synth
from parity import assert_close, rel_l2

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
BF16, F32 = torch.bfloat16, torch.float32
NH, NKV, HD, ROT = 16, 4, 256, 64


def _p(t):
    return P(0) if t is None else P(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from qwen35_b200 import _lib
    return _lib.fused()


def attn_ref32(q, kc, vc, total, nh, nkv):
    """FP32 softmax attention of BF16 q over the first `total` cached positions."""
    grp = nh // nkv
    d = q.shape[-1]
    k = kc[:, :total].float().repeat_interleave(grp, 0)
    v = vc[:, :total].float().repeat_interleave(grp, 0)
    s = torch.einsum("hd,htd->ht", q.float() / math.sqrt(d), k)
    return torch.einsum("ht,htd->hd", torch.softmax(s, -1), v)


@pytest.mark.parametrize("hd,seq", [(256, 1), (256, 37), (256, 300), (128, 200)])
def test_fused_attn_v2(lib, hd, seq):
    g = synth.gen(seq + hd)
    max_seq = 512
    q = torch.randn(NH, hd, generator=g).to(BF16)
    kc = torch.randn(NKV, max_seq, hd, generator=g).to(BF16)
    vc = torch.randn(NKV, max_seq, hd, generator=g).to(BF16)
    out = torch.empty(NH, hd, dtype=BF16, device="cuda")
    dq, dkc, dvc = q.cuda(), kc.cuda(), vc.cuda()  # keep device copies alive across the launch
    lib.launch_fused_attn_v2(_p(dq), _p(dkc), _p(dvc), _p(out), seq, max_seq, hd, NH, NKV, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    assert_close(out.cpu(), attn_ref32(q, kc, vc, seq, NH, NKV), what=f"attn hd={hd} seq={seq}")


def test_layer_mid_attn(lib):
    g = synth.gen(77)
    max_seq, pos = 256, 100
    q = (torch.randn(NH, HD, generator=g) * 2).to(BF16)
    k = (torch.randn(NKV, HD, generator=g) * 2).to(BF16)
    v = torch.randn(NKV, HD, generator=g).to(BF16)
    qn = torch.randn(HD, generator=g) * 0.02
    kn = torch.randn(HD, generator=g) * 0.02
    kc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16)
    vc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16)
    cos, sin = ops.rope_tables(max_seq, ROT, 1e7)
    # oracle: norm + rope (bf16), cache write, attention
    qr = ops.rope_apply(ops.rmsnorm(q, qn), cos[pos], sin[pos], ROT)
    kr = ops.rope_apply(ops.rmsnorm(k, kn), cos[pos], sin[pos], ROT)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    kc_ref[:, pos], vc_ref[:, pos] = kr, v
    ref = attn_ref32(qr, kc_ref, vc_ref, pos + 1, NH, NKV)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    dkc, dvc = kc.cuda(), vc.cuda()
    out = torch.empty(NH, HD, dtype=BF16, device="cuda")
    dqn, dkn, dcos, dsin = qn.cuda(), kn.cuda(), cos.cuda(), sin.cuda()
    lib.layer_mid_attn(_p(dq), _p(dk), _p(dv), _p(out), _p(dqn), _p(dkn), _p(dcos),
                       _p(dsin), _p(dkc), _p(dvc), pos, pos, pos + 1, max_seq, HD, ROT, NH, NKV, P(0))
    assert lib.qwen_last_error() == 0
    torch.cuda.synchronize()
    assert rel_l2(dq, qr) < 4e-3
    assert rel_l2(dkc, kc_ref) < 4e-3
    assert torch.equal(dvc.cpu(), vc_ref)
    assert_close(out.cpu(), ref, what="layer_mid_attn")


@pytest.mark.parametrize("pos,chunk,max_seq", [(0, 32, 1088), (5, 32, 1088), (299, 32, 1088), (299, 300, 1088),
                                               (1000, 64, 1088), (8191, 128, 8192 + 128)])
def test_engine_attn_decode(lib, pos, chunk, max_seq):
    """qwen_attn_decode == oracle.ops.attention_decode (gated output), up to the
    8192-token context of BASELINE config 4 with the engine's split (64 x 128)."""
    g = synth.gen(pos * 3 + chunk)
    nsplit = math.ceil(max_seq / chunk)
    q_all = (torch.randn(NH * 2 * HD, generator=g) * 2).to(BF16)
    k = (torch.randn(NKV * HD, generator=g) * 2).to(BF16)
    v = torch.randn(NKV * HD, generator=g).to(BF16)
    qn = torch.randn(HD, generator=g) * 0.02
    kn = torch.randn(HD, generator=g) * 0.02
    kc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16)
    vc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16)
    cos, sin = ops.rope_tables(max_seq, ROT, 1e7)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    ref = ops.attention_decode(q_all, k, v, qn, kn, cos, sin, kc_ref, vc_ref, pos, NH, NKV, HD, ROT)
    # FP32 version of the same: reuse the oracle's normalised/roped values
    qh = q_all.reshape(NH, 2 * HD)
    qr = ops.rope_apply(ops.rmsnorm(qh[:, :HD], qn), cos[pos], sin[pos], ROT)
    o32 = attn_ref32(qr, kc_ref, vc_ref, pos + 1, NH, NKV)
    gate = ops.sigmoid_bf16(qh[:, HD:]).float()
    ref32 = o32.to(BF16).float() * gate

    dkc, dvc = kc.cuda(), vc.cuda()
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    ws = torch.empty(NH * nsplit * (HD + 2), dtype=F32, device="cuda")
    cnt = torch.zeros(NKV, dtype=torch.int32, device="cuda")
    out = torch.empty(NH * HD, dtype=BF16, device="cuda")
    dqa, dk, dv, dqn, dkn, dcos, dsin = (t.cuda() for t in (q_all, k, v, qn, kn, cos, sin))
    for _ in range(2):  # twice: the split counters must reset themselves
        st = lib.qwen_attn_decode(_p(dqa), _p(dk), _p(dv), _p(dqn), _p(dkn), _p(dcos), _p(dsin), _p(dkc), _p(dvc),
                                  _p(posd), max_seq, NH, NKV, HD, ROT, 1e-6, chunk, nsplit, _p(ws), _p(cnt), _p(out),
                                  P(0))
        assert st == 0
    torch.cuda.synchronize()
    assert int(cnt.abs().sum()) == 0
    assert torch.equal(dvc.cpu(), vc_ref)
    assert rel_l2(dkc, kc_ref) < 4e-3
    assert_close(out.cpu(), ref32, max_rel_err=8e-3, rel_l2_err=4e-3, min_cos=0.9999,
                 what=f"engine attn pos={pos}")
    assert rel_l2(out, ref) < 4e-3


def test_engine_attn_decode_rejects_position_past_cache(lib):
    """A device-side position at or past max_seq is refused by the kernel's own
    check: nothing is read or written and the device error word says why."""
    from qwen35_b200 import _lib
    max_seq, chunk = 64, 32
    nsplit = 2
    g = synth.gen(5)
    q_all = torch.randn(NH * 2 * HD, generator=g).to(BF16).cuda()
    k = torch.randn(NKV * HD, generator=g).to(BF16).cuda()
    v = torch.randn(NKV * HD, generator=g).to(BF16).cuda()
    qn = torch.zeros(HD).cuda()
    kc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16).cuda()
    vc = torch.randn(NKV, max_seq, HD, generator=g).to(BF16).cuda()
    kc0, vc0 = kc.clone(), vc.clone()
    cos, sin = (t.cuda() for t in ops.rope_tables(max_seq, ROT, 1e7))
    posd = torch.tensor([max_seq], dtype=torch.int32, device="cuda")
    ws = torch.empty(NH * nsplit * (HD + 2), dtype=F32, device="cuda")
    cnt = torch.zeros(NKV, dtype=torch.int32, device="cuda")
    out = torch.zeros(NH * HD, dtype=BF16, device="cuda")
    assert _lib.device_error() == 0
    st = lib.qwen_attn_decode(_p(q_all), _p(k), _p(v), _p(qn), _p(qn), _p(cos), _p(sin), _p(kc), _p(vc), _p(posd),
                              max_seq, NH, NKV, HD, ROT, 1e-6, chunk, nsplit, _p(ws), _p(cnt), _p(out), P(0))
    torch.cuda.synchronize()
    assert st == 0
    assert _lib.device_error() == 5  # ERR_POS_RANGE (read and cleared)
    assert torch.equal(kc, kc0) and torch.equal(vc, vc0)
    assert int(cnt.abs().sum()) == 0 and float(out.float().abs().sum()) == 0.0
