"""The allocation-free attention decode entry point (qwen_attn_decode_noalloc).

It exists for callers that cannot allocate device memory where they run the
decode step -- a runtime whose memory pool owns the whole GPU, a foreign
language binding with no device allocator, code that must not cause the
implicit synchronisation of an allocation -- and takes its split-KV scratch
from a fixed 4 MiB array inside libqwen_fused.so instead of caller buffers.

Checked here through the C ABI: calls in a row (the same layout twice with
another head layout and split count between them, and a single-split call)
give the same output and KV-cache update as the allocating qwen_attn_decode
on the same inputs, stay within the attention tolerance of the CPU oracle and
leave torch's device allocation count unchanged; a request larger than the
array is refused without touching the output.  This
file is collected last so a failure here never hides another test's result.
"""

import ctypes
import math

import pytest
import torch

from oracle import ops, synth
from parity import rel_l2

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
I = ctypes.c_int
BF16, F32 = torch.bfloat16, torch.float32
NH, NKV, HD, ROT = 16, 4, 256, 64


def _p(t):
    return P(0) if t is None else P(t.data_ptr())


@pytest.fixture(scope="module")
def lib():
    from qwen35_b200 import _lib
    lib = _lib.fused()
    fn = lib.qwen_attn_decode_noalloc
    fn.restype = I
    fn.argtypes = [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, ctypes.c_float, I, I, P, P]
    return lib


def _inputs(seed, max_seq, nh=NH, nkv=NKV):
    g = synth.gen(seed)
    q_all = (torch.randn(nh * 2 * HD, generator=g) * 2).to(BF16)
    k = (torch.randn(nkv * HD, generator=g) * 2).to(BF16)
    v = torch.randn(nkv * HD, generator=g).to(BF16)
    qn = torch.randn(HD, generator=g) * 0.02
    kn = torch.randn(HD, generator=g) * 0.02
    kc = torch.randn(nkv, max_seq, HD, generator=g).to(BF16)
    vc = torch.randn(nkv, max_seq, HD, generator=g).to(BF16)
    return q_all, k, v, qn, kn, kc, vc


def _call_pair(lib, seed, pos, max_seq, chunk, nsplit, nh, nkv, dcos, dsin, cos, sin):
    """One call of each entry point on the same inputs; returns the outputs,
    the two updated caches and the oracle's output and caches."""
    q_all, k, v, qn, kn, kc, vc = _inputs(seed, max_seq, nh, nkv)
    dq, dk, dv, dqn, dkn = (t.cuda() for t in (q_all, k, v, qn, kn))
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    # existing entry point with caller-provided scratch
    kc_a, vc_a = kc.cuda(), vc.cuda()
    ws = torch.empty(nh * nsplit * (HD + 2), dtype=F32, device="cuda")
    cnt = torch.zeros(nkv, dtype=torch.int32, device="cuda")
    out_a = torch.empty(nh * HD, dtype=BF16, device="cuda")
    assert lib.qwen_attn_decode(_p(dq), _p(dk), _p(dv), _p(dqn), _p(dkn), _p(dcos), _p(dsin), _p(kc_a),
                                _p(vc_a), _p(posd), max_seq, nh, nkv, HD, ROT, 1e-6, chunk, nsplit, _p(ws),
                                _p(cnt), _p(out_a), P(0)) == 0
    # allocation-free entry point: nothing may be allocated on the device
    kc_b, vc_b = kc.cuda(), vc.cuda()
    out_b = torch.full((nh * HD,), 9.0, dtype=BF16, device="cuda")
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    assert lib.qwen_attn_decode_noalloc(_p(dq), _p(dk), _p(dv), _p(dqn), _p(dkn), _p(dcos), _p(dsin), _p(kc_b),
                                        _p(vc_b), _p(posd), max_seq, nh, nkv, HD, ROT, 1e-6, chunk, nsplit,
                                        _p(out_b), P(0)) == 0
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    kc_r, vc_r = kc.clone(), vc.clone()
    ref = ops.attention_decode(q_all, k, v, qn, kn, cos, sin, kc_r, vc_r, pos, nh, nkv, HD, ROT)
    return out_a.cpu(), out_b.cpu(), (kc_a.cpu(), vc_a.cpu()), (kc_b.cpu(), vc_b.cpu()), ref, (kc_r, vc_r)


def test_noalloc_matches_allocating_entry_point_on_two_calls(lib):
    """Two identical calls with a different head layout and split count in
    between (the counters then sit where the previous call kept partials),
    and a single-split call: every output is bit-equal to qwen_attn_decode's
    and within the attention tolerance of the oracle."""
    max_seq, chunk = 1024, 32
    cos, sin = ops.rope_tables(max_seq, ROT, 1e7)
    dcos, dsin = cos.cuda(), sin.cuda()
    cases = [  # (seed, pos, chunk, nsplit, n_heads, n_kv_heads)
        (100, 299, chunk, math.ceil(max_seq / chunk), NH, NKV),
        (101, 777, 64, 16, 8, 2),
        (100, 299, chunk, math.ceil(max_seq / chunk), NH, NKV),
        (102, 500, max_seq, 1, NH, NKV),
    ]
    outs = []
    for call, (seed, pos, ch, nsplit, nh, nkv) in enumerate(cases):
        out_a, out_b, caches_a, caches_b, ref, caches_r = _call_pair(lib, seed, pos, max_seq, ch, nsplit, nh, nkv,
                                                                     dcos, dsin, cos, sin)
        assert torch.equal(out_b, out_a), f"call {call}"
        assert torch.equal(caches_b[0], caches_a[0]) and torch.equal(caches_b[1], caches_a[1])
        assert torch.equal(caches_b[1], caches_r[1])
        assert rel_l2(out_b, ref) < 4e-3, f"call {call} vs oracle"
        outs.append(out_b)
    assert torch.equal(outs[0], outs[2])  # the same call again, after another layout


def test_noalloc_rejects_scratch_beyond_its_limit(lib):
    max_seq = 8192
    chunk, nsplit = 1, 8192  # 16 * 8192 * 258 * 4 bytes of partials: far above 4 MiB
    q_all, k, v, qn, kn, kc, vc = _inputs(7, max_seq)
    cos, sin = ops.rope_tables(max_seq, ROT, 1e7)
    dq, dk, dv, dqn, dkn, dcos, dsin = (t.cuda() for t in (q_all, k, v, qn, kn, cos, sin))
    dkc, dvc = kc.cuda(), vc.cuda()
    posd = torch.tensor([5], dtype=torch.int32, device="cuda")
    out = torch.full((NH * HD,), 9.0, dtype=BF16, device="cuda")
    st = lib.qwen_attn_decode_noalloc(_p(dq), _p(dk), _p(dv), _p(dqn), _p(dkn), _p(dcos), _p(dsin), _p(dkc),
                                      _p(dvc), _p(posd), max_seq, NH, NKV, HD, ROT, 1e-6, chunk, nsplit, _p(out),
                                      P(0))
    assert st != 0
    assert lib.qwen_last_error() != 0
    torch.cuda.synchronize()
    assert bool((out.float() == 9.0).all())
    assert torch.equal(dkc.cpu(), kc)
