"""Generate golden vectors by running the reference's own CUDA kernels.

The kernels are the reference sources compiled unmodified for sm_100a by
``oracle/Makefile`` into ``oracle/_ref``.  Run on a GPU machine:

    python tests/golden/make_golden_gpu.py --out gpu_golden.safetensors

Inputs are seeded on the CPU; every output is produced by a reference launcher
called through ctypes with the argtypes of main.py.  The file is committed as
``tests/golden/gpu_golden.safetensors`` and checked on the CPU by
``tests/test_oracle_golden_gpu_ref.py`` (oracle vs reference kernels).
"""

from __future__ import annotations

import argparse
import ctypes
import os

import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.path.join(REPO, "oracle", "_ref")
P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
BF16 = torch.bfloat16


def fp8(n, k, g):
    w = (torch.randn(n, k, generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    s = torch.pow(10.0, torch.rand((n + 127) // 128, (k + 127) // 128, generator=g) * 2 - 4).to(BF16)
    return w.contiguous(), s.contiguous()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "gpu_golden.safetensors"))
    args = ap.parse_args()
    fused = ctypes.CDLL(os.path.join(REF, "libref_fused.so"))
    fp8lib = ctypes.CDLL(os.path.join(REF, "libref_fp8.so"))
    fused.launch_gemv_v4_extern.argtypes = [P, P, P, P, I, I, I, P]
    fp8lib.fp8_gemm_batch.argtypes = [P, P, P, P, I, I, I, I, P]
    fused.launch_rmsnorm_ip.argtypes = [P, P, I, I, F, P]
    fused.layer_post_o_fp8_mlp.argtypes = [P, P, P, P, P, I, P, P, I, P, P, I, P, P, P, P, P, I, I, I, P]
    fused.launch_delta_rule_decode.argtypes = [P, P, P, P, P, P, P, I, I, P]
    fused.launch_prepare_linear_gates.argtypes = [P, P, P, P, P, P, I, P]
    fused.launch_rmsnorm_gated_decode.argtypes = [P, P, P, P, I, I, F, P]
    fused.layer_mid_attn.argtypes = [P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, P]
    g = torch.Generator().manual_seed(4321)
    out = {}
    keep = []  # device copies must outlive the asynchronous launches that read them

    def c(t):
        d = t.cuda().contiguous()
        keep.append(d)
        return d

    p = lambda t: P(t.data_ptr())  # noqa: E731

    # GEMV in the three scale modes
    n, k = 256, 512
    x = torch.randn(k, generator=g).to(BF16)
    w, s_blk = fp8(n, k, g)
    s_row = torch.pow(10.0, torch.rand(n, 1, generator=g) * 2 - 4).to(BF16)
    s_rb = torch.pow(10.0, torch.rand(n, k // 128, generator=g) * 2 - 4).to(BF16)
    out.update(gemv_x=x, gemv_w=w, gemv_s_blk=s_blk, gemv_s_row=s_row, gemv_s_rb=s_rb)
    for name, s, kb in (("blk", s_blk, k // 128), ("row", s_row, 1), ("rb", s_rb, -(k // 128))):
        y = torch.empty(n, dtype=BF16, device="cuda")
        xd, wd, sd = c(x), c(w), c(s)
        fused.launch_gemv_v4_extern(p(xd), p(wd), p(sd), p(y), n, k, kb, None)
        torch.cuda.synchronize()
        out[f"gemv_y_{name}"] = y.cpu()

    # batched GEMM
    xm = torch.randn(3, k, generator=g).to(BF16)
    ym = torch.empty(3, n, dtype=BF16, device="cuda")
    xmd, wd, sd = c(xm), c(w), c(s_blk)
    fp8lib.fp8_gemm_batch(p(xmd), p(wd), p(sd), p(ym), 3, n, k, k // 128, None)
    torch.cuda.synchronize()
    out.update(gemm_x=xm, gemm_y=ym.cpu())

    # RMSNorm(1+w) in place
    xr = (torch.randn(4, 256, generator=g) * 3).to(BF16)
    wr = torch.randn(256, generator=g) * 0.02
    xrd = c(xr)
    fused.launch_rmsnorm_ip(p(xrd), p(c(wr)), 4, 256, 1e-6, None)
    torch.cuda.synchronize()
    out.update(rms_x=xr, rms_w=wr, rms_y=xrd.cpu())

    # MLP composite
    H, Im = 256, 512
    wg, sg = fp8(Im, H, g)
    wu, su = fp8(Im, H, g)
    wdn, sdn = fp8(H, Im, g)
    hid = (torch.randn(H, generator=g) * 2).to(BF16)
    o = torch.randn(H, generator=g).to(BF16)
    nw = torch.randn(H, generator=g) * 0.02
    bufs = {nm: torch.empty(sz, dtype=BF16, device="cuda") for nm, sz in
            (("output", H), ("ws", Im), ("gate", Im), ("up", Im), ("silu", Im))}
    dev = [c(t) for t in (hid, o, nw, wg, sg, wu, su, wdn, sdn)]
    fused.layer_post_o_fp8_mlp(p(dev[0]), p(dev[1]), p(dev[2]), p(dev[3]), p(dev[4]), Im, p(dev[5]), p(dev[6]), Im,
                               p(dev[7]), p(dev[8]), H, p(bufs["output"]), p(bufs["ws"]), p(bufs["gate"]),
                               p(bufs["up"]), p(bufs["silu"]), H, H // 128, Im // 128, None)
    torch.cuda.synchronize()
    out.update(mlp_hidden=hid, mlp_o=o, mlp_nw=nw, mlp_wg=wg, mlp_sg=sg, mlp_wu=wu, mlp_su=su, mlp_wd=wdn,
               mlp_sd=sdn)
    out.update({f"mlp_{nm}": t.cpu() for nm, t in bufs.items()})
    out["mlp_ws"] = out["mlp_ws"][:H].clone()

    # delta rule decode
    hh, D = 2, 128
    q = torch.randn(hh, D, generator=g).to(BF16)
    kk = torch.randn(hh, D, generator=g).to(BF16)
    v = (torch.randn(hh, D, generator=g) * 2).to(BF16)
    gg = -torch.rand(hh, generator=g) * 2
    beta = torch.rand(hh, generator=g).to(BF16)
    st = torch.randn(hh, D, D, generator=g) * 0.1
    std = c(st)
    od = torch.empty(hh, D, dtype=BF16, device="cuda")
    fused.launch_delta_rule_decode(p(c(q)), p(c(kk)), p(c(v)), p(c(gg)), p(c(beta)), p(std), p(od), hh, D, None)
    torch.cuda.synchronize()
    out.update(delta_q=q, delta_k=kk, delta_v=v, delta_g=gg, delta_beta=beta, delta_state_in=st,
               delta_state_out=std.cpu(), delta_out=od.cpu())

    # gates and gated norm
    hv = 32
    a = (torch.randn(hv, generator=g) * 4).to(BF16)
    b = (torch.randn(hv, generator=g) * 3).to(BF16)
    alog = torch.log(torch.rand(hv, generator=g) * 15 + 1)
    dt = torch.ones(hv)
    go = torch.empty(hv, device="cuda")
    bo = torch.empty(hv, dtype=BF16, device="cuda")
    fused.launch_prepare_linear_gates(p(c(a)), p(c(b)), p(c(alog)), p(c(dt)), p(go), p(bo), hv, None)
    core = (torch.randn(4, D, generator=g) * 2).to(BF16)
    z = (torch.randn(4, D, generator=g) * 2).to(BF16)
    nwg = (1 + torch.randn(D, generator=g) * 0.02).to(BF16)
    gn = torch.empty(4, D, dtype=BF16, device="cuda")
    fused.launch_rmsnorm_gated_decode(p(c(core)), p(c(z)), p(c(nwg)), p(gn), 4, D, 1e-6, None)
    torch.cuda.synchronize()
    out.update(gates_a=a, gates_b=b, gates_alog=alog, gates_dt=dt, gates_g=go.cpu(), gates_beta=bo.cpu(),
               gn_core=core, gn_z=z, gn_w=nwg, gn_out=gn.cpu())

    # full attention: Q/K norm + partial RoPE + KV write + attention (layer_mid_attn)
    nh, nkv, hd, rot, max_seq, pos = 4, 1, 256, 64, 8, 5
    qa = (torch.randn(nh, hd, generator=g) * 2).to(BF16)
    ka = (torch.randn(nkv, hd, generator=g) * 2).to(BF16)
    va = torch.randn(nkv, hd, generator=g).to(BF16)
    qn = torch.randn(hd, generator=g) * 0.02
    kn = torch.randn(hd, generator=g) * 0.02
    kc = torch.randn(nkv, max_seq, hd, generator=g).to(BF16)
    vc = torch.randn(nkv, max_seq, hd, generator=g).to(BF16)
    inv = 1.0 / (1e7 ** (torch.arange(0, rot, 2).float() / rot))
    fr = torch.outer(torch.arange(max_seq).float(), inv)
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos().contiguous(), emb.sin().contiguous()
    qad, kad, kcd, vcd = c(qa), c(ka), c(kc), c(vc)
    ao = torch.empty(nh, hd, dtype=BF16, device="cuda")
    fused.layer_mid_attn(p(qad), p(kad), p(c(va)), p(ao), p(c(qn)), p(c(kn)), p(c(cos)), p(c(sin)), p(kcd),
                         p(vcd), pos, pos, pos + 1, max_seq, hd, rot, nh, nkv, None)
    torch.cuda.synchronize()
    out.update(attn_q=qa, attn_k=ka, attn_v=va, attn_qn=qn, attn_kn=kn, attn_kc_in=kc, attn_vc_in=vc,
               attn_cos=cos, attn_sin=sin, attn_q_out=qad.cpu(), attn_kc_out=kcd.cpu(), attn_vc_out=vcd.cpu(),
               attn_out=ao.cpu(), attn_meta=torch.tensor([nh, nkv, hd, rot, max_seq, pos], dtype=torch.int32))

    out = {kk_: vv.contiguous() for kk_, vv in out.items()}
    save_file(out, args.out)
    print(f"wrote {args.out}: {len(out)} tensors, {sum(t.numel() * t.element_size() for t in out.values())} bytes")


if __name__ == "__main__":
    main()
