"""The reference's default batch-1 decode step, re-driven on the GPU through
the reference's own CUDA kernels (test infrastructure only: a checker).

``QwenEngineFP8Opt.forward`` with one token (main.py:1569-1604) runs
``_decode_step`` (main.py:1509-1547).  For a block-FP8 checkpoint the
per-layer fused path is opt-in (``QWEN_NATIVE_FP8_FUSED``, main.py:343-345),
so by default every layer takes the generic branch (main.py:1518-1541).  This
class replays that branch operation for operation:

=========  ==================================================  =====================
layer in   ``ws = hidden``; ``rmsnorm_ip_kernel(ws)``           main.py:1521-1524, 925-931
full       ``gemv_v4`` q / k / v; ``layer_mid_attn`` (q/k norm, main.py:981-1062
           partial RoPE, KV write, attention); ``out *
           bf16(sigmoid(gate))``; ``gemv_v4`` o_proj
linear     ``gemv_v4`` qkv / a / b / z; conv1d update + SiLU;   main.py:1064-1163
           ``beta = sigmoid(b)``, ``g = -exp(A_log) *
           softplus(a + dt_bias)``; q / k repeated per value
           head; ``delta_rule_decode_kernel``; RMSNormGated;
           ``gemv_v4`` out_proj
layer out  ``layer_post_o_fp8_mlp`` (residual add, RMSNorm,     main.py:1531-1533, 1238-1261
           fused gate/up + SiLU, down, residual add)
final      ``rmsnorm_ip_kernel(norm_f)``; ``gemv_v4`` LM head;  main.py:1596-1603
           first-index argmax
=========  ==================================================  =====================

Every CUDA kernel comes from ``oracle/_ref/libref_fused.so``: the reference's
``fused_kernels.cu`` compiled unmodified for sm_100a by ``oracle/Makefile``.
The torch operations main.py runs between those calls (conv1d update, gates,
gated norm, output gate) are the oracle's restatements in ``oracle.ops``,
evaluated on CUDA tensors.  The rotary tables are built on the device with
main.py:525-533's formula.

Weights use the dict layout of ``qwen35_b200.weights`` (the reference's key
names); the LM head must be block-FP8 (the BF16 head is ``F.linear``).
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import ops

BF16 = torch.bfloat16
F32 = torch.float32
P = ctypes.c_void_p
I = ctypes.c_int

REF_LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")

# argtypes of the reference entry points used here (fused_kernels.cu:940-1356)
_ARGTYPES = {
    "launch_gemv_v4_extern": [P, P, P, P, I, I, I, P],                       # :1328
    "launch_rmsnorm_ip": [P, P, I, I, ctypes.c_float, P],                     # :1055
    "launch_delta_rule_decode": [P, P, P, P, P, P, P, I, I, P],               # :967
    "layer_mid_attn": [P, P, P, P, P, P, P, P, P, P] + [I] * 7 + [P],         # :1224
    "layer_post_o_fp8_mlp": [P, P, P, P, P, I, P, P, I, P, P, I, P, P, P, P, P, I, I, I, P],  # :1156
}


def load_reference_lib(path: str | None = None):
    """ctypes handle of the reference kernels built into oracle/_ref."""
    path = path or os.path.join(REF_LIB_DIR, "libref_fused.so")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} (build it with oracle/Makefile)")
    lib = ctypes.CDLL(path)
    for name, at in _ARGTYPES.items():
        fn = getattr(lib, name)
        fn.argtypes = at
        fn.restype = None
    return lib


def _p(t: torch.Tensor) -> P:
    return P(t.data_ptr())


def _kblk(w_u8: torch.Tensor, scale: torch.Tensor) -> int:
    """The K_blk argument fp8_linear passes (main.py:249-251)."""
    return ops.scale_mode(w_u8.shape[0], scale)


class ReferenceKernelEngine:
    """Batch-1 greedy decode with the reference's decode semantics and kernels.

    ``step(token)`` feeds one token at the current position and returns
    (BF16 logits [V], first-index argmax), like ``oracle.model.OracleModel``.
    """

    def __init__(self, cfg, weights, max_seq: int, device="cuda", lib=None):
        self.cfg = cfg
        self.w = weights
        self.max_seq = max_seq
        self.dev = torch.device(device)
        self.lib = lib or load_reference_lib()
        if not isinstance(weights["lm_head"], tuple):
            raise NotImplementedError("the reference's BF16 LM head is F.linear, not a reference kernel")
        self.rot = int(cfg.head_dim * cfg.partial_rotary_factor)
        # main.py:525-533, on the device as the reference builds them
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, self.rot, 2, device=self.dev).float() / self.rot))
        pos = torch.arange(max_seq, device=self.dev).float()
        freqs = torch.outer(pos, inv)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.cos, self.sin = emb.cos().contiguous(), emb.sin().contiguous()
        H = cfg.hidden_size
        e = lambda n, dt=BF16: torch.empty(n, dtype=dt, device=self.dev)  # noqa: E731
        self.ws = e(H)
        self.res = e(H)
        self.hidden = e(H)
        self.o_buf = e(H)
        I_ = cfg.intermediate_size
        self.gate_buf, self.up_buf, self.silu_buf = e(I_), e(I_), e(I_)
        self.attn_buf = e(cfg.num_attention_heads * cfg.head_dim)
        self.delta_out = e(cfg.linear_num_value_heads * cfg.linear_value_head_dim)
        self.reset()

    def reset(self):
        cfg = self.cfg
        self.pos = 0
        self.k_cache, self.v_cache, self.conv, self.state = {}, {}, {}, {}
        conv_dim = 2 * cfg.linear_num_key_heads * cfg.linear_key_head_dim \
            + cfg.linear_num_value_heads * cfg.linear_value_head_dim
        for i, lt in enumerate(cfg.layer_types):
            if lt == "full_attention":
                shape = (cfg.num_key_value_heads, self.max_seq, cfg.head_dim)
                self.k_cache[i] = torch.zeros(shape, dtype=BF16, device=self.dev)
                self.v_cache[i] = torch.zeros(shape, dtype=BF16, device=self.dev)
            else:
                self.conv[i] = torch.zeros(conv_dim, cfg.linear_conv_kernel_dim, dtype=BF16, device=self.dev)
                self.state[i] = torch.zeros(cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                                            cfg.linear_value_head_dim, dtype=F32, device=self.dev)

    # -- reference kernels ---------------------------------------------------
    def gemv(self, x: torch.Tensor, w_u8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
        """fp8_linear's M == 1 branch (main.py:242-268): launch_gemv_v4_extern."""
        x = x.reshape(-1).contiguous()
        y = torch.empty(w_u8.shape[0], dtype=BF16, device=self.dev)
        self.lib.launch_gemv_v4_extern(_p(x), _p(w_u8), _p(scale), _p(y), w_u8.shape[0], w_u8.shape[1],
                                       _kblk(w_u8, scale), P(0))
        return y

    def rmsnorm_ip(self, x: torch.Tensor, w_f32: torch.Tensor, rows: int = 1):
        """QwenEngineFP8Opt.rmsnorm's decode branch (main.py:925-931)."""
        self.lib.launch_rmsnorm_ip(_p(x), _p(w_f32), rows, x.numel() // rows, ctypes.c_float(self.cfg.rms_norm_eps),
                                   P(0))
        return x

    # -- layers ----------------------------------------------------------------
    def _full(self, h, ly, i):
        cfg = self.cfg
        D, nh, nkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        q_all = self.gemv(h, *ly["q_proj"])
        k = self.gemv(h, *ly["k_proj"])
        v = self.gemv(h, *ly["v_proj"])
        qg = q_all.view(nh, 2 * D)
        q = qg[:, :D].contiguous()  # q_flat (main.py:1011)
        gate = qg[:, D:].reshape(-1)
        self.lib.layer_mid_attn(_p(q), _p(k), _p(v), _p(self.attn_buf), _p(ly["q_norm"]), _p(ly["k_norm"]),
                                _p(self.cos), _p(self.sin), _p(self.k_cache[i]), _p(self.v_cache[i]),
                                self.pos, self.pos, self.pos + 1, self.max_seq, D, self.rot, nh, nkv, P(0))
        out = self.attn_buf[:nh * D]
        gated = (out.float() * ops.sigmoid_bf16(gate).float()).to(BF16)  # main.py:1059
        return self.gemv(gated, *ly["o_proj"])

    def _linear(self, h, ly, i):
        cfg = self.cfg
        kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
        vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
        hv, dk = cfg.linear_num_value_heads, cfg.linear_key_head_dim
        mixed = self.gemv(h, *ly["in_proj_qkv"])
        a = self.gemv(h, *ly["in_proj_a"])
        b = self.gemv(h, *ly["in_proj_b"])
        z = self.gemv(h, *ly["in_proj_z"])
        conv_out, self.conv[i] = ops.conv1d_update(mixed, self.conv[i], ly["conv1d_w"])
        q, k, v = torch.split(conv_out, [kd, kd, vd])
        g, beta = ops.linear_gates(a, b, ly["A_log"], ly["dt_bias"])
        rep = hv // cfg.linear_num_key_heads
        q = q.reshape(cfg.linear_num_key_heads, -1).repeat_interleave(rep, 0).contiguous()
        k = k.reshape(cfg.linear_num_key_heads, -1).repeat_interleave(rep, 0).contiguous()
        v = v.reshape(hv, -1).contiguous()
        g = g.contiguous()
        beta = beta.contiguous()
        self.lib.launch_delta_rule_decode(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(self.state[i]),
                                          _p(self.delta_out), hv, cfg.linear_value_head_dim, P(0))
        core = self.delta_out.view(hv, dk)
        gated = ops.rmsnorm_gated(core, z.reshape(hv, -1), ly["norm_w"], 1e-6)  # main.py:1152-1159
        return self.gemv(gated.reshape(-1), *ly["out_proj"])

    def _post(self, o_out, ly):
        """_mixed_post_o_fp8_mlp (main.py:1238-1261) -> layer_post_o_fp8_mlp."""
        (wg, sg), (wu, su), (wd, sd) = ly["gate_proj"], ly["up_proj"], ly["down_proj"]
        self.lib.layer_post_o_fp8_mlp(_p(self.res), _p(o_out), _p(ly["post_attention_layernorm"]),
                                      _p(wg), _p(sg), wg.shape[0], _p(wu), _p(su), wu.shape[0],
                                      _p(wd), _p(sd), wd.shape[0], _p(self.o_buf), _p(self.ws),
                                      _p(self.gate_buf), _p(self.up_buf), _p(self.silu_buf),
                                      self.cfg.hidden_size, _kblk(wg, sg), _kblk(wd, sd), P(0))
        return self.o_buf

    # -- step --------------------------------------------------------------------
    def hidden_after_layers(self, token: int) -> torch.Tensor:
        hidden = self.w["embed"][int(token)]
        for i, ly in enumerate(self.w["layers"]):
            self.res.copy_(hidden)
            self.ws.copy_(hidden)
            h = self.rmsnorm_ip(self.ws, ly["input_layernorm"])
            if self.cfg.layer_types[i] == "full_attention":
                a = self._full(h, ly, i)
            else:
                a = self._linear(h, ly, i)
            hidden = self._post(a, ly)
        self.hidden.copy_(hidden)
        return self.hidden

    def step(self, token: int):
        """One token; returns (BF16 logits [V], first-index greedy token)."""
        if self.pos >= self.max_seq:
            raise ValueError("position beyond max_seq")
        hidden = self.hidden_after_layers(token)
        h = self.ws
        h.copy_(hidden)
        self.rmsnorm_ip(h, self.w["norm_f"])
        logits = self.gemv(h, *self.w["lm_head"])
        self.pos += 1
        return logits, int(torch.argmax(logits.float()))
