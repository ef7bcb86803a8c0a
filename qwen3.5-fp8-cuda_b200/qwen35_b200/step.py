"""Decode engine on the persistent step kernel: one cooperative launch per token.

Replaces the per-layer launch sequence of ``Qwen35DecodeEngine`` (and the
reference's ~1,000 ctypes calls per token in ``QwenEngineFP8Opt._decode_step``
/ ``forward``, main.py:1509-1604) with a program of stages that one kernel
walks (``include/qwen_step.h``):

    per layer (5 stages):
      full:   RMSNorm + q/k/v GEMVs | norm + RoPE + KV write + attention + gate | o_proj (K slices)
      linear: RMSNorm + in_proj GEMVs with conv1d/SiLU and gate epilogues
              | delta rule (units of 32 value columns) | gated RMSNorm + out_proj (K slices)
      both:   residual + RMSNorm + gate/up + SiLU | down (K slices)
    residual + RMSNorm + LM head + greedy argmax (+ position increment)

The first stage gathers the embedding row of the device-resident token.
Every CTA streams its share of each stage's weights into shared memory ahead
of the dependency chain.  Linear weights are packed once for the kernel
(``qwen_step_pack``); the engine keeps the reference-layout weights it was
given untouched.  Buffers, caches, ``decode()`` / ``generate()`` and graph
capture are those of ``Qwen35DecodeEngine``.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .engine import Qwen35DecodeEngine
from .ops import scale_mode

P = ctypes.c_void_p

GEMV, GDN, ATTN = 0, 1, 2
PRO_PLAIN, PRO_NORM, PRO_EMBED_NORM, PRO_SLICES_NORM = 0, 1, 2, 3
EPI_STORE, EPI_SILU_PAIR, EPI_ARGMAX, EPI_CONV, EPI_GATE_G, EPI_GATE_BETA, EPI_SLICES, EPI_SILU = 0, 2, 3, 4, 5, 6, 9, 10


class StepSeg(ctypes.Structure):
    """``qwen_step_seg`` (include/qwen_step.h)."""
    _fields_ = [("w", P), ("w2", P), ("n", ctypes.c_int), ("epi", ctypes.c_int), ("y", P), ("y2", P),
                ("aux0", P), ("aux1", P), ("aux2", P), ("cw", ctypes.c_int), ("row_offset", ctypes.c_int)]


class StepStage(ctypes.Structure):
    """``qwen_step_stage`` (include/qwen_step.h)."""
    _fields_ = [
        ("kind", ctypes.c_int),
        ("K", ctypes.c_int), ("pro", ctypes.c_int), ("nseg", ctypes.c_int), ("pair", ctypes.c_int),
        ("nslice", ctypes.c_int),
        ("x", P), ("x_rows", ctypes.c_int), ("res", P), ("norm_w", P), ("eps", ctypes.c_float), ("h_out", P),
        ("token", P), ("sl_in", P), ("sl_in_count", ctypes.c_int), ("sl_stride", ctypes.c_int),
        ("sl_out", P), ("sl_rows", ctypes.c_int),
        ("am_ws", P), ("am_key_out", P), ("am_token_out", P), ("pos_inc", P),
        ("seg", StepSeg * 6),
        ("g_q", P), ("g_k", P), ("g_v", P), ("g_g", P), ("g_beta", P), ("g_state", P), ("g_out", P),
        ("g_z", P), ("g_norm_w", P), ("g_eps", ctypes.c_float), ("g_heads", ctypes.c_int),
        ("g_dim", ctypes.c_int), ("g_rep", ctypes.c_int),
        ("a_q", P), ("a_k_new", P), ("a_v_new", P), ("a_q_norm", P), ("a_k_norm", P), ("a_cos", P),
        ("a_sin", P), ("a_k_cache", P), ("a_v_cache", P), ("a_pos", P), ("a_max_seq", ctypes.c_int),
        ("a_heads", ctypes.c_int), ("a_kv", ctypes.c_int), ("a_dim", ctypes.c_int), ("a_rot", ctypes.c_int),
        ("a_eps", ctypes.c_float), ("a_chunk", ctypes.c_int), ("a_nsplit", ctypes.c_int), ("a_ws", P),
        ("a_cnt", P), ("a_out", P),
        ("wbf16", ctypes.c_int), ("shard0", ctypes.c_int), ("shard_n", ctypes.c_int), ("xrank", ctypes.c_int),
        ("cstride", ctypes.c_int),
    ]


def _p(t) -> int | None:
    return None if t is None else t.data_ptr()


def pack_linear(w_u8: torch.Tensor, scale: torch.Tensor, stream=None) -> torch.Tensor:
    """Pack a device [N, K] E4M3 weight and its 128x128 block scales for GEMV
    stages (``qwen_step_pack``); returns the packed bytes (uint8, device)."""
    lib = _lib.fused()
    n, k = w_u8.shape
    kblk = scale_mode(n, scale)
    nbytes = lib.qwen_step_packed_bytes(n, k)
    if nbytes == 0 or kblk != k // 128:
        raise ValueError(f"step kernel needs K % 512 == 0 and 128x128 block scales (N={n}, K={k}, K_blk={kblk})")
    out = torch.empty(nbytes, dtype=torch.uint8, device=w_u8.device)
    st = P(stream if stream is not None else torch.cuda.current_stream(w_u8.device).cuda_stream)
    _lib.check(lib.qwen_step_pack(P(w_u8.data_ptr()), P(scale.data_ptr()), 1 if scale.dtype == torch.float32 else 0,
                                  n, k, kblk, P(out.data_ptr()), st), "qwen_step_pack")
    return out


def pack_linear_bf16(w_bf16: torch.Tensor, stream=None) -> torch.Tensor:
    """Pack a device [N, K] BF16 weight for a ``wbf16`` GEMV stage
    (``qwen_step_pack_bf16``); returns the packed bytes (uint8, device)."""
    lib = _lib.fused()
    n, k = w_bf16.shape
    nbytes = lib.qwen_step_packed_bytes_bf16(n, k)
    if nbytes == 0 or w_bf16.dtype != torch.bfloat16:
        raise ValueError(f"BF16 step GEMV needs a BF16 weight with K % 256 == 0 (N={n}, K={k})")
    out = torch.empty(nbytes, dtype=torch.uint8, device=w_bf16.device)
    st = P(stream if stream is not None else torch.cuda.current_stream(w_bf16.device).cuda_stream)
    _lib.check(lib.qwen_step_pack_bf16(P(w_bf16.contiguous().data_ptr()), n, k, P(out.data_ptr()), st),
               "qwen_step_pack_bf16")
    return out


def create_program(stages) -> P:
    """``qwen_step_create`` over a sequence of ``StepStage``; returns the handle."""
    arr = stages if isinstance(stages, ctypes.Array) else (StepStage * len(stages))(*stages)
    prog = P()
    _lib.check(_lib.fused().qwen_step_create(ctypes.cast(arr, P), len(arr), ctypes.byref(prog)), "qwen_step_create")
    return prog


class Qwen35StepEngine(Qwen35DecodeEngine):
    """Greedy batch-1 decoder whose whole step is one persistent-kernel launch.

    Same constructor, state, buffers and public API (``decode``, ``generate``,
    ``step``, ``capture``, ``reset``) as ``Qwen35DecodeEngine``; only the way
    a step is issued differs.  ``nslice`` fixes the K-slice count of the
    residual projections (default: chosen by the library).
    """

    # Fewest positions per attention split: short splits keep a unit's chain
    # of KV-row round trips short (all splits run at once, one per CTA), more
    # splits make the combine longer; 16 measured best on B200 at 128-4000
    # positions (8: +10-17 us a step, 32: +10 us, 64: +40 us).
    ATTN_CHUNK = 16

    def __init__(self, cfg, weights, max_seq: int = 4096, device="cuda", keep_logits: bool = False,
                 attn_chunk: int | None = None, nslice: int = 0):
        super().__init__(cfg, weights, max_seq=max_seq, device=device, keep_logits=keep_logits,
                         attn_chunk=self.ATTN_CHUNK if attn_chunk is None else attn_chunk, slices=True)
        self.nslice = int(nslice)
        self.packed = {}
        self._setup_shared()
        self._pack_all()
        self.stages = self._build_stages()
        self.prog = self._create_program(self.stages)
        self.grid = self.lib.qwen_step_grid(self.prog)

    # ------------------------------------------------------------------
    # hooks of the tensor-parallel engine (step_tp.py)
    def _setup_shared(self):
        """Place the buffers that stages write (one GPU: nothing to do)."""

    def _create_program(self, stages):
        return create_program(stages)

    def gdn_state(self, i: int) -> torch.Tensor:
        """Layer i's GatedDeltaNet state as [value heads][keys][values] FP32 (a
        copy: the step kernel keeps it as [heads][4 value blocks][keys][32])."""
        st = self.state[i]
        h, k, v = st.shape
        return st.view(h, 4, k, v // 4).permute(0, 2, 1, 3).reshape(h, k, v)

    def _pack_all(self):
        w = self.w
        mats = [w["lm_head"]]
        for ly in w["layers"]:
            for key in ("q_proj", "k_proj", "v_proj", "o_proj", "in_proj_qkv", "in_proj_z", "in_proj_a",
                        "in_proj_b", "out_proj", "gate_proj", "up_proj", "down_proj"):
                if key in ly:
                    mats.append(ly[key])
        for m in mats:
            if isinstance(m, tuple):
                self.packed[m[0].data_ptr()] = pack_linear(m[0], m[1])
            else:  # BF16 LM head (the reference's F.linear head, main.py:1600-1601)
                self.packed[m.data_ptr()] = pack_linear_bf16(m)
        torch.cuda.synchronize(self.device)

    def _pk(self, m):
        return self.packed[(m[0] if isinstance(m, tuple) else m).data_ptr()].data_ptr()

    def _gemv(self, K, pro, segs, x=None, res=None, norm_w=None, h_out=None, pair=0, sl_out=False, nslice=0):
        st = StepStage()
        st.kind = GEMV
        st.K = K
        st.pro = pro
        st.nseg = len(segs)
        st.pair = pair
        st.nslice = nslice
        st.x = _p(x)
        st.res = _p(res)
        st.norm_w = _p(norm_w)
        st.eps = self.cfg.rms_norm_eps
        st.h_out = _p(h_out)
        if pro == PRO_EMBED_NORM:
            st.token = self.token.data_ptr()
            st.x_rows = self.cfg.vocab_size
        if pro == PRO_SLICES_NORM:
            st.sl_in = self.sl_buf.data_ptr()
            st.sl_in_count = 0
            st.sl_stride = self.cfg.hidden_size
        if sl_out:
            st.sl_out = self.sl_buf.data_ptr()
            st.sl_rows = self.cfg.hidden_size
        for i, sg in enumerate(segs):
            st.seg[i] = sg
        return st

    def _seg(self, m, epi, y=None, w2=None, aux0=None, aux1=None, aux2=None, cw=0, row_offset=0):
        s = StepSeg()
        s.w = self._pk(m)
        s.w2 = None if w2 is None else self._pk(w2)
        s.n = (m[0] if isinstance(m, tuple) else m).shape[0]
        s.epi = epi
        s.y = _p(y)
        s.aux0 = _p(aux0)
        s.aux1 = _p(aux1)
        s.aux2 = _p(aux2)
        s.cw = cw
        s.row_offset = row_offset
        return s

    def _attn_stage(self, i, ly):
        cfg = self.cfg
        a = StepStage()
        a.kind = ATTN
        a.a_q, a.a_k_new, a.a_v_new = self.q_all.data_ptr(), self.k_new.data_ptr(), self.v_new.data_ptr()
        a.a_q_norm, a.a_k_norm = ly["q_norm"].data_ptr(), ly["k_norm"].data_ptr()
        a.a_cos, a.a_sin = self.cos.data_ptr(), self.sin.data_ptr()
        a.a_k_cache, a.a_v_cache = self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr()
        a.a_pos = self.pos.data_ptr()
        a.a_max_seq = self.max_seq
        a.a_heads, a.a_kv, a.a_dim = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        a.a_rot = cfg.rotary_dim
        a.a_eps = cfg.rms_norm_eps
        a.a_chunk, a.a_nsplit = self.attn_chunk, self.attn_nsplit
        a.a_ws, a.a_cnt = self.attn_ws.data_ptr(), self.attn_cnt.data_ptr()
        a.a_out = self.attn_out.data_ptr()
        return a

    def _gdn_stage(self, i, ly):
        cfg = self.cfg
        kd = cfg.linear_key_dim
        g = StepStage()
        g.kind = GDN
        base = self.qkv_conv.data_ptr()
        g.g_q, g.g_k, g.g_v = base, base + 2 * kd, base + 4 * kd  # BF16: 2 bytes per element
        g.g_g, g.g_beta = self.g.data_ptr(), self.beta.data_ptr()
        g.g_state = self.state[i].data_ptr()
        g.g_out = self.attn_out.data_ptr()
        g.g_z, g.g_norm_w = self.z.data_ptr(), ly["norm_w"].data_ptr()
        g.g_eps = cfg.rms_norm_eps
        g.g_heads = cfg.linear_num_value_heads
        g.g_dim = cfg.linear_value_head_dim
        g.g_rep = cfg.linear_num_value_heads // cfg.linear_num_key_heads
        return g

    def _build_stages(self):
        cfg, w = self.cfg, self.w
        H, I = cfg.hidden_size, cfg.intermediate_size
        stages = []

        def layer_input(i, ly):
            """pro / res / h_out of a layer's first GEMV: the embedding row for
            layer 0, else the previous layer's residual plus down's slices."""
            if i == 0:
                return dict(pro=PRO_EMBED_NORM, x=w["embed"], h_out=self.hidden, norm_w=ly["input_layernorm"])
            return dict(pro=PRO_SLICES_NORM, res=self.h2, h_out=self.hidden, norm_w=ly["input_layernorm"])

        for i, ly in enumerate(w["layers"]):
            if cfg.layer_types[i] == "full_attention":
                segs = [self._seg(ly["q_proj"], EPI_STORE, y=self.q_all),
                        self._seg(ly["k_proj"], EPI_STORE, y=self.k_new),
                        self._seg(ly["v_proj"], EPI_STORE, y=self.v_new)]
                stages.append(self._gemv(H, segs=segs, **layer_input(i, ly)))
                stages.append(self._attn_stage(i, ly))
                qd = cfg.num_attention_heads * cfg.head_dim
                stages.append(self._gemv(qd, PRO_PLAIN, [self._seg(ly["o_proj"], EPI_SLICES)], x=self.attn_out,
                                         sl_out=True, nslice=self.nslice))
            else:
                segs = [self._seg(ly["in_proj_qkv"], EPI_CONV, y=self.qkv_conv, aux0=ly["conv1d_w"],
                                  aux2=self.conv_state[i], cw=cfg.linear_conv_kernel_dim),
                        self._seg(ly["in_proj_z"], EPI_SILU, y=self.z),  # bf16(silu(z)) for the gated norm
                        self._seg(ly["in_proj_a"], EPI_GATE_G, y=self.g, aux0=ly["A_log"], aux1=ly["dt_bias"]),
                        self._seg(ly["in_proj_b"], EPI_GATE_BETA, y=self.beta)]
                stages.append(self._gemv(H, segs=segs, **layer_input(i, ly)))
                stages.append(self._gdn_stage(i, ly))
                stages.append(self._gemv(cfg.linear_value_dim, PRO_PLAIN, [self._seg(ly["out_proj"], EPI_SLICES)],
                                         x=self.attn_out, sl_out=True, nslice=self.nslice))
            stages.append(self._gemv(H, PRO_SLICES_NORM,
                                     [self._seg(ly["gate_proj"], EPI_SILU_PAIR, y=self.silu, w2=ly["up_proj"])],
                                     res=self.hidden, h_out=self.h2, norm_w=ly["post_attention_layernorm"],
                                     pair=1))
            stages.append(self._gemv(I, PRO_PLAIN, [self._seg(ly["down_proj"], EPI_SLICES)], x=self.silu,
                                     sl_out=True, nslice=self.nslice))
        head = self._gemv(H, PRO_SLICES_NORM, [self._seg(w["lm_head"], EPI_ARGMAX, y=self.logits)], res=self.h2,
                          h_out=self.hidden, norm_w=w["norm_f"])
        head.wbf16 = 0 if isinstance(w["lm_head"], tuple) else 1
        head.am_ws = self.am_ws.data_ptr()
        head.am_key_out = self.key.data_ptr()
        head.am_token_out = self.token.data_ptr()
        head.pos_inc = self.pos.data_ptr()
        stages.append(head)
        return (StepStage * len(stages))(*stages)

    # ------------------------------------------------------------------
    def _launch_step(self, stream):
        _lib.check(self.lib.qwen_step_launch(self.prog, P(stream)), "qwen_step_launch")
        self.launches_per_step = 1
        self.kernels_per_step = 1

    def step_reset(self):
        """Clear the stage counters after an abandoned step (device error 8)."""
        _lib.check(self.lib.qwen_step_reset(self.prog, P(torch.cuda.current_stream(self.device).cuda_stream)),
                   "qwen_step_reset")

    def close(self):
        if getattr(self, "prog", None):
            torch.cuda.synchronize(self.device)
            self.lib.qwen_step_destroy(self.prog)
            self.prog = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
