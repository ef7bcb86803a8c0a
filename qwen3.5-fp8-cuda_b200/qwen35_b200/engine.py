"""Batch-1 greedy decode engine for the Qwen3.5 hybrid decoder on one B200.

Replaces the per-layer Python/ctypes orchestration of
``QwenEngineFP8Opt._decode_step`` / ``forward`` (main.py:1509-1604) with a fixed
sequence of C-ABI launches that is captured once into a CUDA graph:

    embed(token)                                               1 kernel
    per layer (5 kernels each):
      full:   RMSNorm+q/k/v GEMVs | norm+RoPE+KV write+attention+gate | o_proj+residual
      linear: RMSNorm+in_proj GEMVs with conv1d/SiLU and gate epilogues
              | delta rule + gated RMSNorm | out_proj+residual
      both:   RMSNorm+gate/up+SiLU | down+residual
    RMSNorm + LM head + greedy argmax (+ position increment)   1 kernel

Kernels are chained with programmatic dependent launch, so each GEMV starts
streaming its weights while the previous kernel finishes.  The token and the
position live on the device: the graph reads the token written by the
previous replay's argmax, so a greedy loop never leaves the GPU.

PyTorch is used for device buffers, the stream and graph capture only.
"""

from __future__ import annotations

import ctypes
import math
import time

import torch

from . import _lib
from .ops import scale_mode

P = ctypes.c_void_p


def _p(t) -> P:
    return P(0) if t is None else P(t.data_ptr())


def rope_tables(max_pos: int, rotary_dim: int, theta: float):
    """Partial-RoPE tables [max_pos, rotary_dim] FP32 (main.py:525-533), built on the CPU."""
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim))
    pos = torch.arange(max_pos).float()
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


class Qwen35DecodeEngine:
    """Greedy batch-1 decoder over device-resident weights (see ``weights.py``).

    ``gdn_split`` (128-wide value heads only): the GatedDeltaNet step writes
    its un-normed output over 4 CTAs per head and out_proj applies the gated
    RMSNorm in its prologue.  Off by default: one CTA per head doing both
    measured 24 us per step faster on B200 (the step kernel gains 1.1 us,
    out_proj loses 0.4 us, and the wider grid delays out_proj's start).

    ``prefetch=True`` makes every launch pull its successor's weights into L2
    (``cp.async.bulk.prefetch``) while it runs.  It is off by default: on B200
    the prefetches compete with the running launch's own stream and the step
    measured about 8% slower with them.

    ``slices`` (default on): o_proj, out_proj and down write their K-split
    partial rows (``qwen_linear_slices``) instead of reducing them in a last
    CTA and adding the residual; the next launch (gate/up, the next layer's
    in_proj, the LM head) adds the slices in slice order to the residual in
    its prologue and writes the new residual stream.  Same arithmetic, one
    store / fence / atomic / reload chain less per projection.  ``hidden``
    holds the residual stream only once the launch after a layer has run.
    """

    def __init__(self, cfg, weights, max_seq: int = 4096, device="cuda", keep_logits: bool = False,
                 attn_chunk: int | None = None, prefetch: bool = False, gdn_split: bool = False,
                 slices: bool = True):
        self.cfg = cfg
        self.slices = bool(slices)
        self.gdn_split = bool(gdn_split) and cfg.linear_value_head_dim == 128
        self.prefetch = prefetch
        self.w = weights
        self.max_seq = int(max_seq)
        self.device = torch.device(device)
        self.keep_logits = keep_logits
        self.lib = _lib.fused()
        dev = self.device
        H = cfg.hidden_size
        bf, f32 = torch.bfloat16, torch.float32

        def empty(n, dt=bf):
            return torch.empty(n, dtype=dt, device=dev)

        self.hidden = empty(H)
        self.h2 = empty(H)
        # K-slice partial rows of the residual projections (o_proj / out_proj /
        # down) and their count, summed by the next launch's prologue
        self.sl_max = 16
        self.sl_buf = empty(self.sl_max * H, f32)
        self.sl_count = torch.zeros(1, dtype=torch.int32, device=dev)
        qd = cfg.num_attention_heads * cfg.head_dim
        kvd = cfg.num_key_value_heads * cfg.head_dim
        self.q_all = empty(2 * qd)
        self.k_new = empty(kvd)
        self.v_new = empty(kvd)
        self.attn_out = empty(max(qd, cfg.linear_value_dim))
        self.qkv_conv = empty(cfg.conv_dim)
        self.z = empty(cfg.linear_value_dim)
        self.g = empty(cfg.linear_num_value_heads, f32)
        self.beta = empty(cfg.linear_num_value_heads)
        self.silu = empty(cfg.intermediate_size)
        self.logits = empty(cfg.vocab_size) if keep_logits else None
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.key = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.am_ws = torch.zeros(2, dtype=torch.int64, device=dev)
        cos, sin = rope_tables(self.max_seq, cfg.rotary_dim, cfg.rope_theta)
        self.cos, self.sin = cos.to(dev), sin.to(dev)

        # Split-KV attention: one wave of CTAs (KV heads x splits <= SMs); the
        # kernel spreads the current context over the splits, at least
        # attn_chunk positions each.
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.attn_chunk = int(attn_chunk) if attn_chunk is not None else 32
        self.attn_nsplit = max(1, min(sms // max(1, cfg.num_key_value_heads),
                                      math.ceil(self.max_seq / self.attn_chunk)))
        self.attn_ws = empty(cfg.num_attention_heads * self.attn_nsplit * (cfg.head_dim + 2), f32)
        self.attn_cnt = torch.zeros(cfg.num_key_value_heads, dtype=torch.int32, device=dev)

        self.k_cache, self.v_cache, self.conv_state, self.state = {}, {}, {}, {}
        for i, lt in enumerate(cfg.layer_types):
            if lt == "full_attention":
                shape = (cfg.num_key_value_heads, self.max_seq, cfg.head_dim)
                self.k_cache[i] = torch.zeros(shape, dtype=bf, device=dev)
                self.v_cache[i] = torch.zeros(shape, dtype=bf, device=dev)
            else:
                self.conv_state[i] = torch.zeros(cfg.conv_dim, cfg.linear_conv_kernel_dim, dtype=bf, device=dev)
                self.state[i] = torch.zeros(cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                                            cfg.linear_value_head_dim, dtype=f32, device=dev)
        self.graph = None
        self.graph_io = None
        self._h_tok = torch.zeros(1, dtype=torch.int64, pin_memory=True)
        self._h_out = torch.zeros(1, dtype=torch.int64, pin_memory=True)
        # decode() I/O: [0] input token, [2] output token, [3] step sequence number
        # (pinned; the step graph copies [0] in and its last kernel writes [2], [3])
        self._io = torch.zeros(4, dtype=torch.int64, pin_memory=True)
        self._io_np = self._io.numpy()
        self._dseq = torch.zeros(1, dtype=torch.int64, device=dev)
        self._seq = 0
        self.launches_per_step = 0
        self.kernels_per_step = 0

    # ------------------------------------------------------------------
    def gdn_state(self, i: int) -> torch.Tensor:
        """Layer i's GatedDeltaNet state as [value heads][keys][values] FP32."""
        return self.state[i]

    def reset(self):
        """Clear caches and recurrent state; position back to 0."""
        for t in list(self.k_cache.values()) + list(self.v_cache.values()):
            t.zero_()
        for t in list(self.conv_state.values()) + list(self.state.values()):
            t.zero_()
        self.pos.zero_()

    # Bytes of one region a launch may prefetch into L2 for its successor.
    PREFETCH_CAP = 64 << 20

    def _regions(self, *tensors):
        """(pointer, bytes) of the tensors a launch streams, for L2 look-ahead."""
        out = []
        for t in tensors:
            if t is None:
                continue
            out.append((t.data_ptr(), min(t.numel() * t.element_size(), self.PREFETCH_CAP)))
        return out[:4]

    def _plan_step(self):
        """The decode step as a list of (launch(stream), regions it streams)."""
        cfg, lib, w = self.cfg, self.lib, self.w
        H, I = cfg.hidden_size, cfg.intermediate_size
        eps = cfg.rms_norm_eps
        plan = []

        def chk(status, what):
            _lib.check(status, what)

        def resid(st, x, wt, scl, res, out, what):
            """out = res + W x: one launch, or (slices) the K-slice rows that the
            next launch adds to res (it writes out)."""
            if self.slices:
                chk(lib.qwen_linear_slices(_p(x), _p(wt), _p(scl), wt.shape[0], wt.shape[1],
                                           scale_mode(wt.shape[0], scl), _p(self.sl_buf), _p(self.sl_count),
                                           self.sl_max, st), what)
            else:
                chk(lib.qwen_linear_resid(_p(x), _p(wt), _p(scl), wt.shape[0], wt.shape[1],
                                          scale_mode(wt.shape[0], scl), _p(res), _p(out), st), what)

        def take(res):
            """The next launch builds its input from the pending slices plus res."""
            if self.slices:
                chk(lib.qwen_set_slices_input(_p(self.sl_buf), _p(self.sl_count), H, self.sl_max, _p(res)),
                    "slices_input")

        plan.append((lambda st: chk(lib.qwen_embed(_p(w["embed"]), _p(self.token), _p(self.hidden), H, st),
                                    "qwen_embed"), []))
        for i, ly in enumerate(w["layers"]):
            if cfg.layer_types[i] == "full_attention":
                (wq, sq), (wk, sk), (wv, sv), (wo, so) = ly["q_proj"], ly["k_proj"], ly["v_proj"], ly["o_proj"]
                def attn_in(st, i=i, ly=ly, wq=wq, sq=sq, wk=wk, sk=sk, wv=wv, sv=sv):
                    if i > 0:
                        take(self.h2)
                    chk(lib.qwen_attn_in_proj(
                        _p(self.hidden), _p(ly["input_layernorm"]), eps, _p(wq), _p(sq), wq.shape[0], _p(wk),
                        _p(sk), wk.shape[0], _p(wv), _p(sv), wv.shape[0], H, scale_mode(wq.shape[0], sq),
                        _p(self.q_all), _p(self.k_new), _p(self.v_new), st), "attn_in_proj")
                plan.append((attn_in, self._regions(wq, wk, wv)))
                plan.append((lambda st, ly=ly, i=i: chk(lib.qwen_attn_decode(
                    _p(self.q_all), _p(self.k_new), _p(self.v_new), _p(ly["q_norm"]), _p(ly["k_norm"]),
                    _p(self.cos), _p(self.sin), _p(self.k_cache[i]), _p(self.v_cache[i]), _p(self.pos),
                    self.max_seq, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.rotary_dim, eps,
                    self.attn_chunk, self.attn_nsplit, _p(self.attn_ws), _p(self.attn_cnt), _p(self.attn_out), st),
                    "attn_decode"), []))  # a decode step reads pos + 1 cache rows, not the whole cache
                plan.append((lambda st, wo=wo, so=so: resid(st, self.attn_out, wo, so, self.hidden, self.h2, "o_proj"),
                             self._regions(wo)))
            else:
                (wqkv, sqkv), (wz, sz) = ly["in_proj_qkv"], ly["in_proj_z"]
                (wa, sa), (wb, sb), (wo, so) = ly["in_proj_a"], ly["in_proj_b"], ly["out_proj"]
                def gdn_in(st, ly=ly, i=i, wqkv=wqkv, sqkv=sqkv, wz=wz, sz=sz, wa=wa, sa=sa, wb=wb, sb=sb):
                    if i > 0:
                        take(self.h2)
                    chk(lib.qwen_gdn_in_proj(
                        _p(self.hidden), _p(ly["input_layernorm"]), eps, H, scale_mode(wqkv.shape[0], sqkv),
                        _p(wqkv), _p(sqkv), wqkv.shape[0], _p(ly["conv1d_w"]), _p(self.conv_state[i]),
                        cfg.linear_conv_kernel_dim, _p(self.qkv_conv), _p(wz), _p(sz), wz.shape[0],
                        _p(self.z), _p(wa), _p(sa), _p(wb), _p(sb), wa.shape[0], _p(ly["A_log"]),
                        _p(ly["dt_bias"]), _p(self.g), _p(self.beta), st), "gdn_in_proj")
                plan.append((gdn_in, self._regions(wqkv, wz, wa, wb)))
                if self.gdn_split:
                    # recurrent step over 4 CTAs per head; the gated norm runs in
                    # out_proj's prologue (one 128-wide K-block per head)
                    plan.append((lambda st, i=i: chk(lib.qwen_gdn_decode_core(
                        _p(self.qkv_conv), _p(self.g), _p(self.beta), _p(self.state[i]), _p(self.attn_out),
                        cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_value_head_dim, st),
                        "gdn_decode_core"), self._regions(self.state[i])))

                    def out_proj(st, ly=ly, wo=wo, so=so):
                        chk(lib.qwen_set_gated_input(_p(self.z), _p(ly["norm_w"]), eps), "gated_input")
                        resid(st, self.attn_out, wo, so, self.hidden, self.h2, "out_proj")
                    plan.append((out_proj, self._regions(wo)))
                else:
                    plan.append((lambda st, ly=ly, i=i: chk(lib.qwen_gdn_decode(
                        _p(self.qkv_conv), _p(self.g), _p(self.beta), _p(self.state[i]), _p(self.z),
                        _p(ly["norm_w"]), eps, _p(self.attn_out), cfg.linear_num_key_heads,
                        cfg.linear_num_value_heads, cfg.linear_value_head_dim, st), "gdn_decode"),
                        self._regions(self.state[i])))
                    plan.append((lambda st, wo=wo, so=so: resid(st, self.attn_out, wo, so, self.hidden, self.h2,
                                                                 "out_proj"), self._regions(wo)))
            (wg, sg), (wu, su), (wd, sd) = ly["gate_proj"], ly["up_proj"], ly["down_proj"]
            def gate_up(st, ly=ly, wg=wg, sg=sg, wu=wu, su=su):
                take(self.hidden)
                chk(lib.qwen_mlp_gate_up(
                    _p(self.h2), _p(ly["post_attention_layernorm"]), eps, _p(wg), _p(sg), _p(wu), _p(su), I, H,
                    scale_mode(I, sg), _p(self.silu), st), "gate_up")
            plan.append((gate_up, self._regions(wg, wu)))
            plan.append((lambda st, wd=wd, sd=sd: resid(st, self.silu, wd, sd, self.h2, self.hidden, "down"),
                         self._regions(wd)))
        head = w["lm_head"]
        if not isinstance(head, tuple):
            raise NotImplementedError("BF16 LM head: use an FP8 head (cfg.fp8_lm_head=True)")
        wh, sh = head
        def lm_head(st):
            take(self.h2)
            chk(lib.launch_lm_head_argmax(
                _p(self.hidden), _p(w["norm_f"]), eps, _p(wh), _p(sh), wh.shape[0], H, scale_mode(wh.shape[0], sh), 0,
                _p(self.am_ws), _p(self.key), _p(self.token), _p(self.logits), _p(self.pos), st), "lm_head_argmax")
        plan.append((lm_head, self._regions(wh)))
        return plan

    def _launch_step(self, stream):
        """Issue one decode step (with prefetch on, every launch prefetches its successor's regions)."""
        plan = self._plan_step()
        st = P(stream)
        n = len(plan)
        for j, (launch, _) in enumerate(plan):
            if self.prefetch:
                nxt = []
                k = (j + 1) % n
                while not nxt and k != j:
                    nxt = plan[k][1]
                    k = (k + 1) % n
                args = []
                for ptr, nbytes in (nxt + [(0, 0)] * 4)[:4]:
                    args += [P(ptr), nbytes]
                self.lib.qwen_set_prefetch(*args)
            launch(st)
        self.launches_per_step = n
        self.kernels_per_step = n - getattr(self, "collectives_per_step", 0)

    # ------------------------------------------------------------------
    def step_eager(self):
        """Run one decode step without the graph (token and pos on device)."""
        self._launch_step(torch.cuda.current_stream().cuda_stream)

    def capture(self):
        """Capture one decode step into a CUDA graph (state is not advanced)."""
        saved = [t.clone() for t in self._mutable()]
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._launch_step(s.cuda_stream)  # warm-up (sets kernel attributes)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._launch_step(s.cuda_stream)
        # decode(): the same step with its host I/O inside the graph: the input
        # token copied in from pinned memory, the output token and a sequence
        # number written to pinned memory by the last kernel
        gio = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gio, stream=s):
            self.token.copy_(self._io[0:1], non_blocking=True)
            self._launch_step(s.cuda_stream)
            _lib.check(self.lib.qwen_publish_token(_p(self.token), P(self._io.data_ptr() + 16), _p(self._dseq),
                                                   P(s.cuda_stream)), "qwen_publish_token")
        torch.cuda.synchronize(self.device)
        for t, v in zip(self._mutable(), saved):
            t.copy_(v)
        self.graph = g
        self.graph_io = gio
        self._seq = int(self._dseq.item())
        return g

    def _mutable(self):
        return ([self.token, self.key, self.pos, self.hidden, self.h2] + list(self.k_cache.values())
                + list(self.v_cache.values()) + list(self.conv_state.values()) + list(self.state.values()))

    def step(self):
        """One decode step on the device (graph replay if captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self.step_eager()

    # ------------------------------------------------------------------
    # Public API: host token in, host token out (one step end to end).
    def decode(self, token: int) -> int:
        """Feed ``token`` at the current position; return the greedy next token.

        With a captured graph the step's I/O is part of it: the token goes in
        from pinned memory and the host polls the pinned sequence number the
        last kernel writes (bounded: after 2 s it synchronises and raises).
        """
        if self.graph_io is not None:
            io = self._io_np
            io[0] = int(token)
            expect = self._seq + 1
            self.graph_io.replay()
            if io[3] != expect:
                t0 = time.perf_counter()
                while io[3] != expect:
                    if time.perf_counter() - t0 > 2.0:
                        torch.cuda.current_stream().synchronize()
                        if io[3] != expect:
                            raise RuntimeError(f"decode step {expect} did not publish its token")
            self._seq = expect
            return int(io[2])
        self._h_tok[0] = int(token)
        self.token.copy_(self._h_tok, non_blocking=True)
        self.step()
        self._h_out.copy_(self.token, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return int(self._h_out[0])

    def generate(self, prompt, n_new: int):
        """Greedy generation: feed the prompt token by token, then ``n_new`` steps on device."""
        out = []
        nxt = None
        for t in prompt:
            nxt = self.decode(int(t))
        tok = nxt
        for _ in range(n_new):
            out.append(tok)
            tok = self.decode(tok)
        return out, tok

    def position(self) -> int:
        return int(self.pos.item())
