"""Tensor-parallel decode on the persistent step kernel: one process and one
cooperative launch per GPU per token (`qwen_step_create_tp`,
include/qwen_step.h).

Per layer, rank r of W takes (column- then row-parallel, so only two of the
five stages exchange data between GPUs):

* in_proj: the q / k / v / z rows of its GatedDeltaNet heads (value heads
  [32 r / W, 32 (r + 1) / W) and their key heads; the 32-row a / b
  projections are computed whole on every rank), or q / k / v: the rows of
  its attention KV heads (with 8 ranks and 4 KV heads, ranks r and r + 4
  compute the same head); the GatedDeltaNet / attention stage then has all
  its inputs on its own GPU;
* out_proj / o_proj: the K range of its heads for every output row, as FP32
  K-slice rows stored into slots [r x nslice, (r + 1) x nslice) of every
  rank's slice buffer over NVLink as tagged words (value | step-and-stage
  tag); the next stage polls the words for the tag instead of waiting on a
  counter;
* gate/up: a 512-aligned range of the intermediate rows; down: the same
  range of K for every row (K-slice rows to every rank, as above);
* the next stage's prologue sums the W x nslice slices in rank order, so
  every rank holds the same residual stream;
* LM head: a range of vocabulary rows; every CTA folds its packed (logit,
  index) key into every rank's workspace and each rank's CTA 0 finalises.

The buffers written across GPUs (slices, logits, argmax workspace, token,
key, position, counters) live in an arena with the same layout on every rank,
allocated with `qwen_ipc_alloc` and mapped by the peers through CUDA IPC;
everything else is per rank.  Every output row is computed with the same
chunk order as on one GPU, so with the same K-slice arithmetic the results
are bit-identical to the single-GPU engine's.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .step import (EPI_ARGMAX, EPI_CONV, EPI_GATE_BETA, EPI_GATE_G, EPI_SILU, EPI_SILU_PAIR, EPI_SLICES, EPI_STORE, P,
                   PRO_EMBED_NORM, PRO_PLAIN, PRO_SLICES_NORM, Qwen35StepEngine, StepStage)

CHUNK_K, CHUNK_BYTES, TILE_ROWS = 512, 16400, 32


class _DevArray:
    """A device array at a raw address, for ``torch.as_tensor`` (CUDA array interface)."""

    def __init__(self, ptr: int, n: int, dtype):
        typestr = {torch.bfloat16: "<f2", torch.float32: "<f4", torch.int64: "<i8", torch.int32: "<i4"}[dtype]
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2}


def _view(ptr: int, n: int, dtype, device) -> torch.Tensor:
    """torch tensor of `n` elements of `dtype` at device address `ptr` (no copy)."""
    if dtype == torch.bfloat16:  # the interface has no bf16 type: view the bytes as f16, reinterpret
        return torch.as_tensor(_DevArray(ptr, n, torch.bfloat16), device=device).view(torch.bfloat16)
    return torch.as_tensor(_DevArray(ptr, n, dtype), device=device)


class Qwen35StepTPEngine(Qwen35StepEngine):
    """``Qwen35StepEngine`` over `world` GPUs, this process being `rank`.

    Construct it on every rank (same config, weights, seeds and arguments);
    `group` is the process group used to exchange the IPC handles.  The
    public API is the single-GPU engine's: every rank calls ``decode`` /
    ``step`` with the same tokens and gets the same greedy tokens.
    """

    def __init__(self, cfg, weights, rank: int, world: int, group=None, **kw):
        if world not in (1, 2, 4, 8):
            raise ValueError("world must be 1, 2, 4 or 8")
        self.rank, self.world, self.group = int(rank), int(world), group
        self._peers = []
        self._arena = None
        super().__init__(cfg, weights, **kw)

    # ------------------------------------------------------------------
    def _split(self, total: int, what: str):
        """This rank's [lo, hi) of `total` units (contiguous, in rank order)."""
        lo, hi = self.rank * total // self.world, (self.rank + 1) * total // self.world
        if hi <= lo:
            raise ValueError(f"{what}: {total} units cannot be split over {self.world} ranks")
        return lo, hi

    @staticmethod
    def _sub(seg, m, r0: int, r1: int):
        """Restrict `seg` (built over all rows of matrix `m`) to rows [r0, r1):
        the packed weights start at tile r0 / 32, the outputs and per-row
        epilogue operands at row r0."""
        if r0 % TILE_ROWS or r1 <= r0:
            raise ValueError(f"row range [{r0}, {r1}) is not a 32-row-aligned range")
        wt = m[0] if isinstance(m, tuple) else m
        C = wt.shape[1] // (CHUNK_K if isinstance(m, tuple) else 256)
        off = (r0 // TILE_ROWS) * C * CHUNK_BYTES
        seg.w += off
        if seg.w2:
            seg.w2 += off
        seg.n = r1 - r0
        if seg.y:
            seg.y += (4 if seg.epi == EPI_GATE_G else 2) * r0
        if seg.epi == EPI_CONV:  # conv1d weights and conv state: cw BF16 values per channel
            seg.aux0 += 2 * r0 * seg.cw
            seg.aux2 += 2 * r0 * seg.cw
        elif seg.epi == EPI_GATE_G:  # A_log, dt_bias: FP32 per head
            seg.aux0 += 4 * r0
            seg.aux1 += 4 * r0
        elif seg.epi == EPI_ARGMAX:
            seg.row_offset += r0
        return seg

    def _row_parallel(self, m, x, sl, c0: int, c1: int):
        """Chunks [c0, c1) of K of every row of `m`: FP32 K-slice rows into
        slots [rank x nslice, (rank + 1) x nslice) of `sl` on every rank."""
        C = m[0].shape[1] // CHUNK_K
        seg = self._seg(m, EPI_SLICES)
        seg.w += c0 * CHUNK_BYTES
        st = self._gemv((c1 - c0) * CHUNK_K, PRO_PLAIN, [seg], x=x, nslice=self.nslice)
        st.x += 2 * c0 * CHUNK_K
        st.sl_out, st.sl_rows = sl.data_ptr(), self.cfg.hidden_size
        st.xrank, st.cstride = 1, C
        return st

    def _k_chunks(self, lo: int, hi: int, what: str):
        if lo % CHUNK_K or hi % CHUNK_K:
            raise ValueError(f"{what}: K range [{lo}, {hi}) of rank {self.rank} is not 512-aligned")
        return lo // CHUNK_K, hi // CHUNK_K

    def _build_stages(self):
        if self.world == 1:
            return super()._build_stages()
        cfg, w, W, r = self.cfg, self.w, self.world, self.rank
        H = cfg.hidden_size
        stages = []

        def with_slices(st, sl):
            st.sl_in, st.sl_in_count, st.sl_stride = sl.data_ptr(), 0, H
            return st

        for i, ly in enumerate(w["layers"]):
            if i == 0:
                inp = dict(pro=PRO_EMBED_NORM, x=w["embed"], h_out=self.hidden, norm_w=ly["input_layernorm"])
            else:
                inp = dict(pro=PRO_SLICES_NORM, res=self.h2, h_out=self.hidden, norm_w=ly["input_layernorm"])
            if cfg.layer_types[i] == "full_attention":
                nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
                G = nh // nkv
                if W <= nkv:
                    kh0, kh1 = self._split(nkv, "KV heads")
                    qh0, qh1 = kh0 * G, kh1 * G
                else:  # W / nkv ranks share a KV head and split its query heads for o_proj
                    per = W // nkv
                    if W % nkv or G % per:
                        raise ValueError(f"{nkv} KV heads x {G} query heads cannot be split over {W} ranks")
                    kh0, kh1 = r // per, r // per + 1
                    qh0 = kh0 * G + (r % per) * (G // per)
                    qh1 = qh0 + G // per
                segs = [self._sub(self._seg(ly["q_proj"], EPI_STORE, y=self.q_all), ly["q_proj"],
                                  kh0 * G * 2 * hd, kh1 * G * 2 * hd),
                        self._sub(self._seg(ly["k_proj"], EPI_STORE, y=self.k_new), ly["k_proj"], kh0 * hd, kh1 * hd),
                        self._sub(self._seg(ly["v_proj"], EPI_STORE, y=self.v_new), ly["v_proj"], kh0 * hd, kh1 * hd)]
                st = self._gemv(H, segs=segs, **inp)
                stages.append(with_slices(st, self.sl_buf2) if i else st)
                a = self._attn_stage(i, ly)
                a.shard0, a.shard_n = kh0, kh1 - kh0
                stages.append(a)
                c0, c1 = self._k_chunks(qh0 * hd, qh1 * hd, "o_proj")
                stages.append(self._row_parallel(ly["o_proj"], self.attn_out, self.sl_buf, c0, c1))
            else:
                nv, nk = cfg.linear_num_value_heads, cfg.linear_num_key_heads
                dk, dv, rep = cfg.linear_key_head_dim, cfg.linear_value_head_dim, nv // nk
                kd = nk * dk
                hv0, hv1 = self._split(nv, "value heads")
                if hv0 % rep or hv1 % rep:
                    raise ValueError(f"{nv} value heads over {nk} key heads cannot be split over {W} ranks")
                hk0, hk1 = hv0 // rep, hv1 // rep
                qkv = ly["in_proj_qkv"]

                def conv(r0, r1):
                    s = self._seg(qkv, EPI_CONV, y=self.qkv_conv, aux0=ly["conv1d_w"], aux2=self.conv_state[i],
                                  cw=cfg.linear_conv_kernel_dim)
                    return self._sub(s, qkv, r0, r1)

                segs = [conv(hk0 * dk, hk1 * dk), conv(kd + hk0 * dk, kd + hk1 * dk),
                        conv(2 * kd + hv0 * dv, 2 * kd + hv1 * dv),
                        self._sub(self._seg(ly["in_proj_z"], EPI_SILU, y=self.z), ly["in_proj_z"], hv0 * dv,
                                  hv1 * dv),
                        # the per-head gates (one row per value head) are computed whole on every rank
                        self._seg(ly["in_proj_a"], EPI_GATE_G, y=self.g, aux0=ly["A_log"], aux1=ly["dt_bias"]),
                        self._seg(ly["in_proj_b"], EPI_GATE_BETA, y=self.beta)]
                st = self._gemv(H, segs=segs, **inp)
                stages.append(with_slices(st, self.sl_buf2) if i else st)
                g = self._gdn_stage(i, ly)
                g.shard0, g.shard_n = hv0, hv1 - hv0
                stages.append(g)
                c0, c1 = self._k_chunks(hv0 * dv, hv1 * dv, "out_proj")
                stages.append(self._row_parallel(ly["out_proj"], self.attn_out, self.sl_buf, c0, c1))
            # MLP: a 512-aligned range of the intermediate rows, then the same K range of down
            c0, c1 = self._split(cfg.intermediate_size // CHUNK_K, "intermediate chunks")
            gu = self._sub(self._seg(ly["gate_proj"], EPI_SILU_PAIR, y=self.silu, w2=ly["up_proj"]), ly["gate_proj"],
                           c0 * CHUNK_K, c1 * CHUNK_K)
            stages.append(with_slices(self._gemv(H, PRO_SLICES_NORM, [gu], res=self.hidden, h_out=self.h2,
                                                 norm_w=ly["post_attention_layernorm"], pair=1), self.sl_buf))
            stages.append(self._row_parallel(ly["down_proj"], self.silu, self.sl_buf2, c0, c1))
        V = cfg.vocab_size
        t0, t1 = self._split((V + TILE_ROWS - 1) // TILE_ROWS, "LM-head tiles")
        lm = w["lm_head"]
        seg = self._sub(self._seg(lm, EPI_ARGMAX, y=self.logits), lm, t0 * TILE_ROWS, min(t1 * TILE_ROWS, V))
        head = with_slices(self._gemv(H, PRO_SLICES_NORM, [seg], res=self.h2, h_out=self.hidden, norm_w=w["norm_f"]),
                           self.sl_buf2)
        head.wbf16 = 0 if isinstance(lm, tuple) else 1
        head.am_ws = self.am_ws.data_ptr()
        head.am_key_out = self.key.data_ptr()
        head.am_token_out = self.token.data_ptr()
        head.pos_inc = self.pos.data_ptr()
        stages.append(head)
        return (StepStage * len(stages))(*stages)

    def _setup_shared(self):
        """Move every buffer a stage writes into the IPC arena and map the peers'."""
        cfg, dev = self.cfg, self.device
        lib = self.lib
        # K-slice buffers of tagged 8-byte words (16 slots x hidden each, zero:
        # no tag); down writes the second while the other ranks may still read
        # out_proj's / o_proj's from the first
        H = cfg.hidden_size
        self.sl_buf = torch.zeros(2 * self.sl_max * H, dtype=torch.float32, device=dev)
        self.sl_buf2 = torch.zeros_like(self.sl_buf)
        names = ["sl_buf", "sl_buf2", "token", "key", "pos", "am_ws"] + (["logits"] if self.logits is not None else [])
        nstages = 5 * cfg.num_hidden_layers + 1
        layout, off = {}, 0
        for name in names:
            t = getattr(self, name)
            layout[name] = (off, t.numel(), t.dtype)
            off = (off + t.numel() * t.element_size() + 255) // 256 * 256
        cbytes = lib.qwen_step_counter_bytes(nstages)
        layout["__counters"] = (off, cbytes, None)
        total = off + cbytes
        base = P()
        handle = ctypes.create_string_buffer(64)
        _lib.check(lib.qwen_ipc_alloc(total, ctypes.byref(base), handle), "qwen_ipc_alloc")
        self._arena = base
        local = int(base.value)
        for name in names:
            o, n, dt = layout[name]
            fresh = _view(local + o, n, dt, dev)
            fresh.copy_(getattr(self, name))
            setattr(self, name, fresh)
        self._counters = local + layout["__counters"][0]
        # every rank's handle; peers mapped into this process
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=self.group)
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(local)
                continue
            pb = P()
            _lib.check(lib.qwen_p2p_open(ctypes.create_string_buffer(h, 64), ctypes.byref(pb)), "qwen_p2p_open")
            self._peers.append(pb)
            bases.append(int(pb.value))
        self._bases = (P * self.world)(*[P(b) for b in bases])
        self._local = local
        torch.cuda.synchronize(dev)

    def _create_program(self, stages):
        arr = stages if isinstance(stages, ctypes.Array) else (StepStage * len(stages))(*stages)
        prog = P()
        _lib.check(self.lib.qwen_step_create_tp(ctypes.cast(arr, P), len(arr), self.world, self.rank, self._bases,
                                                P(self._local), P(self._counters), ctypes.byref(prog)),
                   "qwen_step_create_tp")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every rank's counters are zero before anyone launches
        return prog

    def close(self):
        """Release the program, the peer mappings and the arena.  Collective:
        every rank calls it (before the process group is destroyed)."""
        if getattr(self, "prog", None) and dist.is_initialized():
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)  # nobody writes into a peer's arena any more
            self.lib.qwen_step_destroy(self.prog)
            self.prog = None
            for pb in self._peers:
                self.lib.qwen_p2p_close(pb)
            self._peers = []
            dist.barrier(group=self.group)
            if self._arena is not None:
                self.lib.qwen_p2p_destroy(self._arena)
                self._arena = None
