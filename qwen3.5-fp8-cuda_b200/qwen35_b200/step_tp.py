"""Tensor-parallel decode on the persistent step kernel: one process and one
cooperative launch per GPU per token.

Every stage of the step is split over the ranks (`qwen_step_create_tp`,
include/qwen_step.h): GEMV stages by 32-row tiles of their output (the
LM head and every projection and MLP matrix shard by output rows, the
residual projections keep their K slices), GatedDeltaNet by value heads and
attention by KV heads (with 8 ranks and 4 KV heads, ranks r and r + 4 compute
the same head).  Each CTA stores its outputs on every rank over NVLink and
arrives on every rank's stage counter, so a rank's next stage reads a
complete, local input vector - the all-gather of the row-parallel outputs is
the stores themselves, and the greedy argmax is reduced by every CTA folding
its packed (logit, index) key into every rank's workspace.  Waits read local
memory only.

The buffers that stages write (stage outputs, K slices, token, key, position,
argmax workspace, logits and the stage counters) live in one arena per rank
with the same layout on every rank, allocated with `qwen_ipc_alloc` and
mapped by the peers through CUDA IPC (handles exchanged over the process
group).  Everything else (weights, caches, recurrent state, the residual
stream) is per rank; the weights are identical on every rank.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .step import P, Qwen35StepEngine, StepStage


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
    def _shard(self, kind: str, total: int):
        W, r = self.world, self.rank
        if W == 1:
            return 0, 0
        if kind == "kv" and total < W:  # more ranks than KV heads: ranks r and r + total share a head
            return r % total, 1
        lo, hi = r * total // W, (r + 1) * total // W
        if hi <= lo:
            raise ValueError(f"{kind}: {total} units cannot be split over {W} ranks")
        return lo, hi - lo

    def _setup_shared(self):
        """Move every buffer a stage writes into the IPC arena and map the peers'."""
        cfg, dev = self.cfg, self.device
        lib = self.lib
        names = ["q_all", "k_new", "v_new", "attn_out", "qkv_conv", "z", "g", "beta", "silu", "sl_buf", "token",
                 "key", "pos", "am_ws"] + (["logits"] if self.logits is not None else [])
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
