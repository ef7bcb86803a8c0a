"""Tensor-parallel decomposition of the decode step, checked on the CPU.

Two gloo ranks shard a seeded tiny-config model with qwen35_b200.tp
(head-parallel attention / GatedDeltaNet, row-split gate/up, column-split
o_proj / out_proj / down with an FP32 all-reduce, vocabulary-split LM head
with a packed-key MAX all-reduce) and run the decode step with the CPU
oracle's op restatements on their shards.  Logits and greedy tokens must
match the unsharded oracle model: the sharding may only change the order of
FP32 additions.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ops
from oracle.model import OracleModel

F32, BF16 = torch.float32, torch.bfloat16
STEPS = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _TPOracle(OracleModel):
    """The oracle step on one rank's shard, with the engine's collectives."""

    def __init__(self, lcfg, lw, max_seq):
        super().__init__(lcfg, lw, max_seq)

    @staticmethod
    def _partial_resid(x, wt, res):
        part = ops.dequant(*wt) @ x.reshape(-1).to(F32)
        dist.all_reduce(part)
        return (res.float() + part.to(BF16).float()).to(BF16)

    def hidden_after_layers(self, token):
        cfg = self.cfg
        hidden = self.w["embed"][token].clone()
        for i, ly in enumerate(self.w["layers"]):
            h = ops.rmsnorm(hidden, ly["input_layernorm"], cfg.rms_norm_eps)
            if cfg.layer_types[i] == "full_attention":
                q_all = ops.gemv(h, *ly["q_proj"])
                k = ops.gemv(h, *ly["k_proj"])
                v = ops.gemv(h, *ly["v_proj"])
                out = ops.attention_decode(q_all, k, v, ly["q_norm"], ly["k_norm"], self.cos, self.sin,
                                           self.k_cache[i], self.v_cache[i], self.pos, cfg.num_attention_heads,
                                           cfg.num_key_value_heads, cfg.head_dim, self.rotary_dim, cfg.rms_norm_eps)
                h2 = self._partial_resid(out, ly["o_proj"], hidden)
            else:
                kd = cfg.linear_num_key_heads * cfg.linear_key_head_dim
                vd = cfg.linear_num_value_heads * cfg.linear_value_head_dim
                mixed = ops.gemv(h, *ly["in_proj_qkv"])
                a = ops.gemv(h, *ly["in_proj_a"])
                b = ops.gemv(h, *ly["in_proj_b"])
                z = ops.gemv(h, *ly["in_proj_z"])
                conv_out, self.conv[i] = ops.conv1d_update(mixed, self.conv[i], ly["conv1d_w"])
                q, k, v = torch.split(conv_out, [kd, kd, vd])
                g, beta = ops.linear_gates(a, b, ly["A_log"], ly["dt_bias"])
                rep = cfg.linear_num_value_heads // cfg.linear_num_key_heads
                q = q.reshape(cfg.linear_num_key_heads, -1).repeat_interleave(rep, 0)
                k = k.reshape(cfg.linear_num_key_heads, -1).repeat_interleave(rep, 0)
                v = v.reshape(cfg.linear_num_value_heads, -1)
                core, self.state[i] = ops.delta_rule_decode(q, k, v, g, beta, self.state[i])
                gated = ops.rmsnorm_gated(core, z.reshape(cfg.linear_num_value_heads, -1), ly["norm_w"],
                                          cfg.rms_norm_eps)
                h2 = self._partial_resid(gated, ly["out_proj"], hidden)
            n = ops.rmsnorm(h2, ly["post_attention_layernorm"], cfg.rms_norm_eps)
            _, _, s = ops.gate_up_silu(n, *ly["gate_proj"], *ly["up_proj"])
            hidden = self._partial_resid(s, ly["down_proj"], h2)
        return hidden

    def step(self, token):
        hidden = self.hidden_after_layers(token)
        h = ops.rmsnorm(hidden, self.w["norm_f"], self.cfg.rms_norm_eps)
        logits = ops.gemv(h, *self.w["lm_head"])
        off = self.w["lm_row_offset"]
        bits = (logits.view(torch.int16).to(torch.int64) & 0xFFFF).tolist()
        key = torch.tensor([max(ops.packed_key(b, off + j) for j, b in enumerate(bits))], dtype=torch.int64)
        dist.all_reduce(key, op=dist.ReduceOp.MAX)
        self.pos += 1
        return logits, ops.key_to_index(int(key.item()))


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "qwen3.5-fp8-cuda_b200"))
    from qwen35_b200.config import qwen35_tiny
    from qwen35_b200.tp import local_config, shard_weights, tp_layout
    from qwen35_b200.weights import random_weights
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        cfg = qwen35_tiny()
        w = random_weights(cfg, seed=11, device="cpu")
        lay = tp_layout(cfg, rank, world)
        full = OracleModel(cfg, w, max_seq=16)
        tp = _TPOracle(local_config(cfg, lay), shard_weights(cfg, w, lay), max_seq=16)
        tok_full = tok_tp = 17
        worst = 0.0
        for _ in range(STEPS):
            lf, tok_full = full.step(tok_full)
            lt, tok_tp = tp.step(tok_tp)
            parts = [torch.zeros_like(lt) for _ in range(world)]
            dist.all_gather(parts, lt)
            lt_all = torch.cat(parts).float()
            err = float((lt_all - lf.float()).norm() / lf.float().norm())
            worst = max(worst, err)
            assert tok_tp == tok_full, (tok_tp, tok_full)
        out[rank] = worst
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_decomposition_matches_oracle(world):
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    assert len(out) == world
    assert max(out.values()) < 2e-3, dict(out)
