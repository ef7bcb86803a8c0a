"""CPU oracle of one batch-1 greedy decode step of the Qwen3.5 hybrid decoder
(test infrastructure only).

It restates the reference's default native-FP8 decode path,
``QwenEngineFP8Opt._decode_step`` generic branch (main.py:1509-1541) and
``forward`` (main.py:1569-1604), with the op restatements of ``oracle.ops``:

  per layer:  res = hidden; h = RMSNorm(1+w)(hidden)            main.py:1521-1524
     full:    full_attention_forward  (main.py:981-1062, layer_mid_attn path)
     linear:  linear_attention_forward (main.py:1064-1163, decode branch)
     hidden = layer_post_o_fp8_mlp(res, attn_out, ...)            main.py:1531
  final:      RMSNorm(norm_f) -> LM head GEMV -> argmax            main.py:1599-1603

The model description is duck-typed: ``cfg`` needs the attributes of
``qwen35_b200.config.Qwen35Config`` and ``weights`` the dict layout of
``qwen35_b200.weights`` (reference key names, main.py:614-715).

Prompt tokens go through the same single-token step as decode tokens (the
reference prefills with batched kernels and the chunked delta rule, which is
the same function up to rounding).
"""

from __future__ import annotations

import torch

from . import ops

BF16 = torch.bfloat16
F32 = torch.float32


class OracleModel:
    def __init__(self, cfg, weights, max_seq: int, device="cpu"):
        self.cfg = cfg
        self.w = weights
        self.max_seq = max_seq
        self.dev = torch.device(device)  # where the caches live: the weights' device
        self.rotary_dim = int(cfg.head_dim * cfg.partial_rotary_factor)
        cos, sin = ops.rope_tables(max_seq, self.rotary_dim, cfg.rope_theta)
        self.cos, self.sin = cos.to(self.dev), sin.to(self.dev)
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

    # -- layers ------------------------------------------------------------
    def _full(self, h, ly, i):
        cfg = self.cfg
        q_all = ops.gemv(h, *ly["q_proj"])
        k = ops.gemv(h, *ly["k_proj"])
        v = ops.gemv(h, *ly["v_proj"])
        out = ops.attention_decode(
            q_all, k, v, ly["q_norm"], ly["k_norm"], self.cos, self.sin,
            self.k_cache[i], self.v_cache[i], self.pos,
            cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, self.rotary_dim,
            cfg.rms_norm_eps)
        return ops.gemv(out, *ly["o_proj"])

    def _linear(self, h, ly, i):
        cfg = self.cfg
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
        return ops.gemv(gated.reshape(-1), *ly["out_proj"])

    # -- step --------------------------------------------------------------
    def hidden_after_layers(self, token: int):
        cfg = self.cfg
        hidden = self.w["embed"][token].clone()
        for i, ly in enumerate(self.w["layers"]):
            res = hidden
            h = ops.rmsnorm(hidden, ly["input_layernorm"], cfg.rms_norm_eps)
            if cfg.layer_types[i] == "full_attention":
                a = self._full(h, ly, i)
            else:
                a = self._linear(h, ly, i)
            hidden = ops.mlp_post(res, a, ly["post_attention_layernorm"],
                                  *ly["gate_proj"], *ly["up_proj"], *ly["down_proj"],
                                  eps=cfg.rms_norm_eps)["output"]
        return hidden

    def step(self, token: int):
        """Process one token; returns (logits BF16 [V], greedy next token)."""
        hidden = self.hidden_after_layers(token)
        h = ops.rmsnorm(hidden, self.w["norm_f"], self.cfg.rms_norm_eps)
        head = self.w["lm_head"]
        logits = ops.gemv(h, *head) if isinstance(head, tuple) else ops.linear_bf16(h, head)
        self.pos += 1
        return logits, ops.argmax_first(logits)
