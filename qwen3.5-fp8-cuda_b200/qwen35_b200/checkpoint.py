"""Block-FP8 safetensors checkpoints: ``config.json`` + ``*.safetensors`` -> engine weights.

Reads the on-disk format the reference loads (``QwenEngineFP8Opt.__init__``
config parsing, main.py:346-370, and ``_load_weights_fp8``, main.py:573-720)
and returns the weights dict ``Qwen35DecodeEngine`` / ``Qwen35TPDecodeEngine``
take (the layout ``weights.random_weights`` produces):

* FP8 linears: ``<name>.weight`` E4M3 ``[N, K]`` plus ``<name>.weight_scale_inv``
  FP32 ``[ceil(N/128), ceil(K/128)]`` -> ``(uint8 bytes, BF16 scale)``; the scale
  is rounded to BF16 as the reference does at load (main.py:596-598);
* an E4M3 weight without a scale tensor: the reference widens it to a BF16
  weight (main.py:599-600), i.e. scale 1 -> here a BF16 scale of ones (same values);
* a BF16 / FP16 / FP32 linear (the reference keeps it BF16 and runs a torch
  matmul): the engine's kernels are FP8-only, so it is quantized here with the
  reference's own 128x128 absmax scheme (``_quantize_bf16_to_fp8``,
  main.py:834-848) and listed in ``info["quantized"]``; ``bf16_linears="error"``
  refuses instead;
* LM head: ``lm_head.weight`` FP8 -> tuple; BF16, or absent (tied to the
  embedding), -> quantized the same way (the reference keeps a BF16 head,
  main.py:615-639: greedy tokens can then differ where its top-2 logits are
  closer than the quantization error);
* ``embed_tokens`` BF16; RMSNorm weights FP32 (main.py:645-669); ``conv1d.weight``
  BF16 ``[C, 1, W]`` -> ``[C, W]``; gated-norm weight FP32 -> BF16 (main.py:695-698);
* ``A_log`` / ``dt_bias`` -> FP32.  The reference keeps their stored dtype
  (main.py:606-610) but its gate kernel reads ``float*``
  (fused_kernels.cu:578-579), so a BF16 copy would be misread there; the values
  are the same.

Keys are looked up under ``model.language_model.`` first, then ``model.``
(text-only exports).  Unlike the reference, a missing tensor raises
``KeyError`` naming it at load.  Keys the decoder does not use (vision tower,
MTP head) are never read: the files are opened lazily and only the needed
tensors are materialised, directly on ``device``.
"""

from __future__ import annotations

import contextlib
import glob
import json
import os

import torch

from .config import Qwen35Config

BLOCK = 128
E4M3_MAX = 448.0
_PREFIXES = ("model.language_model.", "model.")


# ---------------------------------------------------------------- config

def config_from_dict(d: dict) -> Qwen35Config:
    """Architecture from a ``config.json`` dict (main.py:346-370).

    A multimodal config nests the text decoder under ``text_config`` with
    ``rope_parameters``; a text-only one is flat.  The rest of the fields and
    their defaults are the reference's.
    """
    if "text_config" in d:
        tc = dict(d["text_config"])
        rp = tc.get("rope_parameters", {}) or {}
        tc.setdefault("rope_theta", rp.get("rope_theta", 10_000_000))
        tc.setdefault("partial_rotary_factor", rp.get("partial_rotary_factor", 0.25))
        d = tc
    return Qwen35Config(
        hidden_size=d["hidden_size"],
        intermediate_size=d["intermediate_size"],
        num_hidden_layers=d["num_hidden_layers"],
        vocab_size=d["vocab_size"],
        num_attention_heads=d["num_attention_heads"],
        num_key_value_heads=d["num_key_value_heads"],
        head_dim=d.get("head_dim", 256),
        partial_rotary_factor=d.get("partial_rotary_factor", 0.25),
        rope_theta=d.get("rope_theta", 10_000_000),
        linear_num_key_heads=d.get("linear_num_key_heads", 16),
        linear_num_value_heads=d.get("linear_num_value_heads", 32),
        linear_key_head_dim=d.get("linear_key_head_dim", 128),
        linear_value_head_dim=d.get("linear_value_head_dim", 128),
        linear_conv_kernel_dim=d.get("linear_conv_kernel_dim", 4),
        rms_norm_eps=d.get("rms_norm_eps", 1e-6),
        fp8_lm_head=True,
        layer_types=list(d["layer_types"]),
    )


def config_to_dict(cfg: Qwen35Config) -> dict:
    """The ``config.json`` of the multimodal export (``text_config`` + ``rope_parameters``)."""
    tc = {
        "hidden_size": cfg.hidden_size, "intermediate_size": cfg.intermediate_size,
        "num_hidden_layers": cfg.num_hidden_layers, "vocab_size": cfg.vocab_size,
        "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim,
        "linear_num_key_heads": cfg.linear_num_key_heads, "linear_num_value_heads": cfg.linear_num_value_heads,
        "linear_key_head_dim": cfg.linear_key_head_dim, "linear_value_head_dim": cfg.linear_value_head_dim,
        "linear_conv_kernel_dim": cfg.linear_conv_kernel_dim, "rms_norm_eps": cfg.rms_norm_eps,
        "layer_types": list(cfg.layer_types),
        "rope_parameters": {"rope_theta": cfg.rope_theta, "partial_rotary_factor": cfg.partial_rotary_factor},
    }
    return {"text_config": tc, "tie_word_embeddings": False}


def load_config(model_dir: str) -> Qwen35Config:
    with open(os.path.join(model_dir, "config.json")) as f:
        return config_from_dict(json.load(f))


# ---------------------------------------------------------------- quantization

def quantize_block_fp8(w: torch.Tensor, block: int = BLOCK):
    """128x128 absmax block quantization of a 2-D weight (main.py:834-848).

    Per block: ``scale = bf16(max(absmax / 448, 1e-12))``, ``q = e4m3(w / scale)``
    with the ragged edge blocks zero-padded.  Returns ``(uint8 [N, K], BF16
    [ceil(N/block), ceil(K/block)])``; ``q * scale`` dequantizes.
    """
    w = w.to(torch.bfloat16)
    n, k = w.shape
    nb, kb = (n + block - 1) // block, (k + block - 1) // block
    pad = torch.zeros(nb * block, kb * block, dtype=torch.bfloat16, device=w.device)
    pad[:n, :k] = w
    blocks = pad.view(nb, block, kb, block)
    scale = (blocks.abs().amax(dim=(1, 3)) / E4M3_MAX).clamp(min=1e-12).to(torch.bfloat16)
    q = (blocks / scale.view(nb, 1, kb, 1)).to(torch.float8_e4m3fn).reshape(nb * block, kb * block)
    return q[:n, :k].contiguous().view(torch.uint8), scale.contiguous()


# ---------------------------------------------------------------- loading

class _Tensors:
    """Lazy key -> tensor access over every ``*.safetensors`` file of a directory."""

    def __init__(self, model_dir: str, device: str, stack: contextlib.ExitStack):
        from safetensors import safe_open

        self.files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
        if not self.files:
            raise FileNotFoundError(f"no *.safetensors file in {model_dir}")
        self.where = {}
        for fn in self.files:
            h = stack.enter_context(safe_open(fn, framework="pt", device=str(device)))
            for key in h.keys():
                self.where[key] = h
        self.used = set()

    def __contains__(self, key):
        return key in self.where

    def get(self, key):
        self.used.add(key)
        return self.where[key].get_tensor(key)


def load_checkpoint(model_dir: str, cfg: Qwen35Config | None = None, device: str = "cuda",
                    bf16_linears: str = "quantize", info: dict | None = None) -> dict:
    """Engine weights from a block-FP8 safetensors checkpoint directory.

    ``cfg`` defaults to the directory's ``config.json``.  ``info`` (a dict, if
    given) receives ``files``, ``quantized`` (keys quantized at load) and
    ``unused`` (number of tensors in the files the decoder does not read).
    """
    if bf16_linears not in ("quantize", "error"):
        raise ValueError("bf16_linears must be 'quantize' or 'error'")
    cfg = cfg if cfg is not None else load_config(model_dir)
    quantized = []
    with contextlib.ExitStack() as stack:
        ts = _Tensors(model_dir, device, stack)

        def find(*names):
            for pre in _PREFIXES:
                for name in names:
                    if pre + name in ts:
                        return pre + name
            raise KeyError(f"{names[0]} (under {' or '.join(_PREFIXES)}) not in {model_dir}")

        def bf16(key):
            return ts.get(key).to(torch.bfloat16).contiguous()

        def fp32(key):
            return ts.get(key).to(torch.float32).contiguous()

        def linear(key, head=False):
            t = ts.get(key)
            skey = key[: -len(".weight")] + ".weight_scale_inv"
            if t.dtype == torch.float8_e4m3fn:
                n, k = t.shape
                shape = ((n + BLOCK - 1) // BLOCK, (k + BLOCK - 1) // BLOCK)
                if skey in ts:
                    s = ts.get(skey)
                    if tuple(s.shape) != shape:
                        raise ValueError(f"{skey}: shape {tuple(s.shape)}, expected {shape} for a 128x128 "
                                         f"block-scaled [{n}, {k}] weight")
                    s = s.to(torch.bfloat16)
                elif head:
                    raise TypeError("FP8 lm_head is missing block scales")  # main.py:628-630
                else:
                    s = torch.ones(shape, dtype=torch.bfloat16, device=t.device)
                return t.contiguous().view(torch.uint8), s.contiguous()
            if bf16_linears == "error":
                raise TypeError(f"{key}: {t.dtype} linear weight; the decode kernels take block-FP8 only")
            quantized.append(key)
            return quantize_block_fp8(t)

        w = {"embed": bf16(find("embed_tokens.weight")), "norm_f": fp32(find("norm.weight")), "layers": []}
        if "lm_head.weight" in ts:
            w["lm_head"] = linear("lm_head.weight", head=True)
        else:
            if bf16_linears == "error":
                raise TypeError("no lm_head.weight (tied to the embedding): the LM head must be block-FP8")
            quantized.append("lm_head (tied: embed_tokens.weight)")
            w["lm_head"] = quantize_block_fp8(w["embed"])

        for i, lt in enumerate(cfg.layer_types):
            base = f"layers.{i}."

            def key(name):
                return find(base + name)

            ly = {"layer_type": lt,
                  "input_layernorm": fp32(key("input_layernorm.weight")),
                  "post_attention_layernorm": fp32(key("post_attention_layernorm.weight"))}
            if lt == "full_attention":
                for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
                    ly[p] = linear(key(f"self_attn.{p}.weight"))
                ly["q_norm"] = fp32(key("self_attn.q_norm.weight"))
                ly["k_norm"] = fp32(key("self_attn.k_norm.weight"))
            elif lt == "linear_attention":
                for p in ("in_proj_qkv", "in_proj_a", "in_proj_b", "in_proj_z", "out_proj"):
                    ly[p] = linear(key(f"linear_attn.{p}.weight"))
                ly["A_log"] = fp32(key("linear_attn.A_log"))
                ly["dt_bias"] = fp32(key("linear_attn.dt_bias"))
                conv = bf16(key("linear_attn.conv1d.weight"))
                ly["conv1d_w"] = conv.reshape(conv.shape[0], -1).contiguous()
                ly["norm_w"] = fp32(key("linear_attn.norm.weight")).to(torch.bfloat16)
            else:
                raise ValueError(f"layer {i}: unknown layer type {lt!r}")
            for p in ("gate_proj", "up_proj", "down_proj"):
                ly[p] = linear(key(f"mlp.{p}.weight"))
            w["layers"].append(ly)
        if info is not None:
            info["files"] = list(ts.files)
            info["quantized"] = quantized
            info["unused"] = len(set(ts.where) - ts.used)
    cfg.fp8_lm_head = True
    return w


# ---------------------------------------------------------------- writing

def _hf_tensors(w: dict, cfg: Qwen35Config) -> dict:
    pre = "model.language_model."
    out = {pre + "embed_tokens.weight": w["embed"], pre + "norm.weight": w["norm_f"]}

    def put_linear(key, t):
        if isinstance(t, tuple):
            out[key] = t[0].view(torch.float8_e4m3fn)
            out[key[: -len(".weight")] + ".weight_scale_inv"] = t[1].to(torch.float32)
        else:
            out[key] = t

    put_linear("lm_head.weight", w["lm_head"])
    for i, ly in enumerate(w["layers"]):
        b = f"{pre}layers.{i}."
        out[b + "input_layernorm.weight"] = ly["input_layernorm"]
        out[b + "post_attention_layernorm.weight"] = ly["post_attention_layernorm"]
        if ly["layer_type"] == "full_attention":
            for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
                put_linear(f"{b}self_attn.{p}.weight", ly[p])
            out[b + "self_attn.q_norm.weight"] = ly["q_norm"]
            out[b + "self_attn.k_norm.weight"] = ly["k_norm"]
        else:
            for p in ("in_proj_qkv", "in_proj_a", "in_proj_b", "in_proj_z", "out_proj"):
                put_linear(f"{b}linear_attn.{p}.weight", ly[p])
            out[b + "linear_attn.A_log"] = ly["A_log"]
            out[b + "linear_attn.dt_bias"] = ly["dt_bias"]
            c = ly["conv1d_w"]
            out[b + "linear_attn.conv1d.weight"] = c.reshape(c.shape[0], 1, -1)
            out[b + "linear_attn.norm.weight"] = ly["norm_w"]
        for p in ("gate_proj", "up_proj", "down_proj"):
            put_linear(f"{b}mlp.{p}.weight", ly[p])
    return {k: v.detach().to("cpu").contiguous() for k, v in out.items()}


def save_checkpoint(w: dict, cfg: Qwen35Config, model_dir: str, max_shard_bytes: int | None = None) -> list:
    """Write ``w`` (engine layout) as ``config.json`` + safetensors shards in
    the layout ``load_checkpoint`` reads (FP8 weights as E4M3 with FP32
    ``weight_scale_inv``).  Returns the written file names."""
    from safetensors.torch import save_file

    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(config_to_dict(cfg), f, indent=1)
    tensors = _hf_tensors(w, cfg)
    shards, cur, size = [], {}, 0
    for k, t in tensors.items():
        nbytes = t.numel() * t.element_size()
        if cur and max_shard_bytes is not None and size + nbytes > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t
        size += nbytes
    shards.append(cur)
    names = ["model.safetensors"] if len(shards) == 1 else \
        [f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors" for i in range(len(shards))]
    for name, shard in zip(names, shards):
        save_file(shard, os.path.join(model_dir, name), metadata={"format": "pt"})
    return names
