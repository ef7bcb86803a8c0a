"""Block-FP8 safetensors checkpoint loading (qwen35_b200.checkpoint), on the CPU.

Pinned against the reference's own loader: tests/golden/make_golden_cpu.py ran
``QwenEngineFP8Opt._load_weights_fp8`` (main.py:573-720) on the committed
micro checkpoint ``tests/golden/micro_ckpt`` and ``_quantize_bf16_to_fp8``
(main.py:834-848) on a ragged BF16 matrix; the ``load_*`` and ``quant_*``
tensors of cpu_golden.safetensors are its outputs.  Every tensor the
reference loads must come out of ``load_checkpoint`` with the same bits, or,
where the engine needs another form (FP32 ``dt_bias``, ``[C, W]`` conv
weights, block-FP8 for a BF16 linear), with the same values.
"""

import json
import os
import shutil
import sys

import pytest
import torch
from safetensors.torch import load_file, save_file

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "qwen3.5-fp8-cuda_b200"))

from qwen35_b200.checkpoint import (config_from_dict, load_checkpoint, load_config,  # noqa: E402
                                    quantize_block_fp8, save_checkpoint)
from qwen35_b200.config import qwen35_tiny  # noqa: E402
from qwen35_b200.weights import random_weights  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")
MICRO = os.path.join(GOLDEN, "micro_ckpt")
BF16, F32 = torch.bfloat16, torch.float32


@pytest.fixture(scope="module")
def gold():
    return load_file(os.path.join(GOLDEN, "cpu_golden.safetensors"))


def _dequant(w, s):
    n, k = w.shape
    e = s.float().repeat_interleave(128, 0)[:n].repeat_interleave(128, 1)[:, :k]
    return w.view(torch.float8_e4m3fn).float() * e


def _same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)


def test_quantizer_matches_reference(gold):
    q, s = quantize_block_fp8(gold["quant_w_in"])
    assert _same(q, gold["quant_w"]) and _same(s, gold["quant_s"])
    # the all-zero block takes the 1e-12 floor and quantizes to zeros
    assert float(s[1, 0]) == pytest.approx(1e-12, rel=1e-2) and not q[128:256, :128].any()


def test_loader_matches_reference_loader(gold):
    info = {}
    w = load_checkpoint(MICRO, device="cpu", info=info)
    ref = {k[len("load_"):]: v for k, v in gold.items() if k.startswith("load_")}
    checked = set()

    def eq(name, ours):
        assert _same(ours, ref[name]), name
        checked.add(name)

    eq("embed", w["embed"])
    eq("norm_f", w["norm_f"])
    eq("lm_head_w", w["lm_head"][0])
    eq("lm_head_s", w["lm_head"][1])
    for i, ly in enumerate(w["layers"]):
        for name, v in ly.items():
            key = f"L{i}_{name}"
            if isinstance(v, tuple):
                if key + "_w" in ref:
                    eq(key + "_w", v[0])
                    eq(key + "_s", v[1])
                elif name == "in_proj_a":
                    # stored BF16: the reference keeps it, here it is block-FP8
                    # by the reference's own quantizer
                    q, s = quantize_block_fp8(ref[key])
                    assert _same(v[0], q) and _same(v[1], s), key
                    checked.add(key)
                else:
                    # E4M3 without a scale tensor: the reference widens it to
                    # BF16, here it keeps its bytes with unit scales
                    assert torch.equal(_dequant(*v), ref[key].float()), key
                    checked.add(key)
            elif isinstance(v, torch.Tensor):
                if name == "dt_bias":
                    assert v.dtype == F32 and torch.equal(v, ref[key].float()), key
                    checked.add(key)
                elif name == "conv1d_w":
                    assert _same(v, ref[key].reshape(ref[key].shape[0], -1)), key
                    checked.add(key)
                else:
                    eq(key, v)
    assert checked == set(ref), set(ref) - checked
    assert info["quantized"] == ["model.language_model.layers.0.linear_attn.in_proj_a.weight"]
    assert info["unused"] == 2  # vision and MTP tensors are not read


def test_config_parse():
    cfg = load_config(MICRO)
    with open(os.path.join(MICRO, "config.json")) as f:
        tc = json.load(f)["text_config"]
    assert (cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers, cfg.vocab_size) == \
        (tc["hidden_size"], tc["intermediate_size"], tc["num_hidden_layers"], tc["vocab_size"])
    assert cfg.layer_types == tc["layer_types"] and cfg.head_dim == 64 and cfg.rotary_dim == 16
    assert cfg.rope_theta == tc["rope_parameters"]["rope_theta"]
    assert cfg.conv_dim == 256 and cfg.linear_value_dim == 128
    flat = dict(tc, rope_theta=1e6, partial_rotary_factor=0.5)
    del flat["rope_parameters"]
    c2 = config_from_dict(flat)
    assert c2.rope_theta == 1e6 and c2.rotary_dim == 32


def _walk(a, b, path="w"):
    if isinstance(a, torch.Tensor):
        assert _same(a, b), path
    elif isinstance(a, (tuple, list)):
        assert len(a) == len(b), path
        for i, (x, y) in enumerate(zip(a, b)):
            _walk(x, y, f"{path}[{i}]")
    elif isinstance(a, dict):
        assert a.keys() == b.keys(), (path, a.keys() ^ b.keys())
        for k in a:
            _walk(a[k], b[k], f"{path}.{k}")
    else:
        assert a == b, path


def test_round_trip_sharded(tmp_path):
    cfg = qwen35_tiny()
    w = random_weights(cfg, seed=3)
    names = save_checkpoint(w, cfg, str(tmp_path), max_shard_bytes=1 << 20)
    assert len(names) > 1
    info = {}
    w2 = load_checkpoint(str(tmp_path), device="cpu", info=info)
    _walk(w, w2)
    assert load_config(str(tmp_path)) == cfg
    assert info["quantized"] == [] and info["unused"] == 0 and len(info["files"]) == len(names)


def _micro_variant(tmp_path, edit):
    d = str(tmp_path)
    os.makedirs(d, exist_ok=True)
    shutil.copy(os.path.join(MICRO, "config.json"), d)
    t = load_file(os.path.join(MICRO, "model.safetensors"))
    edit(t)
    save_file(t, os.path.join(d, "model.safetensors"))
    return d


def test_tied_head_quantized(tmp_path):
    def drop_head(t):
        del t["lm_head.weight"], t["lm_head.weight_scale_inv"]
    info = {}
    w = load_checkpoint(_micro_variant(tmp_path, drop_head), device="cpu", info=info)
    q, s = quantize_block_fp8(w["embed"])
    assert _same(w["lm_head"][0], q) and _same(w["lm_head"][1], s)
    assert "lm_head (tied: embed_tokens.weight)" in info["quantized"]


def test_bf16_head_quantized(tmp_path):
    head = {}

    def bf16_head(t):
        head["w"] = (torch.randn(320, 128) * 0.02).to(BF16)
        t["lm_head.weight"] = head["w"]
        del t["lm_head.weight_scale_inv"]
    w = load_checkpoint(_micro_variant(tmp_path, bf16_head), device="cpu")
    q, s = quantize_block_fp8(head["w"])
    assert _same(w["lm_head"][0], q) and _same(w["lm_head"][1], s)
    err = (_dequant(q, s) - head["w"].float()).abs().max() / head["w"].float().abs().max()
    assert err < 2 ** -3  # E4M3 keeps 3 mantissa bits


def test_refusals(tmp_path):
    with pytest.raises(TypeError, match="block-FP8 only"):
        load_checkpoint(MICRO, device="cpu", bf16_linears="error")

    def head_without_scale(t):
        del t["lm_head.weight_scale_inv"]
    with pytest.raises(TypeError, match="missing block scales"):
        load_checkpoint(_micro_variant(tmp_path / "a", head_without_scale), device="cpu")

    def drop_key(t):
        del t["model.language_model.layers.1.self_attn.k_norm.weight"]
    with pytest.raises(KeyError, match="layers.1.self_attn.k_norm.weight"):
        load_checkpoint(_micro_variant(tmp_path / "b", drop_key), device="cpu")

    def bad_scale(t):
        t["model.language_model.layers.0.mlp.down_proj.weight_scale_inv"] = torch.ones(2, 2)
    with pytest.raises(ValueError, match="down_proj.weight_scale_inv"):
        load_checkpoint(_micro_variant(tmp_path / "c", bad_scale), device="cpu")
    with pytest.raises(FileNotFoundError):
        load_checkpoint(str(tmp_path), cfg=qwen35_tiny(), device="cpu")


def test_text_only_prefix(tmp_path):
    def strip(t):
        for k in list(t):
            if k.startswith("model.language_model."):
                t["model." + k[len("model.language_model."):]] = t.pop(k)
    w = load_checkpoint(_micro_variant(tmp_path, strip), device="cpu")
    w0 = load_checkpoint(MICRO, device="cpu")
    _walk(w0, w)
