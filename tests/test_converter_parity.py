"""A package written by the reference's own converter opens in this build
unchanged: the reference `npu_llm/tools/convert_smollm2.py` (:174-337) runs
as a subprocess on a random SmolLM2-135M-shaped HF checkpoint (config.json +
model.safetensors, BF16 N(0, 0.02)); `runtime.model.PackageModel` opens the
result with its SHA-256 checks, and every tensor is compared bit for bit
with the source (embedding, norms, BF16 projections) and with this build's
quantiser (int8 weights and FP32 scales).  The converter accepts only the
exact SmolLM2-135M / Qwen2.5-0.5B shapes (convert_smollm2.py:17-32), hence
the full-size checkpoint (134 M parameters, about 270 MB in a temporary
directory).  Skipped when the reference tree is not present."""

import json
import os
from pathlib import Path
import subprocess
import sys

import numpy as np
import pytest
from ml_dtypes import bfloat16

REFERENCE = Path(os.environ.get("HAWKPOINT_REFERENCE", "/root/reference"))
CONVERTER = REFERENCE / "npu_llm" / "tools" / "convert_smollm2.py"

pytestmark = pytest.mark.skipif(not CONVERTER.exists(), reason="reference converter not present")

SHAPE = dict(hidden_size=576, intermediate_size=1536, num_attention_heads=9, num_key_value_heads=3,
             num_hidden_layers=30, vocab_size=49152)


def hf_checkpoint(directory, seed=0):
    """A SmolLM2-135M-shaped HF checkpoint; returns its tensors (BF16)."""
    import torch
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    h, i, L, v = SHAPE["hidden_size"], SHAPE["intermediate_size"], SHAPE["num_hidden_layers"], SHAPE["vocab_size"]
    kv = SHAPE["num_key_value_heads"] * 64

    def normal(*shape):
        return (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)

    def norm(n):  # RMSNorm weights near 1, not all equal
        return (1.0 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16)

    tensors = {"model.embed_tokens.weight": normal(v, h), "model.norm.weight": norm(h)}
    for layer in range(L):
        p = f"model.layers.{layer}"
        tensors.update({
            f"{p}.self_attn.q_proj.weight": normal(h, h),
            f"{p}.self_attn.k_proj.weight": normal(kv, h),
            f"{p}.self_attn.v_proj.weight": normal(kv, h),
            f"{p}.self_attn.o_proj.weight": normal(h, h),
            f"{p}.mlp.gate_proj.weight": normal(i, h),
            f"{p}.mlp.up_proj.weight": normal(i, h),
            f"{p}.mlp.down_proj.weight": normal(h, i),
            f"{p}.input_layernorm.weight": norm(h),
            f"{p}.post_attention_layernorm.weight": norm(h),
        })
    directory.mkdir(parents=True, exist_ok=True)
    save_file(tensors, str(directory / "model.safetensors"))
    config = dict(SHAPE, model_type="llama", rms_norm_eps=1e-5, rope_theta=100000.0, tie_word_embeddings=True)
    (directory / "config.json").write_text(json.dumps(config))
    return {k: t.view(torch.int16).numpy().view(bfloat16) for k, t in tensors.items()}


def bits(a):
    return np.ascontiguousarray(a).view(np.uint8)


@pytest.fixture(scope="module")
def converted(tmp_path_factory):
    root = tmp_path_factory.mktemp("convert")
    src = hf_checkpoint(root / "hf")
    out = root / "package"
    run = subprocess.run([sys.executable, str(CONVERTER), str(root / "hf"), str(out)],
                         capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    return src, out


def test_reference_package_opens_with_checksums(converted):
    from runtime.model import PackageModel

    _, out = converted
    pkg = PackageModel(out, verify=True)
    meta = pkg.metadata
    assert meta["hidden_size"] == 576 and meta["layers"] == 30 and meta["vocab_size"] == 49152
    assert meta["model_family"] == "llama"


def test_every_tensor_matches_the_source_and_this_quantiser(converted):
    from runtime.model import PackageModel
    from runtime.quantize import quantize_per_output_channel

    src, out = converted
    pkg = PackageModel(out, verify=True)
    assert np.array_equal(bits(pkg.raw("token_embedding")), bits(src["model.embed_tokens.weight"]))
    assert np.array_equal(bits(pkg.raw("final_norm")), bits(src["model.norm.weight"]))
    expected_lm = src["model.embed_tokens.weight"]  # tied: the converter quantises the embedding
    checked = 0
    for layer in range(SHAPE["num_hidden_layers"]):
        p = f"model.layers.{layer}"
        mats = {
            "qkv": np.concatenate([src[f"{p}.self_attn.{n}_proj.weight"] for n in "qkv"]),
            "o_proj": src[f"{p}.self_attn.o_proj.weight"],
            "gate_up": np.concatenate([src[f"{p}.mlp.gate_proj.weight"], src[f"{p}.mlp.up_proj.weight"]]),
            "down_proj": src[f"{p}.mlp.down_proj.weight"],
        }
        for name, m in mats.items():
            key = f"layer{layer:02d}.{name}"
            assert np.array_equal(bits(pkg.bf16_projection(key)), bits(m)), key
            q = pkg.quantized(key)
            w8, scale = quantize_per_output_channel(m)
            assert np.array_equal(np.asarray(q.weight), w8), key
            assert np.array_equal(bits(np.asarray(q.scale)), bits(scale)), key
            checked += 1
        assert np.array_equal(bits(pkg.raw(f"layer{layer:02d}.input_norm")), bits(src[f"{p}.input_layernorm.weight"]))
        assert np.array_equal(bits(pkg.raw(f"layer{layer:02d}.post_attn_norm")),
                              bits(src[f"{p}.post_attention_layernorm.weight"]))
        assert not np.asarray(pkg.raw(f"layer{layer:02d}.qkv_bias")).any()  # llama: no bias
    q = pkg.quantized("lm_head")
    w8, scale = quantize_per_output_channel(expected_lm)
    assert np.array_equal(np.asarray(q.weight), w8)
    assert np.array_equal(bits(np.asarray(q.scale)), bits(scale))
    assert checked == 4 * SHAPE["num_hidden_layers"]


def test_reference_package_packs_into_the_engine_layout(converted):
    """The engine's weight blob builds from the converted package (BF16 and
    W8) with every projection in place."""
    from runtime import layout
    from runtime.model import PackageModel

    _, out = converted
    pkg = PackageModel(out, verify=True)
    for weights in ("bf16", "w8"):
        blob, lay = layout.pack(pkg, weights)
        assert blob.size == lay.total
        # the first layer's qkv projection reads back from the blob unchanged
        back = layout.unpack(blob, lay)
        key = "layer00.qkv"
        if weights == "bf16":
            assert np.array_equal(bits(back[key]), bits(pkg.bf16_projection(key)))
