#!/usr/bin/env python3
"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only) at
``--reference`` (default: the ``REFERENCE_ROOT`` environment variable).  It
imports the reference's own NumPy BF16 runtime ``CPUDecoderStage``
(npu_llm/runtime/cpu_backend.py) and its quantiser
(npu_llm/tools/convert_smollm2.py:81-86), runs them on this repository's
seeded random-init models, and writes small ``.npz`` fixtures next to this
script.  Nothing at test time reads the reference; the tests compare the
oracle (and, on a GPU, the engine) against these files.

Cases:
* ``decode_<shape>.npz`` -- teacher-forced decode through every layer the way
  ``NPUDecoder.decode_token`` drives ``CPUDecoderStage`` with ``npu_layers=0``
  (npu_llm/runtime/generate.py:830-846): input ids, per-position argmax and
  top-2 margin, FP32 logits (full for the small shapes; top-32 plus a strided
  sample for the full-size shapes), and the final BF16 hidden state bits.
* ``quantize.npz`` -- the reference quantiser's int8 bytes and FP32 scales on
  the converter test's matrix (seed 7, npu_llm/tests/test_converter.py:15-23)
  and on BF16 projections of the seeded Qwen model.
* ``attention.npz`` -- the reference ``_attention`` on the toy case of
  npu_llm/tests/test_cpu_backend.py:17-52 (seed 42).
"""

import argparse
import hashlib
import importlib.util
import os
from pathlib import Path
import sys

import numpy as np
from ml_dtypes import bfloat16

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "hawkpoint-npu-llm_b200"))

from runtime import synthetic  # noqa: E402


def load_reference(root):
    root = Path(root)
    spec = importlib.util.spec_from_file_location(
        "reference_cpu_backend", root / "npu_llm/runtime/cpu_backend.py"
    )
    backend = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(backend)
    spec = importlib.util.spec_from_file_location(
        "reference_convert", root / "npu_llm/tools/convert_smollm2.py"
    )
    convert = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(convert)
    return backend, convert


def reference_decode(backend, model, ids):
    """Teacher-forced positions through the reference CPU stage."""
    stage = backend.CPUDecoderStage(model, 0, 64)
    embedding = np.asarray(model.raw("token_embedding"), dtype=np.float32)
    layers = model.metadata["layers"]
    out = []
    for position, token in enumerate(ids):
        hidden = backend._bf16(embedding[token])
        for layer in range(layers):
            hidden = stage.layer(hidden, layer, position)
        logits = np.asarray(stage.logits(hidden), dtype=np.float32)
        out.append((logits, np.asarray(hidden).view(np.uint16).copy()))
    return out


def decode_case(backend, name, seed, positions, full_logits, layers=None):
    model = synthetic.build(name, seed=seed, layers=layers)
    ids = synthetic.prompt_ids(model.shape.vocab, positions, seed)
    results = reference_decode(backend, model, ids)
    logits = np.stack([r[0] for r in results])
    hidden = np.stack([r[1] for r in results])
    order = np.argsort(-logits, axis=1, kind="stable")
    top = order[:, :32]
    record = {
        "shape": np.array(name),
        "seed": np.array(seed),
        "layers": np.array(model.shape.layers),
        "ids": np.array(ids, dtype=np.int64),
        "argmax": logits.argmax(axis=1).astype(np.int64),
        "margin": np.take_along_axis(logits, order[:, :1], 1)[:, 0]
        - np.take_along_axis(logits, order[:, 1:2], 1)[:, 0],
        "top_ids": top.astype(np.int64),
        "top_logits": np.take_along_axis(logits, top, 1),
        "final_hidden_bits": hidden,
        "embedding_sha256": np.array(
            hashlib.sha256(np.asarray(model.raw("token_embedding")).tobytes()).hexdigest()
        ),
    }
    if full_logits:
        record["logits"] = logits
    else:
        stride = 151
        record["sample_stride"] = np.array(stride)
        record["sample_logits"] = logits[:, ::stride]
    return record


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"))
    parser.add_argument("--skip-full", action="store_true")
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set REFERENCE_ROOT")
    backend, convert = load_reference(args.reference)

    cases = [
        ("decode_tiny-qwen.npz", dict(name="tiny-qwen", seed=11, positions=20, full_logits=True)),
        ("decode_tiny-llama.npz", dict(name="tiny-llama", seed=12, positions=20, full_logits=True)),
    ]
    if not args.skip_full:
        cases += [
            ("decode_qwen2.5-0.5b.npz", dict(name="qwen2.5-0.5b", seed=0, positions=6, full_logits=False)),
            ("decode_smollm2-135m.npz", dict(name="smollm2-135m", seed=0, positions=6, full_logits=False)),
        ]
    for filename, options in cases:
        record = decode_case(backend, **options)
        np.savez_compressed(HERE / filename, **record)
        print("wrote", filename, "argmax", record["argmax"].tolist())

    # Quantiser: the converter test's matrix plus seeded BF16 projections.
    rng = np.random.default_rng(7)
    matrix = rng.normal(0, 0.2, (32, 64)).astype(np.float32)
    q, scale = convert.quantize_per_output_channel(matrix)
    qwen = synthetic.build("tiny-qwen", seed=11)
    projection = qwen.bf16_projection("layer00.gate_up")
    q2, s2 = convert.quantize_per_output_channel(projection)
    edge = np.zeros((4, 32), np.float32)
    edge[1, 5] = -1e-30
    edge[2, :] = 127.0
    edge[3, ::2] = 0.5
    q3, s3 = convert.quantize_per_output_channel(edge)
    np.savez_compressed(
        HERE / "quantize.npz",
        matrix=matrix, q=q, scale=scale,
        proj_q_head=q2[:48], proj_scale=s2,
        proj_q_sha256=np.array(hashlib.sha256(q2.tobytes()).hexdigest()),
        edge=edge, edge_q=q3, edge_scale=s3,
    )
    print("wrote quantize.npz")

    # Attention toy case of the reference test.
    stage = object.__new__(backend.CPUDecoderStage)
    stage.q_heads, stage.kv_heads, stage.q_per_kv, stage.head_dim = 4, 2, 2, 4
    stage._rope_inv_frequency = np.array([1.0, 0.5], dtype=np.float32)
    stage.key_cache = {0: np.zeros((2, 5, 4), dtype=bfloat16)}
    stage.value_cache = {0: np.zeros((2, 5, 4), dtype=bfloat16)}
    rng = np.random.default_rng(42)
    qkv = rng.normal(size=32).astype(np.float32).astype(bfloat16)
    out = np.asarray(stage._attention(qkv, 0, 3), dtype=np.float32)
    np.savez_compressed(
        HERE / "attention.npz",
        qkv=np.asarray(qkv).view(np.uint16), position=np.array(3), out=out,
        key_cache=np.asarray(stage.key_cache[0]).view(np.uint16),
        value_cache=np.asarray(stage.value_cache[0]).view(np.uint16),
    )
    print("wrote attention.npz")


if __name__ == "__main__":
    main()
