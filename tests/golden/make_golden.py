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
* ``request_<shape>_<weights>.npz`` -- the complete benchmarked requests:
  the prompt, then greedy decoding with the token fed back, the way
  ``NPUDecoder._generate_tokens_core`` drives the CPU stage
  (npu_llm/runtime/generate.py:1110-1158); per position the argmax, top-2
  margin, top-32 logits and a strided sample.  Qwen2.5-0.5B BF16: the
  32-position window of the 40-id prompt + 32 tokens (64 positions);
  SmolLM2-135M BF16: 35 + 16; Qwen2.5-0.5B W8: 32 + 32.  The reference has
  no W8 CPU runtime, so the W8 request comes from this repository's W8
  oracle (its projection arithmetic follows the reference W8 kernels; its
  int8 bytes are pinned by ``quantize.npz``).
* ``serving_qwen2.5-0.5b.npz`` -- four requests of the multi-stream serving
  workload (two opening with its shared 16-token prefix), each with 16
  greedy tokens from the reference CPU stage run alone, with per-token
  top-2 margins.
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


class _ReferenceStep:
    """One position of the reference CPU stage through every layer, as
    ``decode_token`` runs it with ``npu_layers=0``."""

    def __init__(self, backend, model):
        self.backend = backend
        self.stage = backend.CPUDecoderStage(model, 0, 64)
        self.embedding = np.asarray(model.raw("token_embedding"), dtype=np.float32)
        self.layers = model.metadata["layers"]

    def __call__(self, token, position):
        hidden = self.backend._bf16(self.embedding[token])
        for layer in range(self.layers):
            hidden = self.stage.layer(hidden, layer, position)
        return np.asarray(self.stage.logits(hidden), dtype=np.float32)


def greedy_request(step, prompt, new_tokens, context=64):
    """Prompt positions, then greedy tokens fed back; every generated token
    is also fed (its successor's logits are recorded) while the context
    lasts.  Returns (fed ids, logits per position, generated tokens)."""
    ids, rows, generated = [], [], []
    token = None
    for position in range(min(context, len(prompt) + new_tokens)):
        token = prompt[position] if position < len(prompt) else generated[-1]
        logits = step(int(token), position)
        ids.append(int(token))
        rows.append(logits)
        if position >= len(prompt) - 1 and len(generated) < new_tokens:
            generated.append(int(np.argmax(logits)))
    return ids, np.stack(rows), generated


def summarize_logits(logits, stride):
    order = np.argsort(-logits, axis=1, kind="stable")
    top = order[:, :32]
    return {
        "argmax": logits.argmax(axis=1).astype(np.int64),
        "margin": np.take_along_axis(logits, order[:, :1], 1)[:, 0]
        - np.take_along_axis(logits, order[:, 1:2], 1)[:, 0],
        "top_ids": top.astype(np.int32),
        "top_logits": np.take_along_axis(logits, top, 1),
        "sample_stride": np.array(stride),
        "sample_logits": logits[:, ::stride].astype(np.float32),
        "norm": np.linalg.norm(logits, axis=1).astype(np.float32),
    }


def request_case(backend, name, weights, n_prompt, new_tokens, stride):
    model = synthetic.build(name, seed=0).materialize()
    prompt = synthetic.prompt_ids(model.shape.vocab, 40, 1)[:n_prompt]
    if weights == "bf16":
        step = _ReferenceStep(backend, model)
    else:
        sys.path.insert(0, str(REPO))
        from oracle.cpu_decoder import OracleDecoder

        oracle = OracleDecoder(model, weights="w8")
        step = lambda token, position: oracle.step(token, position)  # noqa: E731
    ids, logits, generated = greedy_request(step, prompt, new_tokens)
    record = {"shape": np.array(name), "weights": np.array(weights), "seed": np.array(0),
              "prompt": np.array(prompt, dtype=np.int64), "ids": np.array(ids, dtype=np.int64),
              "generated": np.array(generated, dtype=np.int64),
              "source": np.array("reference CPUDecoderStage" if weights == "bf16" else "repository W8 oracle")}
    record.update(summarize_logits(logits, stride))
    return record


def serving_case(backend, picks=(0, 1, 2, 4), new_tokens=16):
    model = synthetic.build("qwen2.5-0.5b", seed=0).materialize()
    prompts = synthetic.ragged_prompts(model.shape.vocab)
    out = {"picks": np.array(picks, dtype=np.int64)}
    for i in picks:
        step = _ReferenceStep(backend, model)  # a fresh cache per request
        prompt = prompts[i]
        ids, logits, generated = greedy_request(step, prompt, new_tokens, context=len(prompt) + new_tokens - 1)
        summary = summarize_logits(logits[len(prompt) - 1:], 301)
        out[f"prompt_{i}"] = np.array(prompt, dtype=np.int64)
        out[f"generated_{i}"] = np.array(generated, dtype=np.int64)
        out[f"margin_{i}"] = summary["margin"]
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"))
    parser.add_argument("--skip-full", action="store_true")
    parser.add_argument("--only", choices=["all", "requests"], default="all",
                        help="requests: write only the whole-request and serving fixtures")
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set REFERENCE_ROOT")
    backend, convert = load_reference(args.reference)
    if args.only == "requests" or not args.skip_full:
        for name, weights, n_prompt, new_tokens, stride in (("qwen2.5-0.5b", "bf16", 32, 32, 301),
                                                            ("smollm2-135m", "bf16", 35, 16, 97),
                                                            ("qwen2.5-0.5b", "w8", 32, 32, 301)):
            record = request_case(backend, name, weights, n_prompt, new_tokens, stride)
            np.savez_compressed(HERE / f"request_{name}_{weights}.npz", **record)
            print(f"wrote request_{name}_{weights}.npz generated", record["generated"].tolist())
        record = serving_case(backend)
        np.savez_compressed(HERE / "serving_qwen2.5-0.5b.npz", **record)
        print("wrote serving_qwen2.5-0.5b.npz")
    if args.only == "requests":
        return

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
