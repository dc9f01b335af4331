"""The CPU oracle against golden vectors recorded from the reference itself
(tests/golden/make_golden.py imports npu_llm/runtime/cpu_backend.py and
npu_llm/tools/convert_smollm2.py), plus the reference's own known-answer
tests restated: the quantiser bound (npu_llm/tests/test_converter.py:15-23)
and the vectorised attention check (npu_llm/tests/test_cpu_backend.py:17-52).
"""

import hashlib

import numpy as np
import pytest
from ml_dtypes import bfloat16

from oracle.cpu_decoder import OracleDecoder, rope_inverse_frequency, to_bf16
from runtime import synthetic
from runtime.quantize import quantize_per_output_channel


def run_oracle(g):
    model = synthetic.build(str(g["shape"]), seed=int(g["seed"]))
    oracle = OracleDecoder(model)
    logits, hidden = [], []
    for position, token in enumerate(g["ids"]):
        trace = []
        logits.append(oracle.step(int(token), position, trace=trace))
        hidden.append(np.asarray(trace[-1]).view(np.uint16))
    return model, np.stack(logits), np.stack(hidden)


@pytest.mark.parametrize("name", ["tiny-qwen", "tiny-llama"])
def test_oracle_matches_reference_small(name, golden):
    g = golden(f"decode_{name}.npz")
    model, logits, hidden = run_oracle(g)
    assert hashlib.sha256(np.asarray(model.raw("token_embedding")).tobytes()).hexdigest() == str(
        g["embedding_sha256"])
    # same NumPy arithmetic as the reference: BF16 hidden states bit-equal,
    # logits equal up to the host BLAS's summation order
    assert np.mean(hidden != g["final_hidden_bits"]) <= 0.002
    np.testing.assert_allclose(logits, g["logits"], rtol=0, atol=2e-5)
    assert np.array_equal(logits.argmax(axis=1), g["argmax"]) or np.all(
        g["margin"][logits.argmax(axis=1) != g["argmax"]] <= 0.05)


@pytest.mark.parametrize("name", ["qwen2.5-0.5b", "smollm2-135m"])
def test_oracle_matches_reference_full_size(name, golden):
    g = golden(f"decode_{name}.npz")
    positions = 3
    model = synthetic.build(name, seed=int(g["seed"])).materialize()
    oracle = OracleDecoder(model)
    stride = int(g["sample_stride"])
    for position in range(positions):
        logits = oracle.step(int(g["ids"][position]), position)
        np.testing.assert_allclose(logits[::stride], g["sample_logits"][position], rtol=0, atol=1e-4)
        np.testing.assert_allclose(logits[g["top_ids"][position]], g["top_logits"][position], rtol=0, atol=1e-4)
        assert int(np.argmax(logits)) == int(g["argmax"][position]) or g["margin"][position] <= 0.05


def test_oracle_matches_reference_whole_request(golden):
    """The SmolLM2-135M request of the benchmark (35 prompt positions + 16
    greedy tokens) through the oracle, against the reference CPU stage's
    recording: logits at every position and the greedy tokens."""
    g = golden("request_smollm2-135m_bf16.npz")
    model = synthetic.build("smollm2-135m", seed=int(g["seed"])).materialize()
    oracle = OracleDecoder(model)
    stride = int(g["sample_stride"])
    n_prompt = len(g["prompt"])
    generated = []
    for position, token in enumerate(g["ids"]):
        logits = oracle.step(int(token), position)
        np.testing.assert_allclose(logits[::stride], g["sample_logits"][position], rtol=0, atol=1e-4)
        np.testing.assert_allclose(logits[g["top_ids"][position]], g["top_logits"][position], rtol=0, atol=1e-4)
        if position >= n_prompt - 1 and len(generated) < len(g["generated"]):
            generated.append(int(np.argmax(logits)))
    assert generated == g["generated"].tolist()


def test_request_fixtures_are_consistent(golden):
    """Each whole-request fixture feeds its prompt, then its own greedy
    tokens, and its top-1 entries are its argmax."""
    for name in ("request_qwen2.5-0.5b_bf16", "request_smollm2-135m_bf16", "request_qwen2.5-0.5b_w8"):
        g = golden(f"{name}.npz")
        n = len(g["prompt"])
        ids = g["ids"].tolist()
        assert ids[:n] == g["prompt"].tolist()
        assert ids[n:] == g["generated"].tolist()[: len(ids) - n]
        assert np.array_equal(g["top_ids"][:, 0], g["argmax"])
        assert np.all(g["margin"] >= 0)


def test_quantiser_is_bit_exact_with_reference(golden):
    g = golden("quantize.npz")
    q, s = quantize_per_output_channel(g["matrix"])
    assert np.array_equal(q, g["q"]) and np.array_equal(s.view(np.uint32), g["scale"].view(np.uint32))
    model = synthetic.build("tiny-qwen", seed=11)
    q, s = quantize_per_output_channel(model.bf16_projection("layer00.gate_up"))
    assert np.array_equal(q[:48], g["proj_q_head"])
    assert hashlib.sha256(q.tobytes()).hexdigest() == str(g["proj_q_sha256"])
    assert np.array_equal(s.view(np.uint32), g["proj_scale"].view(np.uint32))
    q, s = quantize_per_output_channel(g["edge"])
    assert np.array_equal(q, g["edge_q"]) and np.array_equal(s.view(np.uint32), g["edge_scale"].view(np.uint32))


def test_quantiser_error_bound():
    """npu_llm/tests/test_converter.py:15-23: |q*s - w| <= s/2 per row."""
    rng = np.random.default_rng(7)
    weight = rng.normal(0, 0.2, (32, 64)).astype(np.float32)
    q, scale = quantize_per_output_channel(weight)
    restored = q.astype(np.float32) * scale[:, None]
    assert q.dtype == np.int8 and scale.dtype == np.float32
    assert np.all(np.abs(restored - weight).max(axis=1) <= scale / 2 + 1e-6)


class _ToyModel:
    """Just enough of the package surface for the attention toy case."""

    metadata = {"hidden_size": 16, "intermediate_size": 16, "attention_heads": 4, "kv_heads": 2,
                "head_dim": 4, "layers": 1, "vocab_size": 8, "rope_theta": 10000.0}
    tensors = {}


def test_attention_matches_reference_toy_case(golden):
    """The reference's own attention test inputs (seed 42) and its output."""
    g = golden("attention.npz")
    oracle = OracleDecoder(_ToyModel(), context_length=5)
    # the reference test fixes inv_freq = [1, 0.5]
    inv = np.array([1.0, 0.5], np.float32)
    for p in range(5):
        angle = np.float32(p) * inv
        oracle.cos[p] = np.cos(angle)
        oracle.sin[p] = np.sin(angle)
    qkv = np.asarray(g["qkv"]).view(bfloat16)
    out = np.asarray(oracle.attention(qkv, 0, int(g["position"])), np.float32)
    np.testing.assert_allclose(out, g["out"], rtol=0, atol=0)
    assert np.array_equal(np.asarray(oracle.keys[0]).view(np.uint16), g["key_cache"])
    assert np.array_equal(np.asarray(oracle.values[0]).view(np.uint16), g["value_cache"])


def test_rope_inverse_frequency_is_float32():
    inv = rope_inverse_frequency(1e6, 64)
    assert inv.dtype == np.float32 and inv[0] == 1.0
    assert to_bf16(np.float32(1.00390625)).dtype == bfloat16
