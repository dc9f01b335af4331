"""B200 weight layout: exact round trips on the raw bits (the counterpart of
npu_llm/tests/test_engine_layout.py:191-212 and
npu_llm/tests/test_qwen_engine_layout.py:333-387 for the AIE layouts)."""

import numpy as np
import pytest
from ml_dtypes import bfloat16

from runtime import layout, synthetic


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint16) if a.dtype == np.dtype(bfloat16) else a


@pytest.mark.parametrize("name", ["tiny-qwen", "tiny-llama"])
@pytest.mark.parametrize("fmt", ["bf16", "w8"])
def test_every_tensor_round_trips(name, fmt):
    model = synthetic.build(name, seed=5)
    blob, lay = layout.pack(model, fmt)
    assert blob.size == lay.total
    out = layout.unpack(blob, lay)
    for layer in range(model.shape.layers):
        p = f"layer{layer:02d}"
        for t in layout_projections():
            if fmt == "bf16":
                assert np.array_equal(bits(out[f"{p}.{t}"]), bits(model.bf16_projection(f"{p}.{t}"))), t
            else:
                q = model.quantized(f"{p}.{t}")
                assert np.array_equal(out[f"{p}.{t}"], q.weight), t
                assert np.array_equal(out[f"{p}.{t}.scale"].view(np.uint32), q.scale.view(np.uint32)), t
        for t in ("input_norm", "post_attn_norm"):
            assert np.array_equal(out[f"{p}.{t}"], np.asarray(model.raw(f"{p}.{t}"), np.float32))
        if model.shape.qkv_bias:
            assert np.array_equal(out[f"{p}.qkv_bias"].view(np.uint32),
                                  np.asarray(model.raw(f"{p}.qkv_bias"), np.float32).view(np.uint32))
        else:
            assert not out[f"{p}.qkv_bias"].any()
    assert np.array_equal(bits(out["token_embedding"]), bits(model.raw("token_embedding")))
    if fmt == "bf16":
        assert np.array_equal(bits(out["lm_head"]), bits(model.bf16_projection("lm_head")))


def layout_projections():
    return ("qkv", "o_proj", "gate_up", "down_proj")


def test_row_group_layout_formula():
    """Byte (row r, chunk j) of a packed matrix sits at
    group * K_bytes * 8 + j * 128 + (r % 8) * 16."""
    rows, k = 24, 40
    m = np.arange(rows * k, dtype=np.uint16).reshape(rows, k)
    packed = layout.pack_matrix_bytes(m).view(np.uint16)
    kbytes = k * 2
    for r in range(rows):
        for j in range(kbytes // 16):
            off = (r // 8) * kbytes * 8 + j * 128 + (r % 8) * 16
            assert np.array_equal(packed[off // 2: off // 2 + 8], m[r, j * 8: j * 8 + 8])
    assert np.array_equal(layout.unpack_matrix_bytes(packed.view(np.uint8), rows, kbytes).view(np.uint16), m)


def test_gate_up_pairs_gate_and_up_rows():
    order = layout.gate_up_order(16)
    assert list(order[:8]) == list(range(8))
    assert list(order[8:16]) == list(range(16, 24))
    assert list(order[16:24]) == list(range(8, 16))
    assert sorted(order) == list(range(32))


@pytest.mark.parametrize("name", list(synthetic.SHAPES))
@pytest.mark.parametrize("fmt", ["bf16", "w8"])
def test_offsets_are_aligned_and_disjoint(name, fmt):
    shape = synthetic.SHAPES[name]
    lay = layout.plan(shape, fmt)
    e = layout.element_bytes(fmt)
    spans = []
    for off in lay.layers:
        sizes = {
            "gamma_in": 4 * shape.hidden, "gamma_post": 4 * shape.hidden, "qkv_bias": 4 * shape.qkv_rows,
            "w_qkv": shape.qkv_rows * shape.hidden * e, "w_o": shape.hidden * shape.hidden * e,
            "w_gate_up": 2 * shape.intermediate * shape.hidden * e, "w_down": shape.hidden * shape.intermediate * e,
        }
        if fmt == "w8":
            sizes.update(s_qkv=4 * shape.qkv_rows, s_o=4 * shape.hidden, s_gate_up=8 * shape.intermediate,
                         s_down=4 * shape.hidden)
        for field, size in sizes.items():
            assert off[field] % 256 == 0
            spans.append((off[field], off[field] + size))
    spans.append((lay.w_lm, lay.w_lm + shape.vocab * shape.hidden * e))
    spans.append((lay.embedding, lay.embedding + shape.vocab * shape.hidden * 2))
    spans.sort()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert spans[-1][1] <= lay.total


def test_check_dims_rejects_unsupported_shapes():
    bad = synthetic.with_layers(synthetic.TINY_QWEN, 1)
    layout.check_dims(bad)
    from dataclasses import replace
    with pytest.raises(ValueError):
        layout.check_dims(replace(bad, head_dim=32))
    with pytest.raises(ValueError):
        layout.check_dims(replace(bad, intermediate=520))
