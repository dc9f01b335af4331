"""B200 weight layout: one device blob holding every tensor the engine streams.

The reference packs its weights into AIE tile streams (six GEMV tiles with
uneven row slices, npu_llm/designs/qwen_engine_layout.py:18-190 and
npu_llm/designs/engine_layout.py:11-105).  That layout is an AIE workaround;
this build defines its own for a persistent B200 kernel whose CTAs stream
their share of each projection through a shared-memory ring with bulk copies:

* **Row-group major projections.**  8 consecutive output rows form a *row
  group*.  A group stores its K dimension as 16-byte column chunks, each chunk
  holding the 8 rows' bytes for that column range: byte offset of (row r,
  chunk j) = group * (K_bytes * 8) + j * 128 + (r % 8) * 16.  A CTA's share of
  a projection is a contiguous run of row groups, a K-slice of one group is
  contiguous too, and a warp reading one chunk column touches 128 contiguous
  bytes (bank-conflict free).  The same bytes are the no-swizzle K-major
  8x16-byte "core matrix" arrangement the tensor-core descriptors use.
* **gate_up paired.**  Packed row group 2b holds gate rows 8b..8b+7 and packed
  group 2b+1 the matching up rows, so a CTA always owns both halves of the
  SwiGLU it computes.
* **W8** stores the int8 bytes (bit-identical to the quantiser) in the same
  arrangement (16 columns per chunk) plus one FP32 scale per packed row.
* Norm weights and the q/k/v bias are FP32; the embedding is BF16 row-major.
  Every tensor starts on a 256-byte boundary.

``pack`` builds the blob from a model with the package surface; ``unpack``
inverts it exactly (the round-trip test compares bits).
"""

from dataclasses import dataclass
import ctypes

import numpy as np
from ml_dtypes import bfloat16

from runtime.synthetic import shape_from_metadata

LAYOUT_VERSION = 1
ALIGN = 256
ROW_GROUP = 8
CHUNK = 16

FORMATS = {"bf16": 0, "w8": 1}


def _align(value):
    return (value + ALIGN - 1) // ALIGN * ALIGN


def element_bytes(fmt):
    return 2 if fmt == "bf16" else 1


# -- single-matrix packing ----------------------------------------------------
def pack_matrix_bytes(matrix):
    """[rows, K] array of 1- or 2-byte elements -> row-group-major bytes."""
    m = np.ascontiguousarray(matrix)
    rows = m.shape[0]
    raw = m.view(np.uint8).reshape(rows, -1)
    kbytes = raw.shape[1]
    if rows % ROW_GROUP or kbytes % CHUNK:
        raise ValueError("rows must be a multiple of 8 and K bytes of 16")
    tiles = raw.reshape(rows // ROW_GROUP, ROW_GROUP, kbytes // CHUNK, CHUNK)
    return np.ascontiguousarray(tiles.transpose(0, 2, 1, 3)).reshape(-1)


def unpack_matrix_bytes(blob, rows, kbytes):
    tiles = np.asarray(blob, np.uint8).reshape(
        rows // ROW_GROUP, kbytes // CHUNK, ROW_GROUP, CHUNK
    )
    return np.ascontiguousarray(tiles.transpose(0, 2, 1, 3)).reshape(rows, kbytes)


def gate_up_order(intermediate):
    """Packed row -> original row of the fused [gate; up] matrix."""
    order = np.empty(2 * intermediate, np.int64)
    groups = intermediate // ROW_GROUP
    for b in range(groups):
        base = 2 * b * ROW_GROUP
        order[base: base + ROW_GROUP] = np.arange(b * ROW_GROUP, (b + 1) * ROW_GROUP)
        order[base + ROW_GROUP: base + 2 * ROW_GROUP] = intermediate + np.arange(
            b * ROW_GROUP, (b + 1) * ROW_GROUP
        )
    return order


# -- offsets --------------------------------------------------------------------
LAYER_FIELDS = (
    "gamma_in", "gamma_post", "qkv_bias",
    "w_qkv", "s_qkv", "w_o", "s_o", "w_gate_up", "s_gate_up", "w_down", "s_down",
)


class HbLayerOffsets(ctypes.Structure):
    _fields_ = [(name, ctypes.c_uint64) for name in LAYER_FIELDS]


@dataclass
class Layout:
    shape: object
    fmt: str
    layers: list          # list of dicts field -> offset
    gamma_final: int
    w_lm: int
    s_lm: int
    embedding: int
    total: int

    def layer_table(self):
        table = (HbLayerOffsets * len(self.layers))()
        for i, offsets in enumerate(self.layers):
            for name in LAYER_FIELDS:
                setattr(table[i], name, offsets[name])
        return table


def plan(shape, fmt="bf16"):
    """Offsets of every tensor for a model shape and weight format."""
    if fmt not in FORMATS:
        raise ValueError("weight format must be 'bf16' or 'w8'")
    e = element_bytes(fmt)
    h, i, d = shape.hidden, shape.intermediate, shape.head_dim
    cursor = 0

    def take(nbytes):
        nonlocal cursor
        start = cursor
        cursor = _align(cursor + nbytes)
        return start

    layers = []
    for _ in range(shape.layers):
        off = {}
        off["gamma_in"] = take(4 * h)
        off["gamma_post"] = take(4 * h)
        off["qkv_bias"] = take(4 * shape.qkv_rows)
        off["w_qkv"] = take(shape.qkv_rows * h * e)
        off["s_qkv"] = take(4 * shape.qkv_rows) if fmt == "w8" else 0
        off["w_o"] = take(h * shape.q_heads * d * e)
        off["s_o"] = take(4 * h) if fmt == "w8" else 0
        off["w_gate_up"] = take(2 * i * h * e)
        off["s_gate_up"] = take(4 * 2 * i) if fmt == "w8" else 0
        off["w_down"] = take(h * i * e)
        off["s_down"] = take(4 * h) if fmt == "w8" else 0
        layers.append(off)
    gamma_final = take(4 * h)
    w_lm = take(shape.vocab * h * e)
    s_lm = take(4 * shape.vocab) if fmt == "w8" else 0
    embedding = take(shape.vocab * h * 2)
    return Layout(shape, fmt, layers, gamma_final, w_lm, s_lm, embedding, cursor)


def check_dims(shape, fmt="bf16"):
    """The divisibility the kernels rely on; raises ValueError otherwise."""
    e = element_bytes(fmt)
    problems = []
    if shape.head_dim != 64:
        problems.append("head_dim must be 64")
    if shape.q_heads % shape.kv_heads:
        problems.append("q_heads must be a multiple of kv_heads")
    for name, rows, k in (
        ("qkv", shape.qkv_rows, shape.hidden),
        ("o_proj", shape.hidden, shape.q_heads * shape.head_dim),
        ("gate_up", 2 * shape.intermediate, shape.hidden),
        ("down_proj", shape.hidden, shape.intermediate),
        ("lm_head", shape.vocab, shape.hidden),
    ):
        if rows % ROW_GROUP:
            problems.append(f"{name} rows must be a multiple of 8")
        if (k * e) % CHUNK or k % 32:
            problems.append(f"{name} K must be a multiple of 32")
    if shape.intermediate % ROW_GROUP:
        problems.append("intermediate must be a multiple of 8")
    if problems:
        raise ValueError("; ".join(problems))


# -- packing --------------------------------------------------------------------
def _weights_of(model, name, fmt):
    """(matrix as raw elements, FP32 scales or None) for one projection."""
    if fmt == "w8":
        tensor = model.quantized(name)
        return np.asarray(tensor.weight, np.int8), np.asarray(tensor.scale, np.float32)
    return np.asarray(model.bf16_projection(name)).astype(bfloat16, copy=False), None


def _f32(values):
    return np.asarray(values, dtype=np.float32).reshape(-1)


def pack(model, fmt="bf16"):
    """Build (blob uint8 array, Layout) for a model with the package surface."""
    shape = shape_from_metadata(model.metadata)
    check_dims(shape, fmt)
    lay = plan(shape, fmt)
    blob = np.zeros(lay.total, np.uint8)

    def put(offset, array):
        data = np.ascontiguousarray(array).view(np.uint8).reshape(-1)
        blob[offset: offset + data.size] = data

    h, i, d = shape.hidden, shape.intermediate, shape.head_dim
    for layer, off in enumerate(lay.layers):
        p = f"layer{layer:02d}"
        put(off["gamma_in"], _f32(model.raw(f"{p}.input_norm")))
        put(off["gamma_post"], _f32(model.raw(f"{p}.post_attn_norm")))
        if f"{p}.qkv_bias" in model.tensors:
            put(off["qkv_bias"], _f32(model.raw(f"{p}.qkv_bias")))
        w, s = _weights_of(model, f"{p}.qkv", fmt)
        put(off["w_qkv"], pack_matrix_bytes(w))
        if s is not None:
            put(off["s_qkv"], s)
        w, s = _weights_of(model, f"{p}.o_proj", fmt)
        put(off["w_o"], pack_matrix_bytes(w))
        if s is not None:
            put(off["s_o"], s)
        w, s = _weights_of(model, f"{p}.gate_up", fmt)
        order = gate_up_order(i)
        put(off["w_gate_up"], pack_matrix_bytes(w[order]))
        if s is not None:
            put(off["s_gate_up"], s[order])
        w, s = _weights_of(model, f"{p}.down_proj", fmt)
        put(off["w_down"], pack_matrix_bytes(w))
        if s is not None:
            put(off["s_down"], s)
    put(lay.gamma_final, _f32(model.raw("final_norm")))
    w, s = _weights_of(model, "lm_head", fmt)
    put(lay.w_lm, pack_matrix_bytes(w))
    if s is not None:
        put(lay.s_lm, s)
    embedding = np.asarray(model.raw("token_embedding"), dtype=np.float32).astype(bfloat16)
    put(lay.embedding, embedding)
    return blob, lay


def unpack(blob, lay):
    """Invert ``pack``: dict name -> array in the package's row order.
    Projections come back as BF16 (or (int8, scale) pairs for W8)."""
    shape, fmt = lay.shape, lay.fmt
    e = element_bytes(fmt)
    h, i, d = shape.hidden, shape.intermediate, shape.head_dim
    blob = np.asarray(blob, np.uint8)

    def raw(offset, nbytes):
        return blob[offset: offset + nbytes]

    def matrix(offset, rows, k):
        kb = k * e
        m = unpack_matrix_bytes(raw(offset, rows * kb), rows, kb)
        return m.view(bfloat16) if fmt == "bf16" else m.view(np.int8)

    def scales(offset, rows):
        return raw(offset, 4 * rows).view(np.float32).copy()

    out = {}
    for layer, off in enumerate(lay.layers):
        p = f"layer{layer:02d}"
        out[f"{p}.input_norm"] = raw(off["gamma_in"], 4 * h).view(np.float32).copy()
        out[f"{p}.post_attn_norm"] = raw(off["gamma_post"], 4 * h).view(np.float32).copy()
        out[f"{p}.qkv_bias"] = raw(off["qkv_bias"], 4 * shape.qkv_rows).view(np.float32).copy()
        out[f"{p}.qkv"] = matrix(off["w_qkv"], shape.qkv_rows, h)
        out[f"{p}.o_proj"] = matrix(off["w_o"], h, shape.q_heads * d)
        packed = matrix(off["w_gate_up"], 2 * i, h)
        order = gate_up_order(i)
        restored = np.empty_like(packed)
        restored[order] = packed
        out[f"{p}.gate_up"] = restored
        out[f"{p}.down_proj"] = matrix(off["w_down"], h, i)
        if fmt == "w8":
            out[f"{p}.qkv.scale"] = scales(off["s_qkv"], shape.qkv_rows)
            out[f"{p}.o_proj.scale"] = scales(off["s_o"], h)
            gu = scales(off["s_gate_up"], 2 * i)
            restored_scale = np.empty_like(gu)
            restored_scale[order] = gu
            out[f"{p}.gate_up.scale"] = restored_scale
            out[f"{p}.down_proj.scale"] = scales(off["s_down"], h)
    out["final_norm"] = raw(lay.gamma_final, 4 * h).view(np.float32).copy()
    out["lm_head"] = matrix(lay.w_lm, shape.vocab, h)
    if fmt == "w8":
        out["lm_head.scale"] = scales(lay.s_lm, shape.vocab)
    out["token_embedding"] = raw(lay.embedding, shape.vocab * h * 2).view(bfloat16).reshape(
        shape.vocab, h
    ).copy()
    return out
