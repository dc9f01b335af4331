"""Seeded random-init decoder models with the reference package surface.

The reference's benchmark configurations use random-init weights (there is no
network for checkpoints).  This module builds those models deterministically
from a seed and exposes the same read surface as the reference's
``runtime.model.XDNA1Model`` (``metadata``, ``tensors``, ``raw``,
``bf16_projection``, ``quantized``; npu_llm/runtime/model.py:84-198), so the
engine, the package writer and the CPU oracle all consume one object.

Tensor names and the fused projections follow the reference converter
(npu_llm/tools/convert_smollm2.py:214-311): ``token_embedding``,
``layerNN.{qkv,o_proj,gate_up,down_proj}`` (q|k|v and gate|up row-concatenated),
``layerNN.qkv_bias`` (FP32), ``layerNN.{input_norm,post_attn_norm}``,
``final_norm`` and a tied ``lm_head``.

Value distributions (the benchmark text gives N(0, 0.02) BF16 weights and
RMSNorm weights of 1.0): every weight is ``standard_normal * 0.02`` rounded to
BF16; the Qwen q/k/v bias is drawn the same way and stored as FP32 (a converted
BF16 checkpoint stores its bias the same way).  Each tensor draws from its own
``np.random.default_rng([seed, tensor_index])`` stream, so any single tensor can
be regenerated without the others.
"""

from dataclasses import dataclass, asdict
import numpy as np
from ml_dtypes import bfloat16

from runtime.quantize import quantize_per_output_channel


@dataclass(frozen=True)
class ModelShape:
    family: str            # "llama" (SmolLM2) or "qwen2"
    hidden: int
    intermediate: int
    q_heads: int
    kv_heads: int
    head_dim: int
    layers: int
    vocab: int
    rope_theta: float
    rms_eps: float
    qkv_bias: bool
    context: int = 64

    @property
    def qkv_rows(self):
        return (self.q_heads + 2 * self.kv_heads) * self.head_dim


# SmolLM2-135M and Qwen2.5-0.5B geometry: 30 layers of hidden 576 (9 q / 3 kv heads,
# intermediate 1536, vocab 49152, theta 1e5, eps 1e-5); 24 layers of hidden 896
# (14 q / 2 kv heads, intermediate 4864, vocab 151936, theta 1e6, eps 1e-6, qkv bias).
SMOLLM2_135M = ModelShape("llama", 576, 1536, 9, 3, 64, 30, 49152, 1e5, 1e-5, False)
QWEN25_05B = ModelShape("qwen2", 896, 4864, 14, 2, 64, 24, 151936, 1e6, 1e-6, True)
# Small shapes with the same head geometry, for fast parity cases.
TINY_QWEN = ModelShape("qwen2", 256, 512, 4, 2, 64, 2, 1024, 1e6, 1e-6, True)
TINY_LLAMA = ModelShape("llama", 192, 384, 3, 1, 64, 2, 768, 1e5, 1e-5, False)

SHAPES = {
    "smollm2-135m": SMOLLM2_135M,
    "qwen2.5-0.5b": QWEN25_05B,
    "tiny-qwen": TINY_QWEN,
    "tiny-llama": TINY_LLAMA,
}


def with_layers(shape, layers):
    """The same shape with a different layer count (for short parity runs)."""
    values = asdict(shape)
    values["layers"] = int(layers)
    return ModelShape(**values)


def tensor_names(shape):
    """Every tensor of the package, in the fixed order that seeds them."""
    names = ["token_embedding"]
    for layer in range(shape.layers):
        prefix = f"layer{layer:02d}"
        names += [
            f"{prefix}.qkv",
            f"{prefix}.qkv_bias",
            f"{prefix}.o_proj",
            f"{prefix}.gate_up",
            f"{prefix}.down_proj",
            f"{prefix}.input_norm",
            f"{prefix}.post_attn_norm",
        ]
    names += ["final_norm", "lm_head"]
    return names


def tensor_shape(shape, name):
    h, i = shape.hidden, shape.intermediate
    leaf = name.split(".")[-1]
    if name in ("token_embedding", "lm_head"):
        return (shape.vocab, h)
    return {
        "qkv": (shape.qkv_rows, h),
        "qkv_bias": (shape.qkv_rows,),
        "o_proj": (h, shape.q_heads * shape.head_dim),
        "gate_up": (2 * i, h),
        "down_proj": (h, i),
        "input_norm": (h,),
        "post_attn_norm": (h,),
        "final_norm": (h,),
    }[leaf]


PROJECTIONS = ("qkv", "o_proj", "gate_up", "down_proj")


def metadata_for(shape):
    """Package metadata with the keys the reference converter writes
    (npu_llm/tools/convert_smollm2.py:183-202)."""
    return {
        "format": (
            "xdna1-qwen2-w8a16-v1" if shape.family == "qwen2"
            else "xdna1-smollm2-w8a16-v1"
        ),
        "model_family": shape.family,
        "hidden_size": shape.hidden,
        "intermediate_size": shape.intermediate,
        "attention_heads": shape.q_heads,
        "kv_heads": shape.kv_heads,
        "head_dim": shape.head_dim,
        "layers": shape.layers,
        "vocab_size": shape.vocab,
        "rope_theta": float(shape.rope_theta),
        "rms_norm_eps": float(shape.rms_eps),
        "context_length": shape.context,
        "activation_dtype": "bfloat16",
        "accumulator_dtype": "float32",
    }


def shape_from_metadata(metadata):
    family = metadata.get("model_family", "llama")
    q_heads = int(metadata["attention_heads"])
    kv_heads = int(metadata["kv_heads"])
    head_dim = int(metadata["head_dim"])
    return ModelShape(
        family=family,
        hidden=int(metadata["hidden_size"]),
        intermediate=int(metadata["intermediate_size"]),
        q_heads=q_heads,
        kv_heads=kv_heads,
        head_dim=head_dim,
        layers=int(metadata["layers"]),
        vocab=int(metadata["vocab_size"]),
        rope_theta=float(metadata.get("rope_theta", 10000.0)),
        rms_eps=float(metadata.get("rms_norm_eps", 1e-5)),
        qkv_bias=family == "qwen2",
        context=int(metadata.get("context_length", 64)),
    )


class QuantizedView:
    """``weight`` int8 [rows, K] and ``scale`` float32 [rows] of one projection
    (the surface of npu_llm/runtime/model.py:61-81)."""

    def __init__(self, weight, scale):
        self.weight = weight
        self.scale = scale
        self.shape = tuple(weight.shape)


class SyntheticModel:
    """A random-init model held in host memory."""

    def __init__(self, shape, seed=0):
        self.shape = shape
        self.seed = int(seed)
        self.metadata = metadata_for(shape)
        self.tensors = {}
        for name in tensor_names(shape):
            if name == "qkv_bias" or name.endswith(".qkv_bias"):
                if not shape.qkv_bias:
                    continue
            dims = list(tensor_shape(shape, name))
            leaf = name.split(".")[-1]
            if leaf in PROJECTIONS or name == "lm_head":
                self.tensors[name] = {"shape": dims, "layout": "row_major"}
            elif leaf == "qkv_bias":
                self.tensors[name] = {"shape": dims, "dtype": "float32"}
            else:
                self.tensors[name] = {"shape": dims, "dtype": "bfloat16"}
        self.metadata["tensors"] = self.tensors
        self._index = {name: i for i, name in enumerate(tensor_names(shape))}
        self._cache = {}
        self._quantized = {}

    def _generate(self, name):
        dims = tensor_shape(self.shape, name)
        leaf = name.split(".")[-1]
        if leaf in ("input_norm", "post_attn_norm", "final_norm"):
            return np.ones(dims, dtype=bfloat16)
        if name == "lm_head":
            # Tied embeddings: the LM head is the embedding table.
            return self.bf16("token_embedding")
        rng = np.random.default_rng([self.seed, self._index[name]])
        values = rng.standard_normal(dims, dtype=np.float32) * np.float32(0.02)
        values = values.astype(bfloat16)
        if leaf == "qkv_bias":
            return values.astype(np.float32)
        return values

    def bf16(self, name):
        if name not in self._cache:
            self._cache[name] = self._generate(name)
        return self._cache[name]

    # -- XDNA1Model surface -------------------------------------------------
    def raw(self, name):
        if name not in self.tensors:
            raise KeyError(name)
        return self.bf16(name)

    def bf16_projection(self, name):
        if name not in self.tensors:
            raise KeyError(name)
        return self.bf16(name)

    def quantized(self, name):
        if name not in self._quantized:
            q, scale = quantize_per_output_channel(self.bf16(name))
            self._quantized[name] = QuantizedView(q, scale)
        return self._quantized[name]

    def materialize(self, weights="bf16", threads=None):
        """Generate every tensor (and, for W8, its quantisation) in parallel.

        Each tensor has its own RNG stream, so the result does not depend on
        the order or the thread count."""
        from concurrent.futures import ThreadPoolExecutor
        import os

        names = [n for n in tensor_names(self.shape) if n in self.tensors and n != "lm_head"]
        workers = threads or min(16, os.cpu_count() or 1)
        with ThreadPoolExecutor(workers) as pool:
            for name, value in zip(names, pool.map(self._generate, names)):
                self._cache.setdefault(name, value)
            self.bf16("lm_head")
            if weights == "w8":
                quantizable = [n for n in names if n.split(".")[-1] in PROJECTIONS]
                quantizable.append("lm_head")
                list(pool.map(self.quantized, quantizable))
        return self

    def drop_cache(self):
        self._cache.clear()
        self._quantized.clear()


def build(name_or_shape, seed=0, layers=None):
    shape = SHAPES[name_or_shape] if isinstance(name_or_shape, str) else name_or_shape
    if layers is not None:
        shape = with_layers(shape, layers)
    return SyntheticModel(shape, seed)


def prompt_ids(vocab, count, seed):
    """Seeded uniform token ids in [0, vocab), as the benchmark configs draw them."""
    rng = np.random.default_rng([seed, 0x9E3779B9])
    return [int(v) for v in rng.integers(0, vocab, size=count)]


def ragged_prompts(vocab, count=512, seed=5, shared_len=16):
    """The multi-stream serving workload's prompts: `count` independent
    requests with lengths uniform in [8, 48], every fourth one opening with
    one shared `shared_len`-token prefix (seeded ids stand in for text)."""
    rng = np.random.default_rng(seed)
    shared = rng.integers(0, vocab, shared_len).tolist()
    prompts = []
    for i in range(count):
        length = int(rng.integers(8, 49))
        ids = rng.integers(0, vocab, length).tolist()
        if i % 4 == 0:
            ids = shared + ids[: max(1, length - shared_len)]
        prompts.append([int(t) for t in ids])
    return prompts
