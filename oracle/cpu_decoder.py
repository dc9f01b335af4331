"""CPU oracle for the decoder-engine hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (``runtime.*`` and ``libhawkb200.so``) never calls
it; there is no CPU fallback.

This is a NumPy restatement of the reference's BF16 CPU runtime,
``CPUDecoderStage`` (npu_llm/runtime/cpu_backend.py:11-181), driven the way
``NPUDecoder.decode_token`` drives it with ``npu_layers=0``
(npu_llm/runtime/generate.py:830-846).  Its rounding points are the numeric
contract the CUDA kernels follow: BF16 (round-to-nearest-even) at the
embedding, every projection output, the biased qkv, the rotated q/k, the
attention output, each residual sum, the SwiGLU output and each norm output;
FP32 everywhere else; FP32 logits.

Parity of this restatement is pinned by ``tests/golden/make_golden.py``, which
imports the reference ``CPUDecoderStage`` itself and records its outputs on the
same seeded models (``tests/test_oracle_golden.py`` compares them).

W8 mode has no CPU runtime in the reference.  Its oracle replaces each BF16
projection with the W8 arithmetic of the reference AIE kernels
(npu_llm/kernels/decoder_layer_bf16.cc:64-80 and
npu_llm/kernels/project_w8bf16.cc:14-38): ``bf16((sum_k f32(q) * f32(x)) *
scale_f32)``; W8 logits are the same sum times the scale, kept in FP32.
"""

import numpy as np
from ml_dtypes import bfloat16


def to_bf16(values):
    """Round FP32 values to BF16 (RNE) -- cpu_backend.py:7-8."""
    return np.asarray(values, dtype=np.float32).astype(bfloat16)


def f32(values):
    return np.asarray(values, dtype=np.float32)


def rope_inverse_frequency(theta, head_dim):
    """``1 / theta ** (arange(d/2) / (d/2))`` in float32 (cpu_backend.py:26-32)."""
    half = head_dim // 2
    exponent = np.arange(half, dtype=np.float32) / np.float32(half)
    return (1.0 / (np.float32(theta) ** exponent)).astype(np.float32)


def rope_tables(theta, head_dim, context):
    """cos/sin of ``f32(position) * inv_freq`` for every position
    (cpu_backend.py:78-83), float32 [context, head_dim/2]."""
    inv = rope_inverse_frequency(theta, head_dim)
    cos = np.empty((context, head_dim // 2), np.float32)
    sin = np.empty((context, head_dim // 2), np.float32)
    for position in range(context):
        angle = np.float32(position) * inv
        cos[position] = np.cos(angle)
        sin[position] = np.sin(angle)
    return cos, sin


class OracleDecoder:
    """Single-stream decoder over a model with the package surface."""

    def __init__(self, model, context_length=64, weights="bf16"):
        if weights not in ("bf16", "w8"):
            raise ValueError("weights must be 'bf16' or 'w8'")
        meta = model.metadata
        self.model = model
        self.weights = weights
        self.hidden = int(meta["hidden_size"])
        self.intermediate = int(meta["intermediate_size"])
        self.q_heads = int(meta["attention_heads"])
        self.kv_heads = int(meta["kv_heads"])
        self.head_dim = int(meta["head_dim"])
        self.layers = int(meta["layers"])
        self.vocab = int(meta["vocab_size"])
        self.group = self.q_heads // self.kv_heads
        self.context = int(context_length)
        self.eps = float(meta.get("rms_norm_eps", 1e-5))
        self.cos, self.sin = rope_tables(
            float(meta.get("rope_theta", 10000.0)), self.head_dim, self.context
        )
        shape = (self.kv_heads, self.context, self.head_dim)
        self.keys = [np.zeros(shape, bfloat16) for _ in range(self.layers)]
        self.values = [np.zeros(shape, bfloat16) for _ in range(self.layers)]
        self._f32 = {}
        self._w8 = {}

    # -- parameters ----------------------------------------------------------
    def _param(self, name):
        if name not in self._f32:
            self._f32[name] = f32(self.model.raw(name))
        return self._f32[name]

    def _matrix(self, name):
        key = ("w", name)
        if key not in self._f32:
            self._f32[key] = f32(self.model.bf16_projection(name))
        return self._f32[key]

    def _quantized(self, name):
        if name not in self._w8:
            tensor = self.model.quantized(name)
            self._w8[name] = (f32(tensor.weight), f32(tensor.scale))
        return self._w8[name]

    def reset(self):
        for cache in self.keys + self.values:
            cache.fill(0)

    # -- operators -----------------------------------------------------------
    def project(self, name, x):
        """cpu_backend.py:64-69 (BF16) / decoder_layer_bf16.cc:64-80 (W8)."""
        x32 = f32(to_bf16(x))
        if self.weights == "w8":
            q, scale = self._quantized(name)
            return to_bf16((q @ x32) * scale)
        return to_bf16(self._matrix(name) @ x32)

    def rmsnorm(self, x, gamma_name):
        """cpu_backend.py:71-76: inv = 1/sqrt(mean(x*x) + eps), all float32."""
        v = f32(to_bf16(x))
        mean_square = np.mean(v * v, dtype=np.float32)
        inverse = np.float32(1.0) / np.sqrt(mean_square + np.float32(self.eps))
        return to_bf16(v * inverse * self._param(gamma_name))

    def rotate(self, heads, position):
        """Rotate-half RoPE (cpu_backend.py:78-93)."""
        h = f32(heads)
        half = self.head_dim // 2
        c, s = self.cos[position], self.sin[position]
        lo, hi = h[..., :half], h[..., half:]
        return to_bf16(np.concatenate([lo * c - hi * s, hi * c + lo * s], axis=-1))

    def attention(self, qkv, layer, position):
        """GQA over the cache, writing this position first (cpu_backend.py:95-129)."""
        d = self.head_dim
        nq, nkv = self.q_heads, self.kv_heads
        q = qkv[: nq * d].reshape(nq, d)
        k = qkv[nq * d: (nq + nkv) * d].reshape(nkv, d)
        v = qkv[(nq + nkv) * d:].reshape(nkv, d)
        q = self.rotate(q, position)
        self.keys[layer][:, position] = self.rotate(k, position)
        self.values[layer][:, position] = v
        keys = f32(self.keys[layer][:, : position + 1])
        values = f32(self.values[layer][:, : position + 1])
        grouped = f32(q).reshape(nkv, self.group, d)
        scores = np.einsum("kqd,ksd->kqs", grouped, keys, optimize=True)
        scores = scores * np.float32(d ** -0.5)
        scores = scores - scores.max(axis=-1, keepdims=True)
        weights = np.exp(scores)
        weights = weights / weights.sum(axis=-1, keepdims=True)
        out = np.einsum("kqs,ksd->kqd", weights, values, optimize=True)
        return to_bf16(out.reshape(-1))

    def layer(self, hidden, layer, position):
        """One decoder layer (cpu_backend.py:131-171); returns the new BF16 hidden."""
        p = f"layer{layer:02d}"
        x = self.rmsnorm(hidden, f"{p}.input_norm")
        qkv = f32(self.project(f"{p}.qkv", x))
        if f"{p}.qkv_bias" in self.model.tensors:
            qkv = qkv + self._param(f"{p}.qkv_bias")
        qkv = to_bf16(qkv)
        attended = self.attention(qkv, layer, position)
        h1 = to_bf16(f32(self.project(f"{p}.o_proj", attended)) + f32(hidden))
        x2 = self.rmsnorm(h1, f"{p}.post_attn_norm")
        gate_up = f32(self.project(f"{p}.gate_up", x2))
        gate, up = gate_up[: self.intermediate], gate_up[self.intermediate:]
        clipped = np.clip(gate, np.float32(-80.0), np.float32(80.0))
        act = to_bf16((gate / (np.float32(1.0) + np.exp(-clipped))) * up)
        return to_bf16(f32(self.project(f"{p}.down_proj", act)) + f32(h1))

    def logits(self, hidden):
        """Final norm + FP32 LM head, not rounded (cpu_backend.py:173-181)."""
        x32 = f32(self.rmsnorm(hidden, "final_norm"))
        if self.weights == "w8":
            q, scale = self._quantized("lm_head")
            return ((q @ x32) * scale).astype(np.float32)
        return (self._matrix("lm_head") @ x32).astype(np.float32)

    def embed(self, token_id):
        """``bf16(f32(E[token]))`` (generate.py:830-833)."""
        if not 0 <= token_id < self.vocab:
            raise ValueError("token id outside the vocabulary")
        return to_bf16(f32(self.model.raw("token_embedding")[token_id]))

    def step(self, token_id, position, compute_logits=True, trace=None):
        """One position through every layer; FP32 logits or None."""
        if not 0 <= position < self.context:
            raise ValueError("position outside the context")
        hidden = self.embed(token_id)
        for layer in range(self.layers):
            hidden = self.layer(hidden, layer, position)
            if trace is not None:
                trace.append(hidden.copy())
        if not compute_logits:
            return None
        return self.logits(hidden)


def argmax_first(logits):
    """First index of the maximum, as ``np.argmax`` (generate.py:709-714)."""
    return int(np.argmax(np.asarray(logits, np.float32)))


def greedy_generate(oracle, prompt, new_tokens, start=0):
    """Sequential prefill (only the last prompt position computes logits) then
    greedy decode -- the loop of generate.py:1110-1158 without sampling.
    Returns (generated ids, list of FP32 logits per emitted token)."""
    logits_seen = []
    token = None
    for index in range(start, len(prompt)):
        last = index == len(prompt) - 1
        out = oracle.step(prompt[index], index, compute_logits=last)
        if last:
            logits_seen.append(out)
            token = argmax_first(out)
    generated = [token]
    position = len(prompt)
    while len(generated) < new_tokens:
        out = oracle.step(generated[-1], position)
        logits_seen.append(out)
        generated.append(argmax_first(out))
        position += 1
    return generated, logits_seen
