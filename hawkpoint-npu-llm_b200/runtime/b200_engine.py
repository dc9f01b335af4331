"""Host object of the B200 decoder engine: the counterpart of the reference's
``QwenDecoderEngine`` / ``DecoderEngine`` (npu_llm/runtime/qwen_engine.py:37-102,
npu_llm/runtime/engine.py:29-91).

Differences from the reference object, all on the device side of the
boundary: the embedding gather, the RoPE tables and the K/V append happen on
the GPU, so ``step`` takes the token id instead of an embedding row; the LM
head and the argmax run on the GPU for both model families; the KV cache has
``max_slots`` independent slots (streams).

``context`` (default: the model metadata's ``context_length``, 64 -- the
reference's -- when it has none) may also be a multiple of 64 up to 4096: the cache is then paged (64-position pages, a page table per
slot; ``copy_prefix`` shares whole pages and copies a page only when a slot
writes into a shared one) and the attention splits long histories over
several SMs.  The reference has no counterpart: its cache is fixed at 64.
"""

import ctypes

import numpy as np

from runtime import hb_lib, layout
from runtime.synthetic import shape_from_metadata


def rope_tables(theta, head_dim, context):
    """cos/sin of ``float32(position) * inv_freq`` with
    ``inv_freq = 1 / theta ** (arange(d/2) / (d/2))``, all float32 and
    evaluated by NumPy exactly as the reference host does
    (npu_llm/runtime/qwen_engine.py:44-51, 68-71) -- the device reads the table."""
    half = head_dim // 2
    inv = 1.0 / (np.float32(theta) ** (np.arange(half, dtype=np.float32) / np.float32(half)))
    inv = inv.astype(np.float32)
    cos = np.empty((context, half), np.float32)
    sin = np.empty((context, half), np.float32)
    for position in range(context):
        angle = np.float32(position) * inv
        cos[position] = np.cos(angle)
        sin[position] = np.sin(angle)
    return cos, sin


MAX_CONTEXT = 4096  # longest paged context (64-position pages)


class B200DecoderEngine:
    """All decoder layers + final norm + LM head + argmax of one position per
    call, on one GPU."""

    def __init__(self, model, weights="bf16", device=0, max_slots=1, max_batch=1, blob=None, context=None):
        self._lib = hb_lib.load()
        self._handle = None
        meta = model.metadata
        self.shape = shape_from_metadata(meta)
        layout.check_dims(self.shape, weights)
        # the model metadata's context_length unless the caller names one
        context = int(self.shape.context if context is None else context)
        if context != 64 and (context % 64 or not 64 < context <= MAX_CONTEXT):
            raise ValueError(f"context {context}: must be 64 or a multiple of 64 up to {MAX_CONTEXT}")
        self.weights = weights
        self.layers = self.shape.layers
        self.vocab = self.shape.vocab
        self.context = context
        self.max_slots = int(max_slots)
        self.max_batch = int(max_batch)
        if blob is None:
            blob, lay = layout.pack(model, weights)
        else:
            blob, lay = blob
        self._layout = lay
        self._layer_table = lay.layer_table()
        cos, sin = rope_tables(self.shape.rope_theta, self.shape.head_dim, self.context)
        self._cos = np.ascontiguousarray(cos)
        self._sin = np.ascontiguousarray(sin)
        desc = hb_lib.HbModelDesc()
        desc.abi_version = hb_lib.ABI_VERSION
        desc.family = 1 if self.shape.family == "qwen2" else 0
        desc.hidden = self.shape.hidden
        desc.intermediate = self.shape.intermediate
        desc.q_heads = self.shape.q_heads
        desc.kv_heads = self.shape.kv_heads
        desc.head_dim = self.shape.head_dim
        desc.layers = self.shape.layers
        desc.vocab = self.shape.vocab
        desc.context = self.context
        desc.has_qkv_bias = 1 if any(k.endswith("qkv_bias") for k in model.tensors) else 0
        desc.weight_format = layout.FORMATS[weights]
        desc.max_slots = self.max_slots
        desc.max_batch = self.max_batch
        desc.rms_eps = float(np.float32(self.shape.rms_eps))
        desc.blob_bytes = lay.total
        desc.gamma_final = lay.gamma_final
        desc.w_lm = lay.w_lm
        desc.s_lm = lay.s_lm
        desc.embedding = lay.embedding
        desc.layer_offsets = self._layer_table
        desc.rope_cos = self._cos.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        desc.rope_sin = self._sin.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        handle = ctypes.c_void_p()
        hb_lib.check(self._lib.hb_create(ctypes.byref(desc), int(device), ctypes.byref(handle)))
        self._handle = handle
        try:
            blob = np.ascontiguousarray(blob)
            hb_lib.check(
                self._lib.hb_load_weights(handle, blob.ctypes.data, blob.nbytes, layout.LAYOUT_VERSION),
                handle,
            )
        except Exception:
            self.close()
            raise
        self._logits = np.empty(self.vocab, np.float32)
        self._argmax = ctypes.c_int32(-1)

    # -- helpers ---------------------------------------------------------------
    def _check(self, rc):
        hb_lib.check(rc, self._handle)

    def _live(self):
        if self._handle is None:
            raise RuntimeError("engine is closed")
        return self._handle

    # -- reference engine surface -------------------------------------------------
    def step(self, token_id, position, logits=True, slot=0):
        """One position through every layer.  Returns the FP32 logits (a fresh
        array) or, with ``logits=False``, None after the layers only."""
        h = self._live()
        if logits:
            out = np.empty(self.vocab, np.float32)
            self._check(self._lib.hb_step(
                h, slot, int(token_id), int(position), hb_lib.HB_STEP_LOGITS,
                out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), ctypes.byref(self._argmax)))
            return out
        self._check(self._lib.hb_step(h, slot, int(token_id), int(position), 0, None, None))
        return None

    def step_device_logits(self, token_id, position, slot=0):
        """One position with the LM head, the FP32 logits kept on the device
        for ``sample``; returns the argmax token."""
        h = self._live()
        self._check(self._lib.hb_step(
            h, slot, int(token_id), int(position), hb_lib.HB_STEP_DEVICE_LOGITS, None,
            ctypes.byref(self._argmax)))
        return int(self._argmax.value)

    def sample(self, params, history, uniform, row=0):
        """Select a token on the device from the logits of the last
        ``step_device_logits`` (row 0) -- the reference ``Sampler.select``
        with ``uniform`` as its generator draw.  None when top_p keeps more
        candidates than the device sorts (select on the host then)."""
        from runtime.device_sampler import sample_engine_row

        return sample_engine_row(self._lib, self._live(), self.vocab, row, params, history, uniform)

    def logprobs(self, token, n_top, row=0):
        """(log-probability of ``token``, top ids, top log-probabilities) of
        the logits the last ``step_device_logits`` left on the device."""
        from runtime.device_sampler import engine_logprobs

        return engine_logprobs(self._lib, self._live(), row, token, n_top)

    def device_logits(self, rows=1):
        """Host copy of the FP32 logits the last step left on the device."""
        h = self._live()
        out = np.empty((rows, self.vocab), np.float32)
        self._check(self._lib.hb_read_logits(h, int(rows), out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return out[0] if rows == 1 else out

    def step_argmax(self, token_id, position, slot=0):
        """One position with the LM head; returns only the argmax token."""
        h = self._live()
        self._check(self._lib.hb_step(
            h, slot, int(token_id), int(position), hb_lib.HB_STEP_ARGMAX, None,
            ctypes.byref(self._argmax)))
        return int(self._argmax.value)

    def prefill(self, ids, start=0, slot=0, logits=False):
        """Prefill of ``ids`` at positions start..; returns (argmax of the
        last position, its logits or None).  With max_batch > 1 the positions
        before the last run up to 8 per launch."""
        h = self._live()
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.vocab, np.float32) if logits else None
        self._check(self._lib.hb_prefill(
            h, slot, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ids.size, int(start),
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if logits else None,
            ctypes.byref(self._argmax)))
        return int(self._argmax.value), out

    def generate(self, prompt_ids, new_tokens, start=0, slot=0):
        """Device-resident greedy generation; returns the ``new_tokens`` ids."""
        h = self._live()
        ids = np.ascontiguousarray(prompt_ids, np.int32)
        out = np.empty(int(new_tokens), np.int32)
        self._check(self._lib.hb_generate(
            h, slot, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ids.size, int(start),
            int(new_tokens), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
        return [int(t) for t in out]

    def step_batch(self, slots, tokens, positions, logits=False, device_logits=False):
        """One position of each of several streams; (argmax per row, FP32
        logits or None).  ``device_logits`` keeps the logits on the device
        for ``sample_batch`` without copying them."""
        h = self._live()
        n = len(slots)
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        out = np.empty((n, self.vocab), np.float32) if logits else None
        am = np.empty(n, np.int32)
        ip = ctypes.POINTER(ctypes.c_int32)
        self._check(self._lib.hb_step_batch(
            h, n, s.ctypes.data_as(ip), t.ctypes.data_as(ip), p.ctypes.data_as(ip),
            hb_lib.HB_STEP_DEVICE_LOGITS if device_logits else hb_lib.HB_STEP_ARGMAX,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if logits else None,
            am.ctypes.data_as(ip)))
        return am, out

    # -- batched tensor-core path (hb_step_rows / hb_prefill_tc) ----------------
    MAX_ROWS = 256

    def step_rows(self, slots, tokens, positions, logits=False, out_rows=None):
        """Up to 256 rows through the whole model on the tensor cores (row i:
        tokens[i] at positions[i] of KV slot slots[i]); rows may be several
        consecutive positions of one sequence.  The LM head runs over
        ``out_rows`` (indices into the rows; default every row).  Returns
        (argmax per output row, FP32 logits [outputs, vocab] or None).  BF16
        weights, 64-position cache."""
        h = self._live()
        n = len(slots)
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        if not (s.size == t.size == p.size == n):
            raise ValueError("slots, tokens and positions must have the same length")
        sel = None if out_rows is None else np.ascontiguousarray(out_rows, np.int32)
        n_out = n if sel is None else sel.size
        out = np.empty((n_out, self.vocab), np.float32) if logits else None
        am = np.empty(n_out, np.int32)
        ip = ctypes.POINTER(ctypes.c_int32)
        self._check(self._lib.hb_step_rows(
            h, n, s.ctypes.data_as(ip), t.ctypes.data_as(ip), p.ctypes.data_as(ip), n_out,
            None if sel is None else sel.ctypes.data_as(ip), am.ctypes.data_as(ip),
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if logits else None))
        return am, out

    def prefill_tc(self, ids, start=0, slot=0, logits=False):
        """Prefill of ``ids`` at positions start.. in one batched
        tensor-core pass; (argmax of the last position, its logits or None)."""
        h = self._live()
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.vocab, np.float32) if logits else None
        self._check(self._lib.hb_prefill_tc(
            h, slot, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ids.size, int(start),
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)) if logits else None,
            ctypes.byref(self._argmax)))
        return int(self._argmax.value), out

    def generate_rows(self, ids, n_new, slot=0):
        """Greedy decode through the batched tensor-core step alone: the
        prompt in one prefill pass, then one row per step.  Stops early when
        the cache is full."""
        first, _ = self.prefill_tc(ids, slot=slot)
        out = [int(first)]
        pos = len(ids)
        while len(out) < n_new and pos < self.context:
            am, _ = self.step_rows([slot], [out[-1]], [pos])
            out.append(int(am[0]))
            pos += 1
        return out

    def sample_batch(self, rows, params, histories, uniforms):
        """Device selections for several rows of the last ``step_batch(...,
        device_logits=True)`` in one launch; a token per entry, None where the
        top-p nucleus is too large (select those on the host)."""
        from runtime.device_sampler import sample_engine_rows

        return sample_engine_rows(self._lib, self._live(), self.vocab, rows, params, histories, uniforms)

    def reset(self, slot=None):
        """Forget every cached position (of one slot, or of all)."""
        h = self._live()
        slots = range(self.max_slots) if slot is None else [slot]
        for s in slots:
            self._check(self._lib.hb_reset(h, int(s)))

    def copy_prefix(self, src, dst, n_positions):
        self._check(self._lib.hb_copy_prefix(self._live(), int(src), int(dst), int(n_positions)))

    def hidden(self):
        """BF16 residual stream rows after the last step (as uint16 bits)."""
        out = np.empty((8, self.shape.hidden), np.uint16)
        self._check(self._lib.hb_debug_dump(self._live(), hb_lib.HB_DUMP_HIDDEN, out.ctypes.data, out.nbytes))
        return out

    def kv_cache(self, slot=0):
        """BF16 bits of one slot's cache as [layers, kv_heads, 2 (K, V), context, 64].

        The device stores each position's 64 values as eight 16-byte blocks
        XOR-swizzled by the position (block b at (b ^ (pos & 7)) * 16); this
        view undoes that so it compares directly with the reference's caches."""
        s = self.shape
        raw = np.zeros((s.layers, s.kv_heads, 2, self.context, 8, 8), np.uint16)
        raw.view(np.int32).reshape(-1)[0] = slot
        self._check(self._lib.hb_debug_dump(self._live(), hb_lib.HB_DUMP_KV, raw.ctypes.data, raw.nbytes))
        pos = np.arange(self.context)[:, None]
        block = np.arange(8)[None, :] ^ (pos & 7)          # physical block of logical block b
        out = np.take_along_axis(raw, block[None, None, None, :, :, None], axis=4)
        return np.ascontiguousarray(out.reshape(s.layers, s.kv_heads, 2, self.context, s.head_dim))

    def phase_trace(self):
        """globaltimer stamps [G, 4L+2, 8] of the last launch traced with
        profile(trace=True): per phase its start, inputs ready, weights
        consumed, outputs stored, (unused), producer's first issue of the
        phase, prologue (norm / attention) done, (unused)."""
        g = self._lib.hb_device_sm_count(0)
        out = np.zeros((g, 4 * self.layers + 2, 8), np.uint64)
        self._check(self._lib.hb_debug_dump(self._live(), hb_lib.HB_DUMP_TRACE, out.ctypes.data, out.nbytes))
        return out

    def profile(self, enable=True, trace=False):
        self._check(self._lib.hb_profile(self._live(), (1 if enable else 0) | (2 if trace else 0)))

    def profile_read(self, max_launches=65536, starts=False):
        """Kernel durations (ms) of the launches since the last read; with
        starts=True also each launch's start (ms) relative to the first."""
        buf = np.zeros(max_launches, np.float32)
        st = np.zeros(max_launches, np.float32)
        count = ctypes.c_int(0)
        fp = ctypes.POINTER(ctypes.c_float)
        self._check(self._lib.hb_profile_read(
            self._live(), buf.ctypes.data_as(fp), st.ctypes.data_as(fp), max_launches, ctypes.byref(count)))
        n = count.value
        return (buf[:n].copy(), st[:n].copy()) if starts else buf[:n].copy()

    def set_stream(self, stream_handle):
        self._check(self._lib.hb_set_stream(self._live(), ctypes.c_void_p(stream_handle or None)))

    def test_stall_next(self, limit_ns):
        self._check(self._lib.hb_test_stall_next(self._live(), int(limit_ns)))

    def close(self):
        """Release every device buffer (idempotent)."""
        if self._handle is not None:
            self._lib.hb_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
