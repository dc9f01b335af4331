"""Drop-in ``NPUDecoder`` running the decoder engine on a B200.

Same import path and surface as the reference orchestrator
(``from runtime.generate import NPUDecoder``; npu_llm/runtime/generate.py:41-1316),
so ``api_server.py``, ``chat.py`` and the benchmark scripts run on it
unchanged:

* ``NPUDecoder(model_dir, context_length=64, npu_layers=None)``;
* ``decode_token(token_id, position, *, diagnostics=False, select=None,
  compute_logits=True)`` -> ``(next_token, elapsed[, diagnostics])``;
* ``generate_messages`` / ``generate_text`` / ``generate`` generators,
  ``warmup``, ``reset_prefix_cache``, ``close``;
* attributes ``tokenizer``, ``context_length``, ``model.metadata``,
  ``_engine``, ``_cached_prefix``, ``_prefix_cache_enabled``, ``npu_layers``,
  ``layers``; the same generation statistics keys.

Every layer, the final norm, the LM head and the greedy argmax run on the GPU
in one kernel launch per position (libhawkb200.so); logits are copied to the
host only when a ``select`` callback or diagnostics need them.  There is no
CPU path: ``npu_layers`` other than all layers is rejected.

Host-side helpers outside the engine path (sampling, stop strings, the chat
tokenizer) come from the reference's own ``runtime.sampling``,
``runtime.stopping`` and ``runtime.tokenizer`` when this package is overlaid
on the reference; a standalone install falls back to ``runtime.host_shims``
(greedy decoding only).

Environment: ``HAWKPOINT_PREFIX_CACHE`` (default 1) and ``HAWKPOINT_PROFILE``
as in the reference; ``HAWKPOINT_W8=1`` selects int8 weights;
``HAWKPOINT_DEVICE`` picks the CUDA device (default 0).
"""

from collections import OrderedDict
import gc
import os
import resource
import time

import numpy as np

from runtime.model import open_model

try:  # the reference's host modules, when overlaid
    from runtime.sampling import GREEDY, Sampler, SamplingParams
    from runtime.stopping import StopMatcher, log_softmax, normalize_logprobs, normalize_stop
except ImportError:  # standalone install
    from runtime.host_shims import (  # noqa: F401
        GREEDY, Sampler, SamplingParams, StopMatcher, log_softmax, normalize_logprobs, normalize_stop,
    )
try:
    from runtime.tokenizer import SmolLMTokenizer, StreamDetokenizer
except ImportError:
    SmolLMTokenizer = None
    from runtime.host_shims import StreamDetokenizer

CONTEXT = 64  # the reference's fixed cache (npu_llm/runtime/generate.py:43-44)


def _load_tokenizer(model_dir, family):
    if SmolLMTokenizer is None or not isinstance(model_dir, (str, os.PathLike)):
        return None
    if not os.path.exists(os.path.join(model_dir, "tokenizer.json")):
        return None
    system = (
        "You are Qwen, created by Alibaba Cloud. You are a helpful assistant."
        if family == "qwen2"
        else "You are a helpful AI assistant named SmolLM."
    )
    return SmolLMTokenizer(model_dir, default_system=system)


def prepare_request(vocab, context, max_new_tokens, sampling, stop, logprobs):
    """(sampler, stop matcher, top logprobs) of one request, with the
    reference's argument checks (npu_llm/runtime/generate.py:1022-1035)."""
    if not 0 < max_new_tokens < context:
        raise ValueError(f"max_new_tokens must be between 1 and {context - 1}")
    if sampling is None:
        params = GREEDY
    elif isinstance(sampling, SamplingParams):
        params = sampling
    else:
        params = SamplingParams.from_dict(sampling)
    stop_matcher = StopMatcher(normalize_stop(stop))
    top_logprobs = normalize_logprobs(logprobs)
    return Sampler(params, vocab_size=vocab), stop_matcher, top_logprobs


def logprob_entry(tokenizer, logits, token_id, top_logprobs):
    """OpenAI ``logprobs`` entry of `token_id` from the raw distribution."""
    values = log_softmax(logits)

    def describe(index):
        return {
            "token": tokenizer.decode([int(index)]),
            "logprob": float(values[index]),
            "bytes": list(tokenizer.token_bytes(int(index))),
        }

    entry = describe(token_id)
    top = []
    if top_logprobs:
        count = min(top_logprobs, values.shape[0])
        best = np.argpartition(values, -count)[-count:]
        best = best[np.argsort(values[best])[::-1]]
        top = [describe(i) for i in best]
    entry["top_logprobs"] = top
    return entry


class NPUDecoder:
    """Greedy / sampled generation over the B200 decoder engine."""

    def __init__(self, model_dir, context_length=64, npu_layers=None):
        # 64 is the reference's cache; a multiple of 64 up to 4096 selects
        # the paged cache of the B200 engine (no reference counterpart)
        from runtime.b200_engine import MAX_CONTEXT

        if context_length != CONTEXT and (context_length % 64 or not CONTEXT < context_length <= MAX_CONTEXT):
            raise ValueError(f"context_length must be 64 or a multiple of 64 up to {MAX_CONTEXT}")
        self._closed = False
        self._engine = None
        self.model = open_model(model_dir)
        meta = self.model.metadata
        self.model_family = meta.get("model_family", "llama")
        self.tokenizer = _load_tokenizer(model_dir, self.model_family)
        self.context_length = context_length
        self.hidden_size = int(meta["hidden_size"])
        self.intermediate_size = int(meta["intermediate_size"])
        self.q_heads = int(meta["attention_heads"])
        self.kv_heads = int(meta["kv_heads"])
        self.head_dim = int(meta["head_dim"])
        self.rms_norm_eps = float(meta.get("rms_norm_eps", 1e-5))
        self.layers = int(meta["layers"])
        self.npu_layers = self.layers if npu_layers is None else int(npu_layers)
        if self.npu_layers != self.layers:
            raise ValueError(
                f"npu_layers must be {self.layers}: every layer runs on the GPU "
                "(there is no CPU decoder path)"
            )
        self._profile_enabled = os.environ.get("HAWKPOINT_PROFILE") == "1"
        self._phase_totals = {}
        # Token ids whose keys and values are valid at cache positions 0..n-1
        # (the prefix-cache contract of npu_llm/runtime/generate.py:76-79).
        self._cached_prefix = []
        self._prefix_cache_enabled = os.environ.get("HAWKPOINT_PREFIX_CACHE", "1") != "0"
        weights = "w8" if os.environ.get("HAWKPOINT_W8") == "1" else "bf16"
        device = int(os.environ.get("HAWKPOINT_DEVICE", "0"))
        from runtime.b200_engine import B200DecoderEngine

        # max_batch 8: prompts are prefilled up to 8 positions per launch
        self._engine = B200DecoderEngine(self.model, weights=weights, device=device, max_batch=8,
                                         context=int(context_length))
        self.weights = weights
        self._qwen_embedding_cache = OrderedDict()  # kept for attribute compatibility

    # -- helpers ---------------------------------------------------------------
    def _record_phase(self, name, started):
        if self._profile_enabled:
            self._phase_totals[name] = self._phase_totals.get(name, 0.0) + (time.perf_counter() - started)

    def _eos_id(self):
        if self.tokenizer is not None:
            return self.tokenizer.eos_id
        return None

    @staticmethod
    def _decode_result(logits, start, diagnostics, select=None):
        """Token selection and optional top-5 diagnostics
        (npu_llm/runtime/generate.py:709-730)."""
        values = np.asarray(logits, dtype=np.float32)
        token = int(np.argmax(values)) if select is None else int(select(values))
        elapsed = time.perf_counter() - start
        if not diagnostics:
            return token, elapsed
        top = np.argpartition(values, -5)[-5:]
        top = top[np.argsort(values[top])[::-1]]
        return token, elapsed, {
            "top_token_ids": [int(i) for i in top],
            "top_logits": [float(values[i]) for i in top],
            "top_logit_margin": float(values[top[0]] - values[top[1]]),
        }

    # -- engine step ---------------------------------------------------------------
    def decode_token(self, token_id, position, *, diagnostics=False, select=None, compute_logits=True):
        """One position through the whole model; ``(next_token, elapsed)``.

        ``select`` picks the token from the FP32 logits (default: argmax, taken
        on the GPU without copying the logits back).  ``compute_logits=False``
        (non-final prefill positions) advances the KV cache and returns
        ``(None, elapsed)``.
        """
        if not 0 <= position < self.context_length:
            raise ValueError(f"position outside the {self.context_length}-token context")
        # This step overwrites the cache at `position`: later positions were
        # computed from another history and are no longer reusable.
        del self._cached_prefix[position:]
        if self._engine is None:
            raise RuntimeError("decoder is closed")
        start = time.perf_counter()
        if not compute_logits:
            self._engine.step(token_id, position, logits=False)
            self._record_phase("npu_engine", start)
            return None, time.perf_counter() - start
        if select is None and not diagnostics:
            token = self._engine.step_argmax(token_id, position)
            self._record_phase("npu_engine", start)
            return token, time.perf_counter() - start
        logits = self._engine.step(token_id, position, logits=True)
        self._record_phase("npu_engine", start)
        return self._decode_result(logits, start, diagnostics, select)

    def warmup(self):
        """Run one step, then forget it (npu_llm/runtime/generate.py:895-946)."""
        eos = self._eos_id()
        self.decode_token(eos if eos is not None else 0, 0)
        self._engine.reset()
        self._cached_prefix.clear()

    def reset_prefix_cache(self):
        """Forget the reusable prompt prefix so the next prompt is fully prefilled."""
        self._cached_prefix.clear()

    def _reusable_prefix(self, prompt_ids):
        """Leading prompt positions still valid in the cache; the last prompt
        position is always recomputed for its logits."""
        if not self._prefix_cache_enabled:
            return 0
        shared = 0
        for cached, token in zip(self._cached_prefix, prompt_ids):
            if cached != token:
                break
            shared += 1
        return min(shared, len(prompt_ids) - 1)

    def _prefill_positions(self, prompt_ids, start, end):
        """Run positions [start, end) through the engine's batched prefill;
        returns one timing per position (the batch time shared evenly).  On
        failure the cached prefix keeps only positions before `start`."""
        del self._cached_prefix[start:]
        began = time.perf_counter()
        self._engine.prefill([int(t) for t in prompt_ids[start:end]], start=start)
        elapsed = time.perf_counter() - began
        self._cached_prefix.extend(int(t) for t in prompt_ids[start:end])
        self._record_phase("prefill", began)
        return [elapsed / (end - start)] * (end - start)

    def _sample_step(self, token_id, position, sampler, history, top_logprobs=None):
        """One position with the next token selected on the GPU: argmax for
        greedy parameters, else the reference ``Sampler.select``
        (npu_llm/runtime/sampling.py:416-445) run on logits that never leave
        the device, with the sampler's own generator supplying the one
        ``random()`` its draw consumes.  When the device reports a top-p
        nucleus too large to sort on chip, the generator is rewound and the
        host sampler selects from a copy of the same logits, so the random
        stream is identical either way.  With ``top_logprobs`` the OpenAI
        logprobs entry comes from the device too (float64 log_softmax, as
        npu_llm/runtime/stopping.py:101-109).  Returns (token, seconds,
        entry or None)."""
        from runtime.device_sampler import draws_uniform

        if not 0 <= position < self.context_length:
            raise ValueError(f"position outside the {self.context_length}-token context")
        del self._cached_prefix[position:]
        if self._engine is None:
            raise RuntimeError("decoder is closed")
        start = time.perf_counter()
        engine = self._engine
        argmax = engine.step_device_logits(token_id, position)
        host_logits = None
        if sampler.greedy:
            token = argmax
        else:
            rng = sampler._rng
            state = rng.bit_generator.state
            u = rng.random() if draws_uniform(sampler.params, engine.vocab) else None
            token = engine.sample(sampler.params, history, u)
            if token is None:
                rng.bit_generator.state = state
                host_logits = engine.device_logits()
                token = int(sampler.select(host_logits, history))
        entry = None
        if top_logprobs is not None:
            if host_logits is not None:
                entry = self._logprob_entry(host_logits, token, top_logprobs)
            else:
                count = min(top_logprobs, engine.vocab)
                lp, ids, lps = engine.logprobs(token, count)
                entry = self._logprob_entry_from(token, lp, ids if top_logprobs else [], lps)
        self._record_phase("npu_engine", start)
        if len(self._cached_prefix) == position:
            self._cached_prefix.append(int(token_id))
        return token, time.perf_counter() - start, entry

    def _decode_step(self, token_id, position, **kwargs):
        del self._cached_prefix[position:]
        result = self.decode_token(token_id, position, **kwargs)
        if len(self._cached_prefix) == position:
            self._cached_prefix.append(int(token_id))
        return result

    def _logprob_entry_from(self, token_id, logprob, top_ids, top_values):
        """The same entry from log-probabilities computed on the device."""

        def describe(index, value):
            return {
                "token": self.tokenizer.decode([int(index)]),
                "logprob": float(value),
                "bytes": list(self.tokenizer.token_bytes(int(index))),
            }

        entry = describe(token_id, logprob)
        entry["top_logprobs"] = [describe(i, v) for i, v in zip(top_ids, top_values)]
        return entry

    def _logprob_entry(self, logits, token_id, top_logprobs):
        return logprob_entry(self.tokenizer, logits, token_id, top_logprobs)

    # -- generation ------------------------------------------------------------------
    def _prepare(self, max_new_tokens, sampling, stop, logprobs):
        prepared = prepare_request(self.model.metadata["vocab_size"], self.context_length, max_new_tokens,
                                   sampling, stop, logprobs)
        if getattr(self, "_profile_enabled", False):
            self._phase_totals = {}
        if self.tokenizer is None:
            raise RuntimeError("the model package has no tokenizer; use decode_token with token ids")
        return prepared

    def generate_messages(self, messages, max_new_tokens=16, sampling=None, *, stop=None, logprobs=None):
        """Chat completion over an OpenAI-style message list, windowed to the
        context at turn boundaries; yields ``(text, None[, entries])``
        chunks then ``("", stats[, []])``."""
        sampler, stop_matcher, top_logprobs = self._prepare(max_new_tokens, sampling, stop, logprobs)
        prompt_ids, truncation = self.tokenizer.encode_chat_window(
            messages, self.context_length - max_new_tokens
        )
        yield from self._generate_tokens_core(
            prompt_ids, truncation, max_new_tokens, sampler, stop_matcher, top_logprobs
        )

    def generate_text(self, prompt, max_new_tokens=16, sampling=None, *, stop=None, logprobs=None):
        """Completion of a raw prompt without chat scaffolding."""
        sampler, stop_matcher, top_logprobs = self._prepare(max_new_tokens, sampling, stop, logprobs)
        prompt_ids, truncated = self.tokenizer.encode_prompt_window(
            prompt, self.context_length - max_new_tokens
        )
        yield from self._generate_tokens_core(
            prompt_ids, {"truncated_prompt": truncated}, max_new_tokens, sampler, stop_matcher, top_logprobs
        )

    def generate(self, prompt, max_new_tokens=32, sampling=None, *, stop=None, logprobs=None):
        """Single-prompt chat generation."""
        yield from self.generate_messages(
            [{"role": "user", "content": prompt}],
            max_new_tokens=max_new_tokens, sampling=sampling, stop=stop, logprobs=logprobs,
        )

    def _generate_tokens_core(self, prompt_ids, truncation, max_new_tokens, sampler, stop_matcher, top_logprobs):
        """Serve one request from prepared prompt ids: ingest the uncached
        prompt positions, then emit tokens until the budget, EOS or a stop
        string.  Yields ``(text, None[, entries])`` chunks, then the
        statistics (the chunk and statistics shapes of
        npu_llm/runtime/generate.py:1050-1200)."""
        picker = _TokenPicker(self, sampler, prompt_ids, top_logprobs)
        writer = _ChunkWriter(self.tokenizer, stop_matcher, top_logprobs is not None)
        reused = self._reusable_prefix(prompt_ids)
        prompt_seconds = picker.ingest(prompt_ids, reused)
        eos = self.tokenizer.eos_id
        position = len(prompt_ids)
        token = picker.token
        finish_reason = "length"
        while token != eos:
            chunk = writer.add(token, picker.take_entry())
            if writer.stopped:
                break
            if chunk is not None:
                yield chunk
            if len(writer.tokens) == max_new_tokens:
                break  # the budget is spent: no step for a successor nobody reads
            token = picker.advance(token, position)
            position += 1
        if token == eos or writer.stopped:
            finish_reason = "stop"
        last, reached_stop = writer.finish()
        if reached_stop:
            finish_reason = "stop"
        if last is not None:
            yield last
        stats = self._request_stats(prompt_ids, reused, truncation, writer, finish_reason, sampler,
                                    prompt_seconds, picker.decode_seconds)
        yield ("", stats) if top_logprobs is None else ("", stats, [])

    def _request_stats(self, prompt_ids, reused, truncation, writer, finish_reason, sampler, prompt_seconds,
                       decode_seconds):
        """Statistics of one request under the reference's key names; the
        time to first token is the sum of the prompt positions' step times."""
        ingested = len(prompt_ids) - reused
        steps = len(decode_seconds)
        decoding = sum(decode_seconds)
        ttft = sum(prompt_seconds)
        stats = {
            "prompt_tokens": len(prompt_ids),
            "cached_prompt_tokens": reused,
            "prompt_truncation": truncation,
            "generated_tokens": len(writer.tokens),
            "generated_token_ids": list(writer.tokens),
            "npu_layers": self.npu_layers,
            "cpu_layers": self.layers - self.npu_layers,
            "finish_reason": finish_reason,
            "stop_sequence": writer.stop.matched,
            "ttft_seconds": ttft,
            "prefill_tokens_per_second": ingested / max(1e-9, ttft),
            "decode_steps": steps,
            "decode_seconds": decoding,
            "decode_tokens_per_second": steps / max(1e-9, decoding),
            "peak_ram_mib": resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 1024,
            "sampling": sampler.stats(),
        }
        if getattr(self, "_profile_enabled", False):
            stats["phase_ms"] = {name: round(s * 1000.0, 3) for name, s in self._phase_totals.items()}
        return stats

    def generate_ids(self, prompt_ids, max_new_tokens):
        """Greedy generation from token ids with the whole loop on the device
        (prefix reuse as in ``generate_messages``); returns (ids, stats)."""
        if not 0 < max_new_tokens < self.context_length:
            raise ValueError(f"max_new_tokens must be between 1 and {self.context_length - 1}")
        prompt_ids = [int(t) for t in prompt_ids]
        if not prompt_ids or len(prompt_ids) + max_new_tokens > self.context_length:
            raise ValueError(f"prompt + generated tokens must fit the {self.context_length}-token context")
        reused = self._reusable_prefix(prompt_ids)
        start = time.perf_counter()
        ids = self._engine.generate(prompt_ids, max_new_tokens, start=reused)
        elapsed = time.perf_counter() - start
        self._cached_prefix[reused:] = prompt_ids[reused:] + ids[:-1]
        return ids, {"cached_prompt_tokens": reused, "seconds": elapsed}

    def close(self):
        """Release the GPU engine (idempotent)."""
        if getattr(self, "_closed", False):
            return
        self._closed = True
        engine = getattr(self, "_engine", None)
        if engine is not None:
            engine.close()
        self._engine = None
        self._cached_prefix = []
        gc.collect()


class _TokenPicker:
    """Chooses the token that follows each computed position of one request.

    Three routes, fixed per request: the engine's on-device argmax (greedy
    without logprobs: no logits leave the GPU); selection on the device
    through ``NPUDecoder._sample_step`` (sampled requests whose sampler
    exposes its generator, and greedy requests with logprobs); or the
    sampler's host ``select`` on logits copied back (any other sampler).
    The sampler is consulted once per emitted token, never for prompt
    positions whose successor is known, so its random stream advances as in
    the reference loop.  ``history`` (prompt + generated ids) feeds the
    repetition penalties."""

    def __init__(self, decoder, sampler, prompt_ids, top_logprobs):
        self.decoder = decoder
        self.sampler = sampler
        self.history = list(prompt_ids)
        self.top_logprobs = top_logprobs
        self.entry = None
        self.token = None
        self.decode_seconds = []
        host_select = not (sampler.greedy and top_logprobs is None)
        engine = getattr(decoder, "_engine", None)
        on_device = (
            host_select and engine is not None
            and os.environ.get("HAWKPOINT_DEVICE_SAMPLING", "1") != "0"
            and (sampler.greedy or (getattr(sampler, "_rng", None) is not None and hasattr(sampler, "params")))
        )
        self.route = "device" if on_device else ("host" if host_select else "argmax")

    def _host_choice(self, logits):
        if self.sampler.greedy:
            token = int(np.argmax(logits))
        else:
            token = self.sampler.select(logits, self.history)
        if self.top_logprobs is not None:
            self.entry = self.decoder._logprob_entry(logits, token, self.top_logprobs)
        return token

    def _pick(self, token_id, position):
        """Compute `position` and choose its successor: (token, seconds)."""
        if self.route == "device":
            token, seconds, self.entry = self.decoder._sample_step(
                token_id, position, self.sampler, self.history, self.top_logprobs)
            return token, seconds
        select = self._host_choice if self.route == "host" else None
        return self.decoder._decode_step(token_id, position, select=select)

    def ingest(self, prompt_ids, reused):
        """Compute prompt positions reused..end; only the last one selects a
        token.  With an engine, the positions before it go through batched
        prefill launches.  Returns the per-position seconds."""
        last = len(prompt_ids) - 1
        seconds = []
        begin = reused
        if last > begin and getattr(self.decoder, "_engine", None) is not None:
            seconds += self.decoder._prefill_positions(prompt_ids, begin, last)
            begin = last
        for position in range(begin, last):
            _, elapsed = self.decoder._decode_step(prompt_ids[position], position, compute_logits=False)
            seconds.append(elapsed)
        self.token, elapsed = self._pick(prompt_ids[last], last)
        seconds.append(elapsed)
        return seconds

    def advance(self, token_id, position):
        """Feed the emitted `token_id` at `position`; returns the next token."""
        self.history.append(token_id)
        self.token, elapsed = self._pick(token_id, position)
        self.decode_seconds.append(elapsed)
        return self.token

    def take_entry(self):
        entry, self.entry = self.entry, None
        return entry


class _ChunkWriter:
    """Turns emitted token ids into the request's text chunks.

    Text passes the stream detokenizer and the stop matcher (which holds
    back anything that may begin a stop string).  With logprobs, each
    token's entry is queued under the byte offset where its text starts and
    leaves with the first chunk whose emitted text reaches past that
    offset; on a normal end every queued entry leaves with the last chunk,
    after a stop string only those whose text was emitted."""

    def __init__(self, tokenizer, stop, logprobs):
        self.tokenizer = tokenizer
        self.stop = stop
        self.logprobs = logprobs
        self.detokenizer = StreamDetokenizer(tokenizer)
        self.tokens = []
        self.queue = []      # (byte offset of the token's text, entry), in order
        self.produced = 0    # bytes of text the queued tokens produced
        self.emitted = 0     # bytes of text handed out in chunks
        self.pending_text = ""

    @property
    def stopped(self):
        return self.stop.matched is not None

    def _pack(self, text, flush_all):
        if not self.logprobs:
            return text, None
        self.emitted += len(text.encode("utf-8"))
        count = len(self.queue) if flush_all else sum(1 for offset, _ in self.queue if offset < self.emitted)
        entries = [entry for _, entry in self.queue[:count]]
        del self.queue[:count]
        return text, None, entries

    def add(self, token, entry):
        """Record one emitted token; returns a chunk to yield, or None."""
        self.tokens.append(token)
        if entry is not None:
            self.queue.append((self.produced, entry))
            self.produced += len(self.tokenizer.token_bytes(token))
        text = self.stop.feed(self.detokenizer.push(token))
        if self.stopped:
            self.pending_text = text  # what precedes the stop string goes out last
            return None
        return self._pack(text, False) if text else None

    def finish(self):
        """The final chunk (or None) and whether a stop string ended it."""
        text = self.pending_text
        hit_now = False
        if not self.stopped:
            text = self.stop.feed(self.detokenizer.flush())
            hit_now = self.stopped
            text += self.stop.flush()
        chunk = self._pack(text, not self.stopped)
        has_entries = self.logprobs and len(chunk) == 3 and chunk[2]
        return (chunk if text or has_entries else None), hit_now
