"""Continuous batching behind the reference's OpenAI server.

The reference server hands every request to ``CompletionEngine.generate``,
which holds one lock for the whole generation
(npu_llm/api_server.py:535-678), so concurrent requests run one after
another.  ``BatchingCompletionEngine`` has the engine surface the server's
request handler uses (``models``, ``default_model_id``, ``ready``,
``model_list``, ``model_info``, ``has_model``, ``context_length``,
``prewarm_default``, ``close``, ``generate``), so
``make_handler(BatchingCompletionEngine(...))`` of the unchanged
api_server.py serves the same OpenAI protocol.  ``generate`` no longer
computes anything itself.  It queues the request, and one scheduler thread
per model runs every admitted request together through the engine's
batched step (``MultiStreamServer``): in rows mode, decode rows plus
chunked-prefill rows on the tensor cores, with shared prompt prefixes from
the KV prefix pool.  Each caller's generator yields its own request's text
as the tokens arrive, with the chunks, stop handling, logprobs entries and
final statistics of ``NPUDecoder.generate_messages`` / ``generate_text``.

W8 weights have no batched tensor-core step; their scheduler drives the
persistent kernel's batch of 8 streams (one position per row) instead.
"""

import os
import queue
import resource
import threading
import time

from runtime.generate import _ChunkWriter, _load_tokenizer, logprob_entry, prepare_request
from runtime.model import open_model
from runtime.serving import MultiStreamServer, Request


def default_engine_factory(model, max_slots, weights):
    """The B200 engine of one model on ``HAWKPOINT_DEVICE``."""
    from runtime.b200_engine import B200DecoderEngine

    return B200DecoderEngine(model, weights=weights, device=int(os.environ.get("HAWKPOINT_DEVICE", "0")),
                             max_slots=max_slots, max_batch=8)


class _ModelWorker:
    """One loaded model: tokenizer, engine, and the scheduler thread that
    steps every in-flight request of this model together."""

    def __init__(self, path, engine_factory, weights, max_batch, prefill_chunk, max_rows, prefix_slots,
                 tokenizer_factory=None):
        self.model = open_model(path)
        meta = self.model.metadata
        self.layers = int(meta["layers"])
        self.vocab = int(meta["vocab_size"])
        family = meta.get("model_family", "llama")
        self.tokenizer = (tokenizer_factory or _load_tokenizer)(str(path), family)
        if weights == "w8":  # no batched tensor-core step for int8 weights
            max_batch, prefill_chunk = min(max_batch, 8), 0
        self.engine = engine_factory(self.model, max_batch + prefix_slots, weights)
        self.context = int(self.engine.context)
        self._settings = dict(max_batch=max_batch, prefix_slots=prefix_slots, prefill_chunk=prefill_chunk,
                              max_rows=max_rows)
        self.server = MultiStreamServer(self.engine, **self._settings)
        self.inbox = queue.Queue()
        self._closing = False
        self._thread = threading.Thread(target=self._loop, name="hawkpoint-batch-scheduler", daemon=True)
        self._thread.start()

    def submit(self, req):
        if self._closing:
            raise RuntimeError("the engine is closed")
        self.inbox.put(req)

    def _take(self, block):
        """Move arrived requests into the server; False once closing."""
        while True:
            try:
                req = self.inbox.get(block=block)
            except queue.Empty:
                return True
            if req is None:
                return False
            block = False
            try:
                self.server.submit(req)
            except ValueError as exc:  # does not fit: tell that caller only
                req.listener(req, exc, None)

    def _loop(self):
        while True:
            if not self._take(block=not self.server.busy):
                break
            if not self.server.busy:
                continue
            try:
                self.server.step()
            except Exception as exc:  # a device error ends every request in flight
                self._fail_all(exc)
        closed = RuntimeError("the engine was closed")
        self._fail_all(closed)
        while True:  # requests that arrived after the close
            try:
                req = self.inbox.get_nowait()
            except queue.Empty:
                break
            if req is not None:
                req.listener(req, closed, None)

    def _fail_all(self, exc):
        for req in list(self.server._pending) + [st.req for st in self.server._active]:
            req.listener(req, exc, None)
        self.server = MultiStreamServer(self.engine, **self._settings)
        try:
            self.engine.reset()
        except Exception:
            pass

    def close(self):
        self._closing = True
        self.inbox.put(None)
        self._thread.join(timeout=60)
        self.engine.close()


class BatchingCompletionEngine:
    """The reference server's completion engine, with every concurrent
    request of a model batched on its GPU (see the module docstring).

    ``models``: model id -> record with the package ``path`` (and optional
    ``display_name``, ``context_length``), as the reference catalog lists
    them.  ``engine_factory(model, max_slots, weights)`` builds a model's
    engine (default: the B200 engine); ``max_batch`` streams share a step,
    ``prefill_chunk`` prompt positions per stream per step, at most
    ``max_rows`` rows a step.  ``tokenizer_factory(path, family)`` replaces
    the package's chat tokenizer (tests)."""

    def __init__(self, models, engine_factory=default_engine_factory, max_batch=32, prefill_chunk=16, max_rows=128,
                 prefix_slots=4, weights=None, tokenizer_factory=None):
        if not models:
            raise ValueError("no converted models were found")
        self.models = {model_id: dict(record) for model_id, record in models.items()}
        self.default_model_id = next(iter(self.models))
        self.engine_factory = engine_factory
        self.weights = weights or ("w8" if os.environ.get("HAWKPOINT_W8") == "1" else "bf16")
        self.options = dict(max_batch=max_batch, prefill_chunk=prefill_chunk, max_rows=max_rows,
                            prefix_slots=prefix_slots, tokenizer_factory=tokenizer_factory)
        self._workers = {}
        self._lock = threading.Lock()

    # -- catalogue (the CompletionEngine surface) -----------------------------------
    def model_list(self):
        return [self.model_info(model_id) for model_id in self.models]

    def model_info(self, model_id):
        if model_id not in self.models:
            return None
        return {"id": model_id, "object": "model", "created": 0, "owned_by": "local",
                "name": self.models[model_id].get("display_name", model_id)}

    def has_model(self, model_id):
        return model_id in self.models

    def context_length(self, model_id):
        return int(self.models[model_id].get("context_length", 64))

    @property
    def ready(self):
        return True

    def prewarm_default(self):
        self._worker(self.default_model_id)

    def close(self):
        with self._lock:
            workers, self._workers = list(self._workers.values()), {}
        for worker in workers:
            worker.close()

    def _worker(self, model_id):
        with self._lock:
            worker = self._workers.get(model_id)
            if worker is None:
                worker = _ModelWorker(self.models[model_id]["path"], self.engine_factory, self.weights,
                                      **self.options)
                self._workers[model_id] = worker
            return worker

    # -- one request ------------------------------------------------------------------
    def generate(self, model_id, messages, max_tokens, timeout=None, sampling=None, stop=None, logprobs=None):
        """Queue one chat (message list) or text (string) request and yield
        its ``(text, None[, entries])`` chunks, then ``("", stats[, []])``."""
        worker = self._worker(model_id)
        tok = worker.tokenizer
        if tok is None:
            raise RuntimeError("the model package has no tokenizer")
        sampler, stop_matcher, top_logprobs = prepare_request(worker.vocab, worker.context, max_tokens, sampling,
                                                              stop, logprobs)
        budget = worker.context - max_tokens
        if isinstance(messages, str):
            prompt_ids, truncated = tok.encode_prompt_window(messages, budget)
            truncation = {"truncated_prompt": truncated}
        else:
            prompt_ids, truncation = tok.encode_chat_window(messages, budget)
        events = queue.Queue()
        req = Request(prompt=[int(t) for t in prompt_ids], new_tokens=max_tokens,
                      sampler=None if sampler.greedy else sampler, eos=tok.eos_id,
                      want_logits=top_logprobs is not None,
                      listener=lambda r, token, logits: events.put((token, logits, time.perf_counter())))
        submitted = time.perf_counter()
        deadline = None if timeout is None else submitted + float(timeout)
        worker.submit(req)
        yield from self._stream(req, events, tok, sampler, stop_matcher, top_logprobs, max_tokens, prompt_ids,
                                truncation, submitted, deadline, worker.layers)

    def _stream(self, req, events, tok, sampler, stop_matcher, top_logprobs, max_tokens, prompt_ids, truncation,
                submitted, deadline, layers):
        writer = _ChunkWriter(tok, stop_matcher, top_logprobs is not None)
        eos_seen = False
        token_times = []
        try:
            while True:
                wait = None if deadline is None else max(0.0, deadline - time.perf_counter())
                try:
                    token, logits, at = events.get(timeout=wait)
                except queue.Empty:
                    raise TimeoutError("inference request exceeded its deadline") from None
                if isinstance(token, BaseException):
                    raise token
                if token is None:  # the stream ended (budget or context)
                    break
                token_times.append(at)
                if token == tok.eos_id:
                    eos_seen = True
                    break
                entry = logprob_entry(tok, logits, token, top_logprobs) if top_logprobs is not None else None
                chunk = writer.add(token, entry)
                if writer.stopped:
                    break
                if chunk is not None:
                    yield chunk
                if len(writer.tokens) == max_tokens:
                    break
        finally:
            req.cancelled = True  # a stream nobody reads any more ends at the next step
        finish_reason = "stop" if eos_seen or writer.stopped else "length"
        last, reached_stop = writer.finish()
        if reached_stop:
            finish_reason = "stop"
        if last is not None:
            yield last
        first = token_times[0] if token_times else time.perf_counter()
        ttft = first - submitted
        steps = max(0, len(token_times) - 1)
        decoding = token_times[-1] - first if token_times else 0.0
        stats = {
            "prompt_tokens": len(prompt_ids),
            "cached_prompt_tokens": req.reused_prefix,
            "prompt_truncation": truncation,
            "generated_tokens": len(writer.tokens),
            "generated_token_ids": list(writer.tokens),
            "npu_layers": layers,
            "cpu_layers": 0,
            "finish_reason": finish_reason,
            "stop_sequence": writer.stop.matched,
            "ttft_seconds": ttft,
            "prefill_tokens_per_second": (len(prompt_ids) - req.reused_prefix) / max(1e-9, ttft),
            "decode_steps": steps,
            "decode_seconds": decoding,
            "decode_tokens_per_second": steps / max(1e-9, decoding),
            "peak_ram_mib": resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 1024,
            "sampling": sampler.stats(),
            "queue_seconds": max(0.0, req.admitted - submitted),
        }
        yield ("", stats) if top_logprobs is None else ("", stats, [])
