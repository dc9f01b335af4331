"""Multi-stream serving on one GPU: continuous batching over the engine's
batched decode step (``hb_step_batch``), greedy or sampled per request.

The reference serves one request at a time behind a lock
(npu_llm/api_server.py:646-678); its engine has no batched mode.  Here up to
``max_batch`` independent streams share every kernel launch: each row of a
launch is one stream at its own position -- a prompt token during sequential
prefill (npu_llm/runtime/generate.py:1110-1126, logits unused), or its last
generated token during decode.  A weight-streaming decode step costs about
the same for 8 rows as for 1, so the aggregate rate scales with the batch.

A request may carry a ``sampler`` with the reference ``Sampler`` surface
(``params``, ``greedy``, its generator ``_rng``, ``select``;
npu_llm/runtime/sampling.py:398-453).  The rows of a launch that sample
select on the device in one further launch (``hb_sample_batch``), each
request's own generator supplying its draw, so a seeded request yields the
same tokens as alone; a row whose top-p nucleus is too large for the device
is selected on the host from the same logits with its generator rewound.

With ``prefill_chunk`` set the server drives the engine's batched
tensor-core step instead (``step_rows``, up to ``max_rows`` rows a step):
each decoding stream is one row and each prefilling stream up to
``prefill_chunk`` consecutive prompt positions (chunked prefill), so a
prompt takes a few steps rather than one per position, and the LM head runs
only for the rows whose next token is wanted (the last prompt position and
decode rows).  Sampled rows take their logits to the host and select with
the request's own sampler.

KV slots: ``max_batch`` slots for the running streams plus a small LRU pool
that keeps shared prompt prefixes.  A request whose first ``prefix_tokens``
ids match a kept prefix starts after it (the cached positions are copied into
its slot with ``hb_copy_prefix``), the same reuse rule as the reference's
prefix cache (``min(shared, len - 1)`` positions, generate.py:952-973).
"""

from collections import OrderedDict, deque
from dataclasses import dataclass, field
import time

import numpy as np


@dataclass
class Request:
    prompt: list
    new_tokens: int
    rid: int = 0
    sampler: object = None   # None: greedy
    tokens: list = field(default_factory=list)
    admitted: float = 0.0
    first_token: float = 0.0
    finished: float = 0.0
    reused_prefix: int = 0
    eos: int = None            # a generated eos ends the request (the token is kept)
    cancelled: bool = False    # set by the caller: the stream ends at the next step
    want_logits: bool = False  # rows mode: hand each generated token's FP32 logits to the listener
    listener: object = None    # listener(req, token, logits_or_None) per token; listener(req, None, None) at the end

    @property
    def ttft(self):
        return self.first_token - self.admitted


class _Stream:
    __slots__ = ("req", "slot", "pos", "token", "key")

    def __init__(self, req, slot, pos, token, key):
        self.req, self.slot, self.pos, self.token, self.key = req, slot, pos, token, key


class MultiStreamServer:
    """Runs a list of requests to completion on one engine.

    ``engine`` needs ``step_batch(slots, tokens, positions) -> (argmax, _)``,
    ``copy_prefix(src, dst, n)``, ``max_slots`` and ``context``; it must have
    at least ``max_batch + prefix_slots`` KV slots.  Sampled requests also
    need ``step_batch(..., device_logits=True)``, ``sample_batch`` and
    ``device_logits`` and the engine's ``vocab``."""

    def __init__(self, engine, max_batch=8, prefix_tokens=16, prefix_slots=4, clock=time.perf_counter,
                 prefill_chunk=0, max_rows=128):
        if max_batch < 1:
            raise ValueError("max_batch must be >= 1")
        if engine.max_slots < max_batch + prefix_slots:
            raise ValueError(f"engine has {engine.max_slots} KV slots, needs {max_batch + prefix_slots}")
        if prefill_chunk and not 1 <= max_batch <= max_rows:
            raise ValueError("with prefill_chunk, max_batch must be in [1, max_rows]")
        self.engine = engine
        self.max_batch = max_batch
        self.prefix_tokens = prefix_tokens
        self.clock = clock
        self.prefill_chunk = int(prefill_chunk)
        self.max_rows = int(max_rows)
        self.stream_slots = list(range(max_batch))
        self._pending = deque()                    # submitted, not admitted
        self._free = list(reversed(self.stream_slots))
        self._active = []
        self.prefix_pool = list(range(max_batch, max_batch + prefix_slots))
        self.prefixes = OrderedDict()   # prefix ids -> slot holding their positions
        self.launches = 0
        self.rows = 0

    def _key(self, prompt):
        if self.prefix_tokens > 0 and len(prompt) > self.prefix_tokens:
            return tuple(int(t) for t in prompt[: self.prefix_tokens])
        return None

    def _admit(self, req, free):
        slot = free.pop()
        key = self._key(req.prompt)
        start = 0
        if key is not None and key in self.prefixes:
            self.prefixes.move_to_end(key)
            self.engine.copy_prefix(self.prefixes[key], slot, self.prefix_tokens)
            start = self.prefix_tokens
        req.reused_prefix = start
        req.admitted = self.clock()
        return _Stream(req, slot, start, int(req.prompt[start]), key)

    def _keep_prefix(self, st):
        """Positions [0, prefix_tokens) of st are computed: keep them."""
        if st.key is None or st.key in self.prefixes:
            return
        if self.prefix_pool:
            pslot = self.prefix_pool.pop()
        else:
            _, pslot = self.prefixes.popitem(last=False)
        self.engine.copy_prefix(st.slot, pslot, self.prefix_tokens)
        self.prefixes[st.key] = pslot

    def _sample_rows(self, active, rows):
        """Tokens of the sampled rows of the last launch, on the device."""
        from runtime.device_sampler import draws_uniform

        vocab = self.engine.vocab
        params, histories, uniforms, states = [], [], [], []
        for i in rows:
            req = active[i].req
            rng = req.sampler._rng
            states.append(rng.bit_generator.state)
            params.append(req.sampler.params)
            histories.append(list(req.prompt) + list(req.tokens))
            uniforms.append(rng.random() if draws_uniform(req.sampler.params, vocab) else None)
        tokens = self.engine.sample_batch(rows, params, histories, uniforms)
        host = None
        for k, i in enumerate(rows):
            if tokens[k] is None:  # nucleus beyond the on-chip sort: same draw on the host
                if host is None:
                    host = np.asarray(self.engine.device_logits(rows=len(active))).reshape(len(active), -1)
                req = active[i].req
                req.sampler._rng.bit_generator.state = states[k]
                tokens[k] = int(req.sampler.select(host[i], histories[k]))
        return tokens

    # -- incremental use: submit requests as they arrive, step while busy ------
    def submit(self, req):
        """Queue a request (checked now; admitted in arrival order)."""
        context = self.engine.context
        if not 1 <= len(req.prompt) < context:
            raise ValueError(f"prompt of {len(req.prompt)} ids does not fit a {context}-token context")
        if req.new_tokens < 1:
            raise ValueError("new_tokens must be >= 1")
        self._pending.append(req)

    @property
    def busy(self):
        return bool(self._pending or self._active)

    def step(self):
        """Admit what fits, drop cancelled streams, run one launch."""
        while self._pending and self._free and len(self._active) < self.max_batch:
            self._active.append(self._admit(self._pending.popleft(), self._free))
        still = []
        for st in self._active:
            if st.req.cancelled:
                self._finish(st, self.clock(), self._free)
            else:
                still.append(st)
        self._active = still
        if not self._active:
            return
        if self.prefill_chunk:
            self._active = self._step_rows(self._active, self._free, self.engine.context)
        else:
            self._active = self._step_positions(self._active, self._free, self.engine.context)

    def run(self, requests):
        """Every request to completion; returns them."""
        for req in requests:
            self.submit(req)
        while self.busy:
            self.step()
        return requests

    def _finish(self, st, now, free):
        st.req.finished = now
        free.append(st.slot)
        if st.req.listener is not None:
            st.req.listener(st.req, None, None)

    def _emit(self, st, token, now, logits=None):
        """Record a generated token; True when the stream is done."""
        req = st.req
        req.tokens.append(int(token))
        if len(req.tokens) == 1:
            req.first_token = now
        st.token = int(token)
        if req.listener is not None:
            req.listener(req, int(token), logits)
        return len(req.tokens) >= req.new_tokens or (req.eos is not None and int(token) == req.eos)

    def _step_positions(self, active, free, context):
        """One launch of the persistent kernel: a row per stream, its next
        prompt position or its last token.  Returns the streams still running."""
        slots = [st.slot for st in active]
        tokens = [st.token for st in active]
        positions = [st.pos for st in active]
        sampled = [i for i, st in enumerate(active)
                   if st.pos >= len(st.req.prompt) - 1 and st.req.sampler is not None
                   and not st.req.sampler.greedy]
        if sampled:
            argmax, _ = self.engine.step_batch(slots, tokens, positions, device_logits=True)
            argmax = list(argmax)
            for i, token in zip(sampled, self._sample_rows(active, sampled)):
                argmax[i] = token
        else:
            argmax, _ = self.engine.step_batch(slots, tokens, positions)
        self.launches += 1
        self.rows += len(active)
        now = self.clock()
        still = []
        for st, nxt in zip(active, argmax):
            req = st.req
            done = False
            if st.pos < len(req.prompt) - 1:
                st.token = int(req.prompt[st.pos + 1])        # sequential prefill
            else:
                done = self._emit(st, nxt, now)
            st.pos += 1
            if st.pos == self.prefix_tokens:
                self._keep_prefix(st)
            if done or st.pos >= context:
                self._finish(st, now, free)
            else:
                still.append(st)
        return still

    def _step_rows(self, active, free, context):
        """One batched tensor-core step: a row per decoding stream, then up
        to ``prefill_chunk`` prompt positions per prefilling stream while the
        row budget lasts.  Returns the streams still running."""
        budget = self.max_rows
        plan = []  # (stream, first position, rows)
        for st in active:
            if st.pos >= len(st.req.prompt) - 1:
                plan.append((st, st.pos, 1))
                budget -= 1
        for st in active:
            last_prompt = len(st.req.prompt) - 1
            if st.pos < last_prompt and budget > 0:
                take = min(self.prefill_chunk, last_prompt + 1 - st.pos, budget)
                plan.append((st, st.pos, take))
                budget -= take
        slots, tokens, positions, out_rows, wanted = [], [], [], [], []
        for st, p0, take in plan:
            prompt = st.req.prompt
            for k in range(take):
                p = p0 + k
                slots.append(st.slot)
                positions.append(p)
                tokens.append(int(prompt[p]) if p < len(prompt) else st.token)
            if p0 + take - 1 >= len(prompt) - 1:  # this row's next token is wanted
                out_rows.append(len(slots) - 1)
                wanted.append(st)
        sampled = [j for j, st in enumerate(wanted) if st.req.sampler is not None and not st.req.sampler.greedy]
        need_logits = bool(sampled) or any(st.req.want_logits for st in wanted)
        rows = out_rows or [len(slots) - 1]
        argmax, logits = self.engine.step_rows(slots, tokens, positions, logits=need_logits, out_rows=rows)
        picks = [int(t) for t in argmax[: len(wanted)]]
        for j in sampled:
            req = wanted[j].req
            picks[j] = int(req.sampler.select(np.asarray(logits[j]), list(req.prompt) + list(req.tokens)))
        self.launches += 1
        self.rows += len(slots)
        now = self.clock()
        nxt = {id(st): (picks[j], logits[j] if need_logits and st.req.want_logits else None)
               for j, st in enumerate(wanted)}
        done = set()
        for st, p0, take in plan:
            req = st.req
            before = st.pos
            st.pos = p0 + take
            ended = False
            if id(st) in nxt:
                ended = self._emit(st, nxt[id(st)][0], now, nxt[id(st)][1])
            else:
                st.token = int(req.prompt[st.pos])
            if before < self.prefix_tokens <= st.pos:
                self._keep_prefix(st)
            if ended or st.pos >= context:
                self._finish(st, now, free)
                done.add(id(st))
        return [st for st in active if id(st) not in done]


def run_lanes(servers, requests, new_tokens=16, prefix_tokens=16):
    """Serves ``requests`` on several servers at once, each server's engine
    on its own CUDA stream and each server driven by its own host thread
    (the engine calls release the interpreter lock), so the servers'
    launch sequences overlap on one GPU: a batched step is a chain of
    dependent kernels that leaves most SMs idle between them, and a second
    or third chain fills them.  Requests are assigned to lanes as requests
    are assigned to GPUs (runtime/dispatch.py: requests sharing a prompt
    prefix go to the same lane, where its prefix pool keeps it).  Returns
    the requests; re-raises the first lane's error."""
    import threading

    from runtime import dispatch

    lanes = len(servers)
    prompts = [r.prompt for r in requests]
    groups = [[requests[i] for i in dispatch.shard(prompts, k, lanes, new_tokens, prefix_tokens)]
              for k in range(lanes)]
    errors = [None] * lanes

    def serve(k):
        try:
            servers[k].run(groups[k])
        except BaseException as exc:  # reported after every lane stopped
            errors[k] = exc

    threads = [threading.Thread(target=serve, args=(k,), name=f"hawkpoint-lane-{k}") for k in range(lanes)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for exc in errors:
        if exc is not None:
            raise exc
    return requests
