"""Multi-stream continuous batching (the 512-request ragged serving workload on one GPU): the
scheduler on CPU against a fake causal engine, and on the GPU against
single-stream generation through the same kernels."""

import numpy as np
import pytest

from runtime.serving import MultiStreamServer, Request, run_lanes


class FakeEngine:
    """Causal toy model: the next token is a hash of every token cached in
    the slot up to the position, so a wrong prefix copy, a skipped position
    or a shared slot changes the output."""

    def __init__(self, max_slots, context=64, vocab=1000):
        self.max_slots, self.context, self.vocab = max_slots, context, vocab
        self.cache = [[None] * context for _ in range(max_slots)]
        self.batches = []
        self.copies = []

    def step_batch(self, slots, tokens, positions, device_logits=False):
        assert len(set(slots)) == len(slots), "two rows share a KV slot"
        self.batches.append(len(slots))
        out = []
        self.logits = []
        for s, t, p in zip(slots, tokens, positions):
            self.cache[s][p] = t
            hist = self.cache[s][: p + 1]
            assert None not in hist, f"slot {s} position {p} reads an unwritten position"
            out.append(hash(tuple(hist)) % self.vocab)
            self.logits.append(fake_logits(hist, self.vocab))
        return np.array(out), None

    # the device sampler: the oracle; a top-p nucleus is "too large" here so
    # the server's host fallback runs too
    def sample_batch(self, rows, params, histories, uniforms):
        from oracle.sampling import select_with_uniform

        self.sampled = getattr(self, "sampled", 0) + len(rows)
        return [None if p.top_p < 1.0 else select_with_uniform(self.logits[i], h, p, u)
                for i, p, h, u in zip(rows, params, histories, uniforms)]

    def step_rows(self, slots, tokens, positions, logits=False, out_rows=None):
        """The batched step: every row's position is cached before any row
        reads (rows of one slot see each other); outputs for out_rows."""
        assert len(slots) <= 128
        assert len(set(zip(slots, positions))) == len(slots), "two rows write one slot position"
        self.row_steps = getattr(self, "row_steps", []) + [len(slots)]
        for s, t, p in zip(slots, tokens, positions):
            self.cache[s][p] = t
        rows = range(len(slots)) if out_rows is None else out_rows
        out, lg = [], []
        for i in rows:
            hist = self.cache[slots[i]][: positions[i] + 1]
            assert None not in hist, f"row {i} reads an unwritten position"
            out.append(hash(tuple(hist)) % self.vocab)
            lg.append(fake_logits(hist, self.vocab))
        return np.array(out), (np.stack(lg) if logits else None)

    def device_logits(self, rows=1):
        return np.stack(self.logits[:rows])

    def copy_prefix(self, src, dst, n):
        self.copies.append((src, dst, n))
        self.cache[dst][:n] = self.cache[src][:n]


def fake_logits(hist, vocab):
    return np.random.default_rng(hash(tuple(hist)) % (2 ** 32)).standard_normal(vocab).astype(np.float32)


class OracleSampler:
    """The reference ``Sampler`` surface over the oracle (seeded generator)."""

    def __init__(self, params, vocab, seed):
        self.params, self.vocab = params, vocab
        self._rng = np.random.default_rng(seed)

    @property
    def greedy(self):
        return self.params.greedy_for(self.vocab)

    def select(self, logits, history):
        from oracle import sampling as osamp

        u = self._rng.random() if osamp.draws_uniform(self.params, self.vocab) else None
        return osamp.select_with_uniform(logits, history, self.params, u)


def reference_tokens(prompt, new_tokens, vocab=1000, context=64):
    hist = list(prompt)
    out = []
    while len(out) < new_tokens and len(hist) <= context:
        nxt = hash(tuple(hist)) % vocab
        out.append(nxt)
        if len(hist) == context:
            break
        hist.append(nxt)
    return out


def config5_requests(n=64, seed=0, vocab=1000, new_tokens=16):
    rng = np.random.default_rng(seed)
    shared = rng.integers(0, vocab, 16).tolist()
    reqs = []
    for i in range(n):
        length = int(rng.integers(8, 49))
        ids = rng.integers(0, vocab, length).tolist()
        if i % 4 == 0:
            ids = shared + ids[: max(1, length - 16)]
        reqs.append(Request(prompt=ids, new_tokens=new_tokens, rid=i))
    return reqs


def test_continuous_batching_matches_single_streams():
    eng = FakeEngine(max_slots=12)
    reqs = config5_requests()
    MultiStreamServer(eng, max_batch=8, prefix_slots=4).run(reqs)
    for r in reqs:
        assert r.tokens == reference_tokens(r.prompt, r.new_tokens), r.rid
    assert max(eng.batches) == 8
    # the shared 16-token prefix is computed once and reused afterwards
    reused = [r for r in reqs if r.reused_prefix]
    assert len(reused) >= 10 and all(r.reused_prefix == 16 for r in reused)
    assert eng.copies[0][2] == 16


def test_continuous_batching_with_a_longer_context():
    """Prompts of 60 to 300 positions plus 40 new tokens in a 512-position
    context (the paged engine's range), a third of them opening with the
    same 128 ids (two whole 64-position pages, which a paged engine shares
    instead of copying): the same tokens as single streams, the prefix
    computed once and reused."""
    rng = np.random.default_rng(5)
    shared = rng.integers(0, 1000, 128).tolist()
    reqs = []
    for i in range(24):
        ids = rng.integers(0, 1000, int(rng.integers(60, 301))).tolist()
        reqs.append(Request(prompt=shared + ids if i % 3 == 0 else ids, new_tokens=40, rid=i))
    eng = FakeEngine(max_slots=12, context=512)
    MultiStreamServer(eng, max_batch=8, prefix_tokens=128, prefix_slots=4).run(reqs)
    for r in reqs:
        assert r.tokens == reference_tokens(r.prompt, r.new_tokens, context=512), r.rid
    reused = [r for r in reqs if r.reused_prefix]
    assert len(reused) >= 3 and all(r.reused_prefix == 128 for r in reused)


def _sampled_requests(vocab, seed=0):
    from oracle import sampling as osamp

    reqs = config5_requests(n=24, seed=seed, vocab=vocab, new_tokens=8)
    settings = [None, osamp.Params(temperature=0.9), osamp.Params(temperature=0.8, top_k=40, top_p=0.9),
                osamp.Params(temperature=1.0, repetition_penalty=1.2, logit_bias={3: 2.0})]
    for r in reqs:
        params = settings[r.rid % len(settings)]
        r.sampler = None if params is None else OracleSampler(params, vocab, 100 + r.rid)
    return reqs


def test_sampled_requests_in_continuous_batching():
    """Sampled rows select per request, each with its own generator; the
    tokens equal each request decoded alone with the host sampler, also
    where the device reports a nucleus too large and the host selects."""
    eng = FakeEngine(max_slots=12)
    reqs = _sampled_requests(eng.vocab)
    MultiStreamServer(eng, max_batch=8, prefix_slots=4).run(reqs)
    assert eng.sampled > 0
    alone = _sampled_requests(eng.vocab)
    for r, a in zip(reqs, alone):
        hist, want = list(a.prompt), []
        while len(want) < a.new_tokens:
            nxt = hash(tuple(hist)) % eng.vocab
            if a.sampler is not None and not a.sampler.greedy:
                nxt = a.sampler.select(fake_logits(hist, eng.vocab), list(a.prompt) + want)
            want.append(int(nxt))
            hist.append(int(nxt))
        assert r.tokens == want, r.rid


def test_chunked_prefill_rows_match_single_streams():
    """Rows mode (the batched tensor-core step): prompts advance up to 8
    positions a step, decode streams one; the same tokens as single streams,
    far fewer steps than one position per launch, prefixes reused, the row
    budget respected."""
    eng = FakeEngine(max_slots=36)
    reqs = config5_requests()
    server = MultiStreamServer(eng, max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=48)
    server.run(reqs)
    for r in reqs:
        assert r.tokens == reference_tokens(r.prompt, r.new_tokens), r.rid
    assert max(eng.row_steps) <= 48 and max(eng.row_steps) > 32
    per_position = MultiStreamServer(FakeEngine(max_slots=36), max_batch=32, prefix_slots=4)
    per_position.run(config5_requests())
    assert server.launches < per_position.launches
    # the 8 sharing requests among the first 32 admitted compute the prefix
    # themselves; the 8 admitted later reuse it
    reused = [r for r in reqs if r.reused_prefix]
    assert len(reused) >= 6 and all(r.reused_prefix == 16 for r in reused)


def test_chunked_prefill_rows_with_sampling_and_context_limit():
    eng = FakeEngine(max_slots=12)
    reqs = _sampled_requests(eng.vocab)
    MultiStreamServer(eng, max_batch=8, prefix_slots=4, prefill_chunk=5, max_rows=16).run(reqs)
    alone = _sampled_requests(eng.vocab)
    for r, a in zip(reqs, alone):
        hist, want = list(a.prompt), []
        while len(want) < a.new_tokens:
            nxt = hash(tuple(hist)) % eng.vocab
            if a.sampler is not None and not a.sampler.greedy:
                nxt = a.sampler.select(fake_logits(hist, eng.vocab), list(a.prompt) + want)
            want.append(int(nxt))
            hist.append(int(nxt))
        assert r.tokens == want, r.rid
    eng = FakeEngine(max_slots=2, context=20)
    req = Request(prompt=list(range(18)), new_tokens=10)
    MultiStreamServer(eng, max_batch=1, prefix_slots=1, prefill_chunk=4).run([req])
    assert req.tokens == reference_tokens(req.prompt, 10, context=20)[:3]
    with pytest.raises(ValueError):
        MultiStreamServer(FakeEngine(max_slots=200), max_batch=130, prefix_slots=4, prefill_chunk=4)


def test_context_limit_and_validation():
    eng = FakeEngine(max_slots=2, context=20)
    req = Request(prompt=list(range(18)), new_tokens=10)
    MultiStreamServer(eng, max_batch=1, prefix_slots=1).run([req])
    assert req.tokens == reference_tokens(req.prompt, 10, context=20)[: len(req.tokens)]
    assert len(req.tokens) == 3  # positions 17, 18, 19 produce tokens; then the context is full
    with pytest.raises(ValueError):
        MultiStreamServer(eng, max_batch=1, prefix_slots=1).run([Request(prompt=list(range(20)), new_tokens=1)])
    with pytest.raises(ValueError):
        MultiStreamServer(FakeEngine(max_slots=4), max_batch=8, prefix_slots=0)


def test_lanes_serve_every_request_once_with_prefixes_kept_together():
    """Three lanes (servers on their own engines, one host thread each): the
    same tokens as single streams, every request served by exactly one
    lane.  The shared-prefix group (a quarter of the load, more than a
    lane's fair share) is cut into one piece per lane, and each lane
    computes the prefix once and reuses it for its piece."""
    engines = [FakeEngine(max_slots=12) for _ in range(3)]
    servers = [MultiStreamServer(e, max_batch=8, prefix_slots=4, prefill_chunk=8, max_rows=48) for e in engines]
    reqs = config5_requests(n=96)
    run_lanes(servers, reqs)
    for r in reqs:
        assert r.tokens == reference_tokens(r.prompt, r.new_tokens), r.rid
    rows = [sum(getattr(e, "row_steps", [])) for e in engines]
    assert all(n > 0 for n in rows)
    assert sum(s.rows for s in servers) == sum(rows)
    for e in engines:
        assert e.copies and all(n == 16 for _, _, n in e.copies)
    assert sum(1 for r in reqs if r.reused_prefix) >= 6


def test_a_failing_lane_raises_after_the_others_finish():
    class Broken(FakeEngine):
        def step_rows(self, *args, **kwargs):
            raise RuntimeError("lane fault (planted)")

    good = FakeEngine(max_slots=36)
    servers = [MultiStreamServer(good, max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=48),
               MultiStreamServer(Broken(max_slots=36), max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=48)]
    reqs = config5_requests(n=48)
    with pytest.raises(RuntimeError, match="planted"):
        run_lanes(servers, reqs)
    served = [r for r in reqs if r.tokens and len(r.tokens) == r.new_tokens]
    assert served and all(r.tokens == reference_tokens(r.prompt, r.new_tokens) for r in served)


@pytest.mark.gpu
def test_gpu_lanes_match_one_lane():
    """Two lanes, each an engine on its own CUDA stream driven by its own
    thread, their steps overlapping on the GPU: every request's tokens
    equal the single-lane run's (a row's arithmetic does not depend on the
    other rows of its step, nor on the other lane's kernels)."""
    import torch

    from runtime import layout, synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("tiny-qwen", seed=33).materialize()
    blob = layout.pack(model, "bf16")
    engines, streams = [], []
    try:
        for _ in range(3):
            engines.append(B200DecoderEngine(model, blob=blob, max_slots=36, max_batch=8))
            streams.append(torch.cuda.Stream())
            engines[-1].set_stream(streams[-1].cuda_stream)

        def make():
            rng = np.random.default_rng(12)
            shared = rng.integers(0, model.shape.vocab, 16).tolist()
            reqs = []
            for i in range(60):
                ids = rng.integers(0, model.shape.vocab, int(rng.integers(8, 40))).tolist()
                reqs.append(Request(prompt=shared + ids[:8] if i % 4 == 0 else ids, new_tokens=6, rid=i))
            return reqs

        one = make()
        MultiStreamServer(engines[0], max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=64).run(one)
        two = make()
        servers = [MultiStreamServer(e, max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=64)
                   for e in engines[1:]]
        run_lanes(servers, two)
        assert all(s.rows > 0 for s in servers)
        for a, b in zip(one, two):
            assert a.tokens == b.tokens, a.rid
    finally:
        for e in engines:
            e.close()


@pytest.mark.gpu
def test_gpu_multistream_matches_generate():
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("tiny-qwen", seed=31)
    engine = B200DecoderEngine(model, max_slots=12, max_batch=8)
    try:
        rng = np.random.default_rng(4)
        shared = rng.integers(0, model.shape.vocab, 16).tolist()
        reqs = []
        for i in range(20):
            ids = rng.integers(0, model.shape.vocab, int(rng.integers(8, 40))).tolist()
            if i % 4 == 0:
                ids = shared + ids[:8]
            reqs.append(Request(prompt=ids, new_tokens=6, rid=i))
        server = MultiStreamServer(engine, max_batch=8, prefix_slots=4)
        server.run(reqs)
        assert server.rows > server.launches  # rows really shared launches
        for r in reqs:
            single = engine.generate(r.prompt, r.new_tokens, slot=11)
            assert r.tokens == single, f"request {r.rid}"
        assert any(r.reused_prefix for r in reqs)
    finally:
        engine.close()


@pytest.mark.gpu
def test_gpu_sampled_multistream_matches_each_request_alone():
    """Sampled and greedy requests share launches; each request's tokens
    equal the same request served alone (the batch kernel computes every row
    the same way whatever the other rows are, and each generator supplies
    its own draws)."""
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("tiny-qwen", seed=32)
    vocab = model.shape.vocab
    engine = B200DecoderEngine(model, max_slots=12, max_batch=8)
    try:
        reqs = _sampled_requests(vocab, seed=3)
        for r in reqs:
            r.prompt = [t % vocab for t in r.prompt]
        MultiStreamServer(engine, max_batch=8, prefix_slots=4).run(reqs)
        alone = _sampled_requests(vocab, seed=3)
        for r, a in zip(reqs, alone):
            a.prompt = [t % vocab for t in a.prompt]
            engine.reset()
            MultiStreamServer(engine, max_batch=8, prefix_slots=4).run([a])
            assert r.tokens == a.tokens, r.rid
    finally:
        engine.close()


@pytest.mark.gpu
def test_gpu_chunked_rows_match_batched_single_streams():
    """Rows mode on the tensor-core step: 40 ragged requests, 32 streams,
    8-position prefill chunks.  A row's arithmetic does not depend on the
    other rows of its step, so every request's tokens equal the same
    request generated alone through the batched step."""
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("tiny-qwen", seed=31)
    engine = B200DecoderEngine(model, max_slots=40, max_batch=8)
    try:
        rng = np.random.default_rng(9)
        shared = rng.integers(0, model.shape.vocab, 16).tolist()
        reqs = []
        for i in range(40):
            ids = rng.integers(0, model.shape.vocab, int(rng.integers(8, 40))).tolist()
            if i % 4 == 0:
                ids = shared + ids[:8]
            reqs.append(Request(prompt=ids, new_tokens=6, rid=i))
        server = MultiStreamServer(engine, max_batch=32, prefix_slots=4, prefill_chunk=8, max_rows=64)
        server.run(reqs)
        assert server.rows > 2 * server.launches
        for r in reqs:
            assert r.tokens == engine.generate_rows(r.prompt, r.new_tokens, slot=39), f"request {r.rid}"
        assert any(r.reused_prefix for r in reqs)
    finally:
        engine.close()
