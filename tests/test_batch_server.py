"""BatchingCompletionEngine (runtime/batch_server.py) on CPU: concurrent
requests share batched steps and each gets exactly the tokens it would get
alone; a stop string, a deadline or a dropped reader ends only its own
stream; a device error reaches every request in flight and the next
requests are served again; close fails what is still queued.  The engine
is a causal fake (the next token hashes every cached token of the slot), so
a wrong prefix copy, a skipped position or a shared slot changes the
output."""

import threading
import time

import numpy as np
import pytest

from runtime import synthetic
from runtime.batch_server import BatchingCompletionEngine
from runtime.model import write_package

VOCAB = 1024
EOS = 3


class CausalEngine:
    """step_rows over per-slot token caches; optional failure / delay."""

    def __init__(self, max_slots, context=64):
        self.max_slots, self.context, self.vocab = max_slots, context, VOCAB
        self.cache = [[None] * context for _ in range(max_slots)]
        self.row_steps = []
        self.fail_at = None
        self.delay = 0.0
        self.closed = False

    def step_rows(self, slots, tokens, positions, logits=False, out_rows=None):
        if self.fail_at is not None and len(self.row_steps) == self.fail_at:
            self.fail_at = None
            raise RuntimeError("device fault (planted)")
        time.sleep(self.delay)
        self.row_steps.append(len(slots))
        for s, t, p in zip(slots, tokens, positions):
            self.cache[s][p] = t
        rows = range(len(slots)) if out_rows is None else out_rows
        out = [next_token(self.cache[slots[i]][: positions[i] + 1]) for i in rows]
        return np.array(out, np.int32), None

    def copy_prefix(self, src, dst, n):
        self.cache[dst][:n] = self.cache[src][:n]

    def reset(self, slot=None):
        for s in range(self.max_slots) if slot is None else [slot]:
            self.cache[s] = [None] * self.context

    def close(self):
        self.closed = True


def next_token(history):
    assert None not in history, "a position was read before it was written"
    return hash(tuple(history)) % VOCAB


class Tokenizer:
    eos_id = EOS

    def encode_chat_window(self, messages, budget):
        ids = [10 + (ord(c) % 90) for c in messages[-1]["content"]]
        return ids[-budget:], {"dropped_messages": 0}

    def encode_prompt_window(self, prompt, budget):
        ids = [10 + (ord(c) % 90) for c in prompt]
        return ids[-budget:], False

    def decode(self, ids):
        return "".join(f"<{t}>" for t in ids)

    def token_bytes(self, token_id):
        return f"<{token_id}>".encode()


def alone(prompt_ids, max_tokens, context=64):
    """The tokens a request gets on its own (stops after an eos)."""
    hist, out = list(prompt_ids), []
    while len(out) < max_tokens and len(hist) < context:
        t = next_token(hist)
        out.append(t)
        if t == EOS:
            break
        hist.append(t)
    return out


@pytest.fixture(scope="module")
def package(tmp_path_factory):
    path = tmp_path_factory.mktemp("pkg") / "tiny"
    write_package(synthetic.build("tiny-qwen", seed=3), path)
    return path


@pytest.fixture
def server(package):
    engines = []

    def factory(model, max_slots, weights):
        engines.append(CausalEngine(max_slots))
        return engines[-1]

    engine = BatchingCompletionEngine({"tiny": {"path": str(package)}}, engine_factory=factory, max_batch=16,
                                      prefill_chunk=8, max_rows=48, tokenizer_factory=lambda path, fam: Tokenizer())
    engine.engines = engines
    yield engine
    engine.close()


def collect(chunks):
    text, stats = [], None
    for piece, final, *_ in chunks:
        text.append(piece)
        if final is not None:
            stats = final
    return "".join(text), stats


PROMPTS = [f"request number {i} " + "abcdefghij"[: i % 10] for i in range(24)]


def test_concurrent_requests_match_each_request_alone(server):
    results = [None] * len(PROMPTS)
    start = threading.Barrier(len(PROMPTS))

    def run(i):
        start.wait()
        results[i] = collect(server.generate("tiny", [{"role": "user", "content": PROMPTS[i]}], 10))

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(PROMPTS))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    tok = Tokenizer()
    for i, (text, stats) in enumerate(results):
        prompt_ids, _ = tok.encode_chat_window([{"role": "user", "content": PROMPTS[i]}], 54)
        want = alone(prompt_ids, 10)
        shown = [t for t in want if t != EOS]
        assert stats["generated_token_ids"] == shown, i
        assert text == tok.decode(shown)
        assert stats["finish_reason"] == ("stop" if EOS in want else "length")
        assert stats["prompt_tokens"] == len(prompt_ids) and stats["ttft_seconds"] >= 0
    assert max(server.engines[0].row_steps) > 16  # several streams and prompt chunks per step


def test_stop_string_ends_only_its_request(server):
    tok = Tokenizer()
    ids, _ = tok.encode_prompt_window("stop me", 54)
    want = alone(ids, 12)
    stop = f"<{want[2]}>"
    other, _ = tok.encode_prompt_window("keep going", 54)
    results = {}

    def run(key, prompt, **options):
        results[key] = collect(server.generate("tiny", prompt, 12, **options))

    threads = [threading.Thread(target=run, args=("stop", "stop me"), kwargs={"stop": [stop]}),
               threading.Thread(target=run, args=("other", "keep going"))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    text, stats = results["stop"]
    assert stats["finish_reason"] == "stop" and stop not in text
    assert text == tok.decode(want[:2])
    assert results["other"][1]["generated_token_ids"] == [t for t in alone(other, 12) if t != EOS]


def test_device_error_reaches_every_request_then_recovers(server):
    server.prewarm_default()
    engine = server.engines[0]
    engine.fail_at = len(engine.row_steps) + 2
    errors = []
    start = threading.Barrier(4)

    def run(i):
        start.wait()
        try:
            collect(server.generate("tiny", f"failing {i}", 20))
        except RuntimeError as exc:
            errors.append(str(exc))

    threads = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert len(errors) == 4 and all("planted" in e for e in errors)
    text, stats = collect(server.generate("tiny", "after the fault", 5))
    assert stats["generated_token_ids"] == [t for t in alone(Tokenizer().encode_prompt_window("after the fault", 54)[0], 5)
                                           if t != EOS]


def test_deadline_and_abandoned_readers_end_their_streams(server):
    server.prewarm_default()
    engine = server.engines[0]
    engine.delay = 0.05
    with pytest.raises(TimeoutError):
        collect(server.generate("tiny", "slow request", 30, timeout=0.1))
    gen = server.generate("tiny", "read one chunk", 30)
    next(gen)
    gen.close()  # the reader goes away: its stream is cancelled at the next step
    engine.delay = 0.0
    time.sleep(0.3)
    assert not server._workers["tiny"].server.busy


def test_close_fails_the_requests_in_flight(server):
    server.prewarm_default()
    engine = server.engines[0]
    engine.delay = 0.05
    errors = []

    def run(i):
        try:
            collect(server.generate("tiny", f"long request {i}", 40))
        except RuntimeError as exc:
            errors.append(str(exc))

    threads = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    time.sleep(0.3)
    server.close()
    for t in threads:
        t.join()
    assert len(errors) == 4 and all("closed" in e for e in errors)
    assert engine.closed


def test_a_request_that_cannot_fit_fails_alone(server):
    with pytest.raises(ValueError):
        collect(server.generate("tiny", "x", 64))  # no room left for a prompt position
    text, stats = collect(server.generate("tiny", "fits", 4))
    assert 1 <= stats["generated_tokens"] <= 4


@pytest.mark.gpu
def test_gpu_concurrent_requests_match_batched_single_streams(package):
    """The same server over the B200 engine (tensor-core rows): 16
    concurrent requests; each one's tokens equal that request generated
    alone through the batched step (a row's arithmetic does not depend on
    the other rows of its step)."""
    from runtime.batch_server import default_engine_factory

    engines = []

    def factory(model, max_slots, weights):
        engines.append(default_engine_factory(model, max_slots, weights))
        return engines[-1]

    server = BatchingCompletionEngine({"tiny": {"path": str(package)}}, engine_factory=factory, max_batch=16,
                                      prefill_chunk=8, max_rows=64, tokenizer_factory=lambda path, fam: Tokenizer())
    prompts = PROMPTS[:16]
    results = [None] * len(prompts)
    start = threading.Barrier(len(prompts))

    def run(i):
        start.wait()
        results[i] = collect(server.generate("tiny", prompts[i], 8))

    try:
        threads = [threading.Thread(target=run, args=(i,)) for i in range(len(prompts))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        engine = engines[0]
        tok = Tokenizer()
        for i, (_, stats) in enumerate(results):
            ids, _ = tok.encode_prompt_window(prompts[i], 56)
            engine.reset(19)  # a prefix-pool slot, free now that every request has finished
            want = engine.generate_rows(ids, 8, slot=19)
            shown = []
            for t in want:
                if t == EOS:
                    break
                shown.append(t)
            assert stats["generated_token_ids"] == shown, i
    finally:
        server.close()
