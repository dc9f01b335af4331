"""Token sampling: the oracle against the reference ``Sampler`` (golden
vectors of ``tests/golden/make_sampling_golden.py``), NumPy's summation order,
the C-ABI argument checks, and on a GPU the on-device sampler against the
oracle.

Parity rule for the device sampler: its token must equal the reference's,
except where the oracle's draw ``u`` lies within 1e-5 of a boundary of the
normalised cumulative distribution or a top-p cut lies within 1e-5 of
``top_p`` -- there the float32 ``exp`` of NumPy and of CUDA may differ in the
last bit (a documented near-tie).
"""

import ctypes
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from oracle import sampling as osamp
from runtime import hb_lib

GOLDEN = Path(__file__).resolve().parent / "golden"


def _cases_module():
    spec = importlib.util.spec_from_file_location("sampling_cases", GOLDEN / "make_sampling_golden.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def golden_cases():
    mod = _cases_module()
    tokens = np.load(GOLDEN / "sampling.npz")["tokens"]
    out = []
    for (vocab, scale, spec, seed), expect in zip(mod.cases(), tokens):
        logits, history, bias = mod.build(vocab, scale, spec, seed)
        t, top_p, top_k, rep, pres, freq, _, _ = spec
        params = osamp.Params(temperature=t, top_p=top_p, top_k=top_k, repetition_penalty=rep,
                              presence_penalty=pres, frequency_penalty=freq, logit_bias=bias)
        out.append((logits, history, params, seed, [int(x) for x in expect]))
    return out


def uniforms(params, vocab, seed, steps=2):
    """The generator draws successive selections consume (None: no draw)."""
    rng = np.random.default_rng(seed)
    return [rng.random() if osamp.draws_uniform(params, vocab) else None for _ in range(steps)]


def test_pairwise_sum_is_numpys_order():
    rng = np.random.default_rng(0)
    for n in list(range(1, 140)) + [255, 1000, 8191, 8193, 20001, 151936]:
        for dtype in (np.float32, np.float64):
            x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 1e3], n)).astype(dtype)
            assert osamp.pairwise_sum(x).tobytes() == np.asarray(x.sum(), dtype).tobytes(), (n, dtype)


def test_oracle_matches_reference_sampler():
    cases = golden_cases()
    assert len(cases) == 81
    for logits, history, params, seed, expect in cases:
        us = uniforms(params, logits[0].shape[0], seed)
        got = [osamp.select_with_uniform(logits[i], history, params, us[i]) for i in range(2)]
        assert got == expect, (params, seed)


def test_oracle_log_softmax_matches_reference():
    data = np.load(GOLDEN / "sampling.npz")
    for i, (logits, history, params, seed, expect) in enumerate(golden_cases()):
        values = osamp.log_softmax(logits[0])
        assert abs(values[expect[0]] - data["logprob_token"][i]) < 1e-12
        top = osamp.top_logprobs(values, 5)
        assert top.tolist() == data["logprob_top_ids"][i].tolist()
        assert np.allclose(values[top], data["logprob_top_values"][i], rtol=0, atol=1e-12)


def test_draw_consumes_one_uniform_like_generator_choice():
    rng = np.random.default_rng(5)
    for seed in range(50):
        p = rng.random(300)
        p /= p.sum()
        want = np.random.default_rng(seed).choice(300, p=p)
        assert want == osamp.draw(p, np.random.default_rng(seed).random())


def test_runtime_draw_rule_matches_oracle():
    from runtime.device_sampler import draws_uniform

    for logits, history, params, seed, expect in golden_cases():
        vocab = logits[0].shape[0]
        assert draws_uniform(params, vocab) == osamp.draws_uniform(params, vocab)


def test_sampler_c_abi_rejects_bad_arguments_without_a_gpu():
    lib = hb_lib.load()
    handle = ctypes.c_void_p()
    assert lib.hb_sampler_create(0, 0, ctypes.byref(handle)) == hb_lib.HB_ERR_UNSUPPORTED
    assert lib.hb_sampler_create(1 << 20, 0, ctypes.byref(handle)) == hb_lib.HB_ERR_UNSUPPORTED
    assert lib.hb_sampler_select(None, None, 0, None, None) == hb_lib.HB_ERR_INVALID_ARG
    assert lib.hb_sampler_destroy(None) == hb_lib.HB_OK
    assert lib.hb_sample(None, 0, None, None) == hb_lib.HB_ERR_INVALID_ARG


# -- on the GPU ---------------------------------------------------------------
def _near_tie(logits, history, params, u):
    """True when the oracle's draw or top-p cut sits within 1e-5 of a boundary."""
    scores = np.asarray(logits, np.float32).copy()
    scores = osamp.apply_bias(osamp.apply_penalties(scores, history, params), params.logit_bias)
    scores = scores / params.temperature
    scores = osamp.top_k_mask(scores, params.top_k)
    if params.top_p < 1.0:
        order = np.argsort(scores)[::-1]
        probs = osamp.guarded_softmax(scores[order])
        before = np.cumsum(probs) - probs
        if before.size > 1 and np.min(np.abs(before[1:] - params.top_p)) < 1e-5:
            return True
    scores = osamp.top_p_mask(scores, params.top_p)
    cdf = np.cumsum(osamp.final_distribution(scores))
    cdf /= cdf[-1]
    return bool(np.min(np.abs(cdf - u)) < 1e-5)


@pytest.mark.gpu
def test_device_sampler_matches_reference_golden():
    from runtime.device_sampler import DeviceSampler

    samplers = {}
    mismatches = 0
    try:
        for logits, history, params, seed, expect in golden_cases():
            vocab = logits[0].shape[0]
            dev = samplers.setdefault(vocab, DeviceSampler(vocab))
            us = uniforms(params, vocab, seed)
            for i in range(2):
                got = dev.select(logits[i], history, params, us[i])
                if got != expect[i]:
                    assert got is not None and us[i] is not None and _near_tie(logits[i], history, params, us[i]), (
                        params, seed, i, got, expect[i])
                    mismatches += 1
    finally:
        for dev in samplers.values():
            dev.close()
    assert mismatches <= 1


@pytest.mark.gpu
def test_device_sampler_full_vocabulary_against_oracle():
    """151936-wide logits (the Qwen vocabulary), flat to peaked, every stage;
    a flat distribution under top_p alone keeps more than 4096 candidates and
    must report that (None) instead of guessing."""
    from runtime.device_sampler import DeviceSampler

    rng = np.random.default_rng(11)
    vocab = 151936
    settings = [
        osamp.Params(temperature=1.0),
        osamp.Params(temperature=0.7, top_k=50),
        osamp.Params(temperature=1.0, top_k=3000, top_p=0.9),
        osamp.Params(temperature=0.8, top_p=0.95),
        osamp.Params(temperature=1.1, repetition_penalty=1.2, frequency_penalty=0.3, presence_penalty=0.2,
                     logit_bias={5: 4.0, 77: -100.0, 151935: 2.5}),
        osamp.Params(temperature=0.0, repetition_penalty=1.5),
    ]
    agree = total = unsupported = 0
    with DeviceSampler(vocab) as dev:
        for scale in (0.05, 2.0, 6.0):
            for params in settings:
                for _ in range(3):
                    logits = (rng.standard_normal(vocab) * scale).astype(np.float32)
                    history = rng.integers(0, vocab, 40).tolist()
                    u = rng.random() if osamp.draws_uniform(params, vocab) else None
                    want = osamp.select_with_uniform(logits, history, params, u)
                    got = dev.select(logits, history, params, u)
                    if got is None:
                        # only a top-p nucleus beyond the on-chip sort may say so
                        s = osamp.top_k_mask(osamp.apply_bias(osamp.apply_penalties(
                            logits.copy(), history, params), params.logit_bias) / params.temperature, params.top_k)
                        kept = np.isfinite(osamp.top_p_mask(s, params.top_p)).sum()
                        assert params.top_p < 1.0 and kept > 4096 - 8, (params, scale, kept)
                        unsupported += 1
                        continue
                    total += 1
                    if got == want:
                        agree += 1
                    else:
                        assert _near_tie(logits, history, params, u), (params, scale, got, want)
    assert total >= 40 and agree >= total - 2
    assert unsupported <= 6


@pytest.mark.gpu
def test_engine_samples_its_own_logits_on_the_device():
    """hb_sample on the logits a step left on the device equals the
    standalone sampler on the same logits copied to the host."""
    from oracle.cpu_decoder import OracleDecoder  # noqa: F401  (oracle importable on the box)
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine
    from runtime.device_sampler import DeviceSampler

    model = synthetic.build("tiny-qwen", seed=31)
    engine = B200DecoderEngine(model, max_slots=2, max_batch=8)
    try:
        ids = synthetic.prompt_ids(model.shape.vocab, 6, seed=3)
        params = osamp.Params(temperature=0.9, top_k=40, top_p=0.9, repetition_penalty=1.1,
                              logit_bias={3: 2.0})
        rng = np.random.default_rng(9)
        with DeviceSampler(model.shape.vocab) as dev:
            for pos, tok in enumerate(ids):
                logits = engine.step(tok, pos, logits=True, slot=1)
                engine.step_device_logits(tok, pos, slot=0)
                u = rng.random()
                a = engine.sample(params, ids[:pos + 1], u)
                b = dev.select(logits, ids[:pos + 1], params, u)
                assert a == b == osamp.select_with_uniform(logits, ids[:pos + 1], params, u) or _near_tie(
                    logits, ids[:pos + 1], params, u)
    finally:
        engine.close()


class OracleSampler:
    """The reference ``Sampler``'s surface (``params``, ``greedy``, its seeded
    generator ``_rng``, ``select``) over the oracle."""

    def __init__(self, params, vocab, seed):
        self.params = params
        self.vocab = vocab
        self._rng = np.random.default_rng(seed)

    @property
    def greedy(self):
        return self.params.greedy_for(self.vocab)

    def select(self, logits, history):
        u = self._rng.random() if osamp.draws_uniform(self.params, self.vocab) else None
        return osamp.select_with_uniform(logits, history, self.params, u)


def test_drop_in_falls_back_to_the_host_with_the_same_draw():
    """When the device cannot sort the top-p nucleus, the drop-in rewinds the
    generator and the host sampler selects with the draw the device would
    have used."""
    import types

    from runtime.generate import NPUDecoder

    vocab = 50
    logits = np.random.default_rng(2).standard_normal(vocab).astype(np.float32)
    calls = []

    class FakeEngine:
        def __init__(self):
            self.vocab = vocab

        def step_device_logits(self, token_id, position, slot=0):
            calls.append(("step", token_id, position))
            return 0

        def sample(self, params, history, uniform, row=0):
            calls.append(("sample", uniform))
            return None  # "nucleus too large"

        def device_logits(self, rows=1):
            return logits

    decoder = object.__new__(NPUDecoder)
    decoder.context_length = 64
    decoder._cached_prefix = []
    decoder._profile_enabled = False
    decoder._engine = FakeEngine()
    decoder.model = types.SimpleNamespace(metadata={"vocab_size": vocab})
    params = osamp.Params(temperature=0.8, top_p=0.9)
    sampler = OracleSampler(params, vocab, seed=17)
    token, _, entry = decoder._sample_step(4, 0, sampler, [4])
    assert entry is None
    first_u = np.random.default_rng(17).random()
    assert calls[1] == ("sample", first_u)
    assert token == osamp.select_with_uniform(logits, [4], params, first_u)
    # the stream continues where a host-only run would be
    assert sampler._rng.random() == np.random.default_rng(17).random(2)[1]
    assert decoder._cached_prefix == [4]


@pytest.mark.gpu
def test_drop_in_device_sampling_matches_host_sampling():
    """NPUDecoder's sampled decode step (logits kept on the GPU) selects the
    same tokens as the host sampler on the engine's logits, draw for draw."""
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine
    from runtime.generate import NPUDecoder

    model = synthetic.build("tiny-qwen", seed=43)
    vocab = model.shape.vocab
    params = osamp.Params(temperature=1.0, top_k=200, top_p=0.95, repetition_penalty=1.15,
                          frequency_penalty=0.1, logit_bias={7: 3.0})
    decoder = NPUDecoder(model)
    engine = B200DecoderEngine(model, max_batch=1)
    try:
        dev_sampler, host_sampler = OracleSampler(params, vocab, 5), OracleSampler(params, vocab, 5)
        prompt = synthetic.prompt_ids(vocab, 6, seed=8)
        history = list(prompt)
        for pos, tok in enumerate(prompt[:-1]):
            decoder.decode_token(tok, pos, compute_logits=False)
            engine.step(tok, pos, logits=False)
        tok, pos = prompt[-1], len(prompt) - 1
        for _ in range(12):
            a, _, _ = decoder._sample_step(tok, pos, dev_sampler, history)
            logits = engine.step(tok, pos, logits=True)
            b = host_sampler.select(logits, history)
            if a != b:
                break  # a near-tie; the streams legitimately diverge afterwards
            history.append(a)
            tok, pos = a, pos + 1
        else:
            return
        pytest.fail(f"device {a} != host {b} at position {pos}")
    finally:
        decoder.close()
        engine.close()


def _check_logprobs(got, logits, token, n_top):
    values = osamp.log_softmax(logits)
    tok_lp, ids, lps = got
    assert abs(tok_lp - values[token]) < 1e-9
    want = osamp.top_logprobs(values, n_top)
    assert np.allclose(lps, values[want], rtol=0, atol=1e-9)
    # the same set of entries; equal log-probabilities may come in any order
    assert np.allclose(values[ids], values[want], rtol=0, atol=1e-12)
    assert len(set(ids)) == len(ids)


@pytest.mark.gpu
def test_device_logprobs_match_reference_log_softmax():
    from runtime.device_sampler import DeviceSampler

    data = np.load(GOLDEN / "sampling.npz")
    samplers = {}
    try:
        for i, (logits, history, params, seed, expect) in enumerate(golden_cases()):
            vocab = logits[0].shape[0]
            dev = samplers.setdefault(vocab, DeviceSampler(vocab))
            tok_lp, ids, lps = dev.logprobs(logits[0], expect[0], 5)
            assert abs(tok_lp - data["logprob_token"][i]) < 1e-9
            assert ids == data["logprob_top_ids"][i].tolist()
            assert np.allclose(lps, data["logprob_top_values"][i], rtol=0, atol=1e-9)
        rng = np.random.default_rng(4)
        with DeviceSampler(151936) as dev:
            for scale in (0.05, 3.0):
                for n_top in (0, 1, 20):
                    logits = (rng.standard_normal(151936) * scale).astype(np.float32)
                    logits[rng.integers(0, 151936, 10)] = -np.inf
                    token = int(rng.integers(0, 151936))
                    while not np.isfinite(logits[token]):
                        token = int(rng.integers(0, 151936))
                    _check_logprobs(dev.logprobs(logits, token, n_top), logits, token, n_top)
    finally:
        for dev in samplers.values():
            dev.close()


@pytest.mark.gpu
def test_drop_in_device_logprobs_match_host_entries():
    """Greedy and sampled requests with logprobs: the entries built from the
    device's log-probabilities equal those the host builds from the logits."""
    import types

    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine
    from runtime.generate import NPUDecoder

    model = synthetic.build("tiny-qwen", seed=44)
    vocab = model.shape.vocab
    decoder = NPUDecoder(model)
    engine = B200DecoderEngine(model, max_batch=1)

    class Tok:
        def decode(self, ids):
            return "".join(f"<{t}>" for t in ids)

        def token_bytes(self, t):
            return self.decode([t]).encode()

    decoder.tokenizer = Tok()
    try:
        prompt = synthetic.prompt_ids(vocab, 5, seed=9)
        for params in (osamp.Params(), osamp.Params(temperature=0.9, top_k=100)):
            decoder._engine.reset()
            engine.reset()
            dev_sampler, host_sampler = OracleSampler(params, vocab, 3), OracleSampler(params, vocab, 3)
            history = list(prompt)
            for pos, tok in enumerate(prompt[:-1]):
                decoder.decode_token(tok, pos, compute_logits=False)
                engine.step(tok, pos, logits=False)
            tok, pos = prompt[-1], len(prompt) - 1
            for _ in range(4):
                a, _, entry = decoder._sample_step(tok, pos, dev_sampler, history, top_logprobs=3)
                logits = engine.step(tok, pos, logits=True)
                b = host_sampler.select(logits, history)
                assert a == b
                values = osamp.log_softmax(logits)
                assert abs(entry["logprob"] - values[a]) < 1e-9
                want = osamp.top_logprobs(values, 3)
                assert [e["token"] for e in entry["top_logprobs"]] == [f"<{i}>" for i in want]
                history.append(a)
                tok, pos = a, pos + 1
    finally:
        decoder.close()
        engine.close()


@pytest.mark.gpu
def test_batched_device_sampling_matches_single_rows_at_qwen_vocabulary():
    """hb_sample_batch (one thread block per row) selects what the single
    selection selects on the same logits (the grid-wide kernel at this
    vocabulary), row by row, and reports a flat top-p nucleus as too large
    (None) per row without disturbing the other rows."""
    import dataclasses

    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine
    from runtime.device_sampler import DeviceSampler

    shape = dataclasses.replace(synthetic.TINY_QWEN, vocab=151936)
    model = synthetic.build(shape, seed=45)
    engine = B200DecoderEngine(model, max_slots=4, max_batch=8)
    try:
        ids = synthetic.prompt_ids(shape.vocab, 4, seed=2)
        engine.step_batch([0, 1, 2, 3], ids, [0, 0, 0, 0], device_logits=True)
        logits = engine.device_logits(rows=4)
        params = [osamp.Params(temperature=0.8), osamp.Params(temperature=1.0, top_k=50, top_p=0.9),
                  osamp.Params(temperature=1.0, top_p=0.9),  # flat random-init logits: too large
                  osamp.Params(temperature=0.7, repetition_penalty=1.3, logit_bias={11: 5.0})]
        histories = [ids[:1], ids[:2], ids[:3], ids]
        rng = np.random.default_rng(6)
        uniforms = [rng.random() for _ in params]
        got = engine.sample_batch([0, 1, 2, 3], params, histories, uniforms)
        assert got[2] is None
        with DeviceSampler(shape.vocab) as dev:
            for r in (0, 1, 3):
                single = dev.select(logits[r], histories[r], params[r], uniforms[r])
                assert got[r] == single
                want = osamp.select_with_uniform(logits[r], histories[r], params[r], uniforms[r])
                assert got[r] == want or _near_tie(logits[r], histories[r], params[r], uniforms[r])
    finally:
        engine.close()
