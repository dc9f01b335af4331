"""Host generation loop of the drop-in NPUDecoder, without a GPU: the
decoder is built with ``object.__new__`` and a fake ``decode_token`` that
returns canned logits, the way the reference tests its own loop
(npu_llm/tests/test_decode_loop.py:94-124).  Covers greedy selection, the
prefix cache (:267-311), a failing step (:313-331) and stop strings."""

import types

import numpy as np
import pytest

from runtime.generate import NPUDecoder

EOS = 9
VOCAB = 10


class FakeTokenizer:
    eos_id = EOS

    def __init__(self, prompt_ids):
        self.prompt_ids = list(prompt_ids)

    def encode_chat_window(self, messages, budget):
        return list(self.prompt_ids), {"dropped_messages": 0}

    def encode_prompt_window(self, prompt, budget):
        return list(self.prompt_ids), False

    def decode(self, ids):
        return "".join(f"<{t}>" for t in ids)

    def token_bytes(self, token_id):
        return self.decode([token_id]).encode()


def build(prompt_ids, logits_for):
    decoder = object.__new__(NPUDecoder)
    decoder.model = types.SimpleNamespace(metadata={"vocab_size": VOCAB})
    decoder.context_length = 64
    decoder.tokenizer = FakeTokenizer(prompt_ids)
    decoder.npu_layers = 0
    decoder.layers = 0
    decoder.calls = []
    decoder._cached_prefix = []
    decoder._prefix_cache_enabled = True
    decoder._profile_enabled = False

    def decode_token(token_id, position, *, diagnostics=False, select=None, compute_logits=True):
        logits = np.asarray(logits_for(token_id), np.float32)
        decoder.calls.append((token_id, position, select is not None, compute_logits))
        if not compute_logits:
            return None, 0.001
        return (int(np.argmax(logits)) if select is None else int(select(logits))), 0.001

    decoder.decode_token = decode_token
    return decoder


def run(decoder, max_new_tokens=4, **options):
    text, stats = [], None
    for piece, final, *_ in decoder.generate_messages([{"role": "user", "content": "hi"}], max_new_tokens,
                                                      **options):
        text.append(piece)
        if final is not None:
            stats = final
    return "".join(text), stats


def ramp(token_id):
    logits = np.zeros(VOCAB, np.float32)
    logits[(token_id + 1) % VOCAB] = 5.0
    return logits


def test_greedy_loop_prefills_then_decodes():
    decoder = build([1, 2, 3], ramp)
    text, stats = run(decoder)
    assert stats["generated_token_ids"] == [4, 5, 6, 7]
    assert text == "<4><5><6><7>"
    assert stats["finish_reason"] == "length"
    assert stats["decode_steps"] == 3
    assert stats["decode_seconds"] == 0.003
    assert [c[3] for c in decoder.calls] == [False, False, True, True, True, True]
    assert not any(c[2] for c in decoder.calls)


def test_shared_prompt_prefix_is_not_recomputed():
    decoder = build([1, 2, 3], ramp)
    _, first = run(decoder)
    assert first["cached_prompt_tokens"] == 0
    assert decoder._cached_prefix == [1, 2, 3, 4, 5, 6]
    decoder.tokenizer.prompt_ids = [1, 2, 3, 4, 5, 2]
    decoder.calls.clear()
    _, second = run(decoder)
    assert second["cached_prompt_tokens"] == 5
    assert decoder.calls[0][1] == 5
    assert second["generated_token_ids"] == [3, 4, 5, 6]
    decoder.calls.clear()
    _, repeat = run(decoder)
    assert repeat["cached_prompt_tokens"] == 5
    decoder.tokenizer.prompt_ids = [1, 7, 3]
    decoder.calls.clear()
    _, diverged = run(decoder)
    assert diverged["cached_prompt_tokens"] == 1
    assert decoder.calls[0][:2] == (7, 1)


def test_prefix_cache_can_be_disabled_and_reset():
    decoder = build([1, 2, 3], ramp)
    run(decoder)
    decoder.reset_prefix_cache()
    decoder.calls.clear()
    _, stats = run(decoder)
    assert stats["cached_prompt_tokens"] == 0
    decoder._prefix_cache_enabled = False
    decoder.calls.clear()
    _, stats = run(decoder)
    assert stats["cached_prompt_tokens"] == 0 and len(decoder.calls) == 6


def test_failed_step_invalidates_its_position():
    decoder = build([1, 2, 3], ramp)
    run(decoder)
    original = decoder.decode_token

    def failing(token_id, position, **kwargs):
        if position == 1:
            raise RuntimeError("kernel failure")
        return original(token_id, position, **kwargs)

    decoder.decode_token = failing
    decoder.tokenizer.prompt_ids = [1, 9, 9, 9]
    try:
        run(decoder)
    except RuntimeError:
        pass
    else:
        raise AssertionError("the failing step did not raise")
    assert decoder._cached_prefix == [1]


def test_eos_and_stop_strings_end_generation():
    def to_eos(token_id):
        logits = np.zeros(VOCAB, np.float32)
        logits[EOS if token_id == 7 else 7] = 5.0
        return logits

    _, stats = run(build([1], to_eos), max_new_tokens=6)
    assert stats["generated_token_ids"] == [7] and stats["finish_reason"] == "stop"
    text, stats = run(build([1], ramp), max_new_tokens=8, stop=["<4><"])
    assert text == "<2><3>"
    assert stats["finish_reason"] == "stop" and stats["stop_sequence"] == "<4><"


def test_logprobs_are_reported_per_token():
    decoder = build([1], ramp)
    chunks = list(decoder.generate_messages([{"role": "user", "content": "hi"}], 2, logprobs=2))
    entries = [e for _, _, es in chunks for e in es]
    assert [e["token"] for e in entries] == ["<2>", "<3>"]
    assert all(len(e["top_logprobs"]) == 2 for e in entries)
    assert all(c[2] for c in decoder.calls if c[3])  # a selector was engaged


def test_decode_result_diagnostics():
    logits = np.array([0.0, 3.0, 1.0, 2.9, -1.0, 0.5], np.float32)
    token, elapsed, diag = NPUDecoder._decode_result(logits, 0.0, True)
    assert token == 1 and diag["top_token_ids"][:2] == [1, 3]
    assert abs(diag["top_logit_margin"] - 0.1) < 1e-6


def test_invalid_arguments():
    decoder = build([1], ramp)
    import pytest
    with pytest.raises(ValueError):
        run(decoder, max_new_tokens=64)
    with pytest.raises(ValueError):
        NPUDecoder(object(), context_length=32)
    # longer contexts: whole 64-position pages, at most 4096 (checked before
    # any model or device is touched)
    for context in (100, 4160, 8192):
        with pytest.raises(ValueError, match="multiple of 64"):
            NPUDecoder(object(), context_length=context)


@pytest.mark.gpu
def test_drop_in_batched_prompt_prefill_on_gpu():
    """On the real engine the drop-in prefills the uncached prompt positions
    through batched launches; the tokens equal single-stream generation and
    the prefix cache is reused on a repeated prompt."""
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("tiny-qwen", seed=41)
    prompt = synthetic.prompt_ids(model.shape.vocab, 19, seed=3)
    decoder = NPUDecoder(model)
    try:
        decoder.tokenizer = FakeTokenizer(prompt)
        decoder.tokenizer.eos_id = -1
        _, stats = run(decoder, max_new_tokens=6)
        _, again = run(decoder, max_new_tokens=6)
    finally:
        decoder.close()
    single = B200DecoderEngine(model, max_batch=1)
    try:
        ref = single.generate(prompt, 6)
    finally:
        single.close()
    assert stats["generated_token_ids"] == ref
    assert again["generated_token_ids"] == ref
    assert again["cached_prompt_tokens"] == len(prompt) - 1
