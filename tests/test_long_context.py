"""Paged KV cache (contexts longer than the reference's 64 positions) on the
GPU against the CPU oracle run at the same context length.

The reference fixes its cache at 64 positions (npu_llm/runtime/generate.py:
43-44); beyond that the oracle's per-position attention (scores, max-shifted
softmax, P.V) is the specification.  Same parity rule as the 64-position
engine (tests/test_gpu_engine.py): FP32 logits within max-abs 5e-2 and
relative 1e-2 of the oracle for the 2-layer models, argmax equal except at
documented near-ties; BF16 caches bit-equal except for a small fraction of
one-unit differences.  The cases cross page boundaries (64 positions), run
the split attention (more than 128 positions: several CTAs per head, the
last to arrive combining their partial sums), batched prefill through the
8-row kernel, prefix sharing with copy-on-write, and reset.
"""

import numpy as np
import pytest
from ml_dtypes import bfloat16

from oracle.cpu_decoder import OracleDecoder, greedy_generate
from runtime import layout, synthetic
from runtime.b200_engine import B200DecoderEngine
from test_gpu_engine import ATOL_FULL, NEAR_TIE, RTOL_FULL, assert_logits_close, bits_close

pytestmark = pytest.mark.gpu

CONTEXT = 320  # five pages


@pytest.fixture(scope="module", params=["tiny-qwen", "tiny-llama"])
def paged(request):
    model = synthetic.build(request.param, seed=31)
    engine = B200DecoderEngine(model, max_slots=3, max_batch=8, context=CONTEXT)
    yield model, engine
    engine.close()


def test_teacher_forced_logits_and_cache_match_oracle(paged):
    model, engine = paged
    engine.reset()
    oracle = OracleDecoder(model, context_length=CONTEXT)
    ids = synthetic.prompt_ids(model.shape.vocab, 300, seed=11)
    for position, token in enumerate(ids):
        got = engine.step(token, position, logits=True)
        ref = oracle.step(token, position)
        assert_logits_close(got, ref, f"position {position}")
    kv = engine.kv_cache(0)
    assert kv.shape[3] == CONTEXT
    for layer in range(model.shape.layers):
        for kind, ref in ((0, oracle.keys[layer]), (1, oracle.values[layer])):
            got, want = kv[layer, :, kind, : len(ids)], np.asarray(ref[:, : len(ids)])
            if layer == 0:
                bits_close(got, want)  # from the embedding alone
            else:
                cache_close(got, want)
    assert not kv[:, :, :, len(ids):].any()  # never written: zero, as after a reset


def cache_close(got, ref):
    """K/V of a layer after the first: its input carries the attention
    outputs, summed over up to 300 positions in another order than NumPy's;
    their last-bit differences pass through RMSNorm and the projection, so a
    few percent of the BF16 values move by a few units, all small against
    the tensor's scale."""
    a = np.asarray(got).view(np.uint16)
    b = np.asarray(ref).view(np.uint16)
    assert (a != b).mean() <= 0.05, f"{(a != b).mean():.4f} of BF16 values differ"
    va = a.view(bfloat16).astype(np.float32)
    vb = b.view(bfloat16).astype(np.float32)
    scale = float(np.abs(vb).max())
    assert np.abs(va - vb).max() <= scale * 2 ** -6, (np.abs(va - vb).max(), scale)


def test_batched_prefill_and_batch_rows_match_oracle(paged):
    model, engine = paged
    engine.reset()
    ids = synthetic.prompt_ids(model.shape.vocab, 261, seed=12)
    # 8 positions per launch through the 8-row kernel, then the last with the head
    tok, logits = engine.prefill(ids[:200], slot=0, logits=True)
    oracle = OracleDecoder(model, context_length=CONTEXT)
    for p in range(199):
        oracle.step(ids[p], p, compute_logits=False)
    ref = oracle.step(ids[199], 199)
    assert_logits_close(logits, ref, "prefill position 199")
    # two slots at different depths in one batched step
    engine.prefill(ids[:130], slot=1)
    am, rows = engine.step_batch([0, 1], [ids[200], ids[130]], [200, 130], logits=True)
    assert_logits_close(rows[0], oracle.step(ids[200], 200), "batch row 0")
    other = OracleDecoder(model, context_length=CONTEXT)
    for p in range(130):
        other.step(ids[p], p, compute_logits=False)
    assert_logits_close(rows[1], other.step(ids[130], 130), "batch row 1")
    assert list(am) == [int(np.argmax(r)) for r in rows]


def test_prefix_sharing_copies_a_page_only_on_write(paged):
    model, engine = paged
    engine.reset()
    ids = synthetic.prompt_ids(model.shape.vocab, 150, seed=13)
    alt = synthetic.prompt_ids(model.shape.vocab, 150, seed=14)
    engine.prefill(ids, slot=0)
    kv0 = engine.kv_cache(0)
    # 140 positions: two whole pages shared, 12 rows of the third copied
    engine.copy_prefix(0, 1, 140)
    assert np.array_equal(engine.kv_cache(1)[:, :, :, :140], kv0[:, :, :, :140])
    for p in range(140, 150):
        engine.step(alt[p], p, logits=False, slot=1)
    assert np.array_equal(engine.kv_cache(0), kv0)
    # share two pages again, then rewrite a position inside the shared page 1
    engine.copy_prefix(0, 1, 128)
    got = engine.step(alt[100], 100, logits=True, slot=1)
    assert np.array_equal(engine.kv_cache(0), kv0)  # slot 0's page untouched
    oracle = OracleDecoder(model, context_length=CONTEXT)
    for p in range(100):
        oracle.step(ids[p], p, compute_logits=False)
    assert_logits_close(got, oracle.step(alt[100], 100), "rewritten shared position")
    # slot 0 continues on its own pages
    ref0 = OracleDecoder(model, context_length=CONTEXT)
    for p in range(150):
        ref0.step(ids[p], p, compute_logits=False)
    assert_logits_close(engine.step(alt[0], 150, logits=True, slot=0), ref0.step(alt[0], 150), "slot 0 at 150")


def test_reset_then_generate_across_pages(paged):
    model, engine = paged
    engine.reset(2)
    ids = synthetic.prompt_ids(model.shape.vocab, 60, seed=15)
    device = engine.generate(ids, 80, slot=2)
    engine.reset(2)
    host = [engine.prefill(ids, slot=2)[0]]
    for i in range(79):
        host.append(engine.step_argmax(host[-1], len(ids) + i, slot=2))
    assert device == host
    oracle = OracleDecoder(model, context_length=CONTEXT)
    ref, logits = greedy_generate(oracle, ids, 80)
    for i, (a, b) in enumerate(zip(device, ref)):
        if a != b:
            lg = logits[i]
            top = np.argsort(-lg)[:2]
            assert lg[top[0]] - lg[top[1]] <= NEAR_TIE, f"token {i}: {a} != {b}"
            break  # after a near-tie the sequences legitimately diverge


def test_full_size_split_attention_is_consistent():
    """Qwen2.5-0.5B shape with a 1024-position context: 301 positions run
    one by one (the 1-row kernel splits each head's history over up to three
    CTAs) and through batched prefill (all but the last few positions in the
    8-row kernel, one CTA per head) give the same logits within the
    full-size tolerance, and 40 positions agree with the 64-position engine."""
    model = synthetic.build("qwen2.5-0.5b", seed=3)
    blob = layout.pack(model, "bf16")
    long = B200DecoderEngine(model, max_slots=2, max_batch=8, context=1024, blob=blob)
    try:
        ids = synthetic.prompt_ids(model.shape.vocab, 301, seed=16)
        seq = None
        for p in range(301):
            seq = long.step(ids[p], p, logits=(p == 300), slot=0)
        _, batched = long.prefill(ids, slot=1, logits=True)
        d = np.abs(seq - batched)
        rel = np.linalg.norm(seq - batched) / np.linalg.norm(batched)
        assert d.max() <= ATOL_FULL and rel <= RTOL_FULL, (d.max(), rel)
        long.reset(0)
        _, a = long.prefill(ids[:40], slot=0, logits=True)
    finally:
        long.close()
    short = B200DecoderEngine(model, max_slots=1, max_batch=8, blob=blob)
    try:
        _, b = short.prefill(ids[:40], slot=0, logits=True)
    finally:
        short.close()
    d = np.abs(a - b)
    assert d.max() <= ATOL_FULL and np.linalg.norm(a - b) / np.linalg.norm(b) <= RTOL_FULL


def test_drop_in_decoder_with_a_longer_context():
    """NPUDecoder(model, context_length=256): a 150-id prompt and 40 new
    tokens through the drop-in give the engine's own greedy tokens, and the
    repeated prompt reuses 149 cached positions."""
    from runtime.generate import NPUDecoder
    from test_decode_loop import FakeTokenizer, run

    model = synthetic.build("tiny-qwen", seed=42)
    prompt = synthetic.prompt_ids(model.shape.vocab, 150, seed=17)
    decoder = NPUDecoder(model, context_length=256)
    try:
        assert decoder._engine.context == 256
        decoder.tokenizer = FakeTokenizer(prompt)
        decoder.tokenizer.eos_id = -1
        _, stats = run(decoder, max_new_tokens=40)
        _, again = run(decoder, max_new_tokens=40)
    finally:
        decoder.close()
    engine = B200DecoderEngine(model, max_batch=8, context=256)
    try:
        ref = engine.generate(prompt, 40)
    finally:
        engine.close()
    assert stats["generated_token_ids"] == ref
    assert again["generated_token_ids"] == ref
    assert again["cached_prompt_tokens"] == len(prompt) - 1
