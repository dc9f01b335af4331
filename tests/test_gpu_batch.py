"""The batched tensor-core step (hb_step_rows / hb_prefill_tc) on the GPU.

Its tcgen05 GEMMs sum in a different order than the persistent kernel, so it
is held to the oracle's tolerance (tests/test_gpu_engine.py), not to bit
equality: logits within max-abs / relative bounds, argmax equal except at
BF16 near-ties, K/V cache BF16 values equal except for a small fraction of
small differences.  Rows of one sequence in the same step (chunked
prefill) see each other's keys; rows of different sequences are independent.
"""

import numpy as np
import pytest
from ml_dtypes import bfloat16

from oracle.cpu_decoder import OracleDecoder
from runtime import hb_lib, synthetic
from runtime.b200_engine import B200DecoderEngine
from test_gpu_engine import ATOL_FULL, RTOL_FULL, assert_logits_close

pytestmark = pytest.mark.gpu


def cache_close(a, b, where=""):
    """K/V cache rows from two paths that sum their projections in
    different orders: at most 2 % of the BF16 values differ, none by more
    than 1/16 of the tensor's RMS (a one-unit projection difference grows
    under RoPE's cancellation when a rotated value is small)."""
    va = np.asarray(a).view(np.uint16).view(bfloat16).astype(np.float32)
    vb = np.asarray(b).view(np.uint16).view(bfloat16).astype(np.float32)
    d = np.abs(va - vb)
    rms = float(np.sqrt(np.mean(vb * vb)))
    assert np.mean(d > 0) <= 0.02, f"{where}: {np.mean(d > 0):.4f} of values differ"
    assert d.max() <= rms / 16, f"{where}: max difference {d.max():.3e} (rms {rms:.3e})"


@pytest.fixture(scope="module", params=["tiny-qwen", "tiny-llama"])
def tiny(request):
    model = synthetic.build(request.param, seed=31)
    engine = B200DecoderEngine(model, max_slots=12, max_batch=8)
    yield model, engine
    engine.close()


def test_prefill_tc_matches_oracle_and_sequential_cache(tiny):
    model, engine = tiny
    ids = synthetic.prompt_ids(model.shape.vocab, 23, seed=4)
    oracle = OracleDecoder(model)
    ref = None
    for p, t in enumerate(ids):
        ref = oracle.step(t, p)
    engine.reset()
    am, logits = engine.prefill_tc(ids, slot=1, logits=True)
    assert_logits_close(logits, ref, "prefill_tc last position")
    assert am == int(np.argmax(logits))
    # the same positions one launch each on the persistent kernel
    for p, t in enumerate(ids):
        engine.step(t, p, logits=False, slot=0)
    n = len(ids)
    cache_close(engine.kv_cache(1)[:, :, :, :n], engine.kv_cache(0)[:, :, :, :n], "prefill cache")


def test_prefill_tc_in_one_pass_equals_row_by_row(tiny):
    """A row's arithmetic does not depend on the other rows of its step:
    prefilling 20 positions in one batched pass leaves the same K/V bits and
    the same last-position logits as 20 one-row batched steps."""
    model, engine = tiny
    engine.reset()
    ids = synthetic.prompt_ids(model.shape.vocab, 20, seed=11)
    first, one_pass = engine.prefill_tc(ids, slot=2, logits=True)
    for p, t in enumerate(ids):
        am, last = engine.step_rows([3], [t], [p], logits=p == len(ids) - 1)
    assert np.array_equal(one_pass, last[0])
    assert first == int(am[0])
    n = len(ids)
    assert np.array_equal(engine.kv_cache(2)[:, :, :, :n], engine.kv_cache(3)[:, :, :, :n])


def test_step_above_128_rows_equals_each_sequence_alone(tiny):
    """156 rows in one step (13 prompt positions of each of 12 slots), the
    LM head on each slot's last row: every slot's logits equal the same
    positions prefilled alone (rows are independent of their step)."""
    model, engine = tiny
    engine.reset()
    prompts = [synthetic.prompt_ids(model.shape.vocab, 13, seed=70 + k) for k in range(12)]
    slots = [k for k in range(12) for _ in range(13)]
    tokens = [t for p in prompts for t in p]
    positions = list(range(13)) * 12
    out_rows = [13 * k + 12 for k in range(12)]
    am, logits = engine.step_rows(slots, tokens, positions, logits=True, out_rows=out_rows)
    assert logits.shape == (12, model.shape.vocab)
    for k, p in enumerate(prompts):
        engine.reset(k)
        first, alone = engine.prefill_tc(p, slot=k, logits=True)
        assert np.array_equal(logits[k], alone), k
        assert int(am[k]) == first


def test_step_rows_across_streams_matches_single_rows(tiny):
    """Six sequences at different depths in one step: each row equals that
    sequence's own single-row step (tolerance), its cache row too."""
    model, engine = tiny
    engine.reset()
    lens = [3, 9, 14, 20, 27, 40]
    prompts = [synthetic.prompt_ids(model.shape.vocab, n + 1, seed=50 + n) for n in lens]
    for k, pr in enumerate(prompts):
        engine.prefill(pr[:-1], slot=k)
        engine.copy_prefix(k, 6 + k, len(pr) - 1)
    am, logits = engine.step_rows(list(range(6)), [pr[-1] for pr in prompts], [len(pr) - 1 for pr in prompts],
                                  logits=True)
    for k, pr in enumerate(prompts):
        single = engine.step(pr[-1], len(pr) - 1, logits=True, slot=6 + k)
        assert_logits_close(logits[k], single, f"stream {k}")
        assert int(am[k]) == int(np.argmax(logits[k]))
        p = len(pr) - 1
        cache_close(engine.kv_cache(k)[:, :, :, p], engine.kv_cache(6 + k)[:, :, :, p], f"stream {k}")


def test_chunked_prefill_rows_with_decode_rows(tiny):
    """Five consecutive positions of one sequence and one decode row of
    another in the same step, against the oracle."""
    model, engine = tiny
    engine.reset()
    a = synthetic.prompt_ids(model.shape.vocab, 10, seed=7)
    b = synthetic.prompt_ids(model.shape.vocab, 13, seed=8)
    engine.prefill(a[:5], slot=0)
    engine.prefill(b[:12], slot=1)
    slots = [0, 0, 0, 0, 0, 1]
    tokens = a[5:10] + [b[12]]
    positions = [5, 6, 7, 8, 9, 12]
    _, logits = engine.step_rows(slots, tokens, positions, logits=True)
    oa = OracleDecoder(model)
    ref_a = [oa.step(t, p) for p, t in enumerate(a)]
    ob = OracleDecoder(model)
    ref_b = [ob.step(t, p) for p, t in enumerate(b)]
    for i in range(5):
        assert_logits_close(logits[i], ref_a[5 + i], f"chunk row {i}")
    assert_logits_close(logits[5], ref_b[12], "decode row")


def test_output_rows_select_the_lm_head_rows(tiny):
    """A chunk of five positions of one sequence plus a decode row of
    another, the LM head on the last row of each only: those two outputs
    equal the same rows of an all-rows step (tolerance: the LM head's K split
    follows the output count)."""
    model, engine = tiny
    engine.reset()
    a = synthetic.prompt_ids(model.shape.vocab, 9, seed=17)
    b = synthetic.prompt_ids(model.shape.vocab, 6, seed=18)
    engine.prefill(b[:5], slot=3)
    slots = [2] * 8 + [3]
    tokens = a[:8] + [b[5]]
    positions = list(range(8)) + [5]
    am_all, all_rows = engine.step_rows(slots, tokens, positions, logits=True)
    am_sel, sel = engine.step_rows(slots, tokens, positions, logits=True, out_rows=[7, 8])
    assert sel.shape == (2, model.shape.vocab)
    for j, r in enumerate([7, 8]):
        assert_logits_close(sel[j], all_rows[r], f"output row {r}")
        assert int(am_sel[j]) == int(np.argmax(sel[j]))
    am_only, none = engine.step_rows(slots, tokens, positions, out_rows=[8])
    assert none is None and am_only.shape == (1,)
    with pytest.raises(ValueError):
        engine.step_rows(slots, tokens, positions, out_rows=[9])


def test_step_rows_rejects_bad_rows(tiny):
    model, engine = tiny
    with pytest.raises(ValueError):
        engine.step_rows([0, 0], [1, 2], [3, 3])           # same slot position twice
    with pytest.raises(ValueError):
        engine.step_rows(list(range(257)), [1] * 257, [0] * 257)
    with pytest.raises(ValueError):
        engine.step_rows([0], [model.shape.vocab], [0])     # token outside the vocabulary


def test_batched_path_needs_bf16_weights():
    model = synthetic.build("tiny-qwen", seed=3)
    engine = B200DecoderEngine(model, weights="w8")
    try:
        with pytest.raises(hb_lib.HbError):
            engine.step_rows([0], [1], [0])
    finally:
        engine.close()


def test_full_size_prefill_tc_against_reference(golden):
    """The config-3 prompt (32 positions) in one batched pass: the last
    position's logits against the reference CPU stage, then greedy decode on
    the persistent kernel from the cache the batched pass left."""
    g = golden("request_qwen2.5-0.5b_bf16.npz")
    model = synthetic.build("qwen2.5-0.5b", seed=0).materialize()
    engine = B200DecoderEngine(model, max_batch=8)
    try:
        prompt = [int(t) for t in g["prompt"]]
        n = len(prompt)
        first, logits = engine.prefill_tc(prompt, logits=True)
        stride = int(g["sample_stride"])
        p = n - 1
        err = max(float(np.abs(logits[g["top_ids"][p]] - g["top_logits"][p]).max()),
                  float(np.abs(logits[::stride] - g["sample_logits"][p]).max()))
        rel = float(np.linalg.norm(logits[::stride] - g["sample_logits"][p]) / np.linalg.norm(g["sample_logits"][p]))
        assert err <= ATOL_FULL and rel <= RTOL_FULL, (err, rel)
        tokens = [first]
        for k in range(1, 8):
            tokens.append(engine.step_argmax(tokens[-1], n + k - 1))
        ref = [int(t) for t in g["generated"][:8]]
        margins = g["margin"][n - 1:]
        for k, (a, b) in enumerate(zip(tokens, ref)):
            if a != b:
                assert margins[k] <= 2 * ATOL_FULL, f"token {k}: {a} vs {b}"
                break
        print(f"prefill_tc qwen: last-position max-abs {err:.4f}, rel {rel:.4e}; tokens {tokens}")
    finally:
        engine.close()
