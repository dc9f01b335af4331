"""Runs one of the reference's own entry points, unchanged, inside an overlay
(tests/overlay_kit.py) with the GPU engine replaced by the CPU oracle
engine.  Used by tests/test_reference_overlay.py as a subprocess:

    python tests/overlay_boot.py OVERLAY PACKAGE MODE

MODE ``benchmark`` runs scripts/benchmark_native.py (its JSON report goes
to stdout); ``completion`` drives api_server.CompletionEngine with the
reference's NPUDecoderFactory; ``http`` serves concurrent chat requests
through api_server.make_handler over this build's BatchingCompletionEngine
and, for comparison, the same prompts through CompletionEngine.  The last
two print one JSON object."""

import json
import os
from pathlib import Path
import runpy
import sys
import threading
import urllib.request

OVERLAY, PACKAGE, MODE = Path(sys.argv[1]), sys.argv[2], sys.argv[3]
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(OVERLAY / "npu_llm"))
os.environ["HAWKPOINT_DEVICE_SAMPLING"] = "0"

import overlay_kit  # noqa: E402
import runtime.b200_engine  # noqa: E402  (the overlay's runtime: this build's modules)

runtime.b200_engine.B200DecoderEngine = overlay_kit.OracleEngine

PROMPTS = [
    "Explain why the sky appears blue during the day.",
    "hello how are you today",
    "numbers 0 1 2 3",
    "the weather and light colour",
    "a small model answers questions",
    "thank you",
]


def completion_engine():
    import api_server

    return api_server, api_server.CompletionEngine(
        {"tiny": {"path": PACKAGE, "context_length": 64}}, decoder_factory=api_server.NPUDecoderFactory())


def collect(chunks):
    text, stats = [], None
    for piece, final, *_ in chunks:
        text.append(piece)
        if final is not None:
            stats = final
    return "".join(text), stats


def sequential(engine, max_tokens, chat):
    """Each prompt in turn: as a chat message list, or as raw text (whose
    last token differs between prompts, so random-weight models answer
    each one differently)."""
    out = []
    for prompt in PROMPTS:
        request = [{"role": "user", "content": prompt}] if chat else prompt
        text, stats = collect(engine.generate("tiny", request, max_tokens))
        out.append({"text": text, "ids": stats["generated_token_ids"], "finish": stats["finish_reason"]})
    return out


if MODE == "benchmark":
    script = OVERLAY / "scripts" / "benchmark_native.py"
    sys.argv = [str(script), PACKAGE, "--tokens", "8", "--runs", "2", "--warmup-runs", "1"]
    runpy.run_path(str(script), run_name="__main__")
elif MODE == "completion":
    api_server, engine = completion_engine()
    engine.prewarm_default()
    results = sequential(engine, 8, chat=True)
    texts = sequential(engine, 6, chat=False)
    engine.close()
    print(json.dumps({"chat": results, "text": texts,
                      "engines_closed": all(e.closed for e in overlay_kit.OracleEngine.instances)}))
elif MODE == "http":
    from http.server import ThreadingHTTPServer

    from runtime.batch_server import BatchingCompletionEngine

    api_server, reference_engine = completion_engine()
    expected = sequential(reference_engine, 8, chat=False)
    expected_chat = sequential(reference_engine, 8, chat=True)
    reference_engine.close()

    def oracle_factory(model, max_slots, weights):
        return overlay_kit.OracleEngine(model, weights=weights, max_slots=max_slots)

    engine = BatchingCompletionEngine({"tiny": {"path": PACKAGE, "context_length": 64}},
                                      engine_factory=oracle_factory, max_batch=8, prefill_chunk=8, max_rows=32)
    config = api_server.ServerConfig(api_key="k", queue_capacity=2 * len(PROMPTS), rate_limit_per_minute=10_000)
    httpd = ThreadingHTTPServer(("127.0.0.1", 0), api_server.make_handler(engine, config))
    threading.Thread(target=httpd.serve_forever, daemon=True).start()
    base = f"http://127.0.0.1:{httpd.server_address[1]}/v1"
    answers = [None] * (2 * len(PROMPTS))
    start = threading.Barrier(len(answers))

    def ask(i):
        prompt = PROMPTS[i % len(PROMPTS)]
        if i < len(PROMPTS):   # text completions, then chat completions, all at once
            url, payload = base + "/completions", {"prompt": prompt}
        else:
            url, payload = base + "/chat/completions", {"messages": [{"role": "user", "content": prompt}]}
        body = json.dumps(dict(payload, model="tiny", max_tokens=8)).encode()
        request = urllib.request.Request(url, data=body, headers={"Authorization": "Bearer k",
                                                                  "Content-Type": "application/json"})
        start.wait()
        with urllib.request.urlopen(request, timeout=120) as response:
            answers[i] = json.loads(response.read())

    threads = [threading.Thread(target=ask, args=(i,)) for i in range(len(answers))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    models = json.loads(urllib.request.urlopen(urllib.request.Request(
        f"http://127.0.0.1:{httpd.server_address[1]}/v1/models", headers={"Authorization": "Bearer k"})).read())
    httpd.shutdown()
    batched = [e for e in overlay_kit.OracleEngine.instances if e.row_steps]
    engine.close()
    print(json.dumps({"expected": expected, "expected_chat": expected_chat, "answers": answers, "models": models,
                      "max_rows_per_step": max(batched[0].row_steps) if batched else 0,
                      "row_steps": len(batched[0].row_steps) if batched else 0}))
else:
    raise SystemExit(f"unknown mode {MODE}")
