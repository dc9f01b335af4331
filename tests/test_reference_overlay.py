"""The reference's own callers, unchanged, on this build's runtime (the
INTEGRATION overlay, made in a temporary directory; tests/overlay_kit.py):

* ``scripts/benchmark_native.py`` (:23-123) runs end to end and writes its
  report with ``decoder_engine`` true;
* ``api_server.CompletionEngine`` with the reference's ``NPUDecoderFactory``
  (:535-678, :929-942) loads, warms, serves chat and text requests and
  closes the drop-in ``NPUDecoder``;
* ``api_server.make_handler`` over this build's ``BatchingCompletionEngine``
  serves 12 concurrent OpenAI requests (6 text, 6 chat completions) with
  several streams sharing each batched step, and every answer equals the
  one the serialised CompletionEngine gives for the same prompt.

The engine underneath is the CPU oracle with the B200 engine's Python
surface (no GPU here); the GPU engine's parity with that oracle is covered
by the GPU tests.  Skipped when the reference tree is not present."""

import json
from pathlib import Path
import subprocess
import sys

import pytest

import overlay_kit

pytestmark = pytest.mark.skipif(not overlay_kit.reference_present(), reason="reference tree not present")

BOOT = Path(__file__).resolve().parent / "overlay_boot.py"


@pytest.fixture(scope="module")
def overlay(tmp_path_factory):
    root = tmp_path_factory.mktemp("overlay")
    ov = overlay_kit.build_overlay(root / "ov")
    pkg = overlay_kit.write_tiny_package(root / "pkg")
    return ov, pkg


def boot(overlay, mode):
    ov, pkg = overlay
    run = subprocess.run([sys.executable, str(BOOT), str(ov), str(pkg), mode], capture_output=True, text=True,
                         timeout=600)
    assert run.returncode == 0, run.stderr[-3000:]
    out = run.stdout
    return json.loads(out[out.index("{"):])


def test_benchmark_native_runs_unchanged(overlay):
    report = boot(overlay, "benchmark")
    assert report["configuration"]["decoder_engine"] is True
    assert report["tokens"] == 8 and len(report["runs"]) == 2
    assert report["median_decode_tokens_per_second"] > 0
    for run in report["runs"]:
        stats = run["stats"]
        assert 1 <= stats["generated_tokens"] <= 8
        assert stats["npu_layers"] == 2 and stats["cpu_layers"] == 0
        assert stats["cached_prompt_tokens"] == 0  # --prefix-cache not given: every run prefills


def test_completion_engine_serves_the_drop_in(overlay):
    result = boot(overlay, "completion")
    assert result["engines_closed"]
    for chat in result["chat"]:
        assert len(chat["ids"]) == 8 and chat["finish"] == "length"
    for text in result["text"]:
        assert 1 <= len(text["ids"]) <= 6


def test_openai_server_batches_concurrent_requests(overlay):
    result = boot(overlay, "http")
    expected = result["expected"] + result["expected_chat"]
    assert len(result["answers"]) == len(expected) == 12
    for want, got in zip(expected, result["answers"]):
        choice = got["choices"][0]
        text = choice["text"] if "text" in choice else choice["message"]["content"]
        assert text == want["text"]
        assert choice["finish_reason"] == want["finish"]
    assert len({e["text"] for e in result["expected"]}) > 1  # the prompts really answer differently
    assert result["max_rows_per_step"] > 8  # several streams' rows in one step
    assert [m["id"] for m in result["models"]["data"]] == ["tiny"]
