"""Test infrastructure for running the reference's own callers on this
build's runtime (no GPU): the INTEGRATION overlay, a tiny model package
with a trained chat tokenizer, and an engine with the B200 engine's Python
surface that computes every position with the CPU oracle.

The overlay is made at test time, as INTEGRATION.md describes: a directory
whose ``npu_llm/`` links every entry of the reference's ``npu_llm/`` except
``runtime/``, which links this build's runtime modules plus the
reference's host-only ``sampling``, ``stopping`` and ``tokenizer``; the
reference's ``scripts/benchmark_native.py`` is copied next to it (it finds
``npu_llm/`` from its own resolved path).  Nothing of the reference is
committed."""

import json
import os
from pathlib import Path
import shutil

import numpy as np

REPO = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("HAWKPOINT_REFERENCE", "/root/reference"))
RUNTIME = REPO / "hawkpoint-npu-llm_b200" / "runtime"
HOST_MODULES = ("sampling", "stopping", "tokenizer")


def reference_present():
    return (REFERENCE / "npu_llm" / "api_server.py").exists() and (REFERENCE / "scripts").is_dir()


def build_overlay(root):
    root = Path(root)
    pkg = root / "npu_llm"
    pkg.mkdir(parents=True)
    for entry in (REFERENCE / "npu_llm").iterdir():
        if entry.name != "runtime":
            (pkg / entry.name).symlink_to(entry)
    rt = pkg / "runtime"
    rt.mkdir()
    for module in RUNTIME.glob("*.py"):
        (rt / module.name).symlink_to(module)
    for name in HOST_MODULES:
        target = rt / f"{name}.py"
        if target.exists():
            target.unlink()
        target.symlink_to(REFERENCE / "npu_llm" / "runtime" / f"{name}.py")
    (root / "scripts").mkdir()
    shutil.copy(REFERENCE / "scripts" / "benchmark_native.py", root / "scripts" / "benchmark_native.py")
    return root


CORPUS = [
    "the sky is blue because air scatters short wavelengths more than long ones",
    "a small model answers questions about light colour and the weather",
    "system user assistant hello how are you today thank you",
    "Explain why the sky appears blue during the day.",
    "numbers 0 1 2 3 4 5 6 7 8 9 and punctuation , . ! ?",
] * 30


def write_tokenizer(directory, vocab_size=300):
    """A byte-level BPE with the ChatML markers (trained here; the reference
    chat tokenizer reads tokenizer.json + tokenizer_config.json)."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=["<|im_start|>", "<|im_end|>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(CORPUS, trainer)
    tok.save(str(Path(directory) / "tokenizer.json"))
    (Path(directory) / "tokenizer_config.json").write_text(json.dumps({"eos_token": "<|im_end|>"}))


def write_tiny_package(directory, name="tiny-qwen", seed=7):
    """A synthetic package (random weights) plus a chat tokenizer whose ids
    all fall inside the model's vocabulary."""
    import sys

    sys.path.insert(0, str(RUNTIME.parent))
    from runtime import synthetic
    from runtime.model import write_package

    model = synthetic.build(name, seed=seed)
    write_package(model, directory)
    write_tokenizer(directory)
    return Path(directory)


class OracleEngine:
    """The B200 engine's Python surface (``step``, ``step_argmax``,
    ``prefill``, ``generate``, ``step_rows``, ``copy_prefix``, ``reset``,
    ``close``) over one CPU oracle decoder per KV slot: every position is
    computed by the oracle, so results equal the reference CPU stage's."""

    instances = []

    def __init__(self, model, weights="bf16", device=0, max_slots=8, max_batch=8, context=64, **_):
        import sys

        sys.path.insert(0, str(REPO))
        from oracle.cpu_decoder import OracleDecoder

        self.model = model
        self.max_slots = int(max_slots)
        self.context = int(context)
        self.vocab = int(model.metadata["vocab_size"])
        self.slots = [OracleDecoder(model, context_length=self.context, weights=weights) for _ in range(self.max_slots)]
        self.row_steps = []   # rows per step_rows call
        self.closed = False
        OracleEngine.instances.append(self)

    def step(self, token_id, position, logits=True, slot=0):
        out = self.slots[slot].step(int(token_id), int(position), compute_logits=True)
        return np.asarray(out, np.float32) if logits else None

    def step_argmax(self, token_id, position, slot=0):
        return int(np.argmax(self.step(token_id, position, slot=slot)))

    def prefill(self, ids, start=0, slot=0, logits=False):
        last = None
        for k, t in enumerate(ids):
            last = self.step(t, start + k, slot=slot)
        return int(np.argmax(last)), (last if logits else None)

    def generate(self, prompt_ids, n_new, start=0, slot=0):
        token, _ = self.prefill(list(prompt_ids)[start:], start=start, slot=slot)
        out, pos = [token], len(prompt_ids)
        while len(out) < n_new and pos < self.context:
            out.append(self.step_argmax(out[-1], pos, slot=slot))
            pos += 1
        return out

    def step_rows(self, slots, tokens, positions, logits=False, out_rows=None):
        self.row_steps.append(len(slots))
        results = [self.step(t, p, slot=s) for s, t, p in zip(slots, tokens, positions)]
        rows = range(len(slots)) if out_rows is None else out_rows
        picked = np.stack([results[i] for i in rows])
        return np.argmax(picked, axis=1).astype(np.int32), (picked if logits else None)

    def copy_prefix(self, src, dst, n_positions):
        a, b = self.slots[src], self.slots[dst]
        for cache_a, cache_b in zip(a.keys + a.values, b.keys + b.values):
            cache_b[:, :n_positions] = cache_a[:, :n_positions]

    def reset(self, slot=None):
        for s in (range(self.max_slots) if slot is None else [slot]):
            self.slots[s].reset()

    def close(self):
        self.closed = True
