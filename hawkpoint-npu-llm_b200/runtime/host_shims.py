"""Minimal host-side helpers for running the decoder without the reference's
``runtime.sampling`` / ``runtime.stopping`` / ``runtime.tokenizer`` modules.

Those modules are host logic outside the engine path and are reused
unchanged when this package is overlaid on the reference
(``runtime.generate`` imports them first).  This file only keeps a
standalone install working: greedy selection, stop strings, log-softmax and
incremental UTF-8 detokenisation.  Sampled decoding needs the reference's
``Sampler``.
"""

import numpy as np


class SamplingParams:
    def __init__(self, **options):
        unknown = set(options) - {"temperature", "top_k", "top_p", "seed"}
        if unknown:
            raise ValueError(f"unknown sampling options: {sorted(unknown)}")
        temperature = options.get("temperature", 0.0)
        if temperature not in (None, 0, 0.0):
            raise ValueError(
                "sampled decoding needs the reference runtime.sampling module; "
                "this standalone build decodes greedily"
            )
        self.options = options

    @classmethod
    def from_dict(cls, values):
        if not isinstance(values, dict):
            raise ValueError("sampling must be a dict")
        return cls(**values)

    @classmethod
    def build(cls, **options):
        return cls(**options)


GREEDY = SamplingParams()


class Sampler:
    greedy = True

    def __init__(self, params, vocab_size):
        self.params = params
        self.vocab_size = vocab_size

    def select(self, logits, history):
        return int(np.argmax(logits))

    def stats(self):
        return {"mode": "greedy"}


def normalize_stop(stop):
    if stop is None:
        return []
    if isinstance(stop, str):
        stop = [stop]
    stop = [s for s in stop if s]
    if len(stop) > 4 or not all(isinstance(s, str) for s in stop):
        raise ValueError("stop must be a string or up to four strings")
    return stop


def normalize_logprobs(value):
    if value is None or value is False:
        return None
    if value is True:
        return 0
    value = int(value)
    if not 0 <= value <= 20:
        raise ValueError("logprobs must be between 0 and 20")
    return value


def log_softmax(logits):
    x = np.asarray(logits, np.float64)
    shifted = x - x.max()
    return (shifted - np.log(np.exp(shifted).sum())).astype(np.float32)


class StopMatcher:
    """Withholds text that may still grow into a stop string."""

    def __init__(self, stops):
        self.stops = list(stops)
        self.pending = ""
        self.matched = None

    def feed(self, text):
        if self.matched is not None:
            return ""
        self.pending += text
        for stop in self.stops:
            at = self.pending.find(stop)
            if at >= 0:
                self.matched = stop
                out, self.pending = self.pending[:at], ""
                return out
        keep = 0
        for stop in self.stops:
            for n in range(min(len(stop) - 1, len(self.pending)), 0, -1):
                if self.pending.endswith(stop[:n]):
                    keep = max(keep, n)
                    break
        out = self.pending[: len(self.pending) - keep]
        self.pending = self.pending[len(self.pending) - keep:]
        return out

    def flush(self):
        out, self.pending = self.pending, ""
        return out if self.matched is None else ""


class StreamDetokenizer:
    """Emits text only once its UTF-8 bytes are complete."""

    def __init__(self, tokenizer):
        self.tokenizer = tokenizer
        self.buffer = b""

    def push(self, token_id):
        self.buffer += self.tokenizer.token_bytes(int(token_id))
        try:
            text = self.buffer.decode("utf-8")
        except UnicodeDecodeError as exc:
            if exc.reason == "unexpected end of data":
                text = self.buffer[: exc.start].decode("utf-8", errors="replace")
                self.buffer = self.buffer[exc.start:]
                return text
            text = self.buffer.decode("utf-8", errors="replace")
        self.buffer = b""
        return text

    def flush(self):
        text = self.buffer.decode("utf-8", errors="replace")
        self.buffer = b""
        return text
