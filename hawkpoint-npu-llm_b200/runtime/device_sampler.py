"""On-device token selection (``hb_sample`` / ``hb_sampler_*``).

Runs the reference's ``Sampler.select`` pipeline (npu_llm/runtime/sampling.py:
416-445) on FP32 logits in device memory.  The one random number a draw
consumes stays on the host: the caller passes the request generator's next
``random()`` -- exactly what ``Generator.choice`` would have consumed -- so a
seeded request reproduces the reference's token stream.

``params`` is any object with the reference ``SamplingParams`` fields
(``temperature``, ``top_p``, ``top_k``, ``repetition_penalty``,
``presence_penalty``, ``frequency_penalty``, ``logit_bias``).  A selection
returns the token id, or ``None`` when ``top_p`` keeps more candidates than
the device sorts on chip (4096); the caller then selects on the host.
"""

import ctypes

import numpy as np

from runtime import hb_lib


def draws_uniform(params, vocab):
    """Whether the reference's selection consumes one ``random()`` for these
    parameters (it draws unless the parameters are greedy or temperature is 0)."""
    neutral = (params.repetition_penalty == 1.0 and params.presence_penalty == 0.0
               and params.frequency_penalty == 0.0)
    in_vocab_bias = any(0 <= int(t) < vocab for t in (params.logit_bias or {}))
    greedy = neutral and (params.temperature == 0.0 or params.top_k == 1) and not in_vocab_bias
    return not greedy and params.temperature != 0.0


class SamplingArgs:
    """The ``hb_sampling`` struct for one selection, with the arrays it points
    to kept alive: history reduced to its unique in-vocabulary tokens and
    their counts (np.unique, as sampling.py:346-353 does), logit bias to its
    in-vocabulary entries."""

    def __init__(self, params, history, vocab, uniform):
        hist = np.asarray(list(history) if history is not None else [], np.int64)
        if hist.size:
            tokens, counts = np.unique(hist, return_counts=True)
            keep = (tokens >= 0) & (tokens < vocab)
            tokens, counts = tokens[keep], counts[keep]
        else:
            tokens, counts = np.zeros(0, np.int64), np.zeros(0, np.int64)
        self.h_tok = np.ascontiguousarray(tokens, np.int32)
        self.h_cnt = np.ascontiguousarray(counts, np.float32)
        bias = {int(t): float(v) for t, v in (params.logit_bias or {}).items() if 0 <= int(t) < vocab}
        self.b_tok = np.ascontiguousarray(list(bias.keys()), np.int32)
        self.b_val = np.ascontiguousarray(list(bias.values()), np.float32)
        ip = ctypes.POINTER(ctypes.c_int32)
        fp = ctypes.POINTER(ctypes.c_float)
        self.struct = hb_lib.HbSampling(
            temperature=params.temperature, top_p=params.top_p,
            repetition_penalty=params.repetition_penalty, presence_penalty=params.presence_penalty,
            frequency_penalty=params.frequency_penalty, top_k=int(params.top_k),
            n_history=self.h_tok.size, history_tokens=self.h_tok.ctypes.data_as(ip),
            history_counts=self.h_cnt.ctypes.data_as(fp), n_bias=self.b_tok.size,
            bias_tokens=self.b_tok.ctypes.data_as(ip), bias_values=self.b_val.ctypes.data_as(fp),
            uniform=0.0 if uniform is None else float(uniform))


def _result(rc, token, engine=None):
    if rc == hb_lib.HB_ERR_UNSUPPORTED:
        return None
    hb_lib.check(rc, engine)
    return int(token.value)


class DeviceSampler:
    """A standalone device sampler for ``vocab``-wide host logits."""

    def __init__(self, vocab, device=0):
        self._lib = hb_lib.load()
        self.vocab = int(vocab)
        handle = ctypes.c_void_p()
        hb_lib.check(self._lib.hb_sampler_create(self.vocab, int(device), ctypes.byref(handle)))
        self._handle = handle

    def select(self, logits, history, params, uniform):
        logits = np.ascontiguousarray(logits, np.float32)
        if logits.shape != (self.vocab,):
            raise ValueError(f"logits must have shape ({self.vocab},)")
        args = SamplingArgs(params, history, self.vocab, uniform)
        token = ctypes.c_int32()
        rc = self._lib.hb_sampler_select(self._handle, logits.ctypes.data, 0, ctypes.byref(args.struct),
                                         ctypes.byref(token))
        return _result(rc, token)

    def logprobs(self, logits, token, n_top):
        """(log-probability of ``token``, top ids, top log-probabilities) of
        the reference's float64 log_softmax of ``logits``."""
        logits = np.ascontiguousarray(logits, np.float32)
        if logits.shape != (self.vocab,):
            raise ValueError(f"logits must have shape ({self.vocab},)")
        return _logprobs_call(self._lib.hb_sampler_logprobs, (self._handle, logits.ctypes.data, 0), token, n_top)

    def close(self):
        if self._handle:
            self._lib.hb_sampler_destroy(self._handle)
            self._handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _logprobs_call(fn, lead, token, n_top, engine=None):
    tok_lp = ctypes.c_double()
    ids = np.zeros(max(1, int(n_top)), np.int32)
    vals = np.zeros(max(1, int(n_top)), np.float64)
    dp = ctypes.POINTER(ctypes.c_double)
    rc = fn(*lead, int(token), int(n_top), ctypes.byref(tok_lp), ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            vals.ctypes.data_as(dp))
    hb_lib.check(rc, engine)
    return float(tok_lp.value), ids[:n_top].tolist(), vals[:n_top].tolist()


def engine_logprobs(lib, handle, row, token, n_top):
    """Log-probabilities from row ``row`` of an engine's device logits."""
    return _logprobs_call(lib.hb_logprobs, (handle, int(row)), token, n_top, handle)


def sample_engine_row(lib, handle, vocab, row, params, history, uniform):
    """Select from row ``row`` of the logits an engine step left on the device
    (``HB_STEP_DEVICE_LOGITS``); None when the host must select instead."""
    args = SamplingArgs(params, history, vocab, uniform)
    token = ctypes.c_int32()
    rc = lib.hb_sample(handle, int(row), ctypes.byref(args.struct), ctypes.byref(token))
    return _result(rc, token, handle)


def sample_engine_rows(lib, handle, vocab, rows, params, histories, uniforms):
    """Several selections from a batched step's device logits in one launch."""
    n = len(rows)
    args = [SamplingArgs(p, h, vocab, u) for p, h, u in zip(params, histories, uniforms)]
    structs = (hb_lib.HbSampling * n)(*[a.struct for a in args])
    rows_arr = np.ascontiguousarray(rows, np.int32)
    out = np.empty(n, np.int32)
    ip = ctypes.POINTER(ctypes.c_int32)
    rc = lib.hb_sample_batch(handle, n, rows_arr.ctypes.data_as(ip), structs, out.ctypes.data_as(ip))
    hb_lib.check(rc, handle)
    return [None if t < 0 else int(t) for t in out]
