#!/usr/bin/env python3
"""Benchmark of the B200 decoder engine on the Qwen2.5-0.5B decode workload (config 3, the metric's):

    Qwen2.5-0.5B-shaped BF16 decoder, random-init N(0, 0.02) weights (seed 0),
    a 40-id seeded prompt windowed to the 32 positions that leave room for 32
    generated tokens in the 64-token context (the reference's prompt budget,
    npu_llm/runtime/generate.py:1021-1023), sequential prefill, then greedy
    decode of 32 tokens, batch 1.

One step = one such request.  Reported (one JSON line from rank 0):

* ``value``: decode tokens/s with every input resident in HBM -- the whole
  request runs as back-to-back kernel launches with the greedy token fed back
  on the device (hb_generate); the decode time is measured with CUDA events
  around each launch on the engine's stream (31 decode steps per request, the
  reference's decode_steps / decode_seconds).
* ``e2e``: the same metric through the public ``NPUDecoder.decode_token`` API
  (one call per position, host<->device copies and a sync per call).
* ``roofline``: the decode kernel's algorithmic bytes per launch (the BF16
  weights every token must stream, plus the KV history) / its mean launch
  time, against the measured HBM peak.
* ``cpu_baseline``: the CPU oracle (a NumPy port of the reference's BF16 CPU
  runtime) on a bounded sample of the same request.

``--impl reference`` times the reference path itself -- the CPU runtime
(port), the only implementation of this engine that runs off the NPU -- on
this host's cores.  Multi-GPU (torchrun): every rank runs the same requests on
its own GPU (independent replicas, weak scaling); the time is the max over
ranks.  The synthetic weights are larger than L2 (1 GB per token), so no L2
flush is needed between steps.
"""

import argparse
import contextlib
import json
import os
from pathlib import Path
import statistics
import subprocess
import sys
import time

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "hawkpoint-npu-llm_b200"))
sys.path.insert(0, str(REPO))

PROMPT_SEED = 1
MODEL_SEED = 0
PROMPT_DRAWN = 40
NEW_TOKENS = 32
METRIC = "decode_tokens_per_second"
# Algorithmic bytes per decoded token: BF16 weights of every layer
# (715,653,120) + LM head (272,269,312) + norm weights (87,808) + FP32 qkv
# bias (110,592); plus 24 layers x 512 bytes of K/V history per position.
WEIGHT_BYTES = 988_120_832
KV_BYTES_PER_POSITION = 24 * 512


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the config 1/2/4/5 measurements (profiling runs of config 3 only)")
    p.add_argument("--profile-rows", type=int, default=0, metavar="N",
                   help="profiling entry: run the N-row batched tensor-core step --warmup + --steps times "
                        "and print its mean time (no metric line)")
    p.add_argument("--workload", choices=["config3", "config5"], default="config3",
                   help="config5: the metric line is config 5's aggregate tokens/s (512 ragged requests split "
                        "over the ranks, batched tensor-core step), one step = one pass over every request")
    p.add_argument("--profile-gemv", action="store_true",
                   help="profiling entry: config 2 (standalone GEMV shapes) only, one JSON line per shape")
    return p.parse_args()


LOCAL_DEVICE = [0]  # this rank's GPU (collectives name it explicitly)


def dist_setup(n):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    LOCAL_DEVICE[0] = local
    # the drop-in NPUDecoder (e2e leg) opens its engine on HAWKPOINT_DEVICE
    os.environ["HAWKPOINT_DEVICE"] = str(local)
    if world > 1:
        from datetime import timedelta
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        kwargs = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kwargs["device_id"] = torch.device("cuda", local)  # one communicator, bound to this GPU
        # short timeout: a rank that stops answering ends the others' next collective
        dist.init_process_group(backend, timeout=timedelta(seconds=60), **kwargs)
    return rank, world, local


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", LOCAL_DEVICE[0]) if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", LOCAL_DEVICE[0]) if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_over_ranks(value, world):
    """Every rank's value, in rank order."""
    if world == 1:
        return [value]
    import torch
    import torch.distributed as dist
    dev = torch.device("cuda", LOCAL_DEVICE[0]) if dist.get_backend() == "nccl" else "cpu"
    out = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(world)]
    dist.all_gather(out, torch.tensor([value], dtype=torch.float64, device=dev))
    return [float(t.item()) for t in out]


def config5_requests(vocab, n=512, new_tokens=16, seed=MODEL_SEED + 5):
    """Config 5: 8 x 64 independent requests, prompt lengths U[8, 48],
    every fourth request opening with one shared 16-token prefix, 16 greedy
    tokens each (seeded ids stand in for real prompts)."""
    from runtime import synthetic
    from runtime.serving import Request

    return [Request(prompt=ids, new_tokens=new_tokens, rid=i)
            for i, ids in enumerate(synthetic.ragged_prompts(vocab, n, seed))]


MULTISTREAM_MODES = {
    # the batched tensor-core step: 3 lanes (engines on their own streams,
    # their steps overlapping on the GPU), each 128 streams, prompts in
    # chunks of 32 positions, up to 256 rows a step
    "rows": {"max_slots": 132, "lanes": 3, "server": {"max_batch": 128, "prefill_chunk": 32, "max_rows": 256}},
    # the persistent decoder kernel: 8 streams a launch, one position each
    "persistent": {"max_slots": 12, "server": {"max_batch": 8}},
}


def run_multistream(model, blob, device, rank, world, mode="rows", passes=1, warmup=1, clocks=None):
    """Config 5 on this rank's shard (requests split over ranks, no
    collective on the token path): continuous batching, shared prefixes
    reused from the KV prefix pool.  ``warmup`` untimed passes over the same
    requests capture every launch sequence the ``passes`` timed passes
    replay (each pass a fresh server: prefixes are recomputed every pass)."""
    import numpy as np
    import torch
    from runtime import dispatch
    from runtime.b200_engine import B200DecoderEngine
    from runtime.serving import MultiStreamServer, Request, run_lanes

    spec = MULTISTREAM_MODES[mode]
    lanes = spec.get("lanes", 1)
    everything = config5_requests(model.shape.vocab)
    mine = dispatch.shard([r.prompt for r in everything], rank, world, 16)
    engines, streams = [], []
    for _ in range(lanes):
        engine = B200DecoderEngine(model, device=device, blob=blob, max_slots=spec["max_slots"], max_batch=8)
        streams.append(torch.cuda.Stream(device=device))
        engine.set_stream(streams[-1].cuda_stream)
        engines.append(engine)

    def requests():
        return [Request(prompt=everything[i].prompt, new_tokens=everything[i].new_tokens, rid=i) for i in mine]

    def one_pass():
        servers = [MultiStreamServer(engine, **spec["server"]) for engine in engines]
        reqs = requests()
        if lanes == 1:
            servers[0].run(reqs)
        else:
            run_lanes(servers, reqs)
        return reqs, servers

    try:
        for _ in range(max(1, warmup)):
            one_pass()
        torch.cuda.synchronize()
        barrier(world)
        launches_total = 0
        sampler = clocks if clocks is not None else contextlib.nullcontext()
        with sampler:
            t0 = time.perf_counter()
            for _ in range(passes):
                reqs, servers = one_pass()
                launches_total += sum(s.launches for s in servers)
            torch.cuda.synchronize()
            wall = time.perf_counter() - t0
        barrier(world)
    finally:
        for engine in engines:
            engine.close()
    tokens = passes * sum(len(r.tokens) for r in reqs)
    all_tokens = sum_over_ranks(float(tokens), world)
    walls = gather_over_ranks(wall, world)
    launches = gather_over_ranks(float(sum(s.launches for s in servers)), world)
    t_max = max(walls)
    return {
        "workload": "config 5: 512 requests, prompts U[8,48], 25% share a 16-token prefix, 16 greedy tokens",
        "mode": mode, "server": spec["server"],
        "requests": len(everything), "requests_this_rank": len(reqs),
        "value": all_tokens / t_max, "unit": "tokens/s", "lanes": lanes,
        "p50_ttft_ms": 1000 * float(np.median([r.ttft for r in reqs])),
        "passes": passes, "tokens_per_pass": int(all_tokens) // passes,
        "wall_s_per_rank": walls, "launches_per_rank": [int(v) for v in launches],
        "launches_total_rank0": launches_total,
        "slowest_rank": int(np.argmax(walls)),
        "launches_rank0": sum(s.launches for s in servers), "rows_rank0": sum(s.rows for s in servers),
        "prefix_reuses_rank0": sum(1 for r in reqs if r.reused_prefix),
    }


def prefill_launches(n_prompt, batch=8):
    """Launches before the one that yields the first token: the engine
    prefills positions 0 .. n_prompt-2 in launches of up to `batch`
    consecutive positions (batch 1: one per position)."""
    return -(-(n_prompt - 1) // batch)


def run_long_context(device, peak, context=4096, n_new=16):
    """Greedy decode of the Qwen shape (BF16) with the paged cache of a
    4096-position context, at several prompt depths: per depth the median
    decode launch and its HBM bytes (the streamed weights plus the K/V
    history every layer reads at the mean decode position)."""
    import numpy as np
    from runtime import layout, synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("qwen2.5-0.5b", seed=MODEL_SEED).materialize()
    shape = model.shape
    eng = B200DecoderEngine(model, device=device, max_batch=8, context=context)
    rows = []
    try:
        ids_all = synthetic.prompt_ids(shape.vocab, context - 64, seed=MODEL_SEED + 3)
        for depth in (256, 1024, 2048, context - 64):
            ids = ids_all[:depth]
            first = eng.generate(ids, n_new)
            eng.profile(True)
            eng.profile_read()
            for _ in range(2):
                assert eng.generate(ids, n_new) == first
            n_pre = prefill_launches(depth)
            ms = eng.profile_read().reshape(2, n_pre + n_new)
            eng.profile(False)
            dec = float(np.median(ms[:, n_pre + 1:]))
            lay = layout.plan(shape, "bf16")
            streamed = lay.total - shape.vocab * shape.hidden * 2
            kv = shape.layers * shape.kv_heads * 2 * (depth + n_new // 2) * shape.head_dim * 2
            rows.append({"depth": depth, "decode_launch_ms": dec, "decode_tokens_per_second": 1000.0 / dec,
                         "kv_bytes_per_token": int(kv),
                         "hbm_frac": (streamed + kv) / (dec / 1000.0) / 1e9 / peak})
    finally:
        eng.close()
    return {"context": context, "new_tokens": n_new, "depths": rows}


def run_other_configs(device, peak):
    """Configs 1, 2 and 4 on this GPU (single-GPU runs only): decode
    of the SmolLM2-135M shape (BF16) and of the Qwen shape in W8, and the
    standalone GEMV shapes with HBM GB/s against the roofline."""
    import numpy as np
    import torch
    from runtime import layout, synthetic
    from runtime.b200_engine import B200DecoderEngine

    out = {}
    for key, name, weights, n_prompt, n_new in (("config1_smollm2_135m_bf16", "smollm2-135m", "bf16", 35, 16),
                                                 ("config4_qwen_w8", "qwen2.5-0.5b", "w8", 32, 32)):
        model = synthetic.build(name, seed=MODEL_SEED).materialize()
        eng = B200DecoderEngine(model, weights=weights, device=device, max_batch=8)  # batched prefill
        try:
            ids = synthetic.prompt_ids(model.shape.vocab, 40, seed=MODEL_SEED + 1)[:n_prompt]
            first = eng.generate(ids, n_new)
            eng.profile(True)
            eng.profile_read()
            for _ in range(3):
                assert eng.generate(ids, n_new) == first
            n_pre = prefill_launches(n_prompt)
            ms = eng.profile_read().reshape(3, n_pre + n_new)
            eng.profile(False)
            parity = golden_parity(eng, name, weights)
        finally:
            eng.close()
        lay = layout.plan(model.shape, weights)
        streamed = lay.total - model.shape.vocab * model.shape.hidden * 2  # the embedding is read one row at a time
        dec = float(np.median(ms[:, n_pre + 1:]))
        out[key] = {"decode_tokens_per_second": 1000.0 / dec, "decode_launch_ms": dec,
                    "ttft_ms": float(ms[:, :n_pre + 1].sum(axis=1).mean()),
                    "weight_bytes_per_token": int(streamed),
                    "hbm_frac": streamed / (dec / 1000.0) / 1e9 / peak, "parity": parity}
    out["long_context_qwen_bf16"] = run_long_context(device, peak)
    # config 2: y = W x (BF16 out) and the LM head with a fused argmax;
    # rotating weight copies keep every launch's weights out of L2
    dev = torch.device("cuda", device)
    stream = torch.cuda.Stream(device=dev)
    rng = np.random.default_rng(MODEL_SEED + 2)
    out["config2_gemv"] = measure_gemv(dev, stream, rng, peak)
    return out


CONFIG2_SHAPES = ((896, 896), (4864, 896), (896, 4864), (576, 1536), (151936, 896))


def measure_gemv(dev, stream, rng, peak, n=40):
    """Config 2: hb_gemv on each shape at batch 1 and 8 (the LM head with the
    fused argmax and no logits), W and x ~ N(0, 1) in BF16; 5 warm-up and n
    timed back-to-back launches on `stream`, rotating over copies of W that
    together exceed L2 (256 MB) so every launch reads HBM."""
    import ctypes
    import numpy as np
    import torch
    from ml_dtypes import bfloat16
    from runtime import hb_lib, layout

    lib = hb_lib.load()
    gemv = []
    for rows, k in CONFIG2_SHAPES:
        w = rng.standard_normal((rows, k), dtype=np.float32).astype(bfloat16)
        packed = torch.from_numpy(layout.pack_matrix_bytes(w)).to(dev)
        copies = [packed] + [packed.clone() for _ in range(max(0, -(-256 * 2**20 // packed.numel()) - 1))]
        head = rows == 151936
        for batch in (1, 8):
            x = torch.from_numpy(rng.standard_normal((batch, k), dtype=np.float32).astype(bfloat16).view(np.int16)).to(dev)
            y = torch.empty((batch, rows), dtype=torch.int16, device=dev)
            am = torch.empty(batch, dtype=torch.int32, device=dev)
            nscr = lib.hb_gemv_scratch_bytes(rows, batch)
            scr = torch.zeros(nscr, dtype=torch.uint8, device=dev)
            flags = (hb_lib.HB_GEMV_OUT_NONE | hb_lib.HB_GEMV_ARGMAX) if head else hb_lib.HB_GEMV_OUT_BF16

            def launch(i):
                hb_lib.check(lib.hb_gemv(copies[i % len(copies)].data_ptr(), None, 0, rows, k, x.data_ptr(), batch,
                                         y.data_ptr(), flags, am.data_ptr(), scr.data_ptr(), nscr,
                                         ctypes.c_void_p(stream.cuda_stream)))
            with torch.cuda.stream(stream):
                for i in range(5):
                    launch(i)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for i in range(n):
                    launch(i)
                e1.record(stream)
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) * 1000.0 / n
            nbytes = rows * k * 2 + batch * k * 2 + (0 if head else batch * rows * 2)
            gemv.append({"rows": rows, "k": k, "batch": batch, "argmax": head, "us": us,
                         "gbs": nbytes / (us * 1e-6) / 1e9, "hbm_frac": nbytes / (us * 1e-6) / 1e9 / peak})
        del copies, packed
    return gemv



def barrier(world):
    if world > 1:
        import torch.distributed as dist
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[LOCAL_DEVICE[0]])
        else:
            dist.barrier()


def workload_prompt(vocab):
    from runtime import synthetic
    ids = synthetic.prompt_ids(vocab, PROMPT_DRAWN, PROMPT_SEED)
    return ids[: 64 - NEW_TOKENS]


def measured_peak():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def golden_parity(engine, name, weights):
    """Teacher-forced logits of `engine` at every position of the committed
    reference request (tests/golden/request_<name>_<weights>.npz, written by
    the reference CPU runtime): max |d| and ||d|| / ||ref|| over the
    reference's top-32 entries and a strided sample, worst position; argmax
    agreement count."""
    import numpy as np

    path = REPO / "tests" / "golden" / f"request_{name}_{weights}.npz"
    if not path.exists():
        return None
    g = np.load(path)
    stride = int(g["sample_stride"])
    worst_abs, worst_rel, agree = 0.0, 0.0, 0
    for p, t in enumerate(g["ids"]):
        got = engine.step(int(t), p, logits=True)
        sample = got[::stride]
        ref = g["sample_logits"][p]
        err = max(float(np.abs(got[g["top_ids"][p]] - g["top_logits"][p]).max()), float(np.abs(sample - ref).max()))
        worst_abs = max(worst_abs, err)
        worst_rel = max(worst_rel, float(np.linalg.norm(sample - ref) / np.linalg.norm(ref)))
        agree += int(int(np.argmax(got)) == int(g["argmax"][p]))
    engine.reset()
    return {"positions": int(len(g["ids"])), "max_abs": worst_abs, "rel": worst_rel, "argmax_equal": agree,
            "reference": str(g["source"]), "tolerance": {"max_abs": 0.1, "rel": 3e-2}}


def profiled_traffic():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    path = REPO / "profiles" / "decoder_kernel_qwen25_decode.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":")[1].strip().replace(",", ""))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, index):
        self.proc = None
        self.index = index
        self.path = Path("/tmp") / f"hb_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.path.exists():
            return None
        mhz, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                mhz.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(mhz)}


# ---------------------------------------------------------------- CPU oracle --
def cpu_host():
    """What the CPU arm runs on: logical CPUs, model name, the BLAS library
    NumPy calls and its thread pool size."""
    info = {"nproc": os.cpu_count() or 1, "cpu_model": None, "blas": None, "blas_threads": None}
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                info["cpu_model"] = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    try:
        from threadpoolctl import threadpool_info
        for pool in threadpool_info():
            if pool.get("user_api") == "blas":
                info["blas"] = f"{pool.get('internal_api')} {pool.get('version')}"
                info["blas_threads"] = pool.get("num_threads")
                break
    except Exception:
        pass
    return info


class OracleRequest:
    """The config-3 request on the CPU oracle (the NumPy port of the
    reference's BF16 CPU runtime): the prompt's positions fill the KV cache
    once, untimed; each sample then times `decode_steps` greedy steps from
    the first generated position (rewriting the same positions every time,
    so each sample sees the same cache as the request)."""

    def __init__(self, model, prompt):
        from oracle.cpu_decoder import OracleDecoder, argmax_first

        self.oracle = OracleDecoder(model)
        self.argmax = argmax_first
        self.prompt = list(prompt)
        last = None
        for p, t in enumerate(self.prompt):
            last = self.oracle.step(t, p, compute_logits=(p == len(self.prompt) - 1))
        self.first = self.argmax(last)

    def sample(self, decode_steps):
        """Decode tokens/s over `decode_steps` greedy steps, and the seconds."""
        token, pos = self.first, len(self.prompt)
        t0 = time.perf_counter()
        for _ in range(decode_steps):
            token = self.argmax(self.oracle.step(token, pos))
            pos += 1
        seconds = time.perf_counter() - t0
        return decode_steps / seconds, seconds

    def describe(self, decode_steps):
        n = len(self.prompt)
        return (f"{decode_steps} greedy decode steps of the config-3 request (positions {n}..{n + decode_steps - 1}) "
                f"after an untimed fill of its {n} prompt positions")


def pinned_blas(threads):
    """Context manager pinning NumPy's BLAS pool to `threads` (torchrun sets
    OMP_NUM_THREADS=1 for every rank; the CPU arm uses the whole host)."""
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=threads, user_api="blas")


def run_reference(args, rank, world):
    if rank != 0:
        return
    from runtime import synthetic

    model = synthetic.build("qwen2.5-0.5b", seed=MODEL_SEED).materialize()
    prompt = workload_prompt(model.shape.vocab)
    decode_steps = 16
    threads = os.cpu_count() or 1
    with pinned_blas(threads):
        req = OracleRequest(model, prompt)
        for _ in range(args.warmup):
            req.sample(2)
        rates, secs = [], []
        for _ in range(args.steps):
            rate, sec = req.sample(decode_steps)
            rates.append(rate)
            secs.append(sec)
        host = cpu_host()
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * statistics.median(secs),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(len(prompt), world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": host["blas_threads"] or threads,
                         "kind": "port", "sample": req.describe(decode_steps),
                         "nproc": host["nproc"], "cpu_model": host["cpu_model"], "blas": host["blas"],
                         "weights": "BF16 weights converted to FP32 once at load (the reference converts "
                                    "them on every projection, cpu_backend.py:64-69, which is slower)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(n_prompt, world):
    """The `config` object both arms print."""
    return {"workload": "qwen2.5-0.5b-bf16 greedy decode (config 3)", "prompt_positions": n_prompt,
            "new_tokens": NEW_TOKENS, "decode_steps": NEW_TOKENS - 1, "batch": 1,
            "parallelism": f"replicas x{world}",
            "l2": "weights 1 GB per token > 126 MB L2, no flush needed"}


# ---------------------------------------------------------------- B200 arm --
def run_b200(args, rank, world, local):
    import numpy as np
    import torch
    from runtime import layout, synthetic
    from runtime.b200_engine import B200DecoderEngine
    from runtime.generate import NPUDecoder

    device = local if torch.cuda.is_available() else 0
    torch.cuda.set_device(device)
    model = synthetic.build("qwen2.5-0.5b", seed=MODEL_SEED).materialize()
    prompt = workload_prompt(model.shape.vocab)
    n_prompt = len(prompt)
    decode_steps = NEW_TOKENS - 1
    n_pre = prefill_launches(n_prompt)             # batched prefill launches
    launches_per_step = n_pre + NEW_TOKENS

    blob = layout.pack(model, "bf16")
    engine = B200DecoderEngine(model, device=device, blob=blob, max_batch=8)  # batched prefill
    stream = torch.cuda.Stream(device=device)
    engine.set_stream(stream.cuda_stream)

    def one_request():
        return engine.generate(prompt, NEW_TOKENS)

    for _ in range(args.warmup):
        ref_tokens = one_request()
    torch.cuda.synchronize()
    engine.profile(True)
    engine.profile_read()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            tokens = one_request()
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    total_ms = ev0.elapsed_time(ev1)
    # per-launch events: [prefill launches..., decode launches...] per request
    dur, start = engine.profile_read(starts=True)
    dur = dur.reshape(args.steps, launches_per_step)
    start = start.reshape(args.steps, launches_per_step)
    engine.profile(False)
    assert tokens == ref_tokens, "greedy tokens changed between identical requests"
    decode_launch_ms = dur[:, n_pre + 1:]
    # device time of each segment, launch gaps included
    end = start + dur
    prefill_ms = end[:, n_pre] - start[:, 0]          # through the first generated token
    decode_seg_ms = end[:, -1] - start[:, n_pre + 1]
    local_time = float(decode_seg_ms.sum())
    t_max = max_over_ranks(local_time, world)
    value = (decode_steps * args.steps * world) / (t_max / 1000.0)
    ms_per_step = max_over_ranks(total_ms, world) / args.steps

    # roofline of the decode kernel (positions n_prompt .. n_prompt+30)
    mean_pos = n_prompt + (decode_steps - 1) / 2.0
    alg_bytes = WEIGHT_BYTES + KV_BYTES_PER_POSITION * (mean_pos + 1)
    launch_ms = float(decode_launch_ms.mean())
    achieved = alg_bytes / (launch_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()

    # prefix-cache replay: the same prompt again reuses 31 positions
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    engine.generate(prompt, 1, start=n_prompt - 1)
    ttft_cached_ms = 1000 * (time.perf_counter() - t0)

    # TTFT through the batched tensor-core prefill: the 32 prompt positions
    # in one launch sequence, the LM head on the last one (device events on
    # the engine's stream; host row upload and argmax read-back included)
    for _ in range(3):
        tc_first, _ = engine.prefill_tc(prompt)
    ttft_tc = []
    for _ in range(max(5, args.steps)):
        ev0.record(stream)
        tc_first, _ = engine.prefill_tc(prompt)
        ev1.record(stream)
        torch.cuda.synchronize()
        ttft_tc.append(ev0.elapsed_time(ev1))
    ttft_tc_ms = float(np.median(ttft_tc))
    tc_first = {"token": int(tc_first), "equals_persistent": int(tc_first) == ref_tokens[0]}

    parity = {"config3": golden_parity(engine, "qwen2.5-0.5b", "bf16")} if rank == 0 else None

    # e2e through the public decode_token API (host copies + sync per call)
    engine.close()
    decoder = NPUDecoder(model)
    for _ in range(max(1, args.warmup - 1)):
        run_decode_token_request(decoder, prompt)
    barrier(world)
    e2e_decode = 0.0
    e2e_ttft = []
    for _ in range(args.steps):
        generated, ttft, dec = run_decode_token_request(decoder, prompt)
        e2e_decode += dec
        e2e_ttft.append(ttft)
    assert generated == ref_tokens, "decode_token path disagrees with the device-resident path"
    e2e_t = max_over_ranks(e2e_decode, world)
    e2e_value = decode_steps * args.steps * world / e2e_t
    decoder.close()

    multistream = multistream_persistent = None
    if not args.no_extras:
        multistream = run_multistream(model, blob, device, rank, world, "rows")
        multistream_persistent = run_multistream(model, blob, device, rank, world, "persistent")
    others = run_other_configs(device, measured_peak()[0]) if world == 1 and not args.no_extras else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        with pinned_blas(threads):
            req = OracleRequest(model, prompt)
            req.sample(2)
            rate, _ = req.sample(16)
            host = cpu_host()
        cpu = {"value": rate, "unit": "tokens/s", "cores": host["blas_threads"] or threads, "kind": "port",
               "sample": req.describe(16), "nproc": host["nproc"], "cpu_model": host["cpu_model"],
               "blas": host["blas"]}

    if rank == 0:
        step_state_bytes = 32 * 4 - 16  # StepState: 3x8 ints + 4 ints
        result_bytes = 64               # Result: control block + 8 token ids
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(n_prompt, world),
            "ttft_ms": float(np.median(prefill_ms)),
            "ttft_cached_ms": ttft_cached_ms,
            "e2e_ttft_ms": 1000 * statistics.median(e2e_ttft),
            "decode_launch_ms": launch_ms,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(),
                         "traffic_source": "ncu dram__bytes_read+write of one decode launch, "
                                           "profiles/decoder_kernel_qwen25_decode.md (not measured in this run)",
                         "peak_kind": peak_kind, "algorithmic_bytes_per_launch": alg_bytes},
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    # decode_token runs one launch per position
                    "h2d_bytes_per_step": (n_prompt + NEW_TOKENS - 1) * step_state_bytes,
                    "d2h_bytes_per_step": (n_prompt + NEW_TOKENS - 1) * result_bytes},
            "gpu_launches": launches_per_step * args.steps,
            "parity": parity,
            "multistream": multistream,
            "multistream_persistent": multistream_persistent,
            "ttft_tc_ms": ttft_tc_ms,
            "ttft_tc_first_token": tc_first,
            "other_configs": others,
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)


def run_config5(args, rank, world, local):
    """Config 5 as the metric line: aggregate generated tokens/s of the 512
    requests (split over the ranks by prefix affinity, no collective on the
    token path), --warmup untimed then --steps timed passes, time = the
    slowest rank's wall clock (host scheduling included)."""
    import torch
    from runtime import layout, synthetic

    device = local if torch.cuda.is_available() else 0
    torch.cuda.set_device(device)
    model = synthetic.build("qwen2.5-0.5b", seed=MODEL_SEED).materialize()
    blob = layout.pack(model, "bf16")
    clocks = ClockSampler(device)
    ms = run_multistream(model, blob, device, rank, world, "rows", passes=args.steps, warmup=args.warmup,
                         clocks=clocks)
    if rank != 0:
        return
    spec = MULTISTREAM_MODES["rows"]
    # per step (mean over rank 0's steps): slot, token and position of every row
    # plus the output-row list go up as int32; the argmax of every output row and
    # the 64-byte control block come back (output rows <= rows: upper bounds)
    rows_per_step = ms["rows_rank0"] / max(1, ms["launches_rank0"])
    h2d = int(round(16 * rows_per_step))
    d2h = int(round(4 * rows_per_step + 64))
    peak, peak_kind = measured_peak()
    launch_s = max(ms["wall_s_per_rank"]) / max(1, args.steps * ms["launches_rank0"])
    line = {
        "metric": "config5_generated_tokens_per_second", "value": ms["value"], "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * max(ms["wall_s_per_rank"]) / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": ms["workload"], "requests": ms["requests"], "parallelism": f"requests split x{world}",
                   "server": spec["server"], "lanes": spec.get("lanes", 1), "l2": "weights 1 GB per step > 126 MB L2"},
        "p50_ttft_ms": ms["p50_ttft_ms"], "lanes": ms["lanes"],
        "wall_s_per_rank": ms["wall_s_per_rank"], "launches_per_rank_per_pass": ms["launches_per_rank"],
        "slowest_rank": ms["slowest_rank"], "rows_rank0_per_pass": ms["rows_rank0"],
        "prefix_reuses_rank0": ms["prefix_reuses_rank0"],
        # every step streams the whole BF16 model once for all its rows
        "roofline": {"bound": "hbm", "achieved": WEIGHT_BYTES / launch_s / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": WEIGHT_BYTES / launch_s / 1e9 / peak, "traffic": None, "peak_kind": peak_kind,
                     "note": "weight bytes per batched step x steps of all lanes / wall time (scheduling "
                             "included; the lanes' steps overlap)"},
        "e2e": {"value": ms["value"], "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "the server is the public Python API: token ids in and out through host memory every "
                        "launch sequence, so the metric is already end to end"},
        # kernels per batched step: embedding+norm, 7 per layer (qkv, attention, o,
        # norm, gate/up, down, norm) less the last layer's norm, final norm, LM
        # head, argmax: 3 + 7 x 24 = 171 (rank 0's timed passes)
        "gpu_launches": ms["launches_total_rank0"] * (3 + 7 * 24),
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_decode_token_request(decoder, prompt):
    """The reference's greedy loop over decode_token: sequential prefill
    (logits only at the last position), then decode steps; returns
    (generated ids, ttft seconds, decode seconds)."""
    decoder.reset_prefix_cache()
    ttft = 0.0
    token = None
    last = len(prompt) - 1
    for p, t in enumerate(prompt):
        token, elapsed = decoder.decode_token(t, p, compute_logits=(p == last))
        ttft += elapsed
    generated = [token]
    decode = 0.0
    pos = len(prompt)
    while len(generated) < NEW_TOKENS:
        token, elapsed = decoder.decode_token(generated[-1], pos)
        generated.append(token)
        decode += elapsed
        pos += 1
    return generated, ttft, decode


def run_profile_rows(args, n):
    """The batched tensor-core step on its own, for ncu captures: n rows
    (stream i in KV slot i at position 40, the Qwen2.5-0.5B shape, BF16)."""
    import torch
    from runtime import synthetic
    from runtime.b200_engine import B200DecoderEngine

    model = synthetic.build("qwen2.5-0.5b", seed=MODEL_SEED).materialize()
    engine = B200DecoderEngine(model, max_slots=max(n, 8) + 4, max_batch=8)
    try:
        tokens = synthetic.prompt_ids(model.shape.vocab, n, seed=MODEL_SEED + 9)
        rows = (list(range(n)), tokens, [40] * n)
        for _ in range(args.warmup):
            engine.step_rows(*rows)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            engine.step_rows(*rows)
        ms = 1000 * (time.perf_counter() - t0) / max(1, args.steps)
        print(f"profile-rows {n}: {ms:.3f} ms per step (host wall, {args.steps} steps)", flush=True)
    finally:
        engine.close()


def run_profile_gemv():
    """Config 2 on its own (the standalone GEMV shapes), for ncu launch lists
    beside the CUDA-event times it prints."""
    import numpy as np
    import torch

    dev = torch.device("cuda", 0)
    for r in measure_gemv(dev, torch.cuda.Stream(device=dev), np.random.default_rng(MODEL_SEED + 2),
                          measured_peak()[0]):
        print(json.dumps(r), flush=True)


def main():
    args = parse()
    if args.profile_gemv:
        run_profile_gemv()
        return
    if args.profile_rows:
        run_profile_rows(args, args.profile_rows)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.workload == "config5":
            run_config5(args, rank, world, local)
        else:
            run_b200(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
