#!/usr/bin/env python3
"""Decode benchmark of the promptboot_b200 engine: batched decode (config 3) as
the headline, with the single-sequence, sampler, linear-sweep and long-context
configurations (configs 0, 1, 2, 4) as extra keys of the same JSON line.

Config 3 (the headline): the config-0 model (seeded synthetic Qwen2.5-0.5B
Q4_0, PBTQW25 v1), 256 independent sequences in total, each with a 512-token
uniform random prompt (numpy default_rng(0x5eed0000 + global_index)) and its own
SamplingState(global_index), decoding 1,024 tokens (positions 512..1535) with
the interactive sampler (penalty 1.1 over the whole history, T 0.7, top-k 20,
top-p 0.8).  One step = one sampled token for every sequence: sampler + 24-layer
forward + lm_head, all device resident.  The sequences are split over the
ranks, 256/N contiguous ones per GPU (strong scaling); ranks share nothing.

The whole 1,024-step decode runs; `--warmup` steps come first, then `--steps`
timed steps sit at evenly spaced positions across the rest of the range (each
bracketed by a barrier + synchronize and CUDA events on the engine stream, max
over ranks), so the figure is the mean over config 3's decode range, not its
cheapest end.  Between them the other steps run untimed; some carry the
end-to-end measurement (the host-buffer C ABI: sample + decode_batch) and some
carry per-kernel-class CUDA events for the roofline.

`--impl reference` times the reference's decode arithmetic on the host cores
instead (the CPU restatement in oracle/, the reference's Rust cannot be built
here), one sequence per host thread at the same stratified contexts.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decoded tok/s, Qwen2.5-0.5B Q4_0 batch 256 at 1/2/4/8 B200; % HBM roofline"
UNIT = "tok/s"
WEIGHT_BYTES = 346206720          # Q4_0 layer weights + Q8_0 lm_head + f32 biases/norms per token
KV_BYTES_PER_POSITION = 24576     # K and V of one position, 24 layers
LOGIT_BYTES = 151936 * 4


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20, help="timed decode steps (config 3)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seqs", type=int, default=256, help="sequences in total (split over GPUs)")
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--decode", type=int, default=1024, help="decode steps per sequence")
    p.add_argument("--e2e-steps", type=int, default=8)
    p.add_argument("--cpu-tokens", type=int, default=3, help="CPU-baseline tokens per stratum")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra-configs", action="store_true",
                   help="skip the config 0/1/2/4 keys")
    p.add_argument("--op", choices=["attention", "qmatvec", "matvec-sweep", "sampler", "decode1",
                                    "longctx"],
                   default=None,
                   help="time one operator or configuration alone (the small cases of the "
                        "ncu captures) instead of the decode bench")
    p.add_argument("--op-rows", type=int, default=192, help="--op: sequences")
    p.add_argument("--op-positions", type=int, default=520, help="--op attention: context")
    p.add_argument("--op-shape", default="151936x896", help="--op qmatvec: ROWSxCOLS")
    p.add_argument("--op-wtype", type=int, default=3, help="--op qmatvec: 2 Q4_0, 3 Q8_0")
    return p.parse_args(argv)


# ----------------------------------------------------------------- helpers

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1400.0, "fallback"


def strata(first: int, last: int, k: int) -> list[int]:
    """k distinct indices evenly spread over [first, last] (midpoints of k equal
    strata)."""
    span = last - first + 1
    if k > span:
        raise ValueError(f"{k} timed steps do not fit in {span} positions")
    return [first + int((j + 0.5) * span / k) for j in range(k)]


def step_bytes_at(seqs: int, position: int) -> float:
    """Algorithmic HBM bytes of one decode step of `seqs` sequences evaluating
    `position`: the weights once, every sequence's KV of positions 0..position
    read and this position's written, and its logits row written."""
    return WEIGHT_BYTES + seqs * ((position + 1) * KV_BYTES_PER_POSITION + KV_BYTES_PER_POSITION
                                  + LOGIT_BYTES)


def class_bytes_at(cls: str, seqs: int, position: int) -> float:
    """Algorithmic bytes of all launches of kernel class `cls` in one step of
    `seqs` sequences evaluating `position`."""
    if cls == "attention":
        # per layer: positions 0..position of K (512 B) and V (512 B), q in, out
        return 24 * seqs * ((position + 1) * 1024.0 + 2 * 896 * 4)
    if cls == "gemv":
        mats = [(896, 896), (128, 896), (128, 896), (896, 896), (4864, 896), (4864, 896),
                (896, 4864)]
        return 24 * sum(r * k // 32 * 18 + seqs * (k * 4 + r * 4) for r, k in mats)
    if cls == "lm_head":
        return 151936 * 28 * 34 + seqs * (896 * 4 + 151936 * 4)
    if cls == "sampler":
        return seqs * (151936 * 4 + (position + 1) * 4)
    return 0.0


def profiled_traffic(kernel_class: str, seqs: int, mean_ctx: float):
    """DRAM bytes per launch at this workload, scaled from the committed ncu
    captures of smaller cases (profiles/traffic.json), where one covers the class."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    if kernel_class == "attention" and "attention" in d:
        return seqs * mean_ctx * d["attention"]["dram_bytes_per_sequence_position"]
    if kernel_class == "gemv" and "gemv" in d:
        return d["gemv"]["dram_bytes_per_launch_b256"] * seqs / 256.0 if seqs >= 9 else None
    return None


# What bounds each kernel class in practice (from the ncu captures).
LIMITERS = {
    "attention": "f32->f64 widening of every q.k product on the XU pipe in the scores launch; "
                 "latency of the softmax + PV launch; HBM traffic close to the algorithmic "
                 "1024 B per sequence-position",
    "gemv": "per-block binary32 epilogue (three rounded operations per row, sequence and "
            "block) on the FMA pipe, and per-chunk latency for the 8-sequence tiles",
    "lm_head": "per-block binary32 epilogue on the FMA pipe",
}

KC = {"embed": 0, "norm": 1, "gemv": 2, "rope_kv": 3, "attention": 4, "quant": 5, "swiglu": 6,
      "lm_head": 7, "argmax": 8, "sampler": 9}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms from before
    the timed region (the first sample is awaited, so the sampler is running
    when the region starts) and summarised over the samples whose timestamps
    fall inside the region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.path = pathlib.Path(tempfile.mkstemp(prefix="pb_clocks_", suffix=".csv")[1])
        self.device = device
        self.proc = None
        self.window = None

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0
            while time.time() < deadline and self.path.stat().st_size == 0:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark(self, t0: float, t1: float):
        """Wall-clock bounds (time.time()) of the timed region."""
        self.window = (t0, t1)

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.06)  # one more sample after the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        import datetime
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 10 and f[2].isdigit():
                    try:
                        ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    except ValueError:
                        continue
                    rows.append((ts, f[1:]))
        except OSError:
            pass
        finally:
            self.path.unlink(missing_ok=True)
        if self.window:
            t0, t1 = self.window
            inside = [r for ts, r in rows if t0 <= ts <= t1]
            if not inside:  # a region shorter than the period: the first sample after it began
                after = [r for ts, r in rows if ts >= t0]
                inside = after[:1]
            rows = inside
        else:
            rows = [r for _, r in rows]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(int(r[1]) for r in rows),
                "sm_max_mhz": max(int(r[2]) for r in rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


from promptboot_b200.shard import (aggregate_throughput, barrier, max_over_ranks,  # noqa: E402
                                   partition)


def model_image(rank: int, world: int):
    from promptboot_b200 import pbtqw25
    if rank == 0:
        img = pbtqw25.load_or_synthesize(0)
    barrier(world)
    if rank != 0:
        img = pbtqw25.load_or_synthesize(0)
    return img


class Events:
    """A CUDA-event pair on one stream."""

    def __init__(self, stream):
        import torch
        self.stream = stream
        self.a = torch.cuda.Event(enable_timing=True)
        self.b = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.a.record(self.stream)
        return self

    def __exit__(self, *exc):
        self.b.record(self.stream)

    def ms(self) -> float:
        self.b.synchronize()
        return self.a.elapsed_time(self.b)


# ------------------------------------------------------------ config 3 (GPU)

def run_config3(args, world, rank, local, img):
    """The headline: strong-scaled batched decode over the whole decode range."""
    import ctypes
    import torch
    from promptboot_b200 import _lib, api, shard
    lib = _lib.load()
    first, count = partition(args.seqs, rank, world)
    S, P, D = count, args.prompt, args.decode
    C = (P + D + 4) // 4 * 4   # positions 0 .. P + D - 1 evaluated
    model = api.ModelView(img, device=local)
    eng = api.InferenceEngine(model, max_seqs=S, max_context=C)
    seqs = np.arange(S, dtype=np.uint32)
    gidx = first + np.arange(S)
    prompts = np.stack([shard.prompt_for(g, P) for g in gidx])
    t_prefill = time.perf_counter()
    status, _, errs = eng.prefill_batch(seqs, prompts, D + 1)  # + the prefill's own token
    if status:
        raise RuntimeError(f"prefill failed: {errs[0].tuple()}")
    prefill_s = time.perf_counter() - t_prefill
    states = api.SamplingStates([shard.sampling_seed(g) for g in gidx])
    stream = torch.cuda.ExternalStream(lib.pb_engine_stream(eng._h))

    # decode step i evaluates position P + i; warm-up first, then the timed
    # steps spread over the rest, each followed by one end-to-end step (for
    # the first e2e_steps strata spread over the range) and one step with every
    # kernel class bracketed by CUDA events.
    W, K = args.warmup, args.steps
    timed = strata(W, D - 3, K)
    e2e_at = {timed[int((j + 0.5) * K / args.e2e_steps)] + 1 for j in range(min(args.e2e_steps, K))}
    profile_at = {t + 2 for t in timed}
    done = 0

    def advance_to(i):
        nonlocal done
        if i > done:
            st, _, errs = eng.generate(seqs, states, i - done, want_tokens=False)
            if st:
                raise RuntimeError(f"decode failed: {[e.tuple() for e in errs if e.status][:1]}")
            done = i

    timed_ms, e2e_ms, launches = [], [], 0
    ms16 = (ctypes.c_double * 16)()
    cnt16 = (ctypes.c_uint64 * 16)()
    class_ms = {k: 0.0 for k in KC}
    class_n = {k: 0 for k in KC}
    class_bytes = {k: 0.0 for k in KC}
    clock = ClockSampler(local)
    with clock:
        w0 = time.time()
        for i in range(D):
            if i in timed:
                advance_to(i)
                barrier(world)
                torch.cuda.synchronize()
                l0 = lib.pb_engine_launch_count(eng._h)
                torch.cuda.nvtx.range_push("pb_timed")  # ncu --nvtx --nvtx-include pb_timed/
                with Events(stream) as ev:
                    st, _, errs = eng.generate(seqs, states, 1, want_tokens=False)
                torch.cuda.nvtx.range_pop()
                ms = ev.ms()
                torch.cuda.synchronize()
                barrier(world)
                if st:
                    raise RuntimeError(f"timed step failed: {[e.tuple() for e in errs if e.status][:1]}")
                launches += lib.pb_engine_launch_count(eng._h) - l0
                timed_ms.append(max_over_ranks(ms, world))
                done = i + 1
            elif i in e2e_at:
                advance_to(i)
                barrier(world)
                torch.cuda.synchronize()
                with Events(stream) as ev:
                    st, ids, _ = eng.sample(seqs, states)
                    st2, _, errs = eng.decode_batch(seqs, ids, require_greedy=False)
                ms = ev.ms()
                barrier(world)
                if st or st2:
                    raise RuntimeError(f"e2e step failed: {st} {st2}")
                e2e_ms.append(max_over_ranks(ms, world))
                done = i + 1
            elif i in profile_at:
                advance_to(i)
                lib.pb_engine_profile(eng._h, 0xFFFF)
                st, _, errs = eng.generate(seqs, states, 1, want_tokens=False)
                torch.cuda.synchronize()
                lib.pb_engine_profile_read(eng._h, ms16, cnt16)
                lib.pb_engine_profile(eng._h, 0)
                if st:
                    raise RuntimeError("profiled step failed")
                for name, k in KC.items():
                    class_ms[name] += ms16[k]
                    class_n[name] += cnt16[k]
                    class_bytes[name] += class_bytes_at(name, S, P + i)
                done = i + 1
        advance_to(D)
        clock.mark(w0, time.time())
    total_ms = sum(timed_ms)
    value = aggregate_throughput(S * K, world, total_ms)
    e2e_value = aggregate_throughput(S * len(e2e_ms), world, sum(e2e_ms))
    hbm, _, peak_kind = measured_peaks()
    dominant = max(class_ms, key=class_ms.get)
    dom_ms, dom_n = class_ms[dominant], class_n[dominant]
    achieved = class_bytes[dominant] / (dom_ms / 1000.0) / 1e9 if dom_ms > 0 else None
    mean_pos = float(np.mean([P + t for t in timed]))
    sbytes = float(np.mean([step_bytes_at(S, P + t) for t in timed]))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": total_ms / K,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8xint4->f32/f64",
        "data": "synthetic (seeded random-init weights, uniform random prompts)",
        "config": {"workload": "config 3 batched decode", "global_batch": args.seqs,
                   "seqs_per_gpu": S, "prompt": P, "decode_tokens": D, "context_capacity": C,
                   "timed_positions": [P + t for t in timed],
                   "timed_position_range": [P + timed[0], P + timed[-1]],
                   "mean_timed_position": mean_pos,
                   "parallelism": f"sequence-partitioned {args.seqs}/{world} per GPU, no collective",
                   "l2": "inputs larger than L2 (346 MB weights + KV per step)",
                   "prefill_s": round(prefill_s, 3)},
        "e2e": {"value": e2e_value, "unit": UNIT, "steps": len(e2e_ms),
                "positions": sorted(P + i for i in e2e_at),
                "api": "pb_engine_sample + pb_engine_decode_batch with host token/state buffers",
                "h2d_bytes_per_step": 40 * S, "d2h_bytes_per_step": 48 * S + 4},
        "gpu_launches": int(launches),
        "step_roofline": {"bound": "hbm", "bytes_per_step": sbytes,
                          "achieved": sbytes / (total_ms / K) / 1e6, "peak": hbm, "unit": "GB/s",
                          "frac": sbytes / (total_ms / K) / 1e6 / hbm},
        "roofline": {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": hbm,
                     "unit": "GB/s", "frac": (achieved / hbm) if achieved else None,
                     "traffic": profiled_traffic(dominant, S, mean_pos + 1.0),
                     "algorithmic_bytes_per_launch": class_bytes[dominant] / max(dom_n, 1),
                     "peak_source": peak_kind, "limiter": LIMITERS.get(dominant),
                     "launches": int(dom_n), "avg_launch_us": 1000.0 * dom_ms / max(dom_n, 1),
                     "profiled_steps": len(profile_at),
                     "ms_per_step_by_class": {k: round(v / max(len(profile_at), 1), 4)
                                              for k, v in class_ms.items()}},
        "clocks": clock.summary(),
    }
    eng.close()
    model.close()
    return line


def cpu_config3(img, positions, tokens: int):
    """The oracle's decode (forward + sampler) on every host thread, one
    sequence per thread, `tokens` tokens from each of the given contexts."""
    import oracle
    cores = oracle.cpu_cores()
    oracle.bench_decode(img, positions[0], 1, cores, cores)  # page in the weights
    rates = [oracle.bench_decode(img, p, tokens, cores, cores) for p in positions]
    value = len(rates) / sum(1.0 / r for r in rates)  # tokens/s over equal token counts
    return {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{cores} sequences (one per host thread) x {tokens} decode tokens from "
                      f"each of the contexts {positions}, oracle/ C restatement (-O3 -mavx2)"}


# ------------------------------------------------- configs 0, 1, 2, 4 (GPU)

def run_config0(img, local):
    """Config 0: one sequence, 64-token prompt (default_rng(0x5eed0000)), 64
    sampled tokens with seed 1 through the device-resident generate loop;
    e2e through the REPL's host-buffer calls (sample_token_with_repetition,
    then decode_selected with host logits)."""
    import torch
    from promptboot_b200 import api, shard
    view = api.ModelView(img, device=local)
    eng = api.InferenceEngine(view, max_seqs=2, max_context=160)
    prompt = shard.prompt_for(0, 64)
    stream = torch.cuda.ExternalStream(eng.stream())
    # warm-up on slot 1
    assert eng.prefill_batch([1], prompt[None, :], 80)[0] == 0
    assert eng.generate([1], [api.SamplingState(1)], 8, want_tokens=False)[0] == 0
    assert eng.prefill_batch([0], prompt[None, :], 80)[0] == 0
    state = api.SamplingState(1)
    torch.cuda.synchronize()
    with Events(stream) as ev:
        st, _, _ = eng.generate([0], [state], 64, want_tokens=False)
    ms = ev.ms()
    assert st == 0
    # e2e: the REPL loop with host buffers, wall clock (every call synchronizes)
    eng.reset(1)
    logits = np.zeros(api.VOCAB, dtype=np.uint32)
    eng.prefill(prompt, 80, logits, seq=1)
    seen = np.zeros(api.SEEN_BYTES, dtype=np.uint8)
    rstate = api.SamplingState(1)
    history = list(prompt)
    t0 = time.perf_counter()
    for _ in range(64):
        tok = api.sample_token_with_repetition(logits, history, seen, rstate)
        history.append(tok)
        eng.decode_selected(tok, logits, seq=1)
    e2e_s = time.perf_counter() - t0
    eng.close()
    view.close()
    hbm = measured_peaks()[0]
    per_token = ms / 64 / 1000.0
    return {"workload": "config 0 single sequence (64-token prompt, 64 sampled tokens, seed 1)",
            "value": 1.0 / per_token, "unit": UNIT, "ms_per_token": per_token * 1000.0,
            "roofline": {"bound": "hbm", "bytes_per_token": WEIGHT_BYTES,
                         "achieved": WEIGHT_BYTES / per_token / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": WEIGHT_BYTES / per_token / 1e9 / hbm},
            "e2e": {"value": 64 / e2e_s, "unit": UNIT,
                    "api": "pb_sample_token_with_repetition + pb_engine_decode_selected, host logits",
                    # sampler: logits, history (96 ids on average), length, state, seen
                    # bitmap in; row, state, penalized logits out.  decode_selected:
                    # slot, token, position in; error word, status, greedy id and
                    # bits, logits out.
                    "h2d_bytes_per_step": LOGIT_BYTES + 4 * 96 + 4 + 16 + 18992 + 12,
                    "d2h_bytes_per_step": 2 * LOGIT_BYTES + 16 + 16 + 8 + 4 + 8}}


def cpu_config0(img):
    import oracle
    rate = oracle.bench_decode(img, 64, 8, 1, 1)
    return {"value": rate, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": "1 sequence x 8 decode tokens (forward + sampler) from context 64 on one "
                      "host thread, oracle/ C restatement"}


def sampler_batch_inputs(rows=256, vocab=151936, hist=512):
    """Config 1: rows of N(0, 3^2) logits with 5 positions raised by 12
    (default_rng(7)), 512 history ids per row."""
    rng = np.random.default_rng(7)
    logits = (rng.standard_normal((rows, vocab)) * 3.0).astype(np.float32)
    for r in range(rows):
        logits[r, rng.integers(0, vocab, 5)] += 12.0
    history = rng.integers(0, vocab, (rows, hist), dtype=np.int64).astype(np.uint32)
    return logits, history


def run_config1(local):
    """Config 1: the 256-row sampler batch; every timed call gets a fresh copy of
    the logits (the penalty mutates them; copy untimed); mean of 10 after 3."""
    import ctypes
    import torch
    from promptboot_b200 import _lib
    lib = _lib.load()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rows, vocab, hist = 256, 151936, 512
    logits, history = sampler_batch_inputs(rows, vocab, hist)
    src = torch.from_numpy(logits).cuda()
    work = torch.empty_like(src)
    hist_d = torch.from_numpy(history.reshape(-1).view(np.int32)).cuda()
    offs = torch.arange(rows, dtype=torch.int64, device="cuda") * hist
    lens = torch.full((rows,), hist, dtype=torch.int32, device="cuda")
    states0 = np.zeros((rows, 2), dtype=np.uint64)
    for r in range(rows):  # per-row SamplingState(7 + row)
        st = _lib.PbSamplingState()
        lib.pb_sampling_state_init(ctypes.byref(st), 7 + r)
        states0[r] = [st.state, st.draws]
    states = torch.from_numpy(states0.view(np.int64)).cuda()
    out = torch.empty((rows, 4), dtype=torch.int32, device="cuda")
    call = lambda: lib.pb_sample_batch_device(P(work), vocab, rows, P(hist_d), P(offs), P(lens),
                                              P(states), P(out), None)
    for _ in range(3):
        work.copy_(src)
        assert call() == 0
    total = 0.0
    for _ in range(10):
        work.copy_(src)
        with Events(torch.cuda.current_stream()) as ev:
            call()
        total += ev.ms()
    us = total / 10 * 1000.0
    nbytes = rows * (vocab * 4 + hist * 8)
    hbm = measured_peaks()[0]
    return {"workload": "config 1 sampler batch (256 rows x 151,936, history 512)",
            "us_per_batch": us, "value": rows / (us * 1e-6), "unit": "rows/s",
            "roofline": {"bound": "hbm", "bytes_per_batch": nbytes,
                         "achieved": nbytes / (us * 1e-6) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": nbytes / (us * 1e-6) / 1e9 / hbm}}


def cpu_config1():
    import oracle
    logits, history = sampler_batch_inputs(16)
    state = oracle.SamplingState(7)
    t0 = time.perf_counter()
    for r in range(16):
        st, _, _ = oracle.sample_with_repetition(logits[r], history[r], state)
        assert st == 0
    dt = time.perf_counter() - t0
    return {"value": 16 / dt, "unit": "rows/s", "cores": 1, "kind": "port",
            "sample": "16 rows of the config-1 batch on one host thread, oracle/ C restatement"}


SWEEP_SHAPES = [("q 896x896 Q4_0", ("L", 0, 19), 896, 896, 18),
                ("k 128x896 Q4_0", ("L", 0, 16), 128, 896, 18),
                ("gate 4864x896 Q4_0", ("L", 0, 12), 4864, 896, 18),
                ("down 896x4864 Q4_0", ("L", 0, 11), 896, 4864, 18),
                ("head 151936x896 Q4_0 (tied embedding)", 0, 151936, 896, 18),
                ("head 151936x896 Q8_0", 290, 151936, 896, 34)]


def run_config2(img, local):
    """Config 2: the engine's matvec (pb_model_matvec_device) on the model's own
    tensors at B in {1, 8, 64, 256}; each timed call after a 256 MB write that
    flushes L2, mean of 10 after 3.  Bytes = W + B*K*4 + B*N*4, flops = 2*B*N*K."""
    import ctypes
    import torch
    from promptboot_b200 import _lib, api, pbtqw25
    lib = _lib.load()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    view = api.ModelView(img, device=local)
    hbm = measured_peaks()[0]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    out = []
    for name, tid, n, k, bpb in SWEEP_SHAPES:
        if isinstance(tid, tuple):
            tid = pbtqw25.layer_tensor(tid[1], tid[2])
        for bsz in (1, 8, 64, 256):
            x = torch.randn(bsz, k, device="cuda")
            y = torch.empty(bsz, n, device="cuda")
            for _ in range(3):
                assert lib.pb_model_matvec_device(view._h, tid, P(x), bsz, P(y), None) == 0
            total = 0.0
            for _ in range(10):
                flush.fill_(1.0)
                with Events(torch.cuda.current_stream()) as ev:
                    lib.pb_model_matvec_device(view._h, tid, P(x), bsz, P(y), None)
                total += ev.ms()
            assert lib.pb_model_matvec_status(view._h, None) == 0
            us = total / 10 * 1000.0
            nbytes = n * k // 32 * bpb + bsz * k * 4 + bsz * n * 4
            gbs = nbytes / (us * 1e-6) / 1e9
            out.append({"shape": name, "batch": bsz, "us": round(us, 2), "alg_bytes": nbytes,
                        "GB_s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                        "int8_TOPS": round(2.0 * bsz * n * k / (us * 1e-6) / 1e12, 2),
                        "path": "tensor-core" if bsz >= 9 else "cuda-core"})
    view.close()
    return {"workload": "config 2 linear sweep (engine matvec on model tensors)",
            "l2": "256 MB write between timed calls", "cases": out}


def cpu_config2(img):
    import oracle
    from promptboot_b200 import pbtqw25
    rng = np.random.default_rng(2)
    res = {}
    for name, tid, n, k in (("gate 4864x896 Q4_0", pbtqw25.layer_tensor(0, 12), 4864, 896),
                            ("head 151936x896 Q8_0", 290, 151936, 896)):
        w = pbtqw25.tensor_view(img, tid)
        staging = oracle.prepare_q8(rng.standard_normal(k).astype(np.float32))
        fn = oracle.q8_matvec if tid == 290 else oracle.q4_matvec
        fn(w, staging, n, k)
        reps = 3 if tid == 290 else 50
        t0 = time.perf_counter()
        for _ in range(reps):
            fn(w, staging, n, k)
        us = (time.perf_counter() - t0) / reps * 1e6
        nbytes = n * k // 32 * (34 if tid == 290 else 18) + k * 4 + n * 4
        res[name] = {"batch": 1, "us": round(us, 1), "GB_s": round(nbytes / (us * 1e-6) / 1e9, 2)}
    return {"value": res["gate 4864x896 Q4_0"]["GB_s"], "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "B = 1 matvecs on one host thread (oracle/ C restatement, AVX2 block dots)",
            "cases": res}


def run_config4(img, local, rank, world, K: int = 8, warmup: int = 2):
    """Config 4: 8 sequences in total (8/N per GPU) at 30,000 prompt positions,
    decoding to 31,024.  The KV cache of the prompt is seeded N(0, 0.25) values
    restored into each slot (attention's arithmetic does not depend on how the
    cache was filled); K timed single steps sit at evenly spaced positions over
    30,000..31,023, each after a reset, restore and one untimed step there."""
    import torch
    from promptboot_b200 import api, shard
    first, S = partition(8, rank, world)
    P, D = 30000, 1024
    C = P + D
    view = api.ModelView(img, device=local)
    eng = api.InferenceEngine(view, max_seqs=S, max_context=C)
    seqs = np.arange(S, dtype=np.uint32)
    ids = np.stack([shard.prompt_for(first + s, C) for s in range(S)])
    g = torch.Generator(device="cuda").manual_seed(4000 + first)
    for s in range(S):
        region = eng.kv_tensor(s)
        region.normal_(0.0, 0.5, generator=g)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(eng.stream())
    states = api.SamplingStates([shard.sampling_seed(first + s) for s in range(S)])
    positions = strata(P + 1, P + D - 2, K)

    def place(pos):
        for s in range(S):
            eng.reset(s)
            eng.restore(ids[s, :pos - 1], C - pos + 1, seq=s)
        st, _, _ = eng.decode_batch(seqs, ids[:, pos - 1], require_greedy=False)
        assert st == 0

    place(positions[0])
    assert eng.generate(seqs, states, warmup, want_tokens=False)[0] == 0
    times, attn_ms, attn_bytes = [], 0.0, 0.0
    import ctypes
    from promptboot_b200 import _lib
    lib = _lib.load()
    ms16 = (ctypes.c_double * 16)()
    cnt16 = (ctypes.c_uint64 * 16)()
    for pos in positions:
        place(pos)
        barrier(world)
        torch.cuda.synchronize()
        with Events(stream) as ev:
            st, _, _ = eng.generate(seqs, states, 1, want_tokens=False)
        times.append(max_over_ranks(ev.ms(), world))
        assert st == 0
        lib.pb_engine_profile(eng._h, 1 << KC["attention"])
        assert eng.generate(seqs, states, 1, want_tokens=False)[0] == 0
        torch.cuda.synchronize()
        lib.pb_engine_profile_read(eng._h, ms16, cnt16)
        lib.pb_engine_profile(eng._h, 0)
        attn_ms += ms16[KC["attention"]]
        attn_bytes += class_bytes_at("attention", S, pos + 1)
    eng.close()
    view.close()
    hbm = measured_peaks()[0]
    total = sum(times)
    sbytes = float(np.mean([step_bytes_at(S, p) for p in positions]))
    return {"workload": "config 4 long-context decode (8 sequences, positions 30,000..31,023)",
            "value": aggregate_throughput(S * K, world, total), "unit": UNIT, "n_gpus": world,
            "ms_per_step": total / K, "timed_positions": positions,
            "kv": "seeded N(0, 0.25) cache restored at each timed position",
            "step_roofline": {"bound": "hbm", "bytes_per_step": sbytes,
                              "achieved": sbytes / (total / K) / 1e6, "peak": hbm, "unit": "GB/s",
                              "frac": sbytes / (total / K) / 1e6 / hbm},
            "attention_roofline": {"bound": "hbm",
                                   "achieved": attn_bytes / (attn_ms / 1000.0) / 1e9,
                                   "peak": hbm, "unit": "GB/s",
                                   "frac": attn_bytes / (attn_ms / 1000.0) / 1e9 / hbm,
                                   "ms_per_step": attn_ms / K}}


def cpu_config4(img):
    import oracle
    threads = min(4, oracle.cpu_cores())
    rate = oracle.bench_decode(img, 30000, 1, threads, threads)
    return {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{threads} sequences x 1 decode token from context 30,000 on {threads} "
                      "host threads, oracle/ C restatement"}


def int8_peak(local):
    """A dense int8 GEMM through the library path torch exposes (cuBLASLt,
    torch._int_mm, 8192^3), best of 10 CUDA-event timings: the int8 tensor
    roofline beside the contraction's achieved rate."""
    import torch
    try:
        a = torch.randint(-64, 64, (8192, 8192), dtype=torch.int8, device="cuda")
        b = torch.randint(-64, 64, (8192, 8192), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a, b)
        best = None
        for _ in range(10):
            with Events(torch.cuda.current_stream()) as ev:
                torch._int_mm(a, b)
            ms = ev.ms()
            best = ms if best is None else min(best, ms)
        return {"tops": 2 * 8192 ** 3 / (best * 1e-3) / 1e12,
                "method": "torch._int_mm (cuBLASLt) int8 8192^3, best of 10, CUDA events"}
    except Exception as exc:  # noqa: BLE001
        return {"tops": None, "method": f"unavailable: {exc}"}


# --------------------------------------------------------- single operators

def run_op(args):
    """One operator through the C ABI on seeded synthetic device inputs: 3
    untimed calls, then the mean of 10 timed with CUDA events.  The qmatvec
    operator includes its per-call tile-image build and activation quantization."""
    import ctypes
    import torch
    from promptboot_b200 import _lib
    lib = _lib.load()
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    g = torch.Generator(device="cuda").manual_seed(7)
    rows = args.op_rows
    if args.op == "attention":
        cap = (args.op_positions + 11) // 4 * 4
        kv = torch.randn(rows * 24 * 4 * cap * 64, device="cuda", generator=g) * 0.5
        q = torch.randn(rows, 896, device="cuda", generator=g)
        out = torch.empty(rows, 896, device="cuda")
        pos = (ctypes.c_uint32 * rows)(*([args.op_positions - 1] * rows))
        call = lambda: lib.pb_attention_device(P(q), P(kv), cap, 0, pos, rows, 0, P(out), None, None)
        desc = {"rows": rows, "positions": args.op_positions}
    else:
        m, k = (int(v) for v in args.op_shape.split("x"))
        bpb = 18 if args.op_wtype == 2 else 34
        nb = m * k // 32
        rng = np.random.default_rng(7)
        w = rng.integers(0, 256, (nb, bpb), dtype=np.uint8)
        w[:, :2] = (np.abs(rng.standard_normal(nb) * 0.02) / 8).astype(np.float16).view(np.uint8).reshape(nb, 2)
        w = torch.from_numpy(w.reshape(-1)).cuda()
        x = torch.randn(rows, k, device="cuda", generator=g)
        y = torch.empty(rows, m, device="cuda")
        call = lambda: lib.pb_qmatvec_device(args.op_wtype, P(w), m, k, P(x), rows, P(y), None)
        desc = {"rows": rows, "shape": args.op_shape, "wtype": args.op_wtype}
    for _ in range(3):
        if call() != 0:
            raise RuntimeError(f"{args.op} failed: {lib.pb_last_error_string()}")
    torch.cuda.synchronize()
    with Events(torch.cuda.current_stream()) as ev:
        for _ in range(10):
            call()
    print(json.dumps({"op": args.op, **desc, "ms_per_call": ev.ms() / 10}), flush=True)


# ---------------------------------------------------------------- drivers

def run_reference(args, world, rank):
    """The reference arm: the decode arithmetic on the host cores (oracle/ C
    restatement) at the same stratified contexts as the timed GPU steps, one
    sequence per host thread, one token per thread per step."""
    if rank != 0:
        return
    import oracle
    from promptboot_b200 import pbtqw25
    img = pbtqw25.load_or_synthesize(0)
    cores = oracle.cpu_cores()
    positions = [args.prompt + t for t in strata(args.warmup, args.decode - 3, args.steps)]
    for _ in range(max(args.warmup, 1)):
        oracle.bench_decode(img, positions[0], 1, cores, cores)
    rates = [oracle.bench_decode(img, p, 1, cores, cores) for p in positions]
    value = len(rates) / sum(1.0 / r for r in rates)
    sample = (f"{cores} sequences (one per host thread) x 1 decode token at each of the "
              f"{len(positions)} timed contexts {positions[0]}..{positions[-1]}, "
              f"oracle/ C restatement (-O3 -mavx2)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cores / value * 1000.0, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8xint4->f32/f64",
            "data": "synthetic (seeded random-init weights, uniform random prompts)",
            "config": {"workload": "config 3 batched decode (CPU sample)", "seqs": cores,
                       "timed_positions": positions},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import torch
    torch.cuda.set_device(local)
    img = model_image(rank, world)
    line = run_config3(args, world, rank, local, img)
    extras = {}
    if not args.no_extra_configs:
        extras["config4"] = run_config4(img, local, rank, world)
    if rank == 0:
        if not args.no_cpu_baseline and world == 1:
            positions = [args.prompt + t for t in strata(args.warmup, args.decode - 3, 4)]
            line["cpu_baseline"] = cpu_config3(img, positions, args.cpu_tokens)
        else:
            line["cpu_baseline"] = None
        if not args.no_extra_configs and world == 1:
            extras["config0"] = run_config0(img, local)
            extras["config1_sampler"] = run_config1(local)
            extras["config2_sweep"] = run_config2(img, local)
            extras["int8_tensor_peak_measured"] = int8_peak(local)
            if not args.no_cpu_baseline:
                extras["config0"]["cpu_baseline"] = cpu_config0(img)
                extras["config1_sampler"]["cpu_baseline"] = cpu_config1()
                extras["config2_sweep"]["cpu_baseline"] = cpu_config2(img)
                extras["config4"]["cpu_baseline"] = cpu_config4(img)
        line.update(extras)
        print(json.dumps(line), flush=True)
    return line


def main():
    args = parse()
    if args.op == "matvec-sweep":
        from promptboot_b200 import pbtqw25
        print(json.dumps(run_config2(pbtqw25.load_or_synthesize(0), 0)), flush=True)
        return
    if args.op == "sampler":
        print(json.dumps(run_config1(0)), flush=True)
        return
    if args.op == "decode1":
        from promptboot_b200 import pbtqw25
        print(json.dumps(run_config0(pbtqw25.load_or_synthesize(0), 0)), flush=True)
        return
    if args.op == "longctx":
        from promptboot_b200 import pbtqw25
        print(json.dumps(run_config4(pbtqw25.load_or_synthesize(0), 0, 0, 1,
                                     K=max(1, min(args.steps, 8)), warmup=1)), flush=True)
        return
    if args.op:
        run_op(args)
        return
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
