#!/usr/bin/env python3
"""Benchmark: greedy decode tokens/s of the ragged continuous-batching engine.

Workload (BASELINE configuration 3 shape, full-size decoder, one B200 per rank):
64 utterances per GPU with T_enc drawn from 5-30 s of audio (8x-subsampled
frames) and EOS forced at a drawn length of 20-220 generated tokens, from
seeded N(0, 1) encoder outputs and seeded random-init bf16 decoder weights
(there is no network for checkpoints or audio).  One bench step = submit the
64 utterances, decode all of them to their forced EOS (prefill + packed decode
steps), collect the tokens.

  value  generated tokens / device time of all engine GPU work (cross-K/V
         projection + step graphs, CUDA events on the engine stream), inputs
         resident; max over ranks; N ranks each run the same per-GPU workload.
  e2e    the same count / wall time through the C ABI from host buffers:
         ct_engine_submit_encoded (H2D of the fp32 encoder rows) + run + poll
         (D2H of the tokens), every step.

`--impl reference` times the reference's own CPU implementation (its
backends/cpu/backend.c driven by its model.h, prebuilt under oracle/_ref/) on
a bounded sample of the same workload with one utterance per host thread.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))

METRIC = "decode tokens/s (ragged continuous batch, greedy)"
BATCH = 64


def workload(seed: int = 0, batch: int = BATCH):
    import inputs
    case = inputs.ragged_decode_case(batch, seed=seed, t_lo=5.0, t_hi=30.0, l_lo=20, l_hi=220)
    enc = inputs.enc_outputs(case["T_enc"], case["enc_seed"])
    return case, enc


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier_max(world, value: float) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch
        import torch.distributed as dist
        dist.barrier()
        torch.cuda.synchronize()


class ReferenceCPU:
    """The reference's CPU decode (its model.h driving its backends/cpu/backend.c,
    prebuilt as oracle/_ref/libref_decode_cpu.so) on a bounded sample of the
    workload: the first n_threads utterances (one per host thread, as
    run_files_parallel does with one CPU "device" per core), each decoded to
    min(its forced length, cap) tokens, cross K/V precompute and 10-row
    prefill included.  Rate = generated tokens / wall seconds."""

    def __init__(self, case, enc, n_threads: int, cap: int):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import inputs as _in
        import pyoracle as po
        self.po = po
        W = importlib.import_module("cohere-transcribe_b200.weights")
        L = po.ref_lib("libref_decode_cpu.so")
        if L is None:
            raise RuntimeError("oracle/_ref/libref_decode_cpu.so not built (build() with the reference tree)")
        self.L = po.bind_ref_decode(L)
        self.wb = W.make_blob(W.FULL_DIMS, seed=0, parts=("dec",))
        self.ws = W.weights_struct(self.wb)
        self.L.refh_bind_weights(ctypes.addressof(self.ws))
        n = n_threads
        idx = np.arange(n) % len(case["T_enc"])
        self.n = n
        self.T_enc = np.ascontiguousarray(case["T_enc"][idx], dtype=np.int32)
        self.Tm = int(self.T_enc.max())
        self.enc = np.ascontiguousarray(enc[idx, :self.Tm], dtype=np.float32)
        self.forced = np.ascontiguousarray(np.minimum(case["forced_len"][idx], cap), dtype=np.int32)
        self.prompt = np.array(_in.ctb.PROMPT_FULL, np.int32)
        self.sample = (f"first {n} utterances of the workload (T_enc {int(self.T_enc.min())}-{int(self.T_enc.max())}),"
                       f" each cross-K/V + 10-token prefill + greedy decode to min(forced length, {cap}) tokens"
                       f" ({int(self.forced.sum())} tokens), one utterance per host thread")

    def run(self):
        po = self.po
        tokens = np.zeros((self.n, 1024), np.int32)
        n_tok = np.zeros(self.n, np.int32)
        secs = self.L.refh_parallel_decode(self.n, self.n, po.fp(self.enc), po.ip(self.T_enc), self.Tm,
                                           po.ip(self.prompt), len(self.prompt), po.ip(self.forced),
                                           po.ip(tokens), po.ip(n_tok))
        return int(self.forced.sum()), secs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=32, help="token cap per utterance of the CPU sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--precision", type=int, default=1)
    ap.add_argument("--batch", type=int, default=BATCH, help="utterances per GPU per step (profiling cases)")
    ap.add_argument("--kv-pages", type=int, default=0, help="page-pool size (0 = engine default)")
    ap.add_argument("--max-len", type=int, default=0, help="cap the forced lengths (profiling cases)")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel-class profiling pass")
    ap.add_argument("--no-pdl", action="store_true", help="launch step kernels without programmatic dependent launch")
    args = ap.parse_args()

    world, rank, local = dist_setup(args.gpus)
    pk, pk_kind = peaks()
    case, enc = workload(0, args.batch)
    if args.max_len > 0:
        case["forced_len"] = np.minimum(case["forced_len"], args.max_len).astype(np.int32)
    nb = args.batch
    tokens_per_step = int(case["forced_len"].sum())
    ncores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)

    cfg = {"workload": f"config 3 shape: {nb} ragged utterances/GPU, T_enc from U(5,30) s, EOS forced at U{{20..220}}",
           "global_batch": nb * world, "decoder": "8 x 1024, 8 heads, FFN 4096, vocab 16384 (model.h dims)",
           "tokens_per_step_per_gpu": tokens_per_step, "prompt_tokens": 10,
           "kv": "bf16 pages of 16 rows", "l2": "not flushed: per-step working set (268 MB weights + KV) > 126 MB L2",
           "parallelism": f"replicas x{world} (utterance sharding, no collective)"}

    if args.impl == "reference":
        if rank != 0:
            return
        ref = ReferenceCPU(case, enc, ncores, args.cpu_tokens)
        for _ in range(args.warmup):
            ref.run()
        toks, secs = 0, 0.0
        for _ in range(args.steps):
            t, s = ref.run()
            toks += t
            secs += s
        v = toks / secs
        line = {"metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1000.0 / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
                "data": "synthetic", "config": cfg,
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": ncores, "kind": "reference",
                                 "sample": ref.sample},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    abi = importlib.import_module("cohere-transcribe_b200.abi")
    W = importlib.import_module("cohere-transcribe_b200.weights")
    lib = abi.load()
    wb = W.make_blob(W.FULL_DIMS, seed=0, parts=("dec",))
    ws = W.weights_struct(wb)
    dev = local if world > 1 else 0
    eng = abi.Engine(lib, dev, wb, ws, max_slots=256, max_rows=1024, precision=args.precision,
                     kv_pages=args.kv_pages, no_pdl=int(args.no_pdl))
    # host inputs: the encoder rows of every utterance (fp32, host memory)
    enc_rows = [np.ascontiguousarray(enc[b, :case["T_enc"][b]]) for b in range(nb)]
    h2d = int(sum(x.nbytes for x in enc_rows))
    d2h = int(4 * tokens_per_step)

    def one_step(e, step_times):
        for b in range(nb):
            e.submit(b, enc_rows[b], int(case["forced_len"][b]))
        while True:
            s0 = e.stats()["step_ms"]
            left = e.step(1)
            step_times.append(e.stats()["step_ms"] - s0)
            if left <= 0:
                break
        out = e.poll()
        assert len(out) == nb
        return out

    for _ in range(args.warmup):
        one_step(eng, [])
    if eng.status() != 0:
        raise RuntimeError("device status set during warm-up")
    barrier(world)
    s0 = eng.stats()
    step_times = []
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            one_step(eng, step_times)
        wall = time.perf_counter() - t0
    s1 = eng.stats()
    barrier(world)
    status = eng.status()
    eng.close()
    dev_ms = (s1["step_ms"] - s0["step_ms"]) + (s1["admit_ms"] - s0["admit_ms"])
    dev_ms_max = barrier_max(world, dev_ms)
    wall_max = barrier_max(world, wall)
    tokens = tokens_per_step * args.steps * world
    value = tokens / (dev_ms_max / 1000.0)
    e2e = tokens / wall_max
    dt = {k: s1[k] - s0[k] for k in s1}

    # Per-kernel-class device times: one more bench step on an engine whose step
    # graphs carry CUDA event nodes around the attention and FFN launches of
    # every layer (kept out of the timed run: event nodes serialise neighbours).
    if not args.no_profile:
        prof = abi.Engine(lib, dev, wb, ws, max_slots=256, max_rows=1024, precision=args.precision,
                          kv_pages=args.kv_pages, profile=1)
        one_step(prof, [])
        p0 = prof.stats()
        r0 = prof.profile_report()
        one_step(prof, [])
        p1 = prof.stats()
        r1 = prof.profile_report()
        prof.close()
        breakdown = {k: {"ms_per_step": (v[0] - r0.get(k, [0, 0])[0]) / max(1, p1["steps"] - p0["steps"]),
                         "launch_groups_per_step": (v[1] - r0.get(k, [0, 0])[1]) / max(1, p1["steps"] - p0["steps"])}
                     for k, v in r1.items()}
        d = {k: p1[k] - p0[k] for k in p1}
    else:
        d = {k: 0.0 for k in dt}
        breakdown = {}
    classes = {
        "paged cross-attention": (d["cross_attn_ms"], d["cross_kv_bytes"]),
        "paged self-attention": (d["self_attn_ms"], d["self_kv_bytes"]),
        "FFN GEMMs (tcgen05)": (d["ffn_ms"], d["ffn_bytes"]),
    }
    dom = max(classes, key=lambda k: classes[k][0])
    ms, byts = classes[dom]
    launches = d["steps"] * 8 * (2 if "GEMM" in dom else 1)
    achieved = (byts / (ms / 1000.0)) / 1e9 if ms > 0 else 0.0
    traffic = None
    tpath = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as fh:
            traffic = json.load(fh).get(dom)
    roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "peak_kind": pk_kind, "traffic": traffic,
            "algorithmic_bytes_per_launch": byts / max(1, launches), "avg_launch_ms": ms / max(1, launches),
            "measured": "CUDA event nodes around every launch of the class in one profiled bench step"}
    shares = {k: v[0] / max(1e-9, d["step_ms"]) for k, v in classes.items()}

    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "p50_step_ms": statistics.median(step_times) if step_times else None,
            "decode_steps_per_bench_step": dt["steps"] / args.steps,
            "admit_ms_per_step": dt["admit_ms"] / args.steps,
            "gpu_launches": int(dt["kernel_launches"]),
            "roofline": roof, "time_shares": shares, "profiled_step_breakdown": breakdown, "clocks": clk.summary(), "device_status": status,
            "precision": "bf16 weights, activations as bf16 hi+lo planes, fp32 accumulate" if args.precision else
            "bf16 weights and activations, fp32 accumulate"}
    if rank == 0 and world == 1 and not args.no_cpu:
        ref = ReferenceCPU(case, enc, ncores, args.cpu_tokens)
        t, s = ref.run()
        line["cpu_baseline"] = {"value": t / s, "unit": "tokens/s", "cores": ncores, "kind": "reference",
                                "sample": ref.sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
