#!/usr/bin/env python3
"""Benchmark: decode tokens/s, RTFx and p50 step latency of the engine.

Workload (full-size model, one B200 per rank): 64
utterances per GPU of U(5, 30) s of seeded 16 kHz test signals (a few tones
plus noise), EOS forced at U{20..220} generated tokens, seeded random-init bf16
weights (there is no network for checkpoints or audio).  With N GPUs the job
is 64 * N utterances, dispatched to the ranks by queued audio seconds
(cohere-transcribe_b200/dispatch.py); each rank runs its own engine on its
shard, with no collective on the data path (NCCL carries only the barrier and
the max / sum of the timings).

One bench step runs three legs (A and B over that batch, C alone):

  A  decode: submit the 64 utterances' encoder rows (host fp32, seeded
     N(0, 1)), decode all to their forced EOS, poll the tokens.
       value  generated tokens / device time of the engine's GPU work (cross-K/V
              projection into pages + packed step graphs; CUDA events on the
              engine stream), inputs resident; summed over ranks / max time.
       e2e    the same count / wall time of the C-ABI calls from host buffers
              (H2D of the encoder rows, D2H of the tokens), every step.
       p50_step_ms  median device time of one packed decode step.
  B  transcribe: submit the 64 utterances as 16 kHz samples
     (ct_engine_submit_audio); the engine computes their log-mel on the GPU,
     encodes them as one packed ragged batch (48 Conformer layers), admits and
     decodes them; poll the tokens.
       rtfx.value  audio seconds / device time (front-end + encoder + admission + decode)
       rtfx.e2e    audio seconds / wall time of the C-ABI calls from host samples
  C  configuration 2 (batch 1): one 30 s utterance of seeded N(0, 1) log-mel
     (ct_engine_submit_mel), encoded, admitted and decoded alone to EOS forced
     at the 200th token; reported under "config2" (p50 step latency at batch 1,
     decode tokens/s, RTFx), beside the configuration-3 headline.
  S  (optional, not in the default legs) configuration 4: a stream of
     --stream-n utterances of seeded log-mel with Poisson arrivals at 200/s
     (or all at t = 0 with --stream-saturated), log-normal lengths, 3 tokens
     per audio second, replayed in real time by cohere-transcribe_b200/stream.py
     after the timed legs; reported under "config4" (latency p50 / p95, tokens/s,
     RTFx over the stream's wall time).  --stream-config 5 replays configuration
     5 instead (32768 utterances at 1600/s plus 64 five-minute inputs as 30 s /
     29 s-hop windows), each rank its share by queued audio seconds; reported
     under "config5" with tokens and audio summed over ranks and the worst
     rank's wall time.

Precision: the headline runs --precision 0, bf16 weights and bf16 activations
with fp32 accumulation (the configurations' "bf16 weights with fp32
accumulate").  On one GPU legs A and B then run once more at the other
precision (--precision 1: activations carried as bf16 hi + lo planes, close to
fp32) on a fresh engine, reported under "precision_compare".

`--impl reference` times the reference's own CPU implementation (its
backends/cpu/backend.c driven by its model.h, prebuilt under oracle/_ref/) on
bounded samples of the same workload, one utterance per host thread: greedy
decode from the same encoder rows (tokens/s), and full transcription
(log-mel front-end + encoder + decode) of 1 s cuts of the audio (RTFx).
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

METRIC = "decode tokens/s and RTFx per B200 (ragged continuous batch); p50 step latency"
BATCH = 64
CPU_CUT_S = 1.0        # seconds of log-mel per utterance in the CPU transcription sample
CPU_CUT_TOKENS = 8     # generated-token cap per utterance in the CPU transcription sample
CFG2_SECONDS, CFG2_TOKENS = 30.0, 200   # configuration 2: one 30 s utterance, EOS forced at the 200th token
CUDA_REF_SAMPLE = 16   # utterances in the reference CUDA backend's decode sample

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one ncu capture
# per kernel class, on a smaller case than the bench's, with the units that
# capture processed.  The bench scales it to its own launches by units, for the
# classes whose traffic grows in proportion to them.
NCU_TRAFFIC = {
    # profiles/attn_paged_decode.md: one cross launch, 64 rows over 14,080
    # encoder keys (57,671,680 algorithmic bytes): 59.356672 MB read + 0.566016 MB
    # written.  Unit: algorithmic byte (the K/V rows the launch must read).
    "paged cross-attention": {"bytes": 59.356672e6 + 0.566016e6, "units": 14080 * 4096.0,
                              "unit": "algorithmic byte", "source": "profiles/attn_paged_decode.md"},
    # profiles/gemm_decode_ffn_lmhead.md: one layer's FFN1 + FFN2 at 64 rows,
    # bf16 activations (17,432,576 algorithmic bytes): 8.759552 + 9.262848 MB
    # read, 0 written.  Unit: algorithmic byte (weights + activations of the
    # two launches).
    "decode FFN GEMMs (tcgen05)": {"bytes": 8.759552e6 + 9.262848e6, "units": 17432576.0,
                                   "unit": "algorithmic byte", "source": "profiles/gemm_decode_ffn_lmhead.md"},
    # profiles/gemm_persistent_encoder_ffn1.md: layer 0's FFN1 over 3,545 packed
    # rows: 31.509504 MB read + 24.338688 MB written.  Unit: packed row.  The
    # 13.1 MB of weights do not grow with the rows, so the scaled figure is an
    # upper bound at larger batches.
    "encoder FFN1 GEMM (tcgen05, persistent)": {"bytes": 31.509504e6 + 24.338688e6, "units": 3545.0,
                                                "unit": "packed row",
                                                "source": "profiles/gemm_persistent_encoder_ffn1.md"},
}


# Sharding weight of a generated token against an audio second: on one B200
# the packed encoder takes ~0.059 ms per audio second (65 ms for 1,110 s) and
# a 64-sequence decode step ~0.0102 ms per sequence (0.653 ms), so about 6
# generated tokens cost as much as one second of audio.
DECODE_TOKENS_PER_AUDIO_S = 6.0


def workload(seed: int = 0, batch: int = BATCH, rank: int = 0, world: int = 1):
    """Configuration 3: seconds ~ U(5, 30), forced lengths ~ U{20..220}; log-mel
    N(0, 1) [128, 100 s + 1] per utterance; encoder rows N(0, 1) [T_enc, 1024].
    With world > 1 the job is batch * world utterances, dispatched least
    queued work first, where an utterance's work is its audio seconds plus its
    forced token count / DECODE_TOKENS_PER_AUDIO_S (the forced lengths are
    drawn independently of the durations, so audio seconds alone would leave
    the ranks' decode work unequal); this rank's shard is returned (inputs
    seeded per utterance, so a shard is generated alone)."""
    import inputs
    disp = importlib.import_module("cohere-transcribe_b200.dispatch")
    full = inputs.ragged_decode_case(batch * world, seed=seed, t_lo=5.0, t_hi=30.0, l_lo=20, l_hi=220)
    work = full["seconds"] + full["forced_len"] / DECODE_TOKENS_PER_AUDIO_S
    idx = np.array([i for i, _ in disp.shard(list(range(batch * world)), work, rank, world)], np.int64)
    case = {k: (v[idx] if isinstance(v, np.ndarray) else v) for k, v in full.items()}
    case["index"] = idx
    T_enc = case["T_enc"]
    enc = np.zeros((len(idx), int(T_enc.max()), 1024), np.float32)
    for j, (i, t) in enumerate(zip(idx, T_enc)):
        rng = np.random.default_rng([full["enc_seed"], int(i)])
        enc[j, :t] = rng.standard_normal((int(t), 1024), dtype=np.float32)
    T_mel = np.array([inputs.ctb.t_mel_of_seconds(x) for x in case["seconds"]], np.int32)
    # 16 kHz signals (a few tones plus noise) of the drawn durations
    audio = [inputs.audio(float(x), 10_000 * (seed + 1) + int(i)) for i, x in zip(idx, case["seconds"])]
    case["T_mel"] = T_mel
    return case, enc, audio


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


def dist_setup():
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


def all_reduce(world, value: float, op: str) -> float:
    """Max or sum over ranks (host-side bookkeeping; no collective touches the data path)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch
        import torch.distributed as dist
        dist.barrier()
        torch.cuda.synchronize()


class ReferenceCPU:
    """The reference's CPU path (its model.h driving its backends/cpu/backend.c,
    prebuilt as oracle/_ref/libref_decode_cpu.so) on bounded samples of the
    workload, one utterance per host thread (as run_files_parallel does with one
    CPU "device" per core):
      decode      the n_threads utterances nearest the workload's mean forced
                  length and mean T_enc: cross K/V + 10-row prefill + greedy
                  decode from the workload's encoder rows to each utterance's
                  forced length (cap > 0 caps it) -> tokens/s.  The sample's
                  tokens per utterance then average the workload's, so the
                  per-utterance cross-K/V and prefill cost is spread over as
                  many tokens as in the GPU run.
      transcribe  encoder + decode of the first CPU_CUT_S seconds of each
                  utterance's log-mel, to min(forced, CPU_CUT_TOKENS) tokens
                  -> RTFx (audio seconds / wall seconds)."""

    def __init__(self, case, enc, audio, n_threads: int, cap: int):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import inputs as _in
        import pyoracle as po
        self.po = po
        W = importlib.import_module("cohere-transcribe_b200.weights")
        L = po.ref_lib("libref_decode_cpu.so")
        if L is None:
            raise RuntimeError("oracle/_ref/libref_decode_cpu.so not built (build() with the reference tree)")
        self.L = po.bind_ref_decode(L)
        self.wb = W.make_blob(W.FULL_DIMS, seed=0)
        self.ws = W.weights_struct(self.wb)
        self.L.refh_bind_weights(ctypes.addressof(self.ws))
        n = n_threads
        f_all, te_all = case["forced_len"].astype(np.float64), case["T_enc"].astype(np.float64)
        # distance to the means, the forced length weighted 3x: the threads then
        # finish close together (wall time = the longest thread)
        near = 3.0 * np.abs(f_all - f_all.mean()) / f_all.mean() + np.abs(te_all - te_all.mean()) / te_all.mean()
        idx = np.resize(np.argsort(near, kind="stable"), n)
        self.n = n
        self.T_enc = np.ascontiguousarray(case["T_enc"][idx], dtype=np.int32)
        self.Tm = int(self.T_enc.max())
        self.enc = np.ascontiguousarray(enc[idx, :self.Tm], dtype=np.float32)
        forced = case["forced_len"][idx]
        self.forced = np.ascontiguousarray(np.minimum(forced, cap) if cap > 0 else forced, dtype=np.int32)
        self.workload_mean_tokens = float(f_all.mean())
        self.prompt = np.array(_in.ctb.PROMPT_FULL, np.int32)
        cut = _in.ctb.t_mel_of_seconds(CPU_CUT_S)
        self.T_mel_cut = np.full(n, cut, np.int32)
        self.audio_cut = [np.ascontiguousarray(audio[i][:int(CPU_CUT_S * 16000)]) for i in idx]
        self.M = ctypes.CDLL(os.path.join(po.REF_DIR, "libref_mel.so"))
        self.M.refmel_compute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        self.forced_cut = np.ascontiguousarray(np.minimum(case["forced_len"][idx], CPU_CUT_TOKENS), dtype=np.int32)
        self.sample = (f"{n} utterances of the workload nearest its mean forced length and mean T_enc (T_enc "
                       f"{int(self.T_enc.min())}-{int(self.T_enc.max())}, mean {self.T_enc.mean():.0f}; forced "
                       f"{int(self.forced.min())}-{int(self.forced.max())} tokens, mean {self.forced.mean():.0f} "
                       f"against the workload's {self.workload_mean_tokens:.0f}), each cross-K/V + 10-token prefill"
                       f" + greedy decode to its forced length" + (f" capped at {cap}" if cap > 0 else "") +
                       f" ({int(self.forced.sum())} tokens), one utterance per host thread")
        self.sample_rtfx = (f"first {n} utterances of the workload cut to their first {CPU_CUT_S:g} s of audio,"
                            f" each log-mel front-end + encoder (48 layers) + prefill + greedy decode to"
                            f" {CPU_CUT_TOKENS} tokens, one utterance per host thread")

    def decode(self, warm: bool = False):
        """One timed sample (tokens, seconds).  warm: a short untimed pass (two
        tokens per thread on the shortest encoder rows) that pages in the code
        and the weights."""
        po = self.po
        tokens = np.zeros((self.n, 1024), np.int32)
        n_tok = np.zeros(self.n, np.int32)
        forced, T_enc, Tm, enc = self.forced, self.T_enc, self.Tm, self.enc
        if warm:
            forced = np.full(self.n, 2, np.int32)
            T_enc = np.full(self.n, int(self.T_enc.min()), np.int32)
            Tm = int(T_enc[0])
            enc = np.ascontiguousarray(self.enc[:, :Tm])
        secs = self.L.refh_parallel_decode(self.n, self.n, po.fp(enc), po.ip(T_enc), Tm,
                                           po.ip(self.prompt), len(self.prompt), po.ip(forced),
                                           po.ip(tokens), po.ip(n_tok))
        return int(forced.sum()), secs

    def transcribe(self):
        po = self.po
        tokens = np.zeros((self.n, 1024), np.int32)
        n_tok = np.zeros(self.n, np.int32)
        t0 = time.perf_counter()
        mel = np.zeros((self.n, 128, int(self.T_mel_cut[0])), np.float32)
        for b, x in enumerate(self.audio_cut):   # the reference front-end (one host thread)
            self.M.refmel_compute(x.ctypes.data, len(x), mel[b].ctypes.data)
        secs = time.perf_counter() - t0
        secs += self.L.refh_parallel_transcribe(self.n, self.n, po.fp(mel), int(self.T_mel_cut[0]),
                                                po.ip(self.T_mel_cut), po.ip(self.prompt), len(self.prompt),
                                                po.ip(self.forced_cut), po.ip(tokens), po.ip(n_tok))
        return self.n * CPU_CUT_S, secs


class ReferenceCUDA:
    """The reference's own CUDA backend on this GPU: backends/cuda/backend.cu
    compiled from the reference sources for sm_100a (oracle/Makefile
    `ref-cuda`), driven by the reference's model.h decode loop through
    oracle/ref_harness.c -- the kernels this repository replaces, on the same
    B200 and inputs.  Measured on bounded samples (wall time of the harness
    call: encoder-row upload, cross K/V precompute, per-utterance prefill and
    the batched decode loop with its host argmax, as model.h runs them):
      decode    the n utterances of the workload nearest its mean forced length
                and mean T_enc (the CPU sample's rule), decoded together to
                their forced lengths -> tokens/s;
      config2   one 30 s utterance's encoder rows (T_enc 376), 200 tokens at
                batch 1 -> tokens/s and ms per token."""

    def __init__(self, ws, case, enc, n: int):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import pyoracle as po
        self.po = po
        L = po.ref_lib("libref_decode_cuda.so")
        self.L = po.bind_ref_decode(L) if L is not None else None
        self.ws = ws
        f_all, te_all = case["forced_len"].astype(np.float64), case["T_enc"].astype(np.float64)
        near = 3.0 * np.abs(f_all - f_all.mean()) / f_all.mean() + np.abs(te_all - te_all.mean()) / te_all.mean()
        idx = np.sort(np.argsort(near, kind="stable")[:n])
        self.T_enc = np.ascontiguousarray(case["T_enc"][idx], dtype=np.int32)
        self.Tm = int(self.T_enc.max())
        self.enc = np.ascontiguousarray(enc[idx, :self.Tm], dtype=np.float32)
        self.forced = np.ascontiguousarray(case["forced_len"][idx], dtype=np.int32)
        self.sample = (f"{len(idx)} utterances of the workload nearest its mean forced length and mean T_enc "
                       f"(T_enc {int(self.T_enc.min())}-{self.Tm}, forced {int(self.forced.min())}-"
                       f"{int(self.forced.max())} tokens, {int(self.forced.sum())} in all) decoded as one batch")

    def _decode(self, wb, enc, T_enc, forced):
        po, L = self.po, self.L
        import inputs as _in
        B = len(T_enc)
        prompt = np.array(_in.ctb.PROMPT_FULL, np.int32)
        tokens = np.zeros((B, 1024), np.int32)
        n_tok = np.zeros(B, np.int32)
        L.backend_weights_upload_blob(wb.ptr(), wb.nbytes)
        L.refh_bind_weights(ctypes.addressof(self.ws))
        L.backend_init(0)
        secs = L.refh_decode_from_enc(B, po.fp(enc), po.ip(T_enc), enc.shape[1], po.ip(prompt), len(prompt),
                                      po.ip(forced), po.null_i(), po.ip(tokens), po.ip(n_tok), po.null_i(),
                                      po.null_f())
        L.backend_destroy()
        return int(forced.sum()), secs

    def run(self, wb):
        if self.L is None:
            return None
        t, s_ = self._decode(wb, self.enc, self.T_enc, self.forced)
        enc2 = np.random.default_rng([0, 620]).standard_normal((1, 376, 1024), dtype=np.float32)
        t2, s2 = self._decode(wb, enc2, np.array([376], np.int32), np.array([CFG2_TOKENS], np.int32))
        return {"value": t / s_, "unit": "tokens/s", "kind": "reference CUDA backend (backends/cuda/backend.cu, "
                "sm_100a) on this B200", "sample": self.sample, "sample_tokens": t,
                "config2": {"tokens_per_s": t2 / s2, "ms_per_token": 1000.0 * s2 / t2,
                            "sample": f"one utterance of T_enc 376 (30 s) from encoder rows, {t2} tokens"}}


def config2_summary(dev, wall_s, step_times, K):
    """Configuration 2 (batch 1, one 30 s utterance, 200 tokens) from K timed runs:
    device times from the engine's CUDA events (encoder, admission, steps),
    wall time of the C-ABI calls from the host log-mel to the polled tokens."""
    dec_ms = dev["admit_ms"] + dev["step_ms"]
    all_ms = dec_ms + dev["enc_ms"]
    return {"workload": f"config 2: one {CFG2_SECONDS:g} s utterance of seeded N(0, 1) log-mel, batch 1, "
                        f"EOS forced at token {CFG2_TOKENS}",
            "p50_step_ms": statistics.median(step_times) if step_times else None,
            "steps_per_run": len(step_times) // K if K else None,
            "decode_tokens_per_s": CFG2_TOKENS * K / (dec_ms / 1000.0) if dec_ms > 0 else None,
            "rtfx": CFG2_SECONDS * K / (all_ms / 1000.0) if all_ms > 0 else None,
            "e2e_rtfx": CFG2_SECONDS * K / wall_s if wall_s > 0 else None,
            "encoder_ms": dev["enc_ms"] / K, "decode_ms": dec_ms / K, "wall_ms": 1000.0 * wall_s / K}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=0,
                    help="token cap per utterance of the CPU decode sample (0 = each utterance's forced length)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-cuda-ref", action="store_true", help="skip the reference CUDA backend leg")
    ap.add_argument("--precision", type=int, default=0, choices=[0, 1],
                    help="0: bf16 activations (the configurations' bf16 / fp32-accumulate contract); "
                         "1: activations as bf16 hi+lo planes (near-fp32 activations)")
    ap.add_argument("--no-compare-precision", action="store_true",
                    help="skip timing legs A and B once more at the other precision (one GPU only)")
    ap.add_argument("--batch", type=int, default=BATCH, help="utterances per GPU per step (profiling cases)")
    ap.add_argument("--kv-pages", type=int, default=0, help="page-pool size (0 = engine default)")
    ap.add_argument("--max-len", type=int, default=0, help="cap the forced lengths (profiling cases)")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel-class profiling pass")
    ap.add_argument("--no-pdl", action="store_true", help="launch step kernels without programmatic dependent launch")
    ap.add_argument("--fused-step", type=int, default=0, choices=[0, 1],
                    help="1 = each decode step as one persistent kernel (0 = separate kernels)")
    ap.add_argument("--legs", default="ABC", help="A = decode leg, B = transcription leg, C = configuration 2 "
                    "(batch 1), E = encoder only (profiling cases)")
    ap.add_argument("--max-slots", type=int, default=256, help="engine slots (profiling cases)")
    ap.add_argument("--stream-config", type=int, default=4, choices=[4, 5],
                    help="leg S: configuration 4 (one GPU's stream) or 5 (8x the rate plus long-form windows, "
                         "dispatched over the ranks)")
    ap.add_argument("--stream-n", type=int, default=0,
                    help="leg S: utterances in the stream (0 = the configuration's: 4096, or 32768 for 5)")
    ap.add_argument("--stream-saturated", action="store_true", help="leg S: every utterance arrives at t = 0")
    args = ap.parse_args()

    world, rank, local = dist_setup()
    pk, pk_kind = peaks()
    case, enc, audio = workload(0, args.batch, rank, world)
    if args.max_len > 0:
        case["forced_len"] = np.minimum(case["forced_len"], args.max_len).astype(np.int32)
    nb = len(case["T_enc"])
    tokens_per_step = int(case["forced_len"].sum())
    audio_s = float(case["seconds"].sum())
    ncores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)

    cfg = {"workload": f"config 3: {args.batch} ragged utterances/GPU of U(5,30) s log-mel, EOS forced at U{{20..220}}"
                       + (f"; {args.batch * world} utterances dispatched to {world} GPUs by queued audio seconds"
                          if world > 1 else ""),
           "global_batch": args.batch * world, "model": "encoder 48 x 1280 (8 heads, FFN 5120, dw-K 9), decoder 8 x 1024 "
           "(8 heads, FFN 4096, vocab 16384): model.h dims, random-init bf16",
           "prompt_tokens": 10, "kv": "bf16 pages of 16 rows",
           "l2": "not flushed: per-step working sets (3.8 GB encoder weights, 268 MB decoder weights + KV) > 126 MB L2",
           "parallelism": f"replicas x{world} (utterance sharding, no collective)"}

    if args.impl == "reference":
        if rank != 0:
            return
        ref = ReferenceCPU(case, enc, audio, ncores, args.cpu_tokens)
        for _ in range(args.warmup):
            ref.decode(warm=True)
        toks, secs, aud, tsecs = 0, 0.0, 0.0, 0.0
        for _ in range(args.steps):
            t, s_ = ref.decode()
            toks += t
            secs += s_
            a_, s2 = ref.transcribe()
            aud += a_
            tsecs += s2
        v = toks / secs
        line = {"metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": (secs + tsecs) * 1000.0 / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
                "data": "synthetic", "config": cfg,
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": ncores, "kind": "reference",
                                 "sample": ref.sample, "sample_tokens": int(ref.forced.sum()),
                                 "sample_mean_tokens": float(ref.forced.mean()),
                                 "workload_mean_tokens": ref.workload_mean_tokens},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "rtfx": {"value": aud / tsecs, "e2e": aud / tsecs, "unit": "audio s / s", "cores": ncores,
                         "sample": ref.sample_rtfx}}
        print(json.dumps(line), flush=True)
        return

    abi = importlib.import_module("cohere-transcribe_b200.abi")
    W = importlib.import_module("cohere-transcribe_b200.weights")
    lib = abi.load()
    legs = args.legs.upper()
    # the decode leg alone needs no encoder (a decoder-only blob keeps profiling cases small)
    with_enc = "B" in legs or "E" in legs
    with_c = "C" in legs
    with_s = "S" in legs
    wb = W.make_blob(W.FULL_DIMS, seed=0, parts=("enc", "dec") if (with_enc or with_c or with_s) else ("dec",))
    ws = W.weights_struct(wb)
    dev = local if world > 1 else 0
    enc_frames = int(case["T_mel"].sum())
    # configuration 2: one 30 s utterance of seeded N(0, 1) log-mel [128, 3001]
    mel2 = np.random.default_rng([0, 2]).standard_normal(
        (128, importlib.import_module("cohere-transcribe_b200").t_mel_of_seconds(CFG2_SECONDS)), dtype=np.float32)
    if with_c:
        enc_frames = max(enc_frames, int(mel2.shape[1]))
    enc_utts = nb
    if with_s:   # configuration 4 packs encoder batches of up to 64 utterances of up to 30 s
        enc_utts, enc_frames = max(nb, 64), max(enc_frames, 64 * 3001)

    def make_engine(profile=0):
        return abi.Engine(lib, dev, wb, ws, max_slots=args.max_slots, max_rows=1024, precision=args.precision,
                          kv_pages=args.kv_pages, no_pdl=int(args.no_pdl), profile=profile,
                          fused_step=args.fused_step,
                          enc_max_utts=enc_utts if (with_enc or with_c or with_s) else -1,
                          enc_max_frames=enc_frames)

    eng = make_engine()
    # host inputs: encoder rows (leg A) and log-mel (leg B), fp32 host memory
    enc_rows = [np.ascontiguousarray(enc[b, :case["T_enc"][b]]) for b in range(nb)]
    h2d_a = int(sum(x.nbytes for x in enc_rows))
    h2d_b = int(sum(x.nbytes for x in audio))
    d2h = int(4 * tokens_per_step)

    def leg_a(e, step_times):
        for b in range(nb):
            e.submit(b, enc_rows[b], int(case["forced_len"][b]))
        e.step_times()                       # drop earlier steps' times
        e.run()
        step_times.extend(e.step_times().tolist())
        out = e.poll()
        assert len(out) == nb
        return out

    def leg_b(e):
        if "E" in legs:   # encoder only (profiling cases): front-end + one packed encoder batch
            return e.encode(e.log_mel(audio))
        for b in range(nb):
            e.submit_audio(b, audio[b], int(case["forced_len"][b]))
        e.run()
        out = e.poll()
        assert len(out) == nb
        return out

    def leg_c(e, step_times):
        e.step_times()                       # drop earlier steps' times
        e.submit_mel(0, mel2, CFG2_TOKENS)
        e.run()
        step_times.extend(e.step_times().tolist())
        out = e.poll()
        assert len(out) == 1
        return out

    for _ in range(args.warmup):
        if "A" in legs:
            leg_a(eng, [])
        if with_enc:
            leg_b(eng)
        if with_c:
            leg_c(eng, [])
    if eng.status() != 0:
        raise RuntimeError("device status set during warm-up")
    step_times, step_times_c = [], []
    wall_a = wall_b = wall_c = 0.0
    dev_a = dev_b = enc_ms = 0.0
    dev_c = {"enc_ms": 0.0, "admit_ms": 0.0, "step_ms": 0.0}
    barrier(world)
    s_start = eng.stats()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            if "A" in legs:
                s0 = eng.stats()
                t0 = time.perf_counter()
                leg_a(eng, step_times)
                wall_a += time.perf_counter() - t0
                s1 = eng.stats()
                dev_a += (s1["step_ms"] - s0["step_ms"]) + (s1["admit_ms"] - s0["admit_ms"])
            if with_enc:
                s0 = eng.stats()
                t0 = time.perf_counter()
                leg_b(eng)
                wall_b += time.perf_counter() - t0
                s1 = eng.stats()
                dev_b += (s1["step_ms"] - s0["step_ms"]) + (s1["admit_ms"] - s0["admit_ms"]) + \
                    (s1["enc_ms"] - s0["enc_ms"])
                enc_ms += s1["enc_ms"] - s0["enc_ms"]
            if with_c:
                s0 = eng.stats()
                t0 = time.perf_counter()
                leg_c(eng, step_times_c)
                wall_c += time.perf_counter() - t0
                s1 = eng.stats()
                for k in dev_c:
                    dev_c[k] += s1[k] - s0[k]
    barrier(world)
    s_end = eng.stats()
    status = eng.status()
    launches = int(s_end["kernel_launches"] - s_start["kernel_launches"])
    n_steps = s_end["steps"] - s_start["steps"]
    # batch occupancy of the timed region: packed query rows per step (prefill rows included)
    rows_per_step = (s_end["rows"] - s_start["rows"]) / n_steps if n_steps > 0 else None
    config4 = None
    if with_s:   # configuration 4, after the timed legs (its own wall-clock measurement)
        stream = importlib.import_module("cohere-transcribe_b200.stream")
        disp = importlib.import_module("cohere-transcribe_b200.dispatch")
        warm = stream.stream_case(64, seed=1, saturated=True)
        stream.run_stream(eng, warm, inputs=[warm.log_mel(i) for i in range(64)])
        if args.stream_config == 5:
            n_s = args.stream_n or 32768
            full = stream.config5_case(n_s, seed=0)
            if args.stream_saturated:
                full.arrival_s[:] = 0.0
        else:
            n_s = args.stream_n or 4096
            full = stream.stream_case(n_s, seed=0, saturated=args.stream_saturated)
        mine = [i for i, _ in disp.shard(list(range(len(full.seconds))), full.seconds, rank, world)]
        sc = stream.subset(full, mine)
        mels = [sc.log_mel(i) for i in range(len(sc.seconds))]   # generated before the replay starts
        barrier(world)
        res = stream.run_stream(eng, sc, inputs=mels)
        config4 = res.summary()
        if world > 1:   # whole job: tokens and audio summed, wall time and latency tails the worst rank's
            for k in ("utterances", "generated_tokens", "audio_s"):
                config4[k] = all_reduce(world, float(config4[k]), "sum")
            for k in ("wall_s", "latency_p95_s", "latency_max_s"):
                config4[k] = all_reduce(world, float(config4[k]), "max")
            config4["tokens_per_s"] = config4["generated_tokens"] / config4["wall_s"]
            config4["rtfx"] = config4["audio_s"] / config4["wall_s"]
            config4["latency_p50_s"] = f"rank 0: {config4['latency_p50_s']}"
        arrivals = "all arriving at t = 0" if args.stream_saturated else (
            "Poisson arrivals 1600/s" if args.stream_config == 5 else "Poisson arrivals 200/s")
        config4["workload"] = (f"config {args.stream_config}: {n_s} utterances of seeded N(0, 1) log-mel, {arrivals}"
                               ", log-normal lengths (median 8 s, sigma 0.5, 1-30 s), 3 tokens/s of audio "
                               "+-20% with EOS forced, <= 256 concurrent sequences per GPU, encoder batches <= 64"
                               + (", plus 64 x 300 s long-form inputs as 704 windows of 30 s every 29 s at t = 0"
                                  if args.stream_config == 5 else "")
                               + (f"; dispatched to {world} GPUs by queued audio seconds" if world > 1 else ""))
        status = status or eng.status()
    eng.close()

    K = args.steps
    tokens_all = all_reduce(world, float(tokens_per_step * K), "sum")
    audio_all = all_reduce(world, audio_s * K, "sum")
    dev_a_max = all_reduce(world, dev_a, "max")
    wall_a_max = all_reduce(world, wall_a, "max")
    dev_b_max = all_reduce(world, dev_b, "max")
    wall_b_max = all_reduce(world, wall_b, "max")
    value = tokens_all / (dev_a_max / 1000.0) if dev_a_max > 0 else None
    e2e = tokens_all / wall_a_max if wall_a_max > 0 else None

    # Per-kernel-class device times: one more step of each leg on an engine that
    # records CUDA events between launch groups (kept out of the timed run: the
    # event nodes serialise their neighbours).
    breakdown, rooflines = {}, {}
    if not args.no_profile:
        prof = make_engine(profile=1)
        if "A" in legs:
            leg_a(prof, [])
        if with_enc:
            leg_b(prof)
        p0 = prof.stats()
        r0 = prof.profile_report()
        if "A" in legs:
            leg_a(prof, [])
        if with_enc:
            leg_b(prof)
        p1 = prof.stats()
        r1 = prof.profile_report()
        prof.close()
        d = {k: p1[k] - p0[k] for k in p1}
        breakdown = {k: {"ms": v[0] - r0.get(k, [0, 0])[0], "launch_groups": v[1] - r0.get(k, [0, 0])[1]}
                     for k, v in r1.items()}
        # decode kernels (HBM-bound): algorithmic bytes / device time
        for name, ms_, byts, n_l in (("paged cross-attention", d["cross_attn_ms"], d["cross_kv_bytes"], d["steps"] * 8),
                                     ("paged self-attention", d["self_attn_ms"], d["self_kv_bytes"], d["steps"] * 8),
                                     ("decode FFN GEMMs (tcgen05)", d["ffn_ms"], d["ffn_bytes"], d["steps"] * 16)):
            if ms_ > 0:
                ach = byts / (ms_ / 1000.0) / 1e9
                rooflines[name] = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s",
                                   "frac": ach / pk["hbm_gbs"], "ms_per_step": ms_, "launches": n_l,
                                   "algorithmic_bytes_per_launch": byts / max(1, n_l),
                                   "avg_launch_ms": ms_ / max(1, n_l)}
        # encoder FFN1 GEMM (tensor-bound): 2*T*N*K algorithmic flops per launch
        if "enc_gemm_ffn1" in breakdown and breakdown["enc_gemm_ffn1"]["launch_groups"] > 0:
            R3 = int(sum(int(x) for x in case["T_enc"]))
            n_l = breakdown["enc_gemm_ffn1"]["launch_groups"]
            ms_ = breakdown["enc_gemm_ffn1"]["ms"]
            fl = 2.0 * R3 * 5120 * 1280
            ach = fl / (ms_ / n_l / 1000.0) / 1e12
            rooflines["encoder FFN1 GEMM (tcgen05, persistent)"] = {
                "bound": "tensor", "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / pk["bf16_tflops"], "ms_per_step": ms_, "launches": n_l,
                "algorithmic_flops_per_launch": fl, "avg_launch_ms": ms_ / n_l,
                "note": ("activations as bf16 hi+lo planes: the tensor cores execute 2x the algorithmic flops"
                         if args.precision else "plain bf16 activations: executed = algorithmic flops")}
    # the dominant kernel of the whole bench step by device time
    roof = None
    if rooflines:
        dom = max(rooflines, key=lambda k: rooflines[k]["ms_per_step"])
        r = rooflines[dom]
        traffic, traffic_note = None, None
        if dom in NCU_TRAFFIC:
            t = NCU_TRAFFIC[dom]
            if t["unit"] == "packed row":
                units = float(sum(int(x) for x in case["T_enc"]))
            else:
                units = r["algorithmic_bytes_per_launch"]
            traffic = t["bytes"] / t["units"] * units
            traffic_note = (f"DRAM read + write bytes per launch: the ncu capture in {t['source']} "
                            f"({t['bytes'] / 1e6:.2f} MB over {t['units']:.0f} {t['unit']}s), scaled to this "
                            f"launch's {units:.0f} {t['unit']}s")
        roof = {"kernel": dom, "bound": r["bound"], "achieved": r["achieved"], "peak": r["peak"], "unit": r["unit"],
                "frac": r["frac"], "peak_kind": pk_kind, "traffic": traffic, "traffic_note": traffic_note,
                "avg_launch_ms": r["avg_launch_ms"],
                "measured": "CUDA events between launch groups in one profiled bench step"}

    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": (dev_a_max + dev_b_max) / K, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d_a + h2d_b, "d2h_bytes_per_step": 2 * d2h},
            "rtfx": {"value": audio_all / (dev_b_max / 1000.0) if dev_b_max > 0 else None,
                     "e2e": audio_all / wall_b_max if wall_b_max > 0 else None, "unit": "audio s / s",
                     "audio_s_per_step": audio_s * world, "encoder_ms_per_step": enc_ms / K,
                     "h2d_bytes_per_step": h2d_b, "d2h_bytes_per_step": d2h},
            "p50_step_ms": statistics.median(step_times) if step_times else None,
            "config2": config2_summary(dev_c, wall_c, step_times_c, K) if with_c else None,
            ("config5" if args.stream_config == 5 else "config4"): config4,
            "gpu_launches": launches, "rows_per_step": rows_per_step, "steps_timed": int(n_steps),
            "roofline": roof, "rooflines": rooflines,
            "profiled_step_breakdown": breakdown, "clocks": clk.summary(), "device_status": status,
            "precision": "bf16 weights, activations as bf16 hi+lo planes, fp32 accumulate" if args.precision else
            "bf16 weights and activations, fp32 accumulate"}
    if world == 1 and not args.no_compare_precision and ("A" in legs or with_enc):
        # Legs A and B once more on an engine at the other precision (same
        # inputs, warm-up and step count), so the line carries both.
        other = 1 - args.precision
        e2 = abi.Engine(lib, dev, wb, ws, max_slots=args.max_slots, max_rows=1024, precision=other,
                        kv_pages=args.kv_pages, no_pdl=int(args.no_pdl), fused_step=args.fused_step,
                        enc_max_utts=enc_utts if with_enc else -1, enc_max_frames=enc_frames)
        for _ in range(args.warmup):
            if "A" in legs:
                leg_a(e2, [])
            if with_enc:
                leg_b(e2)
        st2, da, wa, db, wb_ = [], 0.0, 0.0, 0.0, 0.0
        for _ in range(K):
            if "A" in legs:
                s0 = e2.stats()
                t0 = time.perf_counter()
                leg_a(e2, st2)
                wa += time.perf_counter() - t0
                s1 = e2.stats()
                da += (s1["step_ms"] - s0["step_ms"]) + (s1["admit_ms"] - s0["admit_ms"])
            if with_enc:
                s0 = e2.stats()
                t0 = time.perf_counter()
                leg_b(e2)
                wb_ += time.perf_counter() - t0
                s1 = e2.stats()
                db += (s1["step_ms"] - s0["step_ms"]) + (s1["admit_ms"] - s0["admit_ms"]) + (s1["enc_ms"] - s0["enc_ms"])
        st_other = e2.status()
        e2.close()
        line["precision_compare"] = {
            "precision": "bf16 weights, activations as bf16 hi+lo planes, fp32 accumulate" if other else
            "bf16 weights and activations, fp32 accumulate",
            "value": tokens_per_step * K / (da / 1000.0) if da > 0 else None,
            "e2e": tokens_per_step * K / wa if wa > 0 else None, "unit": "tokens/s",
            "p50_step_ms": statistics.median(st2) if st2 else None,
            "rtfx": audio_s * K / (db / 1000.0) if db > 0 else None,
            "rtfx_e2e": audio_s * K / wb_ if wb_ > 0 else None, "device_status": st_other,
            "note": "legs A and B of the same workload, timed after the headline legs on the same GPU"}
    if rank == 0 and world == 1 and not args.no_cpu:
        ref = ReferenceCPU(case, enc, audio, ncores, args.cpu_tokens)
        t, s_ = ref.decode()
        a_, s2 = ref.transcribe()
        line["cpu_baseline"] = {"value": t / s_, "unit": "tokens/s", "cores": ncores, "kind": "reference",
                                "sample": ref.sample, "sample_tokens": int(ref.forced.sum()),
                                "sample_mean_tokens": float(ref.forced.mean()),
                                "workload_mean_tokens": ref.workload_mean_tokens,
                                "rtfx": a_ / s2, "rtfx_sample": ref.sample_rtfx}
    if rank == 0 and world == 1 and not args.no_cuda_ref:
        line["cuda_baseline"] = ReferenceCUDA(ws, case, enc, CUDA_REF_SAMPLE).run(wb)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
