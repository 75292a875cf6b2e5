"""Arrival-driven stream over one engine: configuration 4's workload.

Configuration 4 is a stream of utterances into one GPU, not a static batch:
- Poisson arrivals, mean 200 per second;
- log-normal lengths, median 8 s, clipped to 1-30 s;
- output lengths of 3 tokens per second of audio, +-20% uniform, EOS forced;
- at most 256 sequences decoding at once, encoder batches of up to 64
  utterances.

The reference has no such mode: its `transcribe_batch` (transcribe.c:572-808)
takes a fixed batch and admits nothing once decoding starts. Here the engine
admits new work between steps, and this driver feeds it in arrival order.

`stream_case` draws the workload. Its log-normal sigma is 0.5, since the
configuration leaves it open. `run_stream` replays it in real time against
the wall clock. It submits every utterance whose arrival time has passed,
advances the engine a few steps, and harvests finished utterances. It returns
per-utterance latency (finish time - arrival time) and whole-stream throughput.
With `saturated=True` every utterance arrives at t = 0, which measures capacity
instead of the arrival rate.

`config5_case` is configuration 5's stream, for 1 to 8 GPUs: 32,768 utterances
with configuration 4's lengths and arrivals at 8x the rate (1,600/s). It adds
64 long-form 5-minute inputs, cut into 30 s windows every 29 s (1 s overlap)
that decode as independent utterances, all arriving at t = 0. `subset` takes
one replica's share (see dispatch.shard) and keeps every utterance's seed, so
a shard's inputs equal the full stream's.
"""
from __future__ import annotations

import statistics
import time
from dataclasses import dataclass, field

import numpy as np

def t_mel_of_seconds(sec: float) -> int:
    """Log-mel frames of `sec` seconds at 16 kHz, 10 ms hop (transcribe.c:268)."""
    return 1 + int(round(sec * 16000)) // 160


@dataclass
class StreamCase:
    arrival_s: np.ndarray      # [n] arrival times, seconds from the stream start
    seconds: np.ndarray        # [n] utterance durations
    forced_len: np.ndarray     # [n] generated tokens, EOS forced at the last
    seed: int
    ids: np.ndarray = None     # [n] utterance ids in the full stream (seeds); default 0..n-1
    windows: dict = None       # id -> (long input, first frame, end frame) for long-form windows
    long_frames: int = 0       # log-mel frames of each long-form input

    def __post_init__(self):
        if self.ids is None:
            self.ids = np.arange(len(self.seconds))
        if self.windows is None:
            self.windows = {}
        self._long = (None, None)

    def long_mel(self, j: int) -> np.ndarray:
        """Long-form input j's seeded N(0, 1) log-mel [128, long_frames]."""
        if self._long[0] != j:
            rng = np.random.default_rng([self.seed, 9, j])
            self._long = (j, rng.standard_normal((128, self.long_frames), dtype=np.float32))
        return self._long[1]

    def log_mel(self, i: int) -> np.ndarray:
        """Utterance i's seeded N(0, 1) log-mel [128, T_mel] (generated on demand);
        a long-form window is its frames of the long input."""
        uid = int(self.ids[i])
        if uid in self.windows:
            j, a, b = self.windows[uid]
            return np.ascontiguousarray(self.long_mel(j)[:, a:b])
        rng = np.random.default_rng([self.seed, 7, uid])
        return rng.standard_normal((128, t_mel_of_seconds(float(self.seconds[i]))), dtype=np.float32)


def stream_case(n: int = 4096, seed: int = 0, rate: float = 200.0, median_s: float = 8.0, sigma: float = 0.5,
                lo_s: float = 1.0, hi_s: float = 30.0, tokens_per_s: float = 3.0, jitter: float = 0.2,
                saturated: bool = False) -> StreamCase:
    """Configuration 4's stream (defaults), or a scaled variant of it."""
    if n < 1 or rate <= 0:
        raise ValueError("n >= 1 and rate > 0 required")
    rng = np.random.default_rng(seed)
    gaps = rng.exponential(1.0 / rate, n)
    arrival = np.zeros(n) if saturated else np.cumsum(gaps) - gaps[0]
    secs = np.clip(np.exp(rng.normal(np.log(median_s), sigma, n)), lo_s, hi_s)
    forced = np.maximum(1, np.round(tokens_per_s * secs * rng.uniform(1.0 - jitter, 1.0 + jitter, n)))
    return StreamCase(arrival_s=arrival, seconds=secs, forced_len=forced.astype(np.int32), seed=seed)


def config5_case(n: int = 32768, seed: int = 0, rate: float = 1600.0, longform_n: int = 64,
                 longform_s: float = 300.0, tokens_per_s: float = 3.0, jitter: float = 0.2) -> StreamCase:
    """Configuration 5: configuration 4's draw at 8x the rate, plus the 30 s /
    29 s-hop windows of `longform_n` long inputs, arriving at t = 0."""
    from .dispatch import long_form_windows
    base = stream_case(n, seed=seed, rate=rate, tokens_per_s=tokens_per_s, jitter=jitter)
    T_long = t_mel_of_seconds(longform_s)
    spans = long_form_windows(T_long)
    rng = np.random.default_rng([seed, 5])
    windows, secs = {}, []
    for j in range(longform_n):
        for a, b in spans:
            windows[n + len(secs)] = (j, a, b)
            secs.append((b - a - 1) / 100.0)   # T_mel = 1 + 100 s
    secs = np.array(secs)
    forced = np.maximum(1, np.round(tokens_per_s * secs * rng.uniform(1.0 - jitter, 1.0 + jitter, len(secs))))
    return StreamCase(arrival_s=np.concatenate([base.arrival_s, np.zeros(len(secs))]),
                      seconds=np.concatenate([base.seconds, secs]),
                      forced_len=np.concatenate([base.forced_len, forced.astype(np.int32)]), seed=seed,
                      windows=windows, long_frames=T_long)


def subset(case: StreamCase, idx) -> StreamCase:
    """The utterances `idx` of `case` (one replica's share), same seeds and windows."""
    idx = np.asarray(idx, np.int64)
    return StreamCase(arrival_s=case.arrival_s[idx], seconds=case.seconds[idx], forced_len=case.forced_len[idx],
                      seed=case.seed, ids=case.ids[idx], windows=case.windows, long_frames=case.long_frames)


@dataclass
class StreamResult:
    latency_s: np.ndarray            # [n] finish - arrival
    tokens: dict = field(repr=False)  # utt id -> generated tokens
    wall_s: float = 0.0              # first arrival to last finish
    generated: int = 0
    audio_s: float = 0.0

    def summary(self) -> dict:
        lat = np.sort(self.latency_s)
        return {"utterances": int(len(lat)), "generated_tokens": self.generated, "audio_s": self.audio_s,
                "wall_s": self.wall_s, "tokens_per_s": self.generated / self.wall_s if self.wall_s > 0 else None,
                "rtfx": self.audio_s / self.wall_s if self.wall_s > 0 else None,
                "latency_p50_s": float(statistics.median(lat)),
                "latency_p95_s": float(lat[min(len(lat) - 1, int(np.ceil(0.95 * len(lat))) - 1)]),
                "latency_max_s": float(lat[-1])}


def run_stream(engine, case: StreamCase, steps_per_poll: int = 8, clock=time.perf_counter, sleep=time.sleep,
               inputs=None) -> StreamResult:
    """Replay `case` on `engine` (an abi.Engine, or anything with submit_mel /
    step / poll): submit what has arrived, step, harvest, until every utterance
    has finished.  `inputs[i]` (default case.log_mel(i)) is utterance i's log-mel."""
    n = len(case.seconds)
    order = np.argsort(case.arrival_s, kind="stable")
    arrival = case.arrival_s
    finish = np.full(n, np.nan)
    tokens = {}
    nxt = 0
    live = 0
    t0 = clock()
    while len(tokens) < n:
        now = clock() - t0
        while nxt < n and arrival[order[nxt]] <= now:
            i = int(order[nxt])
            engine.submit_mel(i, inputs[i] if inputs is not None else case.log_mel(i), int(case.forced_len[i]))
            nxt += 1
            live += 1
        if live == 0:                      # idle until the next arrival
            sleep(max(0.0, arrival[order[nxt]] - (clock() - t0)))
            continue
        remaining = engine.step(steps_per_poll)
        done = engine.poll()
        if not done and remaining == 0:
            raise RuntimeError(f"the engine holds no work but {live} submitted utterances never finished")
        t = clock() - t0
        for uid, tk in done.items():
            if uid in tokens:
                raise RuntimeError(f"utterance {uid} finished twice")
            tokens[uid] = tk
            finish[uid] = t
            live -= 1
    lat = finish - arrival
    return StreamResult(latency_s=lat, tokens=tokens, wall_s=float(np.nanmax(finish) - arrival.min()),
                        generated=int(sum(len(v) for v in tokens.values())), audio_s=float(case.seconds.sum()))
