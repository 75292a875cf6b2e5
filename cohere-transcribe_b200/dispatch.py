"""Host-side utterance dispatch across GPUs and long-form windowing.

Scaling is by utterance sharding: one engine per GPU (its own weights, page
pool and encoder batch), fed its own utterances, with no collective on the data
path.  This is the B200 form of the reference's run_files_parallel
(transcribe.c:947-984), which gives each GPU worker thread its own device and a
share of the input files.

`assign` is the dispatcher: each utterance, in arrival order, goes to the
replica with the fewest queued audio seconds (ties to the lowest index).  It is
a pure function of the utterance list, so every rank of a multi-process job
computes the same assignment locally and nothing needs to be exchanged to
agree on it.

`long_form_windows` cuts a long log-mel input into fixed windows decoded as
independent sequences: 30 s windows every 29 s (1 s overlap), the last window
holding the remainder -- a 300 s input gives 11 windows, the last 10 s.
"""
from __future__ import annotations

import heapq

FRAMES_PER_S = 100          # 10 ms hop (transcribe.c:268: T_mel = 1 + n_samples / 160 at 16 kHz)


def t_mel_of_seconds(sec: float) -> int:
    return 1 + int(round(sec * 16000)) // 160


def assign(seconds, n_replicas: int) -> list[int]:
    """Replica index for every utterance: least queued audio seconds first."""
    if n_replicas < 1:
        raise ValueError("n_replicas must be >= 1")
    heap = [(0.0, r) for r in range(n_replicas)]
    out = []
    for s in seconds:
        if s < 0:
            raise ValueError("negative duration")
        load, r = heapq.heappop(heap)
        out.append(r)
        heapq.heappush(heap, (load + float(s), r))
    return out


def shard(items, seconds, rank: int, world: int):
    """The items (with their positions in the full list) dispatched to `rank`."""
    a = assign(seconds, world)
    return [(i, it) for i, (it, r) in enumerate(zip(items, a)) if r == rank]


def long_form_windows(T_mel: int, window_s: float = 30.0, hop_s: float = 29.0) -> list[tuple[int, int]]:
    """[start, end) frame ranges covering T_mel frames with fixed windows of
    window_s seconds every hop_s seconds; the last window ends at T_mel."""
    if T_mel <= 0:
        return []
    win = t_mel_of_seconds(window_s)
    hop = int(round(hop_s * FRAMES_PER_S))
    if hop <= 0 or hop > win:
        raise ValueError("hop must be in (0, window]")
    out = []
    start = 0
    while True:
        end = min(start + win, T_mel)
        out.append((start, end))
        if end >= T_mel:
            return out
        start += hop


def long_form_sample_windows(n_samples: int, window_s: float = 30.0, hop_s: float = 29.0,
                             sr: int = 16000) -> list[tuple[int, int]]:
    """The same windows on the 16 kHz samples: [start, end) sample ranges, each
    window's audio decoded as an independent utterance (its log-mel is computed
    from its own samples, as the reference does for each chunk it cuts,
    transcribe.c:397-535)."""
    if n_samples <= 0:
        return []
    win, hop = int(round(window_s * sr)), int(round(hop_s * sr))
    out = []
    start = 0
    while True:
        end = min(start + win, n_samples)
        out.append((start, end))
        if end >= n_samples:
            return out
        start += hop
