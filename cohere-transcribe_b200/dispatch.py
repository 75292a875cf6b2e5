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

`ReplicaPool` runs one host thread per replica in one process and retires a
replica that fails (an exception, or a non-zero device status word), handing
its unfinished utterances to the others.

`long_form_windows` cuts a long log-mel input into fixed windows decoded as
independent sequences: 30 s windows every 29 s (1 s overlap), the last window
holding the remainder -- a 300 s input gives 11 windows, the last 10 s.
"""
from __future__ import annotations

import heapq
import threading
from collections import deque

FRAMES_PER_S = 100          # 10 ms hop (transcribe.c:268: T_mel = 1 + n_samples / 160 at 16 kHz)


def t_mel_of_seconds(sec: float) -> int:
    return 1 + int(round(sec * 16000)) // 160


def assign(seconds, n_replicas: int) -> list[int]:
    """Replica index for every utterance: least queued audio seconds first.
    Any non-negative per-utterance work measure may stand in for the seconds
    (bench.py weighs audio seconds and forced decode tokens together)."""
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


# ---- in-process replica pool with failure detection ---------------------------
#
# The reference fails stop: a CUDA error or OOM in any worker calls exit(1)
# (backends/cuda/backend.cu:26-33, transcribe.c:306).  Here every replica (one
# engine per GPU) is driven by its own host thread, as run_files_parallel
# gives each GPU worker its own thread (transcribe.c:947-984).  A replica whose
# call raises, or whose device status word reports a bounded wait that ran out,
# is retired: its unfinished utterances go back to the healthy replicas, by the
# same least-queued-audio rule, and the job completes as long as one replica
# stays healthy.  Results a retired replica had already returned are kept.


class ReplicaFailed(RuntimeError):
    pass


class ReplicaPool:
    """Run utterances over `replicas` (objects with the abi.Engine methods used
    here: submit_mel / submit_audio / submit, step, poll, status), one host
    thread each.  `run(items)` takes (utt_id, kind, data, forced_len, seconds)
    tuples, kind in {"mel", "audio", "enc"}, and returns {utt_id: tokens};
    `failed` lists (replica index, reason) of the replicas retired on the way."""

    def __init__(self, replicas, steps_per_poll: int = 8, max_in_flight: int = 256):
        if not replicas:
            raise ValueError("at least one replica")
        self.replicas = list(replicas)
        self.steps_per_poll = steps_per_poll
        self.max_in_flight = max_in_flight
        self.failed = []
        self._cv = threading.Condition()

    def _pick(self, load, healthy):
        return min((load[r], r) for r in healthy)[1]

    def run(self, items):
        n_rep = len(self.replicas)
        queues = [deque() for _ in range(n_rep)]
        load = [0.0] * n_rep
        healthy = set(range(n_rep))
        results = {}
        expected = {it[0] for it in items}
        if len(expected) != len(items):
            raise ValueError("utterance ids must be unique")
        for it in items:                       # initial dispatch: least queued audio seconds
            r = self._pick(load, healthy)
            queues[r].append(it)
            load[r] += float(it[4])
        error = []

        def requeue(lost):
            for it in lost:
                if it[0] in results:
                    continue
                r = self._pick(load, healthy)
                queues[r].append(it)
                load[r] += float(it[4])

        def worker(r):
            eng = self.replicas[r]
            in_flight = {}
            try:
                while True:
                    with self._cv:
                        while not queues[r] and not in_flight and r in healthy and \
                                len(results) < len(expected) and not error:
                            self._cv.wait(0.05)
                        if r not in healthy or len(results) >= len(expected) or error:
                            return
                        batch = []
                        while queues[r] and len(in_flight) + len(batch) < self.max_in_flight:
                            batch.append(queues[r].popleft())
                    for it in batch:
                        uid, kind, data, forced, _sec = it
                        in_flight[uid] = it
                        if kind == "mel":
                            eng.submit_mel(uid, data, forced)
                        elif kind == "audio":
                            eng.submit_audio(uid, data, forced)
                        else:
                            eng.submit(uid, data, forced)
                    if in_flight:
                        eng.step(self.steps_per_poll)
                        done = eng.poll()
                        st = eng.status()
                        if st != 0:
                            raise ReplicaFailed(f"device status {st}")
                        with self._cv:
                            for uid, tk in done.items():
                                it = in_flight.pop(uid, None)
                                if it is None:
                                    continue
                                results[uid] = tk
                                load[r] -= float(it[4])
                            self._cv.notify_all()
            except Exception as exc:          # retire the replica, hand its work on
                with self._cv:
                    healthy.discard(r)
                    self.failed.append((r, repr(exc)))
                    lost = list(in_flight.values()) + list(queues[r])
                    queues[r].clear()
                    load[r] = 0.0
                    if healthy:
                        requeue(lost)
                    elif len(results) < len(expected):
                        error.append(ReplicaFailed("every replica failed; last: " + repr(exc)))
                    self._cv.notify_all()

        threads = [threading.Thread(target=worker, args=(r,), daemon=True) for r in range(n_rep)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if error:
            raise error[0]
        missing = expected - set(results)
        if missing:
            raise ReplicaFailed(f"{len(missing)} utterances were not finished")
        return results
