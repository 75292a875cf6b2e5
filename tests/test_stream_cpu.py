"""CPU tests of the configuration-4 stream driver (cohere-transcribe_b200/stream.py).

The draw follows configuration 4: Poisson arrivals at 200/s, log-normal
lengths (median 8 s, sigma 0.5) clipped to 1-30 s, 3 tokens per audio second
+-20%.  The replay loop runs against a stand-in engine on a virtual clock. The
stand-in decodes one token per live sequence per step, holds at most `slots`
sequences, and admits in submission order. The checks: no utterance is
submitted before it arrives, every utterance finishes exactly once, and the
latencies and totals are the ones the virtual timeline implies.
"""
import importlib

import numpy as np
import pytest

stream = importlib.import_module("cohere-transcribe_b200.stream")


def test_stream_case_distribution():
    c = stream.stream_case(4096, seed=3)
    gaps = np.diff(c.arrival_s)
    assert c.arrival_s[0] == 0.0 and np.all(gaps >= 0)
    assert abs(gaps.mean() - 1 / 200) < 0.0005                   # Poisson, mean 200/s
    assert c.seconds.min() >= 1.0 and c.seconds.max() <= 30.0
    assert abs(np.median(c.seconds) - 8.0) < 0.4                  # log-normal median 8 s
    ratio = c.forced_len / c.seconds
    assert ratio.min() >= 3 * 0.8 - 0.5 and ratio.max() <= 3 * 1.2 + 0.5
    s = stream.stream_case(16, seed=3, saturated=True)
    assert np.all(s.arrival_s == 0)
    m = c.log_mel(5)
    assert m.shape == (128, stream.t_mel_of_seconds(float(c.seconds[5])))
    assert np.array_equal(m, c.log_mel(5))                         # seeded per utterance


class VirtualClock:
    def __init__(self):
        self.t = 0.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += max(0.0, dt)


class StandInEngine:
    """One token per live sequence per step (dt seconds each); FIFO admission
    into at most `slots` sequences; finished sequences are polled."""

    def __init__(self, clock, case, slots=4, dt=0.001):
        self.clock, self.case, self.slots, self.dt = clock, case, slots, dt
        self.queue, self.live, self.ready, self.submit_t = [], {}, {}, {}

    def submit_mel(self, i, mel, forced):
        assert self.clock() >= self.case.arrival_s[i] - 1e-12, "submitted before its arrival"
        assert mel.shape[0] == 128 and forced == self.case.forced_len[i]
        self.submit_t[i] = self.clock()
        self.queue.append((i, forced))

    def step(self, n):
        for _ in range(n):
            while self.queue and len(self.live) < self.slots:
                i, f = self.queue.pop(0)
                self.live[i] = [f, 0]
            if not self.live:
                break
            self.clock.t += self.dt
            for i in list(self.live):
                self.live[i][1] += 1
                if self.live[i][1] >= self.live[i][0]:
                    self.ready[i] = np.full(self.live[i][0], 7, np.int32)
                    del self.live[i]
        return len(self.queue) + len(self.live)

    def poll(self):
        out, self.ready = self.ready, {}
        return out


@pytest.mark.parametrize("saturated", [False, True])
def test_replay_respects_arrivals_and_finishes_everything(saturated):
    case = stream.stream_case(300, seed=11, rate=400.0, median_s=2.0, hi_s=6.0, saturated=saturated)
    clk = VirtualClock()
    eng = StandInEngine(clk, case, slots=8)
    res = stream.run_stream(eng, case, steps_per_poll=4, clock=clk, sleep=clk.sleep,
                            inputs=[np.zeros((128, 4), np.float32)] * len(case.seconds))
    n = len(case.seconds)
    assert sorted(res.tokens) == list(range(n))
    assert all(len(res.tokens[i]) == case.forced_len[i] for i in range(n))
    assert res.generated == int(case.forced_len.sum())
    # a sequence needs forced_len steps once admitted, so latency >= forced_len * dt
    assert np.all(res.latency_s >= case.forced_len * eng.dt - 1e-9)
    assert np.all(np.isfinite(res.latency_s))
    s = res.summary()
    assert s["utterances"] == n and s["latency_p50_s"] <= s["latency_p95_s"] <= s["latency_max_s"]
    assert s["rtfx"] == pytest.approx(case.seconds.sum() / res.wall_s)
    if saturated:   # with everything queued at t = 0 the 8 slots never idle while work remains
        assert res.wall_s <= (case.forced_len.sum() / 8 + case.forced_len.max() + 8) * eng.dt


def test_replay_reports_lost_utterances():
    case = stream.stream_case(3, seed=1, saturated=True)
    clk = VirtualClock()

    class Losing(StandInEngine):
        def step(self, n):
            self.queue.clear()
            return 0

    with pytest.raises(RuntimeError, match="never finished"):
        stream.run_stream(Losing(clk, case), case, clock=clk, sleep=clk.sleep,
                          inputs=[np.zeros((128, 4), np.float32)] * 3)


def test_config5_case_windows_and_shards():
    c = stream.config5_case(200, seed=4, longform_n=3)
    n_win = 3 * 11                                       # 300 s in 30 s windows every 29 s: 11 each
    assert len(c.seconds) == 200 + n_win
    assert np.all(c.arrival_s[200:] == 0)
    assert abs(np.diff(c.arrival_s[:200]).mean() - 1 / 1600) < 0.0003   # 8x configuration 4's rate
    w = [c.windows[200 + k] for k in range(11)]
    assert w[0] == (0, 0, 3001) and w[-1] == (0, 29000, 30001)
    assert np.allclose(c.seconds[200:211], [30.0] * 10 + [10.0])
    a, b = c.log_mel(200), c.log_mel(201)
    assert a.shape == (128, 3001)
    assert np.array_equal(a[:, 2900:], b[:, :101])          # 1 s of overlap between neighbours
    assert np.array_equal(c.log_mel(211), c.long_mel(1)[:, :3001])
    # a replica's share keeps each utterance's input
    disp = importlib.import_module("cohere-transcribe_b200.dispatch")
    mine = [i for i, _ in disp.shard(list(range(len(c.seconds))), c.seconds, 1, 4)]
    sub = stream.subset(c, mine)
    for k in (0, len(mine) // 2, len(mine) - 1):
        assert np.array_equal(sub.log_mel(k), c.log_mel(mine[k]))
    shares = [len(disp.shard(list(range(len(c.seconds))), c.seconds, r, 4)) for r in range(4)]
    assert sum(shares) == len(c.seconds)
