"""Host-side dispatch for utterance sharding (CPU; multi-process with gloo).

The N>1 path has no collective on the data path: every rank computes the same
least-queued-audio assignment locally and runs its own shard.  These tests
check the assignment, the long-form windowing of configuration 5, and a
world-size-2 gloo run in which each rank processes its shard and rank 0
verifies that every utterance was processed exactly once with the result a
single process computes.

Failure detection (ReplicaPool) is tested here on the host, with stand-in
replicas (tests/test_gpu_replica_failure.py repeats it with real engines): one whose step raises (as a failed CUDA call surfaces through the
engine's return code), one whose device status word turns non-zero (as a
bounded device wait that ran out reports itself), and a pool in which every
replica fails.  No GPU is faulted or hung.
"""
import importlib
import os
import socket

import numpy as np
import pytest

disp = importlib.import_module("cohere-transcribe_b200.dispatch")


def test_assign_is_balanced_and_deterministic():
    rng = np.random.default_rng(3)
    secs = rng.uniform(1.0, 30.0, 1000)
    for n in (1, 2, 4, 8):
        a = disp.assign(secs, n)
        assert a == disp.assign(secs, n)
        load = np.zeros(n)
        for s, r in zip(secs, a):
            load[r] += s
        # greedy least-loaded: no replica ends more than one utterance above another
        assert load.max() - load.min() <= secs.max() + 1e-9
        assert set(a) == set(range(n))


def test_assign_prefers_least_loaded_then_lowest_index():
    assert disp.assign([10, 1, 1, 1], 2) == [0, 1, 1, 1]
    assert disp.assign([5, 5, 5], 3) == [0, 1, 2]
    with pytest.raises(ValueError):
        disp.assign([1.0], 0)


def test_long_form_windows_300s():
    T = disp.t_mel_of_seconds(300.0)
    w = disp.long_form_windows(T)
    assert len(w) == 11
    assert w[0] == (0, disp.t_mel_of_seconds(30.0))
    assert all(b[0] - a[0] == 2900 for a, b in zip(w, w[1:]))
    assert all(a[1] - b[0] == 101 for a, b in zip(w, w[1:]))   # 1 s overlap (+ the +1 frame of T_mel)
    assert w[-1][1] == T and (w[-1][1] - w[-1][0] - 1) / 100 == pytest.approx(10.0)
    assert disp.long_form_windows(disp.t_mel_of_seconds(12.0)) == [(0, 1201)]
    assert disp.long_form_windows(0) == []


def test_long_form_sample_windows():
    w = disp.long_form_sample_windows(300 * 16000)
    assert len(w) == 11 and w[-1] == (290 * 16000, 300 * 16000)
    assert all(a[1] - b[0] == 16000 for a, b in zip(w, w[1:]))   # 1 s overlap
    # the frames of each window's own log-mel are the frame windows'
    fw = disp.long_form_windows(disp.t_mel_of_seconds(300.0))
    assert [1 + (e - s) // 160 for s, e in w] == [e - s for s, e in fw]
    assert disp.long_form_sample_windows(65 * 16000) == [(0, 480000), (464000, 944000), (928000, 1040000)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _work(i, secs):
    # stand-in for transcribing utterance i: a deterministic function of it
    return int(np.random.default_rng(i).integers(0, 1 << 30)) ^ int(secs * 1000)


def _rank_main(rank, world, port, secs, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = disp.shard(list(range(len(secs))), secs, rank, world)
        done = {i: _work(i, secs[i]) for i, _ in mine}
        gathered = [None] * world
        dist.all_gather_object(gathered, done)
        if rank == 0:
            q.put(gathered)
    finally:
        dist.destroy_process_group()


def test_sharded_run_two_ranks_gloo():
    import torch.multiprocessing as mp
    secs = list(np.random.default_rng(9).uniform(1.0, 30.0, 37))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, secs, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    seen = {}
    for d in gathered:
        for i, v in d.items():
            assert i not in seen
            seen[i] = v
    assert sorted(seen) == list(range(len(secs)))
    assert all(seen[i] == _work(i, secs[i]) for i in seen)
    a = disp.assign(secs, 2)
    assert sorted(gathered[0]) == [i for i in range(len(secs)) if a[i] == 0]


class FakeReplica:
    """Engine stand-in: one token per live utterance per step; tokens are a
    function of the utterance id, so any replica gives the same result.
    fail_after: raise on that step call; bad_status_after: report a non-zero
    device status word from that step on (a bounded device wait that ran out)."""

    def __init__(self, fail_after=None, bad_status_after=None, delay=0.0):
        self.live, self.ready, self.steps = {}, {}, 0
        self.fail_after, self.bad_status_after, self.delay = fail_after, bad_status_after, delay
        self.seen = []

    def _submit(self, uid, data, forced):
        self.seen.append(uid)
        self.live[uid] = [int(forced), 0]

    submit_mel = submit_audio = submit = _submit

    def step(self, n):
        import time
        self.steps += 1
        if self.fail_after is not None and self.steps >= self.fail_after:
            raise RuntimeError("step failed: -4")
        time.sleep(self.delay)
        for uid in list(self.live):
            f, g = self.live[uid]
            g = min(f, g + n)
            if g >= f:
                self.ready[uid] = (np.arange(f) + uid).astype(np.int32)
                del self.live[uid]
            else:
                self.live[uid][1] = g
        return len(self.live)

    def poll(self):
        out, self.ready = self.ready, {}
        return out

    def status(self):
        return 1 if self.bad_status_after is not None and self.steps >= self.bad_status_after else 0


def _items(n, seed=0):
    rng = np.random.default_rng(seed)
    secs = rng.uniform(1.0, 30.0, n)
    return [(i, "mel", None, int(3 * s) + 1, float(s)) for i, s in enumerate(secs)]


def _check(res, items):
    assert sorted(res) == [it[0] for it in items]
    for uid, _k, _d, f, _s in items:
        assert np.array_equal(res[uid], np.arange(f) + uid)


def test_pool_without_failures_balances_and_finishes_once():
    items = _items(200)
    reps = [FakeReplica() for _ in range(4)]
    pool = disp.ReplicaPool(reps, steps_per_poll=8, max_in_flight=16)
    res = pool.run(items)
    _check(res, items)
    assert pool.failed == []
    assert sum(len(r.seen) for r in reps) == 200 and all(r.seen for r in reps)


def test_pool_requeues_the_work_of_a_failing_replica():
    items = _items(120, seed=1)
    reps = [FakeReplica(delay=0.001), FakeReplica(fail_after=3, delay=0.001), FakeReplica(delay=0.001)]
    pool = disp.ReplicaPool(reps, steps_per_poll=4, max_in_flight=8)
    res = pool.run(items)
    _check(res, items)
    assert [f[0] for f in pool.failed] == [1] and "step failed" in pool.failed[0][1]
    # the failed replica's unfinished utterances ran again on the others
    rerun = set(reps[1].seen) & (set(reps[0].seen) | set(reps[2].seen))
    assert rerun


def test_pool_retires_a_replica_reporting_device_status():
    items = _items(60, seed=2)
    reps = [FakeReplica(bad_status_after=2), FakeReplica()]
    pool = disp.ReplicaPool(reps, steps_per_poll=4, max_in_flight=8)
    res = pool.run(items)
    _check(res, items)
    assert [f[0] for f in pool.failed] == [0] and "device status" in pool.failed[0][1]


def test_pool_raises_when_every_replica_fails():
    items = _items(20, seed=3)
    pool = disp.ReplicaPool([FakeReplica(fail_after=1), FakeReplica(fail_after=2)], steps_per_poll=1)
    with pytest.raises(disp.ReplicaFailed, match="every replica failed"):
        pool.run(items)
    assert sorted(f[0] for f in pool.failed) == [0, 1]
