"""Host-side dispatch for utterance sharding (CPU; multi-process with gloo).

The N>1 path has no collective on the data path: every rank computes the same
least-queued-audio assignment locally and runs its own shard.  These tests
check the assignment, the long-form windowing of configuration 5, and a
world-size-2 gloo run in which each rank processes its shard and rank 0
verifies that every utterance was processed exactly once with the result a
single process computes.
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
