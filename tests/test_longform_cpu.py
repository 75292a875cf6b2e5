"""Long-form chunking (cohere-transcribe_b200/longform.py) on the CPU.

The split points equal the reference's transcribe_file_chunked
(transcribe.c:484-507): against tests/golden/longform_ref.npz, recorded from
the reference built here, and, when that build is present, live on extra
signals.  The chunk-prompt and carry rules follow transcribe.c:381-389 and
:509-520, and the scheduler keeps each input's chunks in order (checked with a
stand-in engine that records what it is given).
"""
import ctypes
import importlib
import math
import os

import numpy as np

import inputs
import pyoracle as po

lf = importlib.import_module("cohere-transcribe_b200.longform")


def _splits(bounds):
    return [s for s, _ in bounds[1:]]


def test_split_points_match_reference():
    gold = np.load(os.path.join(os.path.dirname(inputs.__file__), "longform_ref.npz"))
    for k, (seconds, seed, db, dur, target) in enumerate(inputs.longform_case()):
        x = inputs.speech_like(seconds, seed)
        assert np.float64(x.astype(np.float64).sum()) == gold[f"checksum{k}"]
        b = lf.chunk_bounds(x, db, dur, target)
        assert _splits(b) == gold[f"splits{k}"].tolist(), k
        assert b[0][0] == 0 and b[-1][1] == len(x)
    path = os.path.join(po.REF_DIR, "libref_mel.so")
    if os.path.exists(path):
        R = ctypes.CDLL(path)
        R.refsplit.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                               ctypes.c_void_p, ctypes.c_int]
        for seconds, seed, db, dur, target in [(300.0, 7, math.nan, 0.2, 20.0), (33.3, 8, -35.0, 0.1, 5.0),
                                               (90.0, 9, math.nan, 1.0, 20.0)]:
            x = inputs.speech_like(seconds, seed)
            buf = np.zeros(4096, np.int32)
            n = R.refsplit(x.ctypes.data, len(x), db, dur, target, buf.ctypes.data, len(buf))
            assert _splits(lf.chunk_bounds(x, db, dur, target)) == buf[:n].tolist(), seconds


def test_chunk_prompt_and_carry():
    prompt = list(range(100, 110))
    assert lf.chunk_prompt(prompt, []) == prompt
    assert lf.chunk_prompt(prompt, [7, 8]) == [100, 101, 7, 8] + prompt[2:]
    gen = np.arange(1, 101)          # 100 generated tokens, the last one the EOS
    c = lf.carry_of(gen)
    assert len(c) == 64 and c[-1] == 99 and c[0] == 36
    assert lf.carry_of(np.array([3])) == []
    assert lf.carry_of(np.array([5, 3])) == [5]


class _FakeEngine:
    """Records submissions; 'decodes' chunk c to forced_len tokens of value
    c + 1 (the last one EOS); finishes one chunk per step."""

    def __init__(self):
        self.prompt = None
        self.queue, self.done, self.log = [], {}, []

    def set_prompt(self, p=None):
        self.prompt = None if p is None else list(p)

    def submit_audio(self, uid, x, forced):
        self.log.append((uid, len(x), self.prompt))
        self.queue.append((uid, forced))

    def step(self, n):
        if self.queue:
            uid, forced = self.queue.pop(0)
            self.done[uid] = np.array([uid % 65536 + 1] * (forced - 1) + [3], np.int32)

    def poll(self):
        out, self.done = self.done, {}
        return out


def test_scheduler_orders_chunks_and_carries_context():
    eng = _FakeEngine()
    prompt = list(range(100, 110))
    sch = lf.LongFormScheduler(eng, prompt, forced_len=lambda n: 5)
    xa, xb = inputs.speech_like(130.0, 1202), inputs.speech_like(45.0, 1201)
    sch.add(1, xa)
    sch.add(2, xb)
    out = sch.run()
    na, nb = len(sch.files[1]["bounds"]), len(sch.files[2]["bounds"])
    assert len(out[1]) == na and len(out[2]) == nb and na == 5 and nb == 2
    for fid, n in ((1, na), (2, nb)):
        subs = [s for s in eng.log if s[0] // 65536 == fid]
        assert [s[0] % 65536 for s in subs] == list(range(n))          # chunks in order, one at a time
        assert subs[0][2] == prompt
        for c in range(1, n):                                          # previous chunk's tokens as context
            assert subs[c][2] == prompt[:2] + [c] * 4 + prompt[2:]
