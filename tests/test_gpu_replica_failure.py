"""GPU test of the replica pool's failure path with real engines.

dispatch.ReplicaPool drives one engine per replica from its own host thread
and retires a replica whose call raises or whose device status word is set;
the retired replica's unfinished utterances are decoded by the healthy ones
(the reference instead exits on any CUDA error, backends/cuda/backend.cu:26-33).
The failure is made on the host, as a step call that raises part-way through
the job (the engine underneath stays healthy, so no GPU fault is involved):
two real engines share cuda:0, the second fails after its first step, and
every utterance's tokens must still equal a clean run on one engine.
"""
import importlib

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


class FailingAfter:
    """An engine whose step() raises once it has run `n_ok` times."""

    def __init__(self, eng, n_ok):
        self.eng, self.n_ok, self.calls = eng, n_ok, 0

    def step(self, n=1):
        self.calls += 1
        if self.calls > self.n_ok:
            raise RuntimeError("injected replica failure")
        return self.eng.step(n)

    def __getattr__(self, name):
        return getattr(self.eng, name)


@pytest.fixture(scope="module")
def dec_model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=0, parts=("dec",))
    return wb, wmod.weights_struct(wb)


def test_replica_failure_requeues_to_the_healthy_engine(dec_model):
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    disp = importlib.import_module("cohere-transcribe_b200.dispatch")
    lib = abi.load()
    wb, ws = dec_model
    case = inputs.ragged_decode_case(8, seed=901, l_lo=12, l_hi=48)
    T_enc, forced = case["T_enc"], case["forced_len"]
    enc = inputs.enc_outputs(T_enc, case["enc_seed"])
    items = [(b, "enc", np.ascontiguousarray(enc[b, :T_enc[b]]), int(forced[b]), float(case["seconds"][b]))
             for b in range(len(T_enc))]
    # clean reference: one engine, every utterance
    ref_eng = abi.Engine(lib, 0, wb, ws, max_slots=16)
    try:
        for uid, _k, x, f, _s in items:
            ref_eng.submit(uid, x, f)
        ref_eng.run()
        ref = ref_eng.poll()
        assert ref_eng.status() == 0
    finally:
        ref_eng.close()
    good = abi.Engine(lib, 0, wb, ws, max_slots=16)
    bad = abi.Engine(lib, 0, wb, ws, max_slots=16)
    try:
        pool = disp.ReplicaPool([good, FailingAfter(bad, 1)], steps_per_poll=4, max_in_flight=8)
        got = pool.run(items)
        assert [r for r, _ in pool.failed] == [1], pool.failed
        assert "injected replica failure" in pool.failed[0][1]
        assert set(got) == set(ref)
        for uid in ref:
            assert np.array_equal(got[uid], ref[uid]), uid
        assert good.status() == 0 and bad.status() == 0
    finally:
        good.close()
        bad.close()
