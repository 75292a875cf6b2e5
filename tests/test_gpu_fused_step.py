"""GPU tests of the persistent step kernel (ct_engine_config.fused_step = 1).

The fused step runs the decode step as phases of one launch (grid barriers
between them) and does each phase's arithmetic in the order of the separate
kernels: the same K splits and split-order sums (its split-K partials go
through L2 instead of a cluster's shared memory), the same LayerNorm
statistics, the same attention groups and merges, the same argmax keys.  So
its tokens and its logits must equal the separate-kernel step's bit for bit,
which in turn is checked against the CPU oracle and the reference CUDA backend
(tests/test_gpu_engine.py, tests/test_gpu_reference_cuda.py).

Cases: a ragged batch of six (prefill steps included, logits compared),
configuration 2's batch-1 decode (T_enc 376, 200 tokens), configuration 3's
shape (64 utterances of 5-30 s, EOS forced at U{20..220}: its first step packs
640 prompt rows, five 128-row token tiles), and plain bf16 activations.
"""
import importlib

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def abi():
    a = importlib.import_module("cohere-transcribe_b200.abi")
    a.load()
    return a


@pytest.fixture(scope="module")
def dec_model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=0, parts=("dec",))
    return wb, wmod.weights_struct(wb)


def run(abi, model, enc, T_enc, forced, fused, keep_logits=0, precision=1, max_slots=64):
    wb, ws = model
    B = len(T_enc)
    eng = abi.Engine(abi.load(), 0, wb, ws, max_slots=max_slots, precision=precision, keep_logits=keep_logits,
                     fused_step=fused)
    logits = {}
    try:
        for b in range(B):
            eng.submit(b, enc[b, :T_enc[b]], int(forced[b]))
        if keep_logits:
            while True:
                left = eng.step(1)
                for uid, (g, row) in eng.last_logits().items():
                    logits[(uid, g)] = row
                if left == 0:
                    break
        else:
            eng.run()
        out = eng.poll()
        assert eng.status() == 0
    finally:
        eng.close()
    return out, logits


def test_fused_step_equals_separate_kernels_with_logits(abi, dec_model):
    case = inputs.ragged_decode_case(6, seed=310, l_lo=8, l_hi=40)
    T_enc, forced = case["T_enc"], case["forced_len"]
    enc = inputs.enc_outputs(T_enc, case["enc_seed"])
    ref, ref_lg = run(abi, dec_model, enc, T_enc, forced, fused=0, keep_logits=1)
    got, got_lg = run(abi, dec_model, enc, T_enc, forced, fused=1, keep_logits=1)
    for b in range(len(T_enc)):
        assert np.array_equal(got[b], ref[b]), b
    assert set(got_lg) == set(ref_lg)
    diff = [k for k in ref_lg if not np.array_equal(got_lg[k], ref_lg[k])]
    assert not diff, f"{len(diff)}/{len(ref_lg)} logit rows differ, e.g. {diff[:4]}"


def test_fused_step_configuration2(abi, dec_model):
    T_enc, forced = np.array([376], np.int32), np.array([200], np.int32)
    enc = inputs.enc_outputs(T_enc, seed=620)
    ref, _ = run(abi, dec_model, enc, T_enc, forced, fused=0)
    got, _ = run(abi, dec_model, enc, T_enc, forced, fused=1)
    assert len(got[0]) == 200 and np.array_equal(got[0], ref[0])


def test_fused_step_configuration3_shape(abi, dec_model):
    case = inputs.ragged_decode_case(64, seed=450)
    T_enc, forced = case["T_enc"], case["forced_len"]
    enc = inputs.enc_outputs(T_enc, case["enc_seed"])
    ref, _ = run(abi, dec_model, enc, T_enc, forced, fused=0)
    got, _ = run(abi, dec_model, enc, T_enc, forced, fused=1)
    diff = [b for b in range(64) if not np.array_equal(got[b], ref[b])]
    assert not diff, f"{len(diff)}/64 sequences differ: {diff}"


def test_fused_step_bf16_activations(abi, dec_model):
    case = inputs.ragged_decode_case(5, seed=77, l_lo=10, l_hi=50)
    T_enc, forced = case["T_enc"], case["forced_len"]
    enc = inputs.enc_outputs(T_enc, case["enc_seed"])
    ref, _ = run(abi, dec_model, enc, T_enc, forced, fused=0, precision=0)
    got, _ = run(abi, dec_model, enc, T_enc, forced, fused=1, precision=0)
    for b in range(len(T_enc)):
        assert np.array_equal(got[b], ref[b]), b
