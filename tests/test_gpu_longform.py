"""GPU test of long-form transcription with carried-over context
(cohere-transcribe_b200/longform.py on the engine; transcribe.c:484-532).

Two long inputs are cut at silences; each chunk's prompt carries the previous
chunk's last tokens, so prompts have different lengths and the chunks of one
input run one after another while the two inputs share the engine.  The
scheduler's tokens must equal a strictly sequential chunk-by-chunk run, and a
chunk decoded with a carried-over prompt must agree with the oracle decoding
the same encoder rows with the same prompt (teacher forced, margin rule).
"""
import importlib

import numpy as np
import pytest

import inputs
import pyoracle as po

pytestmark = pytest.mark.gpu
MARGIN_TOL = 2e-3


def _forced(n_samples):
    return min(40, 2 + n_samples // 16000)   # about one token per second of audio


@pytest.fixture(scope="module")
def model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=27)
    return wb, wmod.weights_struct(wb)


def test_long_form_chunks_with_carried_context(model, wmod):
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    lf = importlib.import_module("cohere-transcribe_b200.longform")
    wb, ws = model
    prompt = list(inputs.ctb.PROMPT_FULL)
    xs = {1: inputs.speech_like(70.0, 1301), 2: inputs.speech_like(48.0, 1302)}
    eng = abi.Engine(abi.load(), 0, wb, ws, enc_max_utts=4, enc_max_frames=16000)
    try:
        sch = lf.LongFormScheduler(eng, prompt, forced_len=_forced)
        for fid, x in xs.items():
            sch.add(fid, x)
        got = sch.run()
        # the same chunks one at a time, each waiting for the previous one
        seq = {}
        for fid, x in xs.items():
            carry, seq[fid] = [], []
            for c, (s, e) in enumerate(lf.chunk_bounds(x)):
                eng.set_prompt(lf.chunk_prompt(prompt, carry))
                eng.submit_audio(7000 + c, x[s:e], _forced(e - s))
                eng.run()
                toks = eng.poll()[7000 + c]
                seq[fid].append(toks)
                carry = lf.carry_of(toks)
        eng.set_prompt(None)
        # encoder rows and prompt of file 1's second chunk, for the oracle
        (s, e) = sch.files[1]["bounds"][1]
        rows = eng.encode(eng.log_mel([xs[1][s:e]]))[0]
        assert eng.status() == 0
    finally:
        eng.close()
    for fid in xs:
        assert len(got[fid]) == len(sch.files[fid]["bounds"]) >= 2
        for c, toks in enumerate(got[fid]):
            assert np.array_equal(toks, seq[fid][c]), (fid, c)
    p1 = np.array(lf.chunk_prompt(prompt, lf.carry_of(got[1][0])), np.int32)
    assert len(p1) > 10
    forced = np.array([_forced(e - s)], np.int32)
    out = got[1][1]
    n_p = len(p1)
    force = np.zeros((1, 1024), np.int32)
    force[0, n_p:n_p + len(out)] = out
    T_enc = np.array([rows.shape[0]], np.int32)
    _t, _n, am, mg = po.decode_batch(wmod.FULL_DIMS, ws, rows[None].copy(), T_enc, p1, forced, force_tokens=force)
    checked = 0
    for g in range(forced[0] - 1):
        if mg[0, n_p + g] >= MARGIN_TOL:
            assert out[g] == am[0, n_p + g], g
            checked += 1
    assert checked > 0.7 * (forced[0] - 1)
