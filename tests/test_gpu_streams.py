"""GPU tests of the stream shapes of configurations 4 and 5 (full-size model,
audio in, tokens out), scaled down so they run in seconds.

Configuration 4: utterances arrive over time (log-normal lengths, output
lengths of ~3 tokens per second of audio +-20%, EOS forced) and are admitted
into a running batch as slots free up, with encoder batches packed from
whatever is queued.  Every utterance's tokens must equal those of a run that
admits everything at once: admission order, slot reuse, encoder batch
composition and page reuse must not change any result.

Configuration 5: a long-form input is cut into 30 s windows every 29 s
(cohere-transcribe_b200/dispatch.py) decoded as independent utterances; each
window's tokens must equal the same window decoded alone.
"""
import importlib

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=25)
    return wb, wmod.weights_struct(wb)


def _engine(model, **kw):
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    wb, ws = model
    return abi.Engine(abi.load(), 0, wb, ws, **kw)


def _stream_case(n, seed):
    rng = np.random.default_rng(seed)
    secs = np.clip(np.exp(rng.normal(np.log(2.0), 0.5, n)), 1.0, 4.0)
    forced = np.maximum(2, np.round(3.0 * secs * rng.uniform(0.8, 1.2, n))).astype(np.int32)
    sigs = [inputs.audio(float(s), 500 + i) for i, s in enumerate(secs)]
    return sigs, forced


def test_stream_admission_matches_one_shot(model):
    sigs, forced = _stream_case(24, seed=41)
    eng = _engine(model, max_slots=6, enc_max_utts=8, enc_max_frames=8 * 401)
    try:
        i = 0
        for wave in (5, 3, 7, 4, 5):          # arrivals between steps
            for _ in range(wave):
                eng.submit_audio(i, sigs[i], forced[i])
                i += 1
            eng.step(3)
        eng.run()
        streamed = eng.poll()
        st = eng.stats()
        assert eng.status() == 0
    finally:
        eng.close()
    assert st["admitted"] == 24 and st["enc_utts"] == 24
    eng = _engine(model, max_slots=64, enc_max_utts=32, enc_max_frames=32 * 401)
    try:
        for i in range(24):
            eng.submit_audio(i, sigs[i], forced[i])
        eng.run()
        at_once = eng.poll()
        assert eng.status() == 0
    finally:
        eng.close()
    assert sorted(streamed) == list(range(24))
    for i in range(24):
        assert len(streamed[i]) == forced[i] and streamed[i][-1] == 3
        assert np.array_equal(streamed[i], at_once[i]), i


def test_long_form_windows_decode_independently(model):
    disp = importlib.import_module("cohere-transcribe_b200.dispatch")
    x = inputs.audio(65.0, 4242)
    wins = disp.long_form_sample_windows(len(x))
    assert len(wins) == 3
    eng = _engine(model, max_slots=8, enc_max_utts=4, enc_max_frames=3 * 3001)
    try:
        for k, (s, e) in enumerate(wins):
            eng.submit_audio(k, x[s:e], 24)
        eng.run()
        together = eng.poll()
        alone = {}
        for k, (s, e) in enumerate(wins):
            eng.submit_audio(100 + k, x[s:e], 24)
            eng.run()
            alone[k] = eng.poll()[100 + k]
        assert eng.status() == 0
    finally:
        eng.close()
    for k in range(len(wins)):
        assert len(together[k]) == 24
        assert np.array_equal(together[k], alone[k]), k
