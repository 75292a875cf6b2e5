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


def test_folder_mode_matches_direct_calls(model, tmp_path):
    """The input-folder mode (audio_files.run_folder, transcribe.c:1108-1228) on
    16 kHz PCM WAV files: a short file decodes in one pass and a 48 s file in
    silence-split chunks; the transcripts written equal the vocabulary printout
    of the tokens the engine gives the same samples directly."""
    import wave
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    lf = importlib.import_module("cohere-transcribe_b200.longform")
    af = importlib.import_module("cohere-transcribe_b200.audio_files")
    wb, ws = model
    prompt = list(inputs.ctb.PROMPT_FULL)
    src, dst = tmp_path / "in", tmp_path / "out"
    src.mkdir(); dst.mkdir()
    xs = {"a_short": inputs.speech_like(6.0, 1401), "b_long": inputs.speech_like(48.0, 1302)}
    pcm = {}
    for name, x in xs.items():
        q = np.clip(np.round(x * 32768.0), -32768, 32767).astype("<i2")
        pcm[name] = (q.astype(np.float64) / 32768.0).astype(np.float32)   # what the file decodes to
        with wave.open(str(src / f"{name}.wav"), "wb") as w:
            w.setnchannels(1); w.setsampwidth(2); w.setframerate(16000); w.writeframes(q.tobytes())
    vocab = [f"▁t{i}" for i in range(16384)]
    vocab[3] = "<|endoftext|>"
    eng = abi.Engine(abi.load(), 0, wb, ws, enc_max_utts=4, enc_max_frames=16000)
    try:
        written = af.run_folder(eng, str(src), str(dst), vocab, prompt, forced_len=_forced)
        # direct: the short file in one pass, the long one through the chunk scheduler
        eng.set_prompt(lf.chunk_prompt(prompt, []))
        eng.submit_audio(9000, pcm["a_short"], _forced(len(pcm["a_short"])))
        eng.set_prompt(None)
        eng.run()
        short = eng.poll()[9000]
        sch = lf.LongFormScheduler(eng, prompt, forced_len=_forced)
        sch.add(1, pcm["b_long"])
        long_chunks = sch.run()[1]
        assert eng.status() == 0
    finally:
        eng.close()
    assert [p.rsplit("/", 1)[-1] for p in written] == ["a_short.txt", "b_long.txt"]
    assert (dst / "a_short.txt").read_text() == af.detokenize(short, vocab)
    assert len(long_chunks) >= 2
    assert (dst / "b_long.txt").read_text() == "".join(af.detokenize(t, vocab) for t in long_chunks)
