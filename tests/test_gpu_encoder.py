"""GPU tests of the engine's packed ragged Conformer encoder (ct_engine_encode,
ct_engine_submit_mel) at full width and depth (48 layers, ENC_D 1280) against
the CPU oracle's orc_encoder_forward_batch (model.h:573-609).

Tolerance: the encoder runs its GEMMs on bf16 tensor cores with the
activations split into bf16 hi + lo planes (about 16 mantissa bits) and fp32
accumulation; the oracle is fp32 throughout.  Over 48 layers the difference
stays near 1e-4 of the output scale; ENC_TOL = 2e-3 (max |engine - oracle|
over max |oracle|, per utterance) leaves an order of magnitude.  With plain
bf16 activations (precision 0: one plane, every GEMM input rounded to 8
mantissa bits, fp32 accumulation) the error grows with depth: 7.6e-3 of the
output scale at 30 s; ENC_TOL_BF16 = 2e-2 is the stated tolerance for that
mode.
"""
import ctypes
import importlib

import numpy as np
import pytest

import inputs
import pyoracle as po

pytestmark = pytest.mark.gpu
ENC_TOL = 2e-3
ENC_TOL_BF16 = 2e-2
E2E_MARGIN_TOL = 0.05


def t_enc_of(T_mel):
    t1 = (T_mel + 1) // 2
    t2 = (t1 + 1) // 2
    return ((t2 + 1) // 2).astype(np.int32)


@pytest.fixture(scope="module")
def full_model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=21)
    return wb, wmod.weights_struct(wb)


@pytest.fixture(scope="module")
def abi():
    a = importlib.import_module("cohere-transcribe_b200.abi")
    a.load()
    return a


def oracle_encode(wmod, ws, mel, T_mel):
    B = len(T_mel)
    T_enc = t_enc_of(T_mel)
    out = np.zeros((B, int(T_enc.max()), 1024), np.float32)
    O = po.lib()
    d = po.dims_struct(wmod.FULL_DIMS)
    O.orc_encoder_forward_batch(ctypes.byref(d), ctypes.addressof(ws), po.fp(mel), B, mel.shape[2], po.ip(T_mel),
                                po.ip(T_enc), int(T_enc.max()), po.fp(out))
    return [out[b, :T_enc[b]] for b in range(B)]


def make_engine(abi, model, **kw):
    wb, ws = model
    kw.setdefault("enc_max_utts", 8)
    kw.setdefault("enc_max_frames", 8192)
    return abi.Engine(abi.load(), 0, wb, ws, **kw)


def mels_of(mel, T_mel):
    return [np.ascontiguousarray(mel[b, :, :T_mel[b]]) for b in range(len(T_mel))]


def test_encoder_ragged_batch_vs_oracle(abi, full_model, wmod):
    mel, T_mel = inputs.mel_batch([1.03, 2.41, 0.37], seed=700)
    ref = oracle_encode(wmod, full_model[1], mel, T_mel)
    eng = make_engine(abi, full_model)
    try:
        got = eng.encode(mels_of(mel, T_mel))
        assert eng.status() == 0
    finally:
        eng.close()
    for b in range(len(T_mel)):
        assert got[b].shape == ref[b].shape
        err = float(np.max(np.abs(got[b] - ref[b])) / np.max(np.abs(ref[b])))
        assert err <= ENC_TOL, (b, err)


@pytest.mark.parametrize("precision,tol", [(1, ENC_TOL), (0, ENC_TOL_BF16)])
def test_encoder_long_vs_reference(abi, full_model, precision, tol):
    """The benchmark's lengths: 30 s, 10 s and 1.3 s (T_enc 376, 126 and 17)
    packed in one encoder batch, against the reference's own encoder
    (model.h:573-609 on backends/cpu/backend.c, compiled from the reference
    sources; tests/golden/make_encoder_long.py recorded its rows).  376 and
    126 rows cover several 64-key tiles of the relative-position attention:
    the online-softmax rescaling across tiles, position-table rows
    k - q + T_max - 1 far from the diagonal, and the depthwise-convolution
    halo between tiles.  Same weights as the other tests of this module
    (seed 21).  Both activation precisions: hi+lo planes (the default) and
    plain bf16."""
    import make_encoder_long as mel_long
    gold = np.load(po.os.path.join(po.os.path.dirname(inputs.__file__), "encoder_long_ref.npz"))
    mel, T_mel = mel_long.case()
    assert mel_long.WEIGHT_SEED == 21
    T_enc = t_enc_of(T_mel)
    assert list(T_enc) == [376, 126, 17]
    for b in range(len(T_mel)):
        assert np.isclose(mel[b, :, :T_mel[b]].astype(np.float64).sum(), float(gold[f"checksum{b}"]))
    eng = make_engine(abi, full_model, precision=precision)
    try:
        got = eng.encode(mels_of(mel, T_mel))
        assert eng.status() == 0
    finally:
        eng.close()
    errs = []
    for b in range(len(T_mel)):
        ref = gold[f"enc{b}"]
        assert got[b].shape == ref.shape
        err = float(np.max(np.abs(got[b] - ref)) / np.max(np.abs(ref)))
        errs.append(err)
        # per 64-row tile as well, so an error confined to a later key tile shows
        for r0 in range(0, ref.shape[0], 64):
            e_t = float(np.max(np.abs(got[b][r0:r0 + 64] - ref[r0:r0 + 64])) / np.max(np.abs(ref)))
            assert e_t <= tol, (b, r0, e_t)
    print(f"precision {precision}: encoder max error / output scale per utterance (T_enc 376, 126, 17):", errs)
    assert max(errs) <= tol, errs


@pytest.mark.parametrize("precision", [1, 0])
def test_encoder_batch_invariance_long(abi, full_model, precision):
    """Utterances past one 64-row tile (T_enc 376, 251, 126, 70, 17) encoded
    together equal their runs alone, with both activation precisions."""
    mel, T_mel = inputs.mel_batch([30.0, 20.0, 10.0, 5.55, 1.3], seed=703)
    assert t_enc_of(T_mel).min() < 64 < t_enc_of(T_mel).max()
    mels = mels_of(mel, T_mel)
    eng = make_engine(abi, full_model, precision=precision)
    try:
        together = eng.encode(mels)
        alone = [eng.encode([m])[0] for m in mels]
        assert eng.status() == 0
    finally:
        eng.close()
    for b in range(len(mels)):
        err = float(np.max(np.abs(together[b] - alone[b])))
        assert err <= 1e-6 * float(np.max(np.abs(alone[b]))), (b, err)


def test_encoder_batch_invariance(abi, full_model):
    """An utterance's encoder rows do not depend on the other utterances of
    the packed batch (row-wise GEMMs without K splits; attention and the
    convolutions stop at utterance boundaries; the position table depends only
    on the relative position).  Together the batch has more than 64 rows (the
    persistent GEMM kernel); alone each utterance has fewer (the tile kernel)."""
    mel, T_mel = inputs.mel_batch([2.9, 1.9, 3.27, 0.15, 2.2], seed=701)
    assert t_enc_of(T_mel).sum() > 64 and t_enc_of(T_mel).max() <= 64
    mels = mels_of(mel, T_mel)
    eng = make_engine(abi, full_model)
    try:
        together = eng.encode(mels)
        alone = [eng.encode([m])[0] for m in mels]
        assert eng.status() == 0
    finally:
        eng.close()
    for b in range(len(mels)):
        err = float(np.max(np.abs(together[b] - alone[b])))
        assert err <= 1e-6 * float(np.max(np.abs(alone[b]))), (b, err)


def test_submit_mel_end_to_end(abi, full_model, wmod):
    """Log-mel in, tokens out: equals submitting the engine's own encoder rows,
    and agrees with the oracle's encoder + decoder (teacher forced, at steps
    whose oracle top-2 margin is at least E2E_MARGIN_TOL)."""
    mel, T_mel = inputs.mel_batch([1.5, 0.62, 2.2], seed=702)
    forced = np.array([12, 7, 16], np.int32)
    mels = mels_of(mel, T_mel)
    eng = make_engine(abi, full_model)
    try:
        for b in range(3):
            eng.submit_mel(b, mels[b], forced[b])
        eng.run()
        via_mel = eng.poll()
        enc_rows = eng.encode(mels)
        for b in range(3):
            eng.submit(10 + b, enc_rows[b], forced[b])
        eng.run()
        via_enc = eng.poll()
        stats = eng.stats()
        assert eng.status() == 0
    finally:
        eng.close()
    assert stats["enc_utts"] == 6
    for b in range(3):
        assert np.array_equal(via_mel[b], via_enc[10 + b]), b
    ref = oracle_encode(wmod, full_model[1], mel, T_mel)
    T_enc = t_enc_of(T_mel)
    enc = np.zeros((3, int(T_enc.max()), 1024), np.float32)
    for b in range(3):
        enc[b, :T_enc[b]] = ref[b]
    prompt = np.array(inputs.ctb.PROMPT_FULL, np.int32)
    n_p = len(prompt)
    force = np.zeros((3, 1024), np.int32)
    for b in range(3):
        force[b, n_p:n_p + len(via_mel[b])] = via_mel[b]
    _tok, _n, am, mg = po.decode_batch(wmod.FULL_DIMS, full_model[1], enc, T_enc, prompt, forced, force_tokens=force)
    checked = 0
    for b in range(3):
        assert len(via_mel[b]) == forced[b] and via_mel[b][-1] == 3
        for g in range(forced[b] - 1):
            if mg[b, n_p + g] >= E2E_MARGIN_TOL:
                assert via_mel[b][g] == am[b, n_p + g], (b, g)
                checked += 1
    total = int(forced.sum()) - 3
    print(f"token positions checked (oracle margin >= {E2E_MARGIN_TOL}): {checked}/{total}")
    assert checked >= 0.8 * total, f"checked {checked}/{total}"
