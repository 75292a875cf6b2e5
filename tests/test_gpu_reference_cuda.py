"""The reference's own CUDA backend as a secondary oracle.

oracle/_ref/libref_decode_cuda.so is the reference's model.h driven by
oracle/ref_harness.c on the reference's backends/cuda/backend.cu, compiled
from the reference sources for sm_100a by oracle/Makefile (`make ref-cuda`).
On the same seeded inputs and weights as the engine tests:

* decode from encoder outputs: the engine's logits, teacher forced on the
  engine's tokens, agree with the reference CUDA backend's logits within the
  engine's stated tolerance (LOGIT_RTOL of tests/test_gpu_engine.py), and the
  engine's tokens equal the reference CUDA argmax wherever its top-2 margin is
  at least MARGIN_TOL.  The reference CUDA logits are themselves checked
  against the CPU oracle (fp32 both, summation orders differ).
* the encoder: the reference CUDA encoder (48 layers, full width) on the
  10 s and 1.3 s utterances of tests/golden/encoder_long_ref.npz agrees with
  the reference CPU encoder recorded there, as the engine's does.
"""
import ctypes
import importlib
import os
import time

import numpy as np
import pytest

import inputs
import pyoracle as po

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 5e-3       # engine (bf16 K/V pages, hi+lo planes) vs an fp32 backend: tests/test_gpu_engine.py
REF_RTOL = 1e-4         # reference CUDA vs reference-equivalent CPU oracle, both fp32
MARGIN_TOL = 2e-3
ENC_TOL = 2e-3


def _ref_cuda():
    L = po.ref_lib("libref_decode_cuda.so")
    if L is None:
        pytest.skip("oracle/_ref/libref_decode_cuda.so not built (make -C oracle ref-cuda REF=<reference tree>)")
    return po.bind_ref_decode(L)


@pytest.fixture(scope="module")
def dec_model(wmod):
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=0, parts=("dec",))
    return wb, wmod.weights_struct(wb)


@pytest.fixture(scope="module")
def abi():
    a = importlib.import_module("cohere-transcribe_b200.abi")
    a.load()
    return a


def engine_decode_with_logits(abi, model, enc, T_enc, forced):
    wb, ws = model
    B, cap = len(T_enc), int(forced.max())
    got = np.full((B, cap, 16384), np.nan, np.float32)
    eng = abi.Engine(abi.load(), 0, wb, ws, keep_logits=1)
    try:
        for b in range(B):
            eng.submit(b, enc[b, :T_enc[b]], forced[b])
        while True:
            left = eng.step(1)
            for uid, (g, row) in eng.last_logits().items():
                got[uid, g] = row
            if left == 0:
                break
        out = eng.poll()
        assert eng.status() == 0
    finally:
        eng.close()
    return out, got


def ref_cuda_decode(model, enc, T_enc, forced, force_tokens, cap):
    """Teacher-forced decode on the reference CUDA backend; (argmax, margin, logits)."""
    wb, ws = model
    L = _ref_cuda()
    B, T_max = len(T_enc), enc.shape[1]
    prompt = np.array(inputs.ctb.PROMPT_FULL, np.int32)
    tokens = np.zeros((B, 1024), np.int32)
    n_tok = np.zeros(B, np.int32)
    am = np.full((B, 1024), -1, np.int32)
    mg = np.full((B, 1024), np.nan, np.float32)
    lg = np.zeros((B, cap, 16384), np.float32)
    L.backend_weights_upload_blob(wb.ptr(), wb.nbytes)
    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    L.refh_capture_logits(po.fp(lg), cap)
    t0 = time.perf_counter()
    L.refh_decode_from_enc(B, po.fp(np.ascontiguousarray(enc)), po.ip(T_enc), T_max, po.ip(prompt), len(prompt),
                           po.ip(forced), po.ip(force_tokens), po.ip(tokens), po.ip(n_tok), po.ip(am), po.fp(mg))
    dt = time.perf_counter() - t0
    L.refh_capture_logits(po.null_f(), 0)
    L.backend_destroy()
    return am, mg, lg, dt


def _force(out, B, n_p):
    force = np.zeros((B, 1024), np.int32)
    for b in range(B):
        force[b, n_p:n_p + len(out[b])] = out[b]
    return force


@pytest.mark.parametrize("case_name", ["ragged6", "config2"])
def test_engine_vs_reference_cuda_decode(abi, dec_model, wmod, case_name):
    if case_name == "ragged6":
        case = inputs.ragged_decode_case(6, seed=310, l_lo=8, l_hi=40)
        T_enc, forced = case["T_enc"], case["forced_len"]
        enc = inputs.enc_outputs(T_enc, case["enc_seed"])
    else:   # configuration 2's decode: one 30 s utterance (T_enc 376), EOS forced at token 200
        T_enc, forced = np.array([376], np.int32), np.array([200], np.int32)
        enc = inputs.enc_outputs(T_enc, seed=620)
    B, cap = len(T_enc), int(forced.max())
    n_p = len(inputs.ctb.PROMPT_FULL)
    out, got = engine_decode_with_logits(abi, dec_model, enc, T_enc, forced)
    force = _force(out, B, n_p)
    r_am, r_mg, r_lg, dt = ref_cuda_decode(dec_model, enc, T_enc, forced, force, cap)
    _t, _n, o_am, o_mg, o_lg = po.decode_batch(wmod.FULL_DIMS, dec_model[1], enc, T_enc,
                                               np.array(inputs.ctb.PROMPT_FULL, np.int32), forced,
                                               force_tokens=force, logits_cap=cap)
    worst_e, worst_r, checked, total = 0.0, 0.0, 0, 0
    for b in range(B):
        assert len(out[b]) == forced[b]
        for g in range(forced[b]):
            scale = float(np.max(np.abs(r_lg[b, g])))
            e = float(np.max(np.abs(got[b, g] - r_lg[b, g]))) / scale
            r = float(np.max(np.abs(r_lg[b, g] - o_lg[b, g]))) / scale
            worst_e, worst_r = max(worst_e, e), max(worst_r, r)
            if g < forced[b] - 1:
                total += 1
                if r_mg[b, n_p + g] >= MARGIN_TOL:
                    assert out[b][g] == r_am[b, n_p + g], (b, g, f"checked {checked}/{total}")
                    checked += 1
    msg = (f"{case_name}: engine vs reference CUDA max logit rel err {worst_e:.2e}; reference CUDA vs CPU oracle "
           f"{worst_r:.2e}; tokens checked {checked}/{total}; reference CUDA decode {dt:.2f} s")
    print(msg)
    assert worst_e <= LOGIT_RTOL, msg
    assert worst_r <= REF_RTOL, msg
    assert checked >= 0.8 * total, msg


def test_reference_cuda_encoder_vs_reference_cpu(wmod):
    """The reference CUDA encoder on the 10 s and 1.3 s utterances of the long
    fixture (batch of two) equals the reference CPU encoder there within
    ENC_TOL, and its first tokens equal the CPU run's where the margin allows."""
    import make_encoder_long as mel_long
    gold = np.load(os.path.join(os.path.dirname(inputs.__file__), "encoder_long_ref.npz"))
    L = _ref_cuda()
    mel3, T_mel3 = mel_long.case()
    sel = [1, 2]
    T_mel = np.ascontiguousarray(T_mel3[sel])
    mel = np.ascontiguousarray(mel3[sel][:, :, :int(T_mel.max())])
    wb = wmod.make_blob(wmod.FULL_DIMS, seed=mel_long.WEIGHT_SEED)
    ws = wmod.weights_struct(wb)
    B = len(sel)
    T_enc = np.array([inputs.ctb.t_enc_of(int(t)) for t in T_mel], np.int32)
    prompt = np.array(inputs.ctb.PROMPT_FULL, np.int32)
    forced = np.full(B, mel_long.FORCED, np.int32)
    tokens = np.zeros((B, 1024), np.int32)
    n_tok = np.zeros(B, np.int32)
    am = np.full((B, 1024), -1, np.int32)
    mg = np.full((B, 1024), np.nan, np.float32)
    enc = np.zeros((B, int(T_enc.max()), 1024), np.float32)
    L.backend_weights_upload_blob(wb.ptr(), wb.nbytes)
    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    t0 = time.perf_counter()
    L.refh_transcribe_batch(B, po.fp(mel), mel.shape[2], po.ip(T_mel), po.ip(prompt), len(prompt), po.ip(forced),
                            po.null_i(), po.ip(tokens), po.ip(n_tok), po.ip(am), po.fp(mg), po.fp(enc))
    dt = time.perf_counter() - t0
    L.backend_destroy()
    for i, k in enumerate(sel):
        ref = gold[f"enc{k}"]
        err = float(np.max(np.abs(enc[i, :T_enc[i]] - ref)) / np.max(np.abs(ref)))
        assert err <= ENC_TOL, (k, err)
        g_tok, g_mg = gold[f"tokens{k}"], gold[f"margin{k}"]
        n_p = len(prompt)
        for p in range(n_p, len(g_tok) - 1):
            if g_mg[p] >= 0.05:
                assert tokens[i, p] == g_tok[p], (k, p)
    print(f"reference CUDA encoder + decode of 10 s + 1.3 s: {dt:.2f} s")
