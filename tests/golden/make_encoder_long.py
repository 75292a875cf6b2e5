#!/usr/bin/env python3
"""Record the reference's own encoder output at the benchmark's lengths.

Writes tests/golden/encoder_long_ref.npz: the full-size encoder (48 Conformer
layers at width 1280, model.h dims) of the reference -- its model.h
encoder_forward_batch on its CPU backend, compiled from the reference sources
into oracle/_ref/libref_decode_cpu.so by oracle/Makefile -- run on seeded
N(0, 1) log-mel utterances of 30 s, 10 s and 1.3 s (T_enc 376, 126 and 17),
followed by a short greedy decode (EOS forced at the 6th generated token).

  enc{k}      [T_enc_k, 1024] float32 encoder rows of utterance k
  tokens{k}   the reference's token stream (prompt included)
  argmax{k}   its argmax per generated position (-1 elsewhere)
  margin{k}   its top-2 logit margin per generated position (NaN elsewhere)
  checksum{k} float64 sum of the utterance's log-mel (input drift check)

The relative-position attention of the engine works on 64-key tiles, so 126
and 376 rows cover several key tiles, the online-softmax rescaling between
them and position-table rows far from the diagonal; 1.3 s stays inside one
tile.  The reference runs each utterance in its own process (batch 1): its
encoder treats utterances independently, and the position-table slice it
gives utterance b in a batch holds the same values as a table built for T_b
alone (row T_max - T_b + j and row j of the smaller table are both relative
position T_b - 1 - j).

With --check-oracle the script also runs oracle/oracle.c's
orc_encoder_forward_batch on the same three utterances in one packed batch and
asserts its rows equal the reference's bit for bit.

The reference tree comes from the first argument or $CT_REFERENCE_DIR.  A 30 s
utterance takes the reference's single-threaded CPU backend about 20 minutes.
"""
import ctypes
import importlib
import multiprocessing as mp
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for p in (REPO, os.path.join(REPO, "oracle"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import inputs  # noqa: E402
import pyoracle  # noqa: E402

SECONDS = (30.0, 10.0, 1.3)
MEL_SEED = 710
WEIGHT_SEED = 21
FORCED = 6
OUT = os.path.join(HERE, "encoder_long_ref.npz")


def case():
    """(log-mel batch [3, 128, T_mel_max], T_mel) of the fixture."""
    return inputs.mel_batch(SECONDS, seed=MEL_SEED)


def _one(k: int):
    W = importlib.import_module("cohere-transcribe_b200.weights")
    ctb = importlib.import_module("cohere-transcribe_b200")
    mel, T_mel = case()
    t = int(T_mel[k])
    mk = np.ascontiguousarray(mel[k:k + 1, :, :t])
    L = pyoracle.bind_ref_decode(pyoracle.ref_lib("libref_decode_cpu.so"))
    wb = W.make_blob(W.FULL_DIMS, seed=WEIGHT_SEED)
    ws = W.weights_struct(wb)
    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    prompt = np.array(ctb.PROMPT_FULL, np.int32)
    forced = np.array([FORCED], np.int32)
    T_enc = ctb.t_enc_of(t)
    tokens = np.zeros((1, 1024), np.int32)
    n_tok = np.zeros(1, np.int32)
    am = np.full((1, 1024), -1, np.int32)
    mg = np.full((1, 1024), np.nan, np.float32)
    enc = np.zeros((1, T_enc, 1024), np.float32)
    L.refh_transcribe_batch(1, pyoracle.fp(mk), t, pyoracle.ip(np.array([t], np.int32)), pyoracle.ip(prompt),
                            len(prompt), pyoracle.ip(forced), pyoracle.null_i(), pyoracle.ip(tokens),
                            pyoracle.ip(n_tok), pyoracle.ip(am), pyoracle.fp(mg), pyoracle.fp(enc))
    L.backend_thread_cleanup()
    n = int(n_tok[0])
    return k, enc[0], tokens[0, :n].copy(), am[0, :n].copy(), mg[0, :n].copy()


def check_oracle(out: dict) -> None:
    W = importlib.import_module("cohere-transcribe_b200.weights")
    ctb = importlib.import_module("cohere-transcribe_b200")
    mel, T_mel = case()
    wb = W.make_blob(W.FULL_DIMS, seed=WEIGHT_SEED)
    ws = W.weights_struct(wb)
    T_enc = np.array([ctb.t_enc_of(int(t)) for t in T_mel], np.int32)
    Tm = int(T_enc.max())
    o = np.zeros((len(SECONDS), Tm, 1024), np.float32)
    O = pyoracle.lib()
    d = pyoracle.dims_struct(W.FULL_DIMS)
    O.orc_encoder_forward_batch(ctypes.byref(d), ctypes.addressof(ws), pyoracle.fp(mel), len(SECONDS),
                                mel.shape[2], pyoracle.ip(T_mel), pyoracle.ip(T_enc), Tm, pyoracle.fp(o))
    for k in range(len(SECONDS)):
        assert np.array_equal(o[k, :T_enc[k]], out[f"enc{k}"]), f"oracle differs from the reference, utterance {k}"
    print("oracle equals the reference bit for bit on", SECONDS)


def main(ref: str, check: bool) -> None:
    pyoracle.build(ref)
    mel, T_mel = case()
    with mp.get_context("spawn").Pool(len(SECONDS)) as pool:
        res = pool.map(_one, range(len(SECONDS)))
    out = {}
    for k, enc, tok, am, mg in res:
        out[f"enc{k}"] = enc
        out[f"tokens{k}"] = tok
        out[f"argmax{k}"] = am
        out[f"margin{k}"] = mg
        out[f"checksum{k}"] = np.float64(mel[k, :, :T_mel[k]].astype(np.float64).sum())
    np.savez_compressed(OUT, **out)
    print("wrote", OUT)
    if check:
        check_oracle(out)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    ref_dir = args[0] if args else os.environ.get("CT_REFERENCE_DIR", "")
    if not ref_dir:
        sys.exit("usage: make_encoder_long.py <reference tree> [--check-oracle] (or set CT_REFERENCE_DIR)")
    main(ref_dir, "--check-oracle" in sys.argv)
