#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory from the REFERENCE code.

Needs the reference source tree (argument or $CT_REFERENCE_DIR); it compiles
the reference's own CPU backend, kernel test program and model graph (through
oracle/Makefile into oracle/_ref/) and records their outputs:

  test_kernels_ref_cpu.bin   tests/test_kernels.c of the reference on its CPU
                             backend (LCG seed 0xdeadbeef; 9 kernels)
  struct_offsets_ref.txt     field offsets of the reference weight-table structs
  tiny_e2e_ref.npz           configuration 1 end to end (log-mel -> tokens) on the
                             reference model.h + CPU backend at the tiny dims
  full_decode_ref.npz        full-size decoder: prefill + batched greedy decode of
                             two sequences from seeded encoder outputs
  mel_ref.npz                the log-mel front-end (transcribe.c compute_mel) on
                             seeded 16 kHz signals
  longform_ref.npz           the long-form split points (transcribe.c:484-507) of
                             seeded signals with silences

Inputs are regenerated from seeds by tests/golden/inputs.py; a checksum of
each input is stored with the outputs so drift is detected.
"""
import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, HERE)

import importlib  # noqa: E402

import inputs  # noqa: E402
import pyoracle  # noqa: E402

ctb = importlib.import_module("cohere-transcribe_b200")
W = importlib.import_module("cohere-transcribe_b200.weights")


def main(ref: str) -> None:
    pyoracle.build(ref)
    rdir = pyoracle.REF_DIR

    # 1. the reference kernel test program
    subprocess.run([os.path.join(rdir, "test_kernels_ref"), os.path.join(HERE, "test_kernels_ref_cpu.bin")],
                   check=True, stderr=subprocess.DEVNULL)

    # 2. struct layout of the reference header
    exe = os.path.join(rdir, "struct_offsets_ref")
    subprocess.run(["gcc", "-O0", f"-DMODEL_TYPES_HEADER=\"{ref}/backends/model_types.h\"",
                    "-o", exe, os.path.join(HERE, "struct_offsets.c")], check=True)
    with open(os.path.join(HERE, "struct_offsets_ref.txt"), "w") as fh:
        fh.write(subprocess.run([exe], check=True, capture_output=True, text=True).stdout)

    # 3. configuration 1, tiny, end to end on the reference
    case = inputs.tiny_e2e_case()
    L = pyoracle.bind_ref_decode(pyoracle.ref_lib("libref_decode_tiny.so"))
    wb = W.make_blob(W.TINY_DIMS, seed=case["weight_seed"])
    ws = W.weights_struct(wb, enc_n=2, dec_n=2)
    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    B = case["mel"].shape[0]
    tokens = np.zeros((B, 1024), np.int32)
    n_tok = np.zeros(B, np.int32)
    am = np.full((B, 1024), -1, np.int32)
    mg = np.full((B, 1024), np.nan, np.float32)
    enc_h = np.zeros((B, ctb.t_enc_of(case["T_mel_max"]), 256), np.float32)
    L.refh_transcribe_batch(B, pyoracle.fp(case["mel"]), case["T_mel_max"], pyoracle.ip(case["T_mel"]),
                            pyoracle.ip(case["prompt"]), len(case["prompt"]), pyoracle.ip(case["forced_len"]),
                            pyoracle.null_i(), pyoracle.ip(tokens), pyoracle.ip(n_tok), pyoracle.ip(am),
                            pyoracle.fp(mg), pyoracle.fp(enc_h))
    np.savez_compressed(os.path.join(HERE, "tiny_e2e_ref.npz"), tokens=tokens, n_tok=n_tok, argmax=am,
                        margin=mg, enc_h=enc_h, mel_checksum=np.float64(case["mel"].astype(np.float64).sum()))

    # 4. full-size decoder slice on the reference
    case = inputs.full_decode_case()
    L = pyoracle.bind_ref_decode(pyoracle.ref_lib("libref_decode_cpu.so"))
    wb = W.make_blob(W.FULL_DIMS, seed=case["weight_seed"], parts=("dec",))
    ws = W.weights_struct(wb)
    L.refh_bind_weights(ctypes.addressof(ws))
    L.backend_init(0)
    enc = case["enc_h"]
    B, T_max, _ = enc.shape
    tokens = np.zeros((B, 1024), np.int32)
    n_tok = np.zeros(B, np.int32)
    am = np.full((B, 1024), -1, np.int32)
    mg = np.full((B, 1024), np.nan, np.float32)
    L.refh_decode_from_enc(B, pyoracle.fp(enc), pyoracle.ip(case["T_enc"]), T_max,
                           pyoracle.ip(case["prompt"]), len(case["prompt"]), pyoracle.ip(case["forced_len"]),
                           pyoracle.null_i(), pyoracle.ip(tokens), pyoracle.ip(n_tok), pyoracle.ip(am),
                           pyoracle.fp(mg))
    np.savez_compressed(os.path.join(HERE, "full_decode_ref.npz"), tokens=tokens, n_tok=n_tok, argmax=am,
                        margin=mg, enc_checksum=np.float64(enc.astype(np.float64).sum()))
    make_mel_fixture()
    make_longform_fixture()
    print("golden fixtures written to", HERE)


def make_mel_fixture() -> None:
    """5. the reference front-end (transcribe.c compute_mel) on seeded signals."""
    R = ctypes.CDLL(os.path.join(pyoracle.REF_DIR, "libref_mel.so"))
    R.refmel_compute.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    out = {}
    for k, (seconds, seed) in enumerate(inputs.mel_case()):
        x = inputs.audio(seconds, seed)
        mel = np.zeros((128, 1 + len(x) // 160), np.float32)
        R.refmel_compute(x.ctypes.data, len(x), mel.ctypes.data)
        out[f"mel{k}"] = mel
        out[f"checksum{k}"] = np.float64(x.astype(np.float64).sum())
    np.savez_compressed(os.path.join(HERE, "mel_ref.npz"), **out)


def make_longform_fixture() -> None:
    """6. the reference's long-form split points (transcribe.c:484-507)."""
    R = ctypes.CDLL(os.path.join(pyoracle.REF_DIR, "libref_mel.so"))
    R.refsplit.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                           ctypes.c_void_p, ctypes.c_int]
    out = {}
    for k, (seconds, seed, db, dur, target) in enumerate(inputs.longform_case()):
        x = inputs.speech_like(seconds, seed)
        buf = np.zeros(4096, np.int32)
        n = R.refsplit(x.ctypes.data, len(x), db, dur, target, buf.ctypes.data, len(buf))
        out[f"splits{k}"] = buf[:n].copy()
        out[f"checksum{k}"] = np.float64(x.astype(np.float64).sum())
    np.savez_compressed(os.path.join(HERE, "longform_ref.npz"), **out)


if __name__ == "__main__":
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CT_REFERENCE_DIR", "")
    if not ref_dir:
        sys.exit("usage: make_golden.py <reference tree> (or set CT_REFERENCE_DIR)")
    main(ref_dir)
