"""ctypes bindings for the CPU checker libraries (TEST INFRASTRUCTURE ONLY).

  liboracle.so              this directory's C restatement (oracle.c)
  _ref/libref_cpu.so        the reference's own backends/cpu/backend.c
  _ref/libref_decode_cpu.so the reference's model.h driven by ref_harness.c on
                            the reference CPU backend (full-size dims)
  _ref/libref_decode_tiny.so the same at the tiny configuration's dims
  _ref/libref_decode_cuda.so the reference's model.h on its own CUDA backend
                            (backends/cuda/backend.cu, sm_100a; GPU host only)

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_f = ctypes.POINTER(ctypes.c_float)
_i = ctypes.POINTER(ctypes.c_int)
_u16 = ctypes.POINTER(ctypes.c_uint16)
_vp = ctypes.c_void_p


class Dims(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "enc_d", "enc_ff", "enc_h", "enc_dk", "enc_n", "enc_ck", "sub_ch",
        "dec_d", "dec_ff", "dec_h", "dec_dk", "dec_n", "vocab", "max_seq", "n_mels")]


def dims_struct(d: dict) -> Dims:
    return Dims(**{k: d[k] for k, _ in Dims._fields_})


def build(reference_dir: str | None = None) -> None:
    """Compile liboracle.so (and, given the reference tree, oracle/_ref/)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if reference_dir and os.path.isdir(reference_dir):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={reference_dir}"], check=True)


def fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f)


def ip(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_i)


def u16p(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16)


_lib = None


def lib() -> ctypes.CDLL:
    """The restatement library (built on first use if missing)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        D = ctypes.POINTER(Dims)
        sigs = {
            "orc_layernorm": [_f, _f, _vp, _vp, ctypes.c_int, ctypes.c_int],
            "orc_linear": [_f, _f, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                           ctypes.c_float],
            "orc_add_inplace": [_f, _f, ctypes.c_int],
            "orc_encoder_subsampling": [D, _f, ctypes.c_int, ctypes.c_int, _f, ctypes.c_int, _vp],
            "orc_make_rel_pos_emb": [D, _f, ctypes.c_int],
            "orc_rel_pos_mhsa": [D, _f, _f, ctypes.c_int, _vp],
            "orc_conformer_conv": [D, _f, ctypes.c_int, _vp],
            "orc_sdp_attn": [D, _f, _f, _f, _f, _f, ctypes.c_int, ctypes.c_int],
            "orc_embed": [D, _f, _i, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp],
            "orc_fill_causal_mask": [_f, ctypes.c_int],
            "orc_lm_head": [D, _f, _f, _vp, _vp],
            "orc_argmax": [_f, ctypes.c_int],
            "orc_embed_decode_batch": [D, _f, _i, _i, _i, ctypes.c_int, _vp, _vp, _vp, _vp],
            "orc_lm_head_batch": [D, _f, _f, _vp, _vp, _i, ctypes.c_int],
            "orc_argmax_batch": [D, _i, _f, _i, ctypes.c_int],
            "orc_linear_to_kvcache_batch": [_f, _f, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, _i],
            "orc_sdp_attn_batch_decode": [D, _f, _f, _f, _f, ctypes.c_int, ctypes.c_int, _i],
            "orc_conformer_layer": [D, _f, _f, ctypes.c_int, _vp],
            "orc_encoder_forward_batch": [D, _vp, _f, ctypes.c_int, ctypes.c_int, _i, _i, ctypes.c_int, _f],
            "orc_decode_batch": [D, _vp, ctypes.c_int, _i, ctypes.c_int, _f, _i, ctypes.c_int, _i, _i,
                                 _i, _i, _i, _f],
            "orc_decode_batch_logits": [D, _vp, ctypes.c_int, _i, ctypes.c_int, _f, _i, ctypes.c_int, _i, _i,
                                        _i, _i, _i, _f, _f, ctypes.c_int],
            "orc_compute_mel": [_f, ctypes.c_int, _f],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int if name in ("orc_argmax", "orc_decode_batch", "orc_decode_batch_logits") else None
        _lib = L
    return _lib


def ref_lib(name: str) -> ctypes.CDLL | None:
    """A library under oracle/_ref/ (None when the reference was not built)."""
    path = os.path.join(REF_DIR, name)
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


def bind_ref_decode(L: ctypes.CDLL) -> ctypes.CDLL:
    """Prototypes of ref_harness.c (for any library built from it)."""
    L.refh_bind_weights.argtypes = [_vp]
    L.refh_bind_weights.restype = None
    L.refh_decode_from_enc.argtypes = [ctypes.c_int, _f, _i, ctypes.c_int, _i, ctypes.c_int, _i, _i,
                                       _i, _i, _i, _f]
    L.refh_decode_from_enc.restype = ctypes.c_double
    L.refh_transcribe_batch.argtypes = [ctypes.c_int, _f, ctypes.c_int, _i, _i, ctypes.c_int, _i, _i,
                                        _i, _i, _i, _f, _f]
    L.refh_transcribe_batch.restype = ctypes.c_double
    L.refh_parallel_decode.argtypes = [ctypes.c_int, ctypes.c_int, _f, _i, ctypes.c_int, _i,
                                       ctypes.c_int, _i, _i, _i]
    L.refh_parallel_decode.restype = ctypes.c_double
    if hasattr(L, "refh_parallel_transcribe"):
        L.refh_parallel_transcribe.argtypes = [ctypes.c_int, ctypes.c_int, _f, ctypes.c_int, _i, _i, ctypes.c_int,
                                               _i, _i, _i]
        L.refh_parallel_transcribe.restype = ctypes.c_double
    if hasattr(L, "refh_capture_logits"):
        L.refh_capture_logits.argtypes = [_f, ctypes.c_int]
        L.refh_capture_logits.restype = None
    for fn in ("backend_weights_upload_blob",):
        getattr(L, fn).argtypes = [_vp, ctypes.c_size_t]
        getattr(L, fn).restype = None
    L.backend_init.argtypes = [ctypes.c_int]
    L.backend_init.restype = None
    L.backend_thread_cleanup.argtypes = []
    L.backend_thread_cleanup.restype = None
    return L


def null_i():
    return ctypes.cast(None, _i)


def null_f():
    return ctypes.cast(None, _f)


def decode_batch(dims: dict, wstruct, enc_h: np.ndarray, T_enc: np.ndarray, prompt,
                 forced_len, force_tokens=None, want_margin=True, logits_cap: int = 0):
    """Run orc_decode_batch.  enc_h: [B, T_enc_stride, dec_d] float32.
    Returns (tokens [B,max_seq], n_tok [B], argmax [B,max_seq], margin [B,max_seq]);
    with logits_cap > 0 also logits [B, logits_cap, vocab] of generated tokens
    0 .. logits_cap - 1 (orc_decode_batch_logits)."""
    L = lib()
    d = dims_struct(dims)
    B, stride, _ = enc_h.shape
    ms = dims["max_seq"]
    T_enc = np.ascontiguousarray(T_enc, dtype=np.int32)
    prompt = np.ascontiguousarray(prompt, dtype=np.int32)
    forced = np.ascontiguousarray(forced_len, dtype=np.int32)
    tokens = np.zeros((B, ms), np.int32)
    n_tok = np.zeros(B, np.int32)
    am = np.full((B, ms), -1, np.int32)
    mg = np.full((B, ms), np.nan, np.float32)
    ft = None if force_tokens is None else np.ascontiguousarray(force_tokens, dtype=np.int32)
    lg = np.zeros((B, logits_cap, dims["vocab"]), np.float32) if logits_cap > 0 else None
    L.orc_decode_batch_logits(ctypes.byref(d), ctypes.addressof(wstruct), B, ip(T_enc), stride,
                              fp(np.ascontiguousarray(enc_h, dtype=np.float32)), ip(prompt), len(prompt),
                              ip(forced), ip(ft) if ft is not None else null_i(), ip(tokens), ip(n_tok),
                              ip(am), fp(mg) if want_margin else null_f(),
                              fp(lg) if lg is not None else null_f(), logits_cap)
    if lg is not None:
        return tokens, n_tok, am, mg, lg
    return tokens, n_tok, am, mg


def compute_mel(samples: np.ndarray) -> np.ndarray:
    """Oracle log-mel of 16 kHz samples: [128, 1 + N // 160] (transcribe.c:177-214)."""
    x = np.ascontiguousarray(samples, dtype=np.float32)
    out = np.zeros((128, 1 + len(x) // 160), np.float32)
    lib().orc_compute_mel(fp(x), len(x), fp(out))
    return out
