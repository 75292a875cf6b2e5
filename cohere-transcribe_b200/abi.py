"""ctypes prototypes of libct_b200.so (the C ABI of include/ct_backend.h).

`load()` fails loudly when the library is missing: there is no CPU path.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import LIB_PATH

_f = ctypes.POINTER(ctypes.c_float)
_i = ctypes.POINTER(ctypes.c_int)
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_int = ctypes.c_int
_flt = ctypes.c_float

# name -> (restype, argtypes); weight pointers are passed as void* (host addresses)
SIGNATURES = {
    "backend_init": (None, [_int]),
    "backend_destroy": (None, []),
    "backend_num_devices": (_int, []),
    "backend_thread_cleanup": (None, []),
    "backend_weights_upload_blob": (None, [_vp, _sz]),
    "backend_device_ptr": (_vp, [_vp]),
    "backend_arena_alloc": (_vp, [_sz]),
    "backend_arena_free": (None, [_vp]),
    "backend_htod": (None, [_vp, _vp, _sz]),
    "backend_dtoh": (None, [_vp, _vp, _sz]),
    "backend_layernorm": (None, [_vp, _vp, _vp, _vp, _int, _int]),
    "backend_linear": (None, [_vp, _vp, _vp, _vp, _int, _int, _int]),
    "backend_linear_silu": (None, [_vp, _vp, _vp, _vp, _int, _int, _int]),
    "backend_linear_relu": (None, [_vp, _vp, _vp, _vp, _int, _int, _int]),
    "backend_linear_fmadd": (None, [_vp, _flt, _vp, _vp, _vp, _int, _int, _int]),
    "backend_add_inplace": (None, [_vp, _vp, _int]),
    "backend_encoder_subsampling": (None, [_vp, _int, _int, _vp, _int, _vp, _vp]),
    "backend_make_rel_pos_emb": (None, [_vp, _int]),
    "backend_rel_pos_mhsa": (None, [_vp, _vp, _int, _vp, _vp]),
    "backend_conformer_conv": (None, [_vp, _int, _vp, _vp]),
    "backend_sdp_attn": (None, [_vp, _vp, _vp, _vp, _vp, _int, _int, _vp]),
    "backend_embed": (None, [_vp, _vp, _int, _int, _vp, _vp, _vp, _vp]),
    "backend_fill_causal_mask": (None, [_vp, _int]),
    "backend_lm_head": (None, [_vp, _vp, _vp, _vp]),
    "backend_upload_tokens": (None, [_vp, _int]),
    "backend_graph_replay": (_int, [_int, _int, _int, _int]),
    "backend_graph_begin_capture": (None, [_int]),
    "backend_graph_end_capture": (None, [_int, _int, _int, _int]),
    "backend_decode_set_S": (None, [_int]),
    "backend_decode_inc_S": (None, []),
    "backend_linear_to_kvcache": (None, [_vp, _vp, _vp, _vp, _int, _int]),
    "backend_sdp_attn_devS": (None, [_vp, _vp, _vp, _vp, _vp]),
    "backend_embed_decode": (None, [_vp, _vp, _vp, _vp, _vp]),
    "backend_embed_decode_batch": (None, [_vp, _vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "backend_lm_head_batch": (None, [_vp, _vp, _vp, _vp, _vp, _int]),
    "backend_argmax_batch": (None, [_vp, _vp, _vp, _int]),
    "backend_upload_T_enc": (None, [_vp, _int]),
    "backend_linear_to_kvcache_batch": (None, [_vp, _vp, _vp, _vp, _int, _int, _int, _int]),
    "backend_sdp_attn_batch_decode_sa": (None, [_vp, _vp, _vp, _vp, _int, _int, _vp]),
    "backend_sdp_attn_batch_decode_ca": (None, [_vp, _vp, _vp, _vp, _int, _int, _vp]),
    # extensions
    "ct_device_status": (_int, []),
    "ct_selftest_bounded_wait": (_int, [_int, _int]),
    "ct_sdp_attn_batch_decode_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _int, _int, _vp]),
    # engine (include/ct_engine.h)
    "ct_engine_create": (_int, [_vp, _int, _vp, _sz, _vp, _vp]),
    "ct_engine_destroy": (None, [_vp]),
    "ct_engine_submit_encoded": (_int, [_vp, ctypes.c_longlong, _vp, _int, _int]),
    "ct_engine_step": (_int, [_vp, _int]),
    "ct_engine_run": (_int, [_vp]),
    "ct_engine_poll": (_int, [_vp, _vp, _int, _vp, _int]),
    "ct_engine_stats": (_int, [_vp, _vp]),
    "ct_engine_status": (_int, [_vp]),
    "ct_engine_profile_report": (_int, [_vp, _vp, _int]),
    "ct_engine_encode": (_int, [_vp, _int, _vp, _vp, _vp, _vp]),
    "ct_linear_bf16": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _vp]),
    "ct_engine_submit_mel": (_int, [_vp, ctypes.c_longlong, _vp, _int, _int]),
    "ct_engine_submit_audio": (_int, [_vp, ctypes.c_longlong, _vp, _int, _int]),
    "ct_engine_log_mel": (_int, [_vp, _int, _vp, _vp, _vp]),
    "ct_engine_step_times": (_int, [_vp, _vp, _int]),
    "ct_engine_set_prompt": (_int, [_vp, _vp, _int]),
    "ct_engine_last_logits": (_int, [_vp, _vp, _vp, _vp, _int]),
}


class EngineConfig(ctypes.Structure):
    _fields_ = [("max_slots", _int), ("max_rows", _int), ("kv_pages", _int), ("precision", _int),
                ("n_prompt", _int), ("prompt", _vp), ("profile", _int), ("no_pdl", _int),
                ("enc_max_utts", _int), ("enc_max_frames", _int), ("keep_logits", _int),
                ("fused_step", _int)]


class EngineStats(ctypes.Structure):
    _fields_ = [("steps", ctypes.c_longlong), ("rows", ctypes.c_longlong), ("tokens", ctypes.c_longlong),
                ("admitted", ctypes.c_longlong), ("step_ms", ctypes.c_double), ("admit_ms", ctypes.c_double),
                ("self_attn_ms", ctypes.c_double), ("cross_attn_ms", ctypes.c_double), ("ffn_ms", ctypes.c_double),
                ("self_kv_bytes", ctypes.c_double), ("cross_kv_bytes", ctypes.c_double),
                ("ffn_bytes", ctypes.c_double), ("attn_launches", ctypes.c_longlong),
                ("ffn_launches", ctypes.c_longlong), ("kernel_launches", ctypes.c_longlong),
                ("enc_ms", ctypes.c_double), ("enc_utts", ctypes.c_longlong), ("enc_frames", ctypes.c_longlong)]


class Result(ctypes.Structure):
    _fields_ = [("utt_id", ctypes.c_longlong), ("n_tokens", _int), ("status", _int)]


class Engine:
    """Thin owner of a ct_engine* (one per GPU, driven by one thread)."""

    def __init__(self, lib, device, wb, wstruct, max_slots=256, max_rows=1024, precision=1, kv_pages=0, profile=0,
                 no_pdl=0, enc_max_utts=0, enc_max_frames=0, keep_logits=0, fused_step=0):
        self.lib = lib
        self.wb = wb            # keeps the host blob alive (the engine copies it at creation)
        self.ws = wstruct
        cfg = EngineConfig(max_slots, max_rows, kv_pages, precision, 0, None, profile, no_pdl, enc_max_utts,
                           enc_max_frames, keep_logits, fused_step)
        h = ctypes.c_void_p()
        rc = lib.ct_engine_create(ctypes.byref(h), device, wb.ptr(), wb.nbytes, ctypes.addressof(wstruct),
                                  ctypes.byref(cfg))
        if rc != 0:
            raise RuntimeError(f"ct_engine_create failed: {rc}")
        self.h = h

    def submit(self, utt_id, enc_h, forced_len):
        a = np.ascontiguousarray(enc_h, dtype=np.float32)
        rc = self.lib.ct_engine_submit_encoded(self.h, utt_id, a.ctypes.data, a.shape[0], int(forced_len))
        if rc != 0:
            raise RuntimeError(f"submit failed: {rc}")

    def submit_mel(self, utt_id, mel, forced_len):
        a = np.ascontiguousarray(mel, dtype=np.float32)          # [N_MELS, T_mel]
        rc = self.lib.ct_engine_submit_mel(self.h, utt_id, a.ctypes.data, a.shape[1], int(forced_len))
        if rc != 0:
            raise RuntimeError(f"submit_mel failed: {rc}")

    def submit_audio(self, utt_id, samples, forced_len):
        a = np.ascontiguousarray(samples, dtype=np.float32)      # 16 kHz mono
        rc = self.lib.ct_engine_submit_audio(self.h, utt_id, a.ctypes.data, len(a), int(forced_len))
        if rc != 0:
            raise RuntimeError(f"submit_audio failed: {rc}")

    def log_mel(self, signals):
        """signals: list of 16 kHz float arrays -> list of [128, 1 + len // 160] log-mel."""
        arrs = [np.ascontiguousarray(x, dtype=np.float32) for x in signals]
        n = len(arrs)
        ptrs = (ctypes.c_void_p * n)(*[x.ctypes.data for x in arrs])
        ns = np.array([len(x) for x in arrs], np.int32)
        T = 1 + ns // 160
        out = np.zeros(int(T.sum()) * 128, np.float32)
        rc = self.lib.ct_engine_log_mel(self.h, n, ptrs, ns.ctypes.data, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"log_mel failed: {rc}")
        offs = np.concatenate([[0], np.cumsum(T)]) * 128
        return [out[offs[b]:offs[b + 1]].reshape(128, T[b]) for b in range(n)]

    def encode(self, mels):
        """mels: list of [N_MELS, T_mel] arrays -> list of [T_enc, DEC_D] encoder outputs."""
        arrs = [np.ascontiguousarray(m, dtype=np.float32) for m in mels]
        n = len(arrs)
        ptrs = (ctypes.c_void_p * n)(*[x.ctypes.data for x in arrs])
        T_mel = np.array([x.shape[1] for x in arrs], np.int32)
        t3 = ((((T_mel + 1) // 2) + 1) // 2 + 1) // 2
        out = np.zeros((int(t3.sum()), 1024), np.float32)
        T_enc = np.zeros(n, np.int32)
        rc = self.lib.ct_engine_encode(self.h, n, ptrs, T_mel.ctypes.data, out.ctypes.data, T_enc.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"encode failed: {rc}")
        offs = np.concatenate([[0], np.cumsum(T_enc)])
        return [out[offs[b]:offs[b + 1]] for b in range(n)]

    def set_prompt(self, prompt=None):
        """Prompt for the utterances submitted next (None: the engine default)."""
        if prompt is None:
            rc = self.lib.ct_engine_set_prompt(self.h, None, 0)
        else:
            p = np.ascontiguousarray(prompt, dtype=np.int32)
            rc = self.lib.ct_engine_set_prompt(self.h, p.ctypes.data, len(p))
        if rc != 0:
            raise RuntimeError(f"set_prompt failed: {rc}")

    def step_times(self):
        """Device ms of each step since the previous call (the log is cleared)."""
        out = np.empty(1 << 16, np.float32)
        n = self.lib.ct_engine_step_times(self.h, out.ctypes.data, len(out))
        if n < 0:
            raise RuntimeError(f"step_times failed: {n}")
        return out[:n].copy()

    def step(self, n=1):
        rc = self.lib.ct_engine_step(self.h, n)
        if rc < 0:
            raise RuntimeError(f"step failed: {rc}")
        return rc

    def run(self):
        rc = self.lib.ct_engine_run(self.h)
        if rc < 0:
            raise RuntimeError(f"run failed: {rc}")

    def poll(self, max_results=4096, tok_stride=1024):
        res = (Result * max_results)()
        # uninitialised: only the rows of returned results are written and read
        toks = np.empty((max_results, tok_stride), np.int32)
        n = self.lib.ct_engine_poll(self.h, res, max_results, toks.ctypes.data, tok_stride)
        if n < 0:
            raise RuntimeError(f"poll failed: {n}")
        return {res[i].utt_id: toks[i, :res[i].n_tokens].copy() for i in range(n)}

    def last_logits(self, vocab=16384, max_seqs=1024):
        """Logits of the most recent step: {utt_id: (generated-token index, fp32 [vocab])}."""
        lg = np.empty((max_seqs, vocab), np.float32)
        ids = np.empty(max_seqs, np.int64)
        gi = np.empty(max_seqs, np.int32)
        n = self.lib.ct_engine_last_logits(self.h, lg.ctypes.data, ids.ctypes.data, gi.ctypes.data, max_seqs)
        if n < 0:
            raise RuntimeError(f"last_logits failed: {n}")
        return {int(ids[i]): (int(gi[i]), lg[i].copy()) for i in range(n)}

    def stats(self):
        s = EngineStats()
        self.lib.ct_engine_stats(self.h, ctypes.byref(s))
        return {f: getattr(s, f) for f, _ in EngineStats._fields_}

    def status(self):
        return self.lib.ct_engine_status(self.h)

    def profile_report(self):
        import json
        buf = ctypes.create_string_buffer(1 << 16)
        self.lib.ct_engine_profile_report(self.h, buf, len(buf))
        return json.loads(buf.value.decode())

    def close(self):
        if self.h:
            self.lib.ct_engine_destroy(self.h)
            self.h = None

BACKEND_SYMBOLS = [n for n in SIGNATURES if n.startswith("backend_")]

_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libct_b200.so and set its prototypes (raises if it is not built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"{p} is missing: run __graft_entry__.build() (there is no CPU fallback)")
    L = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = L
    return L


class DeviceArena:
    """Device float buffers carved from the backend arena (backend_arena_alloc),
    mirroring how transcribe.c lays out its arena."""

    def __init__(self, lib: ctypes.CDLL, floats: int):
        self.lib = lib
        self.base = lib.backend_arena_alloc(floats)
        self.cap = floats
        self.off = 0

    def take(self, n: int) -> int:
        n = int(n)
        n = (n + 63) // 64 * 64          # keep every buffer 256-byte aligned
        if self.off + n > self.cap:
            raise MemoryError("arena exhausted")
        p = self.base + 4 * self.off
        self.off += n
        return p

    def put(self, arr: np.ndarray) -> int:
        a = np.ascontiguousarray(arr, dtype=np.float32)
        p = self.take(a.size)
        self.lib.backend_htod(p, a.ctypes.data, a.size)
        return p

    def get(self, ptr: int, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype)
        self.lib.backend_dtoh(out.ctypes.data, ptr, out.nbytes)
        return out
