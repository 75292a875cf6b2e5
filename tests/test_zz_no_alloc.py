"""ct_sdp_attn_batch_decode_noalloc: the batched decode attention for callers
that cannot call cudaMalloc (for example code running under CUDA graph stream
capture, where allocation is rejected, or with a fixed memory budget).  It
keeps its split-KV partials in a static device array instead of allocated
scratch.  Checked through the C ABI against the allocating entry point
backend_sdp_attn_batch_decode_ca on two calls in a row (the second call finds
the first call's data still in the shared array), at the tolerance the other
attention tests use (1e-5 absolute), and against the CPU oracle's batched
decode attention (backends/cpu/backend.c:478-500 restated) at the reference's
own kernel-test tolerance (1e-4 absolute).  A third call gives one item zero
keys: its output row is zero and the device status word reports a bad argument.

This file is named to be collected last, and it sets up its own backend state,
so it runs the same alone in a fresh process and after the other tests.
"""
import ctypes
import importlib

import numpy as np
import pytest

import pyoracle as po

pytestmark = pytest.mark.gpu

TOL = 1e-5
ORACLE_TOL = 1e-4
CT_STATUS_BAD_ARG = 4


def _device_sync():
    import torch
    torch.cuda.synchronize()


def test_noalloc_attention_matches_allocating_entry_point(ctb, wmod):
    abi = importlib.import_module("cohere-transcribe_b200.abi")
    L = abi.load()
    L.backend_init(0)
    try:
        A = abi.DeviceArena(L, 200 << 20)
        for call, (B, stride, seed) in enumerate([(12, 300, 1), (40, 1024, 2)]):
            rng = np.random.default_rng(seed)
            Q = rng.standard_normal((B, 1024), dtype=np.float32) * np.float32(0.3)
            K = rng.standard_normal((B, stride, 1024), dtype=np.float32) * np.float32(0.3)
            V = rng.standard_normal((B, stride, 1024), dtype=np.float32)
            lens = rng.integers(1, stride + 1, B).astype(np.int32)
            lens[:4] = [1, stride, min(128, stride), min(129, stride)]
            qd, kd, vd = A.put(Q), A.put(K), A.put(V)
            ref_d, out_d = A.take(B * 1024), A.take(B * 1024)
            lens_d = A.put(lens.view(np.float32))          # int32 bytes, device copy
            L.backend_upload_T_enc(lens.ctypes.data, B)
            L.backend_sdp_attn_batch_decode_ca(ref_d, qd, kd, vd, stride, B, None)
            ref = A.get(ref_d, (B, 1024))
            rc = L.ct_sdp_attn_batch_decode_noalloc(out_d, qd, kd, vd, lens_d, stride, B, None)
            assert rc == 0, f"call {call}: rc {rc}"
            _device_sync()
            got = A.get(out_d, (B, 1024))
            err = float(np.max(np.abs(got - ref)))
            assert err <= TOL, f"call {call}: max abs err {err}"
            orc = np.zeros((B, 1024), np.float32)
            O = po.lib()
            O.orc_sdp_attn_batch_decode(ctypes.byref(po.dims_struct(wmod.FULL_DIMS)), po.fp(orc), po.fp(Q), po.fp(K),
                                        po.fp(V), stride, B, po.ip(lens))
            err_o = float(np.max(np.abs(got - orc)))
            assert err_o <= ORACLE_TOL, f"call {call}: max abs err vs oracle {err_o}"
        # an item with no keys: defined as a zero row, reported in the status word
        lens0 = lens.copy()
        lens0[5] = 0
        lens0_d = A.put(lens0.view(np.float32))
        rc = L.ct_sdp_attn_batch_decode_noalloc(out_d, qd, kd, vd, lens0_d, stride, B, None)
        assert rc == 0
        _device_sync()
        got0 = A.get(out_d, (B, 1024))
        assert not np.any(got0[5]), "zero-length item must give a zero row"
        keep = np.arange(B) != 5
        assert float(np.max(np.abs(got0[keep] - got[keep]))) <= TOL
        assert L.ct_device_status() == CT_STATUS_BAD_ARG
        assert L.ct_device_status() == 0
        # beyond the static scratch: rejected before any launch
        rc = L.ct_sdp_attn_batch_decode_noalloc(out_d, qd, kd, vd, lens_d, 1024, 65, None)
        assert rc == -2
        assert L.ct_device_status() == 0
    finally:
        L.backend_thread_cleanup()
