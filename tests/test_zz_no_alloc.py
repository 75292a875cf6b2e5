"""ct_sdp_attn_batch_decode_noalloc: the batched decode attention for callers
that cannot call cudaMalloc (for example code running under CUDA graph stream
capture, where allocation is rejected, or with a fixed memory budget).  It
keeps its split-KV partials in a static device array instead of allocated
scratch.  Checked through the C ABI against the allocating entry point
backend_sdp_attn_batch_decode_ca on two calls in a row (the second call finds
the first call's data still in the shared array), at the tolerance the other
attention tests use (1e-5 absolute).

This file is named to be collected last, and it sets up its own backend state,
so it runs the same alone in a fresh process and after the other tests.
"""
import importlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _device_sync():
    import torch
    torch.cuda.synchronize()


def test_noalloc_attention_matches_allocating_entry_point(ctb):
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
        # beyond the static scratch: rejected before any launch
        rc = L.ct_sdp_attn_batch_decode_noalloc(out_d, qd, kd, vd, lens_d, 1024, 65, None)
        assert rc == -2
        assert L.ct_device_status() == 0
    finally:
        L.backend_thread_cleanup()
