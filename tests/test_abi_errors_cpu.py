"""CPU checks of the error behaviour of the extended C ABI (no GPU needed).

The engine and extension entry points return status codes and never exit
(include/ct_engine.h, include/ct_backend.h).  These are the argument checks
that run before any CUDA call, so they behave the same with or without a GPU:
NULL handles and pointers, out-of-range configurations, the no-allocation
attention's size limit, and the GEMM entry point's alignment rules.  On a host
without a GPU, engine creation with valid arguments ends in CT_EDEVICE rather
than a crash.
"""
import ctypes
import importlib

import pytest

CT_EINVAL, CT_EDEVICE = -1, -4
NOALLOC_EINVAL, NOALLOC_ETOOBIG = -1, -2


@pytest.fixture(scope="module")
def lib():
    return importlib.import_module("cohere-transcribe_b200.abi").load()


@pytest.fixture(scope="module")
def abi():
    return importlib.import_module("cohere-transcribe_b200.abi")


def _no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


def test_engine_calls_reject_a_null_handle(lib, abi):
    buf = (ctypes.c_float * 16)()
    res = (abi.Result * 4)()
    stats = abi.EngineStats()
    assert lib.ct_engine_step(None, 1) == CT_EINVAL
    assert lib.ct_engine_run(None) == CT_EINVAL
    assert lib.ct_engine_submit_encoded(None, 0, ctypes.addressof(buf), 1, 5) == CT_EINVAL
    assert lib.ct_engine_submit_mel(None, 0, ctypes.addressof(buf), 1, 5) == CT_EINVAL
    assert lib.ct_engine_submit_audio(None, 0, ctypes.addressof(buf), 16000, 5) == CT_EINVAL
    assert lib.ct_engine_poll(None, res, 4, None, 0) == CT_EINVAL
    assert lib.ct_engine_stats(None, ctypes.byref(stats)) == CT_EINVAL
    assert lib.ct_engine_status(None) == CT_EINVAL
    assert lib.ct_engine_set_prompt(None, None, 0) == CT_EINVAL
    assert lib.ct_engine_step_times(None, ctypes.addressof(buf), 16) == CT_EINVAL
    assert lib.ct_engine_profile_report(None, ctypes.addressof(buf), 64) == CT_EINVAL
    lib.ct_engine_destroy(None)          # a no-op, like free(NULL)


def _create(lib, abi, cfg, blob=True, weights=True):
    h = ctypes.c_void_p()
    data = (ctypes.c_uint8 * 64)()
    w = (ctypes.c_uint8 * 4096)()        # stand-in for the Weights table (never read on these paths)
    rc = lib.ct_engine_create(ctypes.byref(h), 0, ctypes.addressof(data) if blob else None, 64,
                              ctypes.addressof(w) if weights else None,
                              ctypes.byref(cfg) if cfg is not None else None)
    return rc, h


@pytest.mark.parametrize("field,value", [
    ("max_slots", 1025),        # row indices of attention entries are packed in 10 bits
    ("max_rows", 1025),         # one step packs at most 1024 query rows
    ("n_prompt", 97),           # prompts are 1-96 tokens
    ("n_prompt", 11),           # a non-default length needs its own prompt tokens
])
def test_engine_create_rejects_out_of_range_configs(lib, abi, field, value):
    cfg = abi.EngineConfig()
    setattr(cfg, field, value)
    rc, h = _create(lib, abi, cfg)
    assert rc == CT_EINVAL and not h.value


def test_engine_create_rejects_null_arguments(lib, abi):
    assert lib.ct_engine_create(None, 0, None, 0, None, None) == CT_EINVAL
    rc, h = _create(lib, abi, None, blob=False)
    assert rc == CT_EINVAL and not h.value
    rc, h = _create(lib, abi, None, weights=False)
    assert rc == CT_EINVAL and not h.value


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU failure path")
def test_engine_create_without_a_gpu_returns_a_code(lib, abi):
    rc, h = _create(lib, abi, abi.EngineConfig())
    assert rc == CT_EDEVICE and not h.value


def test_noalloc_attention_limits(lib):
    x = (ctypes.c_float * 4)()
    lens = (ctypes.c_int * 4)()
    p = ctypes.addressof(x)
    # a bad argument
    assert lib.ct_sdp_attn_batch_decode_noalloc(p, p, p, p, ctypes.addressof(lens), 0, 1, None) == NOALLOC_EINVAL
    assert lib.ct_sdp_attn_batch_decode_noalloc(p, p, p, p, ctypes.addressof(lens), 128, 0, None) == NOALLOC_EINVAL
    assert lib.ct_sdp_attn_batch_decode_noalloc(None, p, p, p, ctypes.addressof(lens), 128, 1, None) == NOALLOC_EINVAL
    # beyond the static scratch: more than 64 items at MAX_SEQ keys, or one item beyond MAX_SEQ x 64
    assert lib.ct_sdp_attn_batch_decode_noalloc(p, p, p, p, ctypes.addressof(lens), 1024, 65, None) == NOALLOC_ETOOBIG
    assert lib.ct_sdp_attn_batch_decode_noalloc(p, p, p, p, ctypes.addressof(lens), 1024 * 65, 1, None) \
        == NOALLOC_ETOOBIG


def test_linear_bf16_rejects_bad_shapes_and_alignment(lib):
    buf = (ctypes.c_uint8 * 4096)()
    a = (ctypes.addressof(buf) + 255) // 256 * 256      # 256-byte aligned inside buf
    ok = dict(Y=a, ldy=8, X_hi=a, X_lo=None, W=a, bias=None, T=1, K=8, N=8, act=0, stream=None)

    def call(**kw):
        d = dict(ok, **kw)
        return lib.ct_linear_bf16(d["Y"], d["ldy"], d["X_hi"], d["X_lo"], d["W"], d["bias"], d["T"], d["K"],
                                  d["N"], d["act"], d["stream"])
    assert call(K=12) == -1            # K must be a multiple of 8 (16-byte TMA rows)
    assert call(ldy=4) == -1           # ldy >= N
    assert call(act=3) == -1
    assert call(T=0) == -1
    assert call(W=a + 2) == -1         # TMA bases are 16-byte aligned
    assert call(X_lo=a + 8) == -1
    assert call(Y=None) == -1


def test_bounded_wait_selftest_rejects_bad_arguments(lib):
    """ct_selftest_bounded_wait checks its budget (1 us .. 1 s) and code
    (1 .. 255) before any CUDA call."""
    assert lib.ct_selftest_bounded_wait(0, 1) == CT_EINVAL
    assert lib.ct_selftest_bounded_wait(100, 0) == CT_EINVAL
    assert lib.ct_selftest_bounded_wait(100, 256) == CT_EINVAL
    assert lib.ct_selftest_bounded_wait(2000000, 1) == CT_EINVAL
