"""GPU test of the bounded device waits: a wait that runs out ends with a
status code, not a hang or a trap.

Every pipeline wait of the library (mbarrier phases of the GEMM, attention and
encoder kernels, the attention tickets) gives up after a time budget, records a
code in the device status word and returns.  ct_selftest_bounded_wait runs
that same wait on a barrier phase nothing completes, with a short budget; the
test checks the code comes back, that the wait lasted its budget, that the
status word is cleared by the read, and that the context still computes
correctly afterwards (a GEMM through ct_linear_bf16 against torch fp32).
"""
import importlib
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CT_STATUS_TIMEOUT_TMA, CT_STATUS_TIMEOUT_MMA = 1, 2


@pytest.fixture(scope="module")
def lib():
    return importlib.import_module("cohere-transcribe_b200.abi").load()


def test_expired_wait_reports_its_code_and_leaves_the_context_usable(lib):
    import torch
    torch.cuda.init()
    t0 = time.perf_counter()
    assert lib.ct_selftest_bounded_wait(2000, CT_STATUS_TIMEOUT_MMA) == CT_STATUS_TIMEOUT_MMA
    assert time.perf_counter() - t0 >= 2e-3
    # the read cleared the word: a second expiry reports its own code
    assert lib.ct_selftest_bounded_wait(500, CT_STATUS_TIMEOUT_TMA) == CT_STATUS_TIMEOUT_TMA
    # the context still works: a GEMM on the tensor cores agrees with torch fp32
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(64, 1024, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(512, 1024, device="cuda", generator=g) / 32).to(torch.bfloat16)
    y = torch.zeros(64, 512, device="cuda")
    rc = lib.ct_linear_bf16(y.data_ptr(), 512, x.data_ptr(), None, w.data_ptr(), None, 64, 1024, 512, 0, None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    err = float((y - ref).abs().max() / ref.abs().max())
    assert err < 5e-5, err
    assert lib.ct_selftest_bounded_wait(1, 3) == 3

