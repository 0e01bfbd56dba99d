"""Failure detection on the GPU without a fault: a bounded in-kernel wait on a
barrier nothing arrives on gives up, reports FD_ERR_DEVICE_TIMEOUT, and the
CUDA context keeps working."""
import ctypes

import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import decode_reference

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_survives(lib):
    waited = ctypes.c_uint64(0)
    status = lib.fd_selftest_bounded_wait(2_000_000, ctypes.byref(waited))  # 2 ms budget
    assert status == 5, flashdecode.last_error()
    assert 2_000_000 <= waited.value < 500_000_000
    # the context is intact: a normal decode still runs and is correct
    c = cases.custom_case("after_timeout", torch.bfloat16, [300, 7], 32, 8, seed=1)
    t = cases.materialize(c, "cuda", seed=1)
    out = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                   t["block_table"])
    ref, _ = decode_reference(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"])
    assert torch.allclose(out.float().cpu(), ref, atol=2e-3, rtol=1e-2)
    assert flashdecode.device_status() == 0
