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


def test_exchange_merge_times_out_when_a_peer_never_publishes(lib):
    """Cross-GPU split-KV on one GPU with a peer that never runs: rank 0's two
    exchange buffers are both local, only rank 0's step is launched, so rank
    1's flag is never set.  Rank 0's merge kernel must give up after its
    bounded wait (1 s), report FD_ERR_DEVICE_TIMEOUT, write nothing, and leave
    the context usable."""
    B, Hq, Hkv = 2, 32, 8
    c = cases.custom_case("xgpu_timeout", torch.bfloat16, [500, 90], Hq, Hkv, seed=3)
    t = cases.materialize(c, "cuda", seed=3)
    size = lib.fd_xgpu_buffer_size(B, 1, Hq, 2)
    assert size > 0
    bufs, handles = [], []
    for _ in range(2):
        p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        assert lib.fd_xgpu_alloc(size, ctypes.byref(p), h) == 0, flashdecode.last_error()
        bufs.append(p.value)
    try:
        xbufs = (ctypes.c_void_p * 2)(*bufs)
        out = torch.full((B, 1, Hq, 128), 7.0, dtype=torch.bfloat16, device="cuda")
        lse = torch.full((B, Hq), 7.0, dtype=torch.float32, device="cuda")
        nb, page = t["k_cache"].shape[0], t["k_cache"].shape[1]
        status = lib.fd_decode_paged_xgpu(
            t["q"].data_ptr(), t["k_cache"].data_ptr(), t["v_cache"].data_ptr(),
            t["cache_seqlens"].data_ptr(), t["block_table"].data_ptr(), t["block_table"].shape[1],
            B, 1, Hq, Hkv, 128, page, nb, 0, 0, c.softmax_scale, 0, 0, 0, 2, xbufs, 0,
            out.data_ptr(), lse.data_ptr(), None, 0, torch.cuda.current_stream().cuda_stream)
        assert status == 0, flashdecode.last_error()
        assert lib.fd_device_status() == 5  # FD_ERR_DEVICE_TIMEOUT, reported once
        assert bool((out.float() == 7.0).all()) and bool((lse == 7.0).all())  # nothing written
        assert lib.fd_device_status() == 0
    finally:
        for p in bufs:
            lib.fd_xgpu_free(p)
    o2 = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                  t["block_table"])
    ref, _ = decode_reference(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], t["block_table"])
    assert torch.allclose(o2.float().cpu(), ref, atol=2e-3, rtol=1e-2)
