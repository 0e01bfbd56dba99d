"""The no-allocation entry point, fd_decode_paged_noalloc, called through the
C ABI with ctypes.

It serves callers that cannot allocate device memory (a framework allocator
already holding the GPU's memory, or a serving loop that forbids allocation
after start-up); its split scratch is a fixed array inside the library.  The
test compares it with the allocating entry point fd_decode_paged on two calls
in a row (the second call finds the first call's scratch contents), and
checks that a shape needing more scratch than the fixed area is refused.
This file is collected last so a failure here cannot hide another test."""
import ctypes

import pytest
import torch

import flashdecode
from flashdecode import cases

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3
NOALLOC_SCRATCH_BYTES = 8 << 20


def _noalloc(lib, t, c, out, lse):
    return lib.fd_decode_paged_noalloc(
        t["q"].data_ptr(), t["k_cache"].data_ptr(), t["v_cache"].data_ptr(), out.data_ptr(),
        lse.data_ptr(), t["cache_seqlens"].data_ptr(), t["block_table"].data_ptr(),
        t["block_table"].shape[1], c.B, c.Hq, c.Hkv, c.D, c.page, c.num_blocks,
        0 if c.dtype == torch.bfloat16 else 1, 0 if c.dtype == torch.bfloat16 else 1,
        ctypes.c_float(c.softmax_scale), 0, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("which", ["split_heavy", "config2"])
def test_noalloc_matches_allocating_entry_point_twice(lib, which):
    if which == "split_heavy":  # many pairs split across CTAs -> scratch + combine in use
        c = cases.custom_case("noalloc", torch.bfloat16, [5000, 17, 9000, 1, 0, 300, 2049], 32, 8,
                              seed=12)
    else:
        c = cases.config_case(2)
    t = cases.materialize(c, "cuda", seed=12)
    ref_o, ref_l = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                            t["block_table"], softmax_scale=c.softmax_scale,
                                            return_softmax_lse=True)
    for call in range(2):
        out = torch.full_like(ref_o, float("nan"))
        lse = torch.full_like(ref_l, float("nan"))
        status = _noalloc(lib, t, c, out, lse)
        torch.cuda.synchronize()
        assert status == 0, flashdecode.last_error()
        err = (out.float() - ref_o.float()).abs()
        assert bool((err <= ATOL + RTOL * ref_o.float().abs()).all()), (call, float(err.max()))
        fin = torch.isfinite(ref_l)
        assert torch.equal(fin, torch.isfinite(lse)), call
        assert torch.allclose(lse[fin], ref_l[fin], atol=LSE_ATOL), call


def test_noalloc_refuses_shapes_beyond_its_scratch(lib):
    B, Hq, Hkv = 1024, 128, 16
    need = lib.fd_decode_workspace_size(B, Hq, Hkv, 128)
    assert need > NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    status = lib.fd_decode_paged_noalloc(p, p, p, p, None, p, p, 1, B, Hq, Hkv, 128, 16, 1, 0, 0,
                                         ctypes.c_float(0.1), 0, None)
    assert status == 3
    assert "scratch" in flashdecode.last_error()[1]
