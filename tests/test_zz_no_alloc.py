"""The no-allocation entry point, fd_decode_paged_noalloc, called through the
C ABI with ctypes.

It serves callers that cannot allocate device memory (a framework allocator
already holding the GPU's memory, or a serving loop that forbids allocation
after start-up); its split scratch is a fixed array inside the library.  The
tests compare it with the CPU oracle and with the allocating entry point
fd_decode_paged on two calls in a row (the second call finds the first
call's scratch contents), check in a fresh process that it allocates nothing
(free device memory unchanged, no library-owned workspace created), that a
shape needing more scratch than the fixed area is refused, and that shapes
the CUDA-core kernel takes (which use no scratch) are not.  This file is
collected last so a failure here cannot hide another test."""
import ctypes
import json
import os
import subprocess
import sys

import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import decode_reference

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3
NOALLOC_SCRATCH_BYTES = 8 << 20
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _noalloc(lib, t, c, out, lse):
    return lib.fd_decode_paged_noalloc(
        t["q"].data_ptr(), t["k_cache"].data_ptr(), t["v_cache"].data_ptr(), out.data_ptr(),
        lse.data_ptr(), t["cache_seqlens"].data_ptr(), t["block_table"].data_ptr(),
        t["block_table"].shape[1], c.B, c.Hq, c.Hkv, c.D, c.page, c.num_blocks,
        0 if c.dtype == torch.bfloat16 else 1, 0 if c.dtype == torch.bfloat16 else 1,
        ctypes.c_float(c.softmax_scale), 0, torch.cuda.current_stream().cuda_stream)


def _close(out, lse, ref_o, ref_l, what):
    err = (out.float().cpu() - ref_o.float().cpu()).abs()
    assert bool((err <= ATOL + RTOL * ref_o.float().cpu().abs()).all()), (what, float(err.max()))
    fin = torch.isfinite(ref_l.cpu())
    assert torch.equal(fin, torch.isfinite(lse.cpu())), what
    assert torch.allclose(lse.cpu()[fin], ref_l.cpu()[fin], atol=LSE_ATOL), what


def _split_heavy():
    # many pairs split across CTAs -> scratch and the in-kernel merge in use
    return cases.custom_case("noalloc", torch.bfloat16, [5000, 17, 9000, 1, 0, 300, 2049], 32, 8,
                             seed=12)


@pytest.mark.parametrize("which", ["split_heavy", "config2"])
def test_noalloc_matches_allocating_entry_point_twice(lib, which):
    c = _split_heavy() if which == "split_heavy" else cases.config_case(2)
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
        _close(out, lse, ref_o, ref_l, f"call {call}")
    assert lib.fd_device_status() == 0


# Run in a fresh process by test_noalloc_in_a_fresh_process_allocates_nothing
# (argv[1] = repository root): the no-allocation entry point makes the first
# decode calls of the process, and the oracle checks them afterwards.
_FRESH = r"""
import ctypes, json, sys
root = sys.argv[1]
sys.path[:0] = [root, root + "/flashatte-hand_b200", root + "/tests"]
import torch
import flashdecode
from flashdecode import cases
from oracle.decode_ref import decode_reference
from test_zz_no_alloc import ATOL, RTOL, LSE_ATOL, _noalloc
# 256 sequences x 8 KV heads: a 4.5 MiB split scratch, which an allocation
# would take out of the free device memory in 2 MiB pages
g = torch.Generator().manual_seed(3)
lens = torch.randint(100, 700, (256,), generator=g).tolist()
c = cases.custom_case("fresh", torch.bfloat16, lens, 32, 8, page=64, seed=3)
t = cases.materialize(c, "cuda", seed=3)
outs = [torch.full((c.B, 1, c.Hq, c.D), float("nan"), dtype=torch.bfloat16, device="cuda")
        for _ in range(3)]
lses = [torch.full((c.B, c.Hq), float("nan"), dtype=torch.float32, device="cuda") for _ in range(3)]
lib = flashdecode.load_library()
need = int(lib.fd_decode_workspace_size(c.B, c.Hq, c.Hkv, c.D))
torch.cuda.synchronize()
st = [_noalloc(lib, t, c, outs[0], lses[0])]  # first call: module loading, symbol lookup
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
st += [_noalloc(lib, t, c, outs[i], lses[i]) for i in (1, 2)]
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
lib_ws = int(lib.fd_library_workspace_bytes())
ref_o, ref_l = decode_reference(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                t["block_table"], softmax_scale=c.softmax_scale)
fin = torch.isfinite(ref_l)
ok = []
for o, l in zip(outs, lses):
    err = (o.float().cpu() - ref_o).abs()
    ok.append(bool((err <= ATOL + RTOL * ref_o.abs()).all())
              and torch.equal(fin, torch.isfinite(l.cpu()))
              and bool(torch.allclose(l.cpu()[fin], ref_l[fin], atol=LSE_ATOL)))
res = dict(status=st, need=need, free_drop=free0 - free1, lib_ws=lib_ws,
           dev_status=int(lib.fd_device_status()), oracle_ok=ok,
           same=bool(torch.equal(outs[1], outs[2]) and torch.equal(lses[1], lses[2])))
print("RESULT " + json.dumps(res))
"""


def test_noalloc_in_a_fresh_process_allocates_nothing():
    proc = subprocess.run([sys.executable, "-c", _FRESH, ROOT], capture_output=True, text=True,
                          timeout=900, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-3000:]
    line = [x for x in proc.stdout.splitlines() if x.startswith("RESULT ")][-1]
    res = json.loads(line[len("RESULT "):])
    assert res["status"] == [0, 0, 0], res
    assert 4 << 20 <= res["need"] <= NOALLOC_SCRATCH_BYTES, res
    assert res["free_drop"] < (2 << 20), res   # no workspace-sized allocation happened
    assert res["lib_ws"] == 0, res             # the library made no workspace of its own
    assert res["dev_status"] == 0, res
    assert res["oracle_ok"] == [True, True, True], res  # each call against the oracle
    assert res["same"], res                    # and the repeated calls agree exactly


def test_noalloc_refuses_shapes_beyond_its_scratch(lib):
    B, Hq, Hkv = 1024, 128, 16
    need = lib.fd_decode_workspace_size(B, Hq, Hkv, 128)
    assert need > NOALLOC_SCRATCH_BYTES
    buf = torch.zeros(4096, dtype=torch.int32, device="cuda")
    p = buf.data_ptr()
    # a 64-page table row (1024 tokens): long enough for the tensor-core kernel
    status = lib.fd_decode_paged_noalloc(p, p, p, p, None, p, p, 64, B, Hq, Hkv, 128, 16, 1, 0, 0,
                                         ctypes.c_float(0.1), 0, None)
    assert status == 3
    assert "scratch" in flashdecode.last_error()[1]


def test_noalloc_cuda_core_shapes_use_no_scratch(lib):
    """Head dim 64 runs on the CUDA-core kernel, which needs no split scratch:
    a batch whose tensor-core scratch would exceed the fixed area still runs."""
    g = torch.Generator().manual_seed(4)
    lens = torch.randint(0, 40, (1024,), generator=g).tolist()
    c = cases.custom_case("noalloc_simt", torch.bfloat16, lens, 128, 16, D=64, page=16, seed=4)
    assert lib.fd_decode_workspace_size(c.B, c.Hq, c.Hkv, c.D) > NOALLOC_SCRATCH_BYTES
    t = cases.materialize(c, "cuda", seed=4)
    ref_o, ref_l = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                            t["block_table"], softmax_scale=c.softmax_scale,
                                            return_softmax_lse=True)
    for call in range(2):
        out = torch.full_like(ref_o, float("nan"))
        lse = torch.full_like(ref_l, float("nan"))
        status = _noalloc(lib, t, c, out, lse)
        torch.cuda.synchronize()
        assert status == 0, flashdecode.last_error()
        _close(out, lse, ref_o, ref_l, f"call {call}")
