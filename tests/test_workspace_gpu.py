"""Split scratch (workspace) and device status on the GPU.

* The arrival counters of split (sequence, KV head) pairs carry a 52-bit
  launch epoch and are cleared by the CTA that merges the pair: stale
  counters left in a workspace never pass for the current launch's, also
  across the epoch's wrap-around.
* Calls that pass workspace = NULL on different streams get different
  library-owned workspaces, so concurrent streams do not race.
* A block_table entry inside a sequence's range that lies outside the pool is
  reported (FD_ERR_BAD_PAGE through fd_device_status), its rows read as zeros,
  and nothing faults.

Every output is checked against the CPU oracle with the north-star
tolerances (output atol 2e-3 / rtol 1e-2 of the fp32 oracle, LSE 1e-3).
The workspace offsets used below (launch epoch: two 64-bit words at byte 0;
one 64-bit arrival counter per pair from byte 128) are the layout of
fd::workspace_layout in fd_decode_sm100.cu."""
import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import append_reference, decode_reference

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3
FD_ERR_BAD_PAGE = 6
EPOCH_BITS = 52
TICKETS_OFF = 128

# long and short sequences: the long (sequence, KV head) pairs are split over
# many CTAs, so every launch merges partials through the arrival counters
SPLIT_LENS = [5000, 17, 9000, 1, 0, 300, 2049]


def run(t, c, **kw):
    return flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                    t["block_table"], softmax_scale=c.softmax_scale,
                                    return_softmax_lse=True, **kw)


def check(out, lse, ref_o, ref_l, what=""):
    err = (out.float().cpu() - ref_o).abs()
    bad = err > ATOL + RTOL * ref_o.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off, max err {float(err.max()):.3e}"
    fin = torch.isfinite(ref_l)
    assert torch.equal(fin, torch.isfinite(lse.cpu())), f"{what}: LSE finiteness differs"
    assert torch.allclose(lse.cpu()[fin], ref_l[fin], atol=LSE_ATOL), f"{what}: LSE off"


def oracle(t, c, block_table=None, k=None, v=None):
    return decode_reference(t["q"], t["k_cache"] if k is None else k,
                            t["v_cache"] if v is None else v, t["cache_seqlens"],
                            t["block_table"] if block_table is None else block_table,
                            softmax_scale=c.softmax_scale)


def _split_case():
    c = cases.custom_case("wrap", torch.bfloat16, SPLIT_LENS, 32, 8, seed=12)
    return c, cases.materialize(c, "cuda", seed=12)


def test_completed_launch_leaves_every_counter_cleared():
    c, t = _split_case()
    n = flashdecode.workspace_size(c.B, c.Hq, c.Hkv)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    w64 = ws[:16].view(torch.int64)
    tick = ws[TICKETS_OFF:TICKETS_OFF + 8 * c.B * c.Hkv].view(torch.int64)
    ref_o, ref_l = oracle(t, c)
    for i in range(3):
        out, lse = run(t, c, workspace=ws)
        torch.cuda.synchronize()
        check(out, lse, ref_o, ref_l, f"launch {i}")
        assert int(w64[0]) == i + 1 and int(w64[1]) == 0, w64.tolist()
        assert bool((tick == 0).all()), tick.tolist()


def test_stale_counters_across_the_old_20_bit_wrap():
    """Epochs around 2^20: a 20-bit epoch would come back to 1 after 0xFFFFF
    and take counters stamped with epoch 1 (one arrival counted) as current.
    Plant such counters for every pair and decode on across that point."""
    c, t = _split_case()
    n = flashdecode.workspace_size(c.B, c.Hq, c.Hkv)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    w64 = ws[:16].view(torch.int64)
    tick = ws[TICKETS_OFF:TICKETS_OFF + 8 * c.B * c.Hkv].view(torch.int64)
    ref_o, ref_l = oracle(t, c)
    w64[0] = 0xFFFFE
    tick.fill_((1 << 12) | 1)
    for e in (0xFFFFE, 0xFFFFF, 0x100000, 0x100001):
        out, lse = run(t, c, workspace=ws)
        torch.cuda.synchronize()
        check(out, lse, ref_o, ref_l, f"epoch {e:#x}")
        assert int(w64[0]) == e + 1


def test_epoch_wraps_at_2_pow_52():
    """The epoch runs 1 .. 2^52 - 1 and then starts again at 1; every launch
    across that point merges correctly and leaves the counters cleared."""
    c, t = _split_case()
    n = flashdecode.workspace_size(c.B, c.Hq, c.Hkv)
    ws = torch.zeros(n, dtype=torch.uint8, device="cuda")
    w64 = ws[:16].view(torch.int64)
    tick = ws[TICKETS_OFF:TICKETS_OFF + 8 * c.B * c.Hkv].view(torch.int64)
    ref_o, ref_l = oracle(t, c)
    top = (1 << EPOCH_BITS) - 1
    w64[0] = top - 1
    for e, nxt in ((top - 1, top), (top, 1), (1, 2), (2, 3)):
        out, lse = run(t, c, workspace=ws)
        torch.cuda.synchronize()
        check(out, lse, ref_o, ref_l, f"epoch {e:#x}")
        assert int(w64[0]) == nxt and int(w64[1]) == 0
        assert bool((tick == 0).all())


def test_two_streams_get_their_own_workspaces():
    """Two streams decode different batches at the same time, both with
    workspace = NULL: each stream has its own library workspace, and every
    result matches the oracle."""
    lib = flashdecode.load_library()
    ca = cases.custom_case("streamA", torch.bfloat16, SPLIT_LENS, 32, 8, seed=31)
    cb = cases.custom_case("streamB", torch.float16, [9000, 3, 4000, 700, 12000], 28, 4, page=16,
                           seed=32)
    ta, tb = cases.materialize(ca, "cuda", seed=31), cases.materialize(cb, "cuda", seed=32)
    ra, rb = oracle(ta, ca), oracle(tb, cb)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    before = int(lib.fd_library_workspace_bytes())
    torch.cuda.synchronize()
    res_a, res_b = [], []
    for _ in range(25):
        with torch.cuda.stream(sa):
            res_a.append(run(ta, ca))
        with torch.cuda.stream(sb):
            res_b.append(run(tb, cb))
    torch.cuda.synchronize()
    grown = int(lib.fd_library_workspace_bytes()) - before
    need = (flashdecode.workspace_size(ca.B, ca.Hq, ca.Hkv)
            + flashdecode.workspace_size(cb.B, cb.Hq, cb.Hkv))
    assert grown >= need, (grown, need)
    for i, (o, l) in enumerate(res_a):
        check(o, l, *ra, f"stream A call {i}")
    for i, (o, l) in enumerate(res_b):
        check(o, l, *rb, f"stream B call {i}")
    assert flashdecode.device_status() == 0


def test_capture_on_a_stream_with_no_workspace_yet():
    """The first call on a stream may be one being captured into a CUDA graph:
    the library allocates that stream's workspace outside the graph."""
    c, t = _split_case()
    ref_o, ref_l = oracle(t, c)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out, lse = run(t, c)
    for i in range(3):
        g.replay()
        torch.cuda.synchronize()
        check(out, lse, ref_o, ref_l, f"replay {i}")


def _with_zero_page(t, c, bt_bad):
    """Oracle inputs for a table with out-of-pool ids: one extra page of
    zeros at index num_blocks, which the bad entries point to."""
    z = torch.zeros((1,) + tuple(t["k_cache"].shape[1:]), dtype=t["k_cache"].dtype, device="cuda")
    k = torch.cat([t["k_cache"], z])
    v = torch.cat([t["v_cache"], z])
    bt = bt_bad.clone()
    bad = (bt < 0) | (bt >= c.num_blocks)
    bt[bad] = c.num_blocks
    return k, v, bt


@pytest.mark.parametrize("D,page", [(128, 256), (128, 16), (64, 16)])
def test_bad_page_id_is_reported_and_read_as_zeros(D, page):
    """Tensor-core kernel (D = 128) and CUDA-core kernel (D = 64)."""
    lib = flashdecode.load_library()
    assert lib.fd_device_status() == 0
    c = cases.custom_case(f"badpage{D}_{page}", torch.bfloat16, [700, 300, 1500, 64], 32, 8, D=D,
                          page=page, seed=21)
    t = cases.materialize(c, "cuda", seed=21)
    bt = t["block_table"].clone()
    bt[0, 1] = -5
    bt[2, 3] = c.num_blocks + 3
    t_bad = dict(t, block_table=bt)
    out, lse = run(t_bad, c)
    torch.cuda.synchronize()
    assert lib.fd_device_status() == FD_ERR_BAD_PAGE
    assert "num_blocks" in flashdecode.last_error()[1]
    assert lib.fd_device_status() == 0  # read and cleared
    k, v, bt_z = _with_zero_page(t, c, bt.cpu())
    ref_o, ref_l = oracle(t, c, block_table=bt_z, k=k, v=v)
    check(out, lse, ref_o, ref_l, "bad table")
    # the context is intact and a good table reports nothing
    out, lse = run(t, c)
    torch.cuda.synchronize()
    check(out, lse, *oracle(t, c), "good table")
    assert lib.fd_device_status() == 0


def test_append_into_an_unallocated_page_is_reported():
    lib = flashdecode.load_library()
    assert lib.fd_device_status() == 0
    c = cases.custom_case("badappend", torch.bfloat16, [250, 10], 32, 8, page=256, seed=5,
                          pad_blocks=1)
    t = cases.materialize(c, "cuda", seed=5)
    g = torch.Generator(device="cuda").manual_seed(9)
    k_new = torch.randn((c.B, 8, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    v_new = torch.randn_like(k_new)
    # sequence 0 (250 keys) spills into its second table slot, which holds -1
    assert int(t["block_table"][0, 1]) == -1
    kc_ref, vc_ref, _ = append_reference(t["k_cache"], t["v_cache"], k_new, v_new,
                                         t["cache_seqlens"], t["block_table"])
    flashdecode.append_kv(k_new, v_new, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                          t["block_table"])
    torch.cuda.synchronize()
    assert lib.fd_device_status() == FD_ERR_BAD_PAGE
    assert torch.equal(t["k_cache"].cpu(), kc_ref) and torch.equal(t["v_cache"].cpu(), vc_ref)
    assert lib.fd_device_status() == 0
