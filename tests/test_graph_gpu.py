"""Decode calls captured in a CUDA graph and replayed.

A serving loop captures its decode step once and replays it; the operator
must then give the same results as eager calls on whatever the inputs hold
at replay time.  The case that matters: sequences split across CTAs, whose
partial results are merged by the last CTA to arrive, counted per launch
under an epoch the kernel keeps in the workspace (a host-side epoch would be
frozen into the captured launch).  Every replay is checked against the CPU
oracle with the north-star tolerances (output atol 2e-3 / rtol 1e-2 of the
fp32 oracle, LSE 1e-3)."""
import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import decode_reference, dequantize_e4m3

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3

# long and short sequences: the long pairs are split over many CTAs, so
# every launch merges partials
LENS = [5000, 17, 3000, 0, 128, 9000, 1]


def check(out, lse, ref_o, ref_l):
    err = (out.float().cpu() - ref_o).abs()
    bad = err > ATOL + RTOL * ref_o.abs()
    assert not bad.any(), f"{int(bad.sum())} elements off, max err {float(err.max()):.3e}"
    fin = torch.isfinite(ref_l)
    assert torch.equal(fin, torch.isfinite(lse.cpu())), "LSE finiteness differs"
    assert torch.allclose(lse.cpu()[fin], ref_l[fin], atol=LSE_ATOL), "LSE off"


def capture(fn):
    fn()  # eager warm-up: the library workspace and tensor maps exist before capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        res = fn()
    return g, res


def test_graph_replay_matches_oracle_every_time():
    c = cases.custom_case("graph", torch.bfloat16, LENS, 32, 8, page=64, seed=3)
    t = cases.materialize(c, "cuda", seed=3)
    q = t["q"]

    def step():
        return flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True)

    g, (out, lse) = capture(step)
    gen = torch.Generator(device="cuda").manual_seed(7)
    for _ in range(4):
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda", dtype=q.dtype))
        g.replay()
        torch.cuda.synchronize()
        ref_o, ref_l = decode_reference(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale)
        check(out, lse, ref_o, ref_l)


def test_graph_with_several_decodes_per_replay():
    """Three decodes in one graph (as the layers of one step): each launch
    must get its own epoch inside one replay."""
    c = cases.custom_case("graph3", torch.float16, LENS, 28, 4, page=16, seed=5)
    t = cases.materialize(c, "cuda", seed=5)
    gen = torch.Generator(device="cuda").manual_seed(9)
    qs = [torch.randn(t["q"].shape, generator=gen, device="cuda", dtype=t["q"].dtype) for _ in range(3)]

    def step():
        return [flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                         t["block_table"], softmax_scale=c.softmax_scale,
                                         return_softmax_lse=True) for q in qs]

    g, res = capture(step)
    for _ in range(2):
        for q in qs:
            q.copy_(torch.randn(q.shape, generator=gen, device="cuda", dtype=q.dtype))
        g.replay()
        torch.cuda.synchronize()
        for q, (out, lse) in zip(qs, res):
            ref_o, ref_l = decode_reference(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                            t["block_table"], softmax_scale=c.softmax_scale)
            check(out, lse, ref_o, ref_l)


def test_graph_replay_e4m3_cache():
    c = cases.custom_case("graph8", torch.bfloat16, LENS, 32, 8, page=256, seed=11)
    t = cases.materialize_e4m3(c, "cuda", seed=11)
    q = t["q"]

    def step():
        return flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, k_scale=t["k_scale"],
                                        v_scale=t["v_scale"])

    g, (out, lse) = capture(step)
    kd = dequantize_e4m3(t["k_cache"], t["k_scale"])
    vd = dequantize_e4m3(t["v_cache"], t["v_scale"])
    gen = torch.Generator(device="cuda").manual_seed(13)
    for _ in range(3):
        q.copy_(torch.randn(q.shape, generator=gen, device="cuda", dtype=q.dtype))
        g.replay()
        torch.cuda.synchronize()
        ref_o, ref_l = decode_reference(q, kd, vd, t["cache_seqlens"], t["block_table"],
                                        softmax_scale=c.softmax_scale)
        check(out, lse, ref_o, ref_l)
