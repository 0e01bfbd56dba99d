"""Launch-shape routes of the decode, checked against the CPU oracle.

* Short launches — every sequence at most 64 tokens, bounded by the block
  table's width times the page or by max_seqlen_k — run on the CUDA-core
  kernel.
* Launches with few short (sequence, KV head) pairs take one or a few whole
  pairs per CTA on the tensor-core kernel (no pair split, no merge).

Both must give the same results as every other route: output within atol
2e-3 / rtol 1e-2 of the fp32 oracle, LSE (natural log) within 1e-3, for both
16-bit dtypes, multi-token causal queries, fp32 output, a cache append and
e4m3 caches."""
import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import append_reference, decode_reference, dequantize_e4m3

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3


def check(out, lse, ref_o, ref_l, what):
    err = (out.float().cpu() - ref_o).abs()
    bad = err > ATOL + RTOL * ref_o.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off, max err {float(err.max()):.3e}"
    fin = torch.isfinite(ref_l)
    assert torch.equal(fin, torch.isfinite(lse.cpu())), f"{what}: LSE finiteness differs"
    assert torch.allclose(lse.cpu()[fin], ref_l[fin], atol=LSE_ATOL), f"{what}: LSE off"


def query(c, sq, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn((c.B, sq, c.Hq, c.D), generator=g, device="cuda", dtype=c.dtype)


# (lengths, Hq, Hkv, page): table widths of at most 64 tokens
SHORT = [([1, 0, 17, 64], 32, 8, 16), ([3] * 40, 28, 4, 16), ([64, 63, 1, 2, 33], 64, 8, 32),
         ([5, 9], 8, 8, 64)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lens,Hq,Hkv,page", SHORT)
@pytest.mark.parametrize("sq,causal", [(1, False), (2, True), (3, False)])
def test_short_launch_parity(dtype, lens, Hq, Hkv, page, sq, causal):
    c = cases.custom_case("short", dtype, lens, Hq, Hkv, page=page, seed=len(lens) + sq)
    t = cases.materialize(c, "cuda", seed=sq)
    assert c.block_table.shape[1] * page <= 64
    q = query(c, sq, seed=Hq + sq)
    out, lse = flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, causal=causal)
    ref_o, ref_l = decode_reference(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                    t["block_table"], softmax_scale=c.softmax_scale, causal=causal)
    check(out, lse, ref_o, ref_l, "short launch")


def test_short_launch_by_max_seqlen_hint():
    """A wide table, but max_seqlen_k says every sequence is short."""
    c = cases.custom_case("hint_short", torch.bfloat16, [40, 1, 0, 64, 12], 32, 8, page=16, seed=3,
                          pad_blocks=30)
    t = cases.materialize(c, "cuda", seed=3)
    out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, max_seqlen_k=64,
                                        out_dtype=torch.float32)
    ref_o, ref_l = decode_reference(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                    t["block_table"], softmax_scale=c.softmax_scale)
    check(out, lse, ref_o, ref_l, "short by hint")


def test_short_launch_with_append():
    # every sequence owns a page for the appended rows (no out-of-pool ids)
    c = cases.custom_case("short_append", torch.bfloat16, [10, 5, 40], 32, 8, page=16, seed=5)
    t = cases.materialize(c, "cuda", seed=5)
    assert c.block_table.shape[1] * 16 <= 64
    g = torch.Generator(device="cuda").manual_seed(6)
    k_new = torch.randn((c.B, 4, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    v_new = torch.randn_like(k_new)
    kc, vc, lens = append_reference(t["k_cache"], t["v_cache"], k_new, v_new, t["cache_seqlens"],
                                    t["block_table"])
    out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, k=k_new, v=v_new)
    ref_o, ref_l = decode_reference(t["q"], kc, vc, lens, t["block_table"],
                                    softmax_scale=c.softmax_scale)
    check(out, lse, ref_o, ref_l, "short launch with append")


# (lengths, Hq, Hkv, page): few pairs, none longer than 16 tiles (2048 tokens)
ALIGNED = [([2048, 1, 300, 129], 32, 8, 256), ([141] * 16, 32, 4, 16), ([362] * 32, 32, 8, 16),
           ([700, 1500, 128], 28, 4, 64)]


@pytest.mark.parametrize("lens,Hq,Hkv,page", ALIGNED)
@pytest.mark.parametrize("sq,causal", [(1, False), (2, True)])
def test_whole_pair_split_parity(lens, Hq, Hkv, page, sq, causal):
    c = cases.custom_case("aligned", torch.bfloat16, lens, Hq, Hkv, page=page, seed=len(lens))
    t = cases.materialize(c, "cuda", seed=sq)
    q = query(c, sq, seed=7 + sq)
    out, lse = flashdecode.flash_decode(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, causal=causal)
    ref_o, ref_l = decode_reference(q, t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                    t["block_table"], softmax_scale=c.softmax_scale, causal=causal)
    check(out, lse, ref_o, ref_l, "whole-pair split")


@pytest.mark.parametrize("lens,Hq,Hkv,page", ALIGNED[:2])
def test_whole_pair_split_e4m3_cache(lens, Hq, Hkv, page):
    c = cases.custom_case("aligned8", torch.bfloat16, lens, Hq, Hkv, page=page, seed=9)
    t = cases.materialize_e4m3(c, "cuda", seed=9)
    out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, k_scale=t["k_scale"],
                                        v_scale=t["v_scale"])
    kd = dequantize_e4m3(t["k_cache"], t["k_scale"])
    vd = dequantize_e4m3(t["v_cache"], t["v_scale"])
    ref_o, ref_l = decode_reference(t["q"], kd, vd, t["cache_seqlens"], t["block_table"],
                                    softmax_scale=c.softmax_scale)
    check(out, lse, ref_o, ref_l, "whole-pair split, e4m3")
