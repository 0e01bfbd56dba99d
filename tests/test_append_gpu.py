"""GPU parity of the KV-cache append (flash_attn_with_kvcache's k / v
arguments): the cache rows it writes are compared bit-for-bit with the
oracle's restatement, and the attention that follows within atol 2e-3 /
rtol 1e-2 (output) and 1e-3 (LSE) of the fp32 oracle and of flash_attn."""
import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import append_reference, decode_reference

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3


def make(dtype, seqlens, Hq, Hkv, sq, page, seed):
    """Case with pages for L + sq keys per sequence; cache_seqlens = L."""
    alloc = [max(L, 0) + sq for L in seqlens]
    c = cases.custom_case(f"app_{Hq}_{Hkv}_{sq}_{page}", dtype, alloc, Hq, Hkv, page=page, seed=seed)
    t = cases.materialize(c, "cuda", seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    t["q"] = torch.randn((c.B, sq, Hq, c.D), generator=g, device="cuda", dtype=dtype)
    t["k_new"] = torch.randn((c.B, sq, Hkv, c.D), generator=g, device="cuda", dtype=dtype)
    t["v_new"] = torch.randn((c.B, sq, Hkv, c.D), generator=g, device="cuda", dtype=dtype)
    t["cache_seqlens"] = torch.tensor(seqlens, dtype=torch.int32, device="cuda")
    return c, t


def check_attention(c, t, kc_ref, vc_ref, lens, out, lse, causal):
    ref_o, ref_l = decode_reference(t["q"], kc_ref, vc_ref, lens, t["block_table"],
                                    softmax_scale=c.softmax_scale, causal=causal)
    got = out.float().cpu()
    err = (got - ref_o).abs()
    bad = err > ATOL + RTOL * ref_o.abs()
    assert not bad.any(), f"{int(bad.sum())} elements off, max err {float(err.max()):.3e}"
    gl = lse.cpu()
    fin = torch.isfinite(ref_l)
    assert torch.equal(fin, torch.isfinite(gl))
    assert torch.allclose(gl[fin], ref_l[fin], atol=LSE_ATOL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("page", [256, 16])
def test_append_rows_bit_exact(dtype, page):
    seqlens = [0, 15, 16, 255, 256, 1000, -3]
    c, t = make(dtype, seqlens, 32, 8, 4, page, seed=21)
    kc0, vc0 = t["k_cache"].clone(), t["v_cache"].clone()
    kc_ref, vc_ref, _ = append_reference(kc0, vc0, t["k_new"], t["v_new"], t["cache_seqlens"],
                                         t["block_table"])
    flashdecode.append_kv(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                          t["block_table"])
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"].cpu(), kc_ref)
    assert torch.equal(t["v_cache"].cpu(), vc_ref)


@pytest.mark.parametrize("sq,causal", [(1, False), (2, True), (4, True), (3, False)])
@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (28, 4)])
@pytest.mark.parametrize("page", [256, 16])
def test_decode_with_append(sq, causal, Hq, Hkv, page):
    """Append + attention in one call; G * sq > 16 (28/4 with 3 tokens) runs
    the CUDA-core kernel, the rest the tensor-core one."""
    seqlens = [0, 1, 127, 128, 255, 700, 2047]
    c, t = make(torch.bfloat16, seqlens, Hq, Hkv, sq, page, seed=sq * 10 + page)
    kc_ref, vc_ref, lens = append_reference(t["k_cache"], t["v_cache"], t["k_new"], t["v_new"],
                                            t["cache_seqlens"], t["block_table"])
    out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                        t["block_table"], softmax_scale=c.softmax_scale,
                                        return_softmax_lse=True, causal=causal, k=t["k_new"],
                                        v=t["v_new"])
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"].cpu(), kc_ref) and torch.equal(t["v_cache"].cpu(), vc_ref)
    assert torch.equal(t["cache_seqlens"].cpu(), torch.tensor(seqlens, dtype=torch.int32))
    check_attention(c, t, kc_ref, vc_ref, lens, out, lse, causal)


def test_append_past_the_table_is_skipped():
    """Rows whose position has no page are not written and are not attended:
    the attended length is capped by the block table."""
    c, t = make(torch.bfloat16, [250, 10], 32, 8, 1, 256, seed=5)
    # sequence 0 may hold one page only (256 keys); appending 8 rows at 250
    # leaves rows 256..257 without a page.
    sn = 8
    g = torch.Generator(device="cuda").manual_seed(9)
    k_new = torch.randn((c.B, sn, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    v_new = torch.randn((c.B, sn, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    bt = t["block_table"][:, :1].contiguous()
    kc_ref, vc_ref, lens = append_reference(t["k_cache"], t["v_cache"], k_new, v_new,
                                            t["cache_seqlens"], bt)
    out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"], bt,
                                        softmax_scale=c.softmax_scale, return_softmax_lse=True,
                                        k=k_new, v=v_new)
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"].cpu(), kc_ref) and torch.equal(t["v_cache"].cpu(), vc_ref)
    lens = lens.clamp(max=256)
    t2 = dict(t, block_table=bt)
    check_attention(c, t2, kc_ref, vc_ref, lens, out, lse, False)


def test_append_matches_flash_attn():
    """Against the reference's own oracle, flash_attn_with_kvcache(k=, v=),
    run on the same device on a copy of the cache.  flash_attn rounds P to
    bf16 (unit roundoff 2^-8) before P.V, which puts its output up to
    2^-8 * sum_t p_t |v_t| off the fp32 value: on short rows whose output
    cancels that exceeds the 2e-3 atol, so flash_attn is held to that bound
    (computed by the oracle on |V|) and this operator, which keeps P at fp32
    precision, to the plain north-star tolerance."""
    fa = pytest.importorskip("flash_attn.flash_attn_interface")
    for sq, causal in [(1, False), (2, True), (4, True), (2, False)]:
        c, t = make(torch.bfloat16, [0, 255, 256, 3000], 32, 8, sq, 256, seed=40 + sq)
        kc_ref, vc_ref, lens = append_reference(t["k_cache"], t["v_cache"], t["k_new"], t["v_new"],
                                                t["cache_seqlens"], t["block_table"])
        ref_o, ref_l = decode_reference(t["q"], kc_ref, vc_ref, lens, t["block_table"],
                                        softmax_scale=c.softmax_scale, causal=causal)
        kc2, vc2 = t["k_cache"].clone(), t["v_cache"].clone()
        fa_o, fa_l = fa.flash_attn_with_kvcache(
            t["q"], kc2, vc2, t["k_new"], t["v_new"], cache_seqlens=t["cache_seqlens"],
            block_table=t["block_table"].clamp(min=0), softmax_scale=c.softmax_scale,
            causal=causal, return_softmax_lse=True)
        out, lse = flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                            t["block_table"], softmax_scale=c.softmax_scale,
                                            return_softmax_lse=True, causal=causal,
                                            k=t["k_new"], v=t["v_new"])
        torch.cuda.synchronize()
        assert torch.equal(t["k_cache"], kc2) and torch.equal(t["v_cache"], vc2)
        abs_o, _ = decode_reference(t["q"], kc_ref, vc_ref.abs(), lens, t["block_table"],
                                    softmax_scale=c.softmax_scale, causal=causal)
        allow = ATOL + RTOL * ref_o.abs()
        allow_fa = allow + abs_o * 2.0 ** -8
        fa_o, out = fa_o.float().cpu(), out.float().cpu()
        assert bool(((fa_o - ref_o).abs() <= allow_fa).all()), "flash_attn vs fp32 oracle"
        assert bool(((out - ref_o).abs() <= allow).all()), "operator vs fp32 oracle"
        assert bool(((out - fa_o).abs() <= allow + allow_fa).all()), "operator vs flash_attn"
        fa_l = fa_l.float().cpu().reshape(lse.shape)
        assert torch.allclose(fa_l, ref_l, atol=LSE_ATOL)
        assert torch.allclose(lse.cpu(), fa_l, atol=LSE_ATOL)


def test_append_rejects_bad_shapes_before_writing():
    c, t = make(torch.bfloat16, [10, 20], 32, 8, 1, 256, seed=3)
    kc0 = t["k_cache"].clone()
    with pytest.raises(ValueError):
        flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                 t["block_table"], k=t["k_new"])
    with pytest.raises(flashdecode.FlashDecodeError):
        # out_dtype fp16 with bf16 inputs is rejected by the attention half
        flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                 t["block_table"], k=t["k_new"], v=t["v_new"],
                                 out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"], kc0)
