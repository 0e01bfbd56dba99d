"""GPU parity of the e4m3 (FP8) KV-cache path against the fp32 oracle run on
the dequantised cache (k8 * k_scale[h], v8 * v_scale[h]).

The reference has no FP8 path; the tolerance is the north-star one of the
16-bit path (output atol 2e-3 / rtol 1e-2, LSE 1e-3): the query and P are
carried through the e4m3 tensor-core products as three e4m3 parts each, so
the only inputs rounded to 8 bits are the cached keys and values, which the
oracle reads with the same rounding.  Cache rows written by the e4m3 append
are compared byte for byte with the oracle's quantisation."""
import pytest
import torch

import flashdecode
from flashdecode import cases
from oracle.decode_ref import (append_reference_e4m3, decode_reference, dequantize_e4m3)

pytestmark = pytest.mark.gpu

ATOL, RTOL, LSE_ATOL = 2e-3, 1e-2, 1e-3


def oracle(t, c, causal=False, rows=None, kc=None, vc=None, lens=None):
    kd = dequantize_e4m3(t["k_cache"] if kc is None else kc, t["k_scale"])
    vd = dequantize_e4m3(t["v_cache"] if vc is None else vc, t["v_scale"])
    return decode_reference(t["q"], kd, vd, t["cache_seqlens"] if lens is None else lens,
                            t["block_table"], softmax_scale=c.softmax_scale, rows=rows,
                            causal=causal)


def check(out, lse, ref_o, ref_l, rows=None):
    sel = slice(None) if rows is None else list(rows)
    got, exp = out.float().cpu()[sel], ref_o[sel]
    err = (got - exp).abs()
    bad = err > ATOL + RTOL * exp.abs()
    assert not bad.any(), f"{int(bad.sum())} elements off, max err {float(err.max()):.3e}"
    gl, el = lse.cpu()[sel], ref_l[sel]
    fin = torch.isfinite(el)
    assert torch.equal(fin, torch.isfinite(gl)), "LSE finiteness differs"
    assert torch.allclose(gl[fin], el[fin], atol=LSE_ATOL), "LSE off"


def run(t, c, **kw):
    return flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                    t["block_table"], softmax_scale=c.softmax_scale,
                                    return_softmax_lse=True, k_scale=t["k_scale"],
                                    v_scale=t["v_scale"], **kw)


RAGGED = [1, 127, 128, 129, 300, 0, 1000, 2049]


@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (64, 8), (28, 4), (8, 8)])
@pytest.mark.parametrize("page", [256, 16, 64])
def test_fp8_parity(qdtype, Hq, Hkv, page):
    c = cases.custom_case(f"fp8_{Hq}_{Hkv}_{page}", qdtype, RAGGED, Hq, Hkv, page=page, seed=Hq + page)
    t = cases.materialize_e4m3(c, "cuda", seed=5)
    out, lse = run(t, c)
    torch.cuda.synchronize()
    ref_o, ref_l = oracle(t, c)
    check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("out_dtype", [torch.float32])
def test_fp8_fp32_output(out_dtype):
    c = cases.custom_case("fp8_f32", torch.bfloat16, [700, 33, 4096], 32, 8, page=256, seed=2)
    t = cases.materialize_e4m3(c, "cuda", seed=2)
    out, lse = run(t, c, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    ref_o, ref_l = oracle(t, c)
    check(out, lse, ref_o, ref_l)


@pytest.mark.parametrize("sq,causal", [(2, True), (4, True), (2, False)])
def test_fp8_multi_token(sq, causal):
    c = cases.custom_case(f"fp8_mq{sq}", torch.bfloat16, [1, 2, 130, 1000, 257, 0], 32, 8,
                          page=256, seed=sq)
    t = cases.materialize_e4m3(c, "cuda", seed=sq)
    g = torch.Generator(device="cuda").manual_seed(sq)
    t["q"] = torch.randn((c.B, sq, 32, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    out, lse = run(t, c, causal=causal)
    torch.cuda.synchronize()
    ref_o, ref_l = oracle(t, c, causal=causal)
    check(out, lse, ref_o, ref_l)


def test_fp8_config2_full_size_sampled_rows():
    """Config 2's shape (1 GiB of 16-bit KV, 512 MiB as e4m3), rows sampled."""
    c = cases.config_case(2)
    t = cases.materialize_e4m3(c, "cuda", seed=0)
    out, lse = run(t, c)
    torch.cuda.synchronize()
    rows = [0, 17, 38, 63]
    ref_o, ref_l = oracle(t, c, rows=rows)
    check(out, lse, ref_o, ref_l, rows=rows)


def _append_case(sq, page, seed):
    seqlens = [0, 15, 16, 255, 256, 1000]
    c = cases.custom_case(f"fp8app{sq}_{page}", torch.bfloat16, [L + sq for L in seqlens], 32, 8,
                          page=page, seed=seed)
    t = cases.materialize_e4m3(c, "cuda", seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    t["q"] = torch.randn((c.B, sq, 32, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    t["k_new"] = torch.randn((c.B, sq, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    t["v_new"] = torch.randn((c.B, sq, 8, 128), generator=g, device="cuda", dtype=torch.bfloat16)
    t["cache_seqlens"] = torch.tensor(seqlens, dtype=torch.int32, device="cuda")
    return c, t


@pytest.mark.parametrize("page", [256, 16])
def test_fp8_append_bytes_exact(page):
    c, t = _append_case(4, page, seed=31)
    kc_ref, vc_ref, _ = append_reference_e4m3(t["k_cache"], t["v_cache"], t["k_new"], t["v_new"],
                                              t["k_scale"], t["v_scale"], t["cache_seqlens"],
                                              t["block_table"])
    flashdecode.append_kv(t["k_new"], t["v_new"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                          t["block_table"], k_scale=t["k_scale"], v_scale=t["v_scale"])
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"].cpu().view(torch.uint8), kc_ref.view(torch.uint8))
    assert torch.equal(t["v_cache"].cpu().view(torch.uint8), vc_ref.view(torch.uint8))


@pytest.mark.parametrize("sq,causal", [(1, False), (2, True)])
def test_fp8_decode_with_append(sq, causal):
    c, t = _append_case(sq, 256, seed=40 + sq)
    kc_ref, vc_ref, lens = append_reference_e4m3(t["k_cache"], t["v_cache"], t["k_new"],
                                                 t["v_new"], t["k_scale"], t["v_scale"],
                                                 t["cache_seqlens"], t["block_table"])
    out, lse = run(t, c, causal=causal, k=t["k_new"], v=t["v_new"])
    torch.cuda.synchronize()
    assert torch.equal(t["k_cache"].cpu().view(torch.uint8), kc_ref.view(torch.uint8))
    ref_o, ref_l = oracle(t, c, causal=causal, kc=kc_ref, vc=vc_ref, lens=lens)
    check(out, lse, ref_o, ref_l)


def test_fp8_unsupported_shapes_are_refused():
    c = cases.custom_case("fp8_g32", torch.bfloat16, [100, 200], 64, 2, page=256, seed=1)
    t = cases.materialize_e4m3(c, "cuda", seed=1)  # 32 query rows per KV head > 16
    with pytest.raises(flashdecode.FlashDecodeError) as ei:
        run(t, c)
    assert ei.value.code == 2  # FD_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        flashdecode.flash_decode(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                 t["block_table"])  # scales missing


def test_fp8_batch_larger_than_one_launch():
    """More than 512 sequences: the query parts are split per launch chunk
    into the same workspace region, one chunk after the other."""
    lens = [37 + (i * 53) % 700 for i in range(1200)]
    c = cases.custom_case("fp8_big", torch.bfloat16, lens, 32, 8, page=16, seed=9)
    t = cases.materialize_e4m3(c, "cuda", seed=9)
    out, lse = run(t, c)
    torch.cuda.synchronize()
    rows = [0, 1, 511, 512, 513, 1023, 1024, 1199]
    ref_o, ref_l = oracle(t, c, rows=rows)
    check(out, lse, ref_o, ref_l, rows=rows)


@pytest.mark.parametrize("sq", [2, 3])
def test_fp8_multi_token_causal_page16(sq):
    c = cases.custom_case(f"fp8_mq16_{sq}", torch.float16, [5, 16, 17, 900, 0, 2001], 16, 8,
                          page=16, seed=20 + sq)
    t = cases.materialize_e4m3(c, "cuda", seed=20 + sq)
    g = torch.Generator(device="cuda").manual_seed(sq)
    t["q"] = torch.randn((c.B, sq, 16, 128), generator=g, device="cuda", dtype=torch.float16)
    out, lse = run(t, c, causal=True)
    torch.cuda.synchronize()
    ref_o, ref_l = oracle(t, c, causal=True)
    check(out, lse, ref_o, ref_l)
