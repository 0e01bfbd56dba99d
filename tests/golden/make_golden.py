"""Generate golden outputs of the reference's oracle, flash_attn_with_kvcache.

The reference evaluator scores every submission against
flash_attn.flash_attn_interface.flash_attn_with_kvcache
(scripts/evaluate_flashattn_submission.py:232-247; pinned there as
flash_attn 2.6.3, here 2.8.3).  That library is CUDA-only, so this script
runs on a GPU box:

    python tests/golden/make_golden.py --out golden_out

(then copy the files into tests/golden/) and writes ``fa_golden.json`` (case specs, library versions) and
``fa_golden.npz`` (out, lse per case).  With ``--append`` it writes
``fa_golden_append.*`` instead: cases that pass new keys/values (k, v) so
flash_attn first appends them to the paged cache, with 1-4 query tokens and
the bottom-right causal mask.  Inputs are rebuilt bit-identically on any
machine from the specs (CPU generator, fixed seeds), so only outputs are
stored.  Page size is 256 because flash_attn's paged path requires a
multiple of 256.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "flashatte-hand_b200"))

from flashdecode import cases  # noqa: E402

DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}

# Small seeded cases: GQA groups 1/4/7/8, ragged lengths incl. 0, 1, tile and
# page boundaries, both dtypes, a scaled query.
CASE_SPECS = [
    dict(name="bf16_g4_ragged", dtype="bf16", seqlens=[1, 255, 256, 257, 600, 129, 0, 1000], Hq=32, Hkv=8, seed=1),
    dict(name="fp16_g8_ragged", dtype="fp16", seqlens=[17, 511, 768, 3], Hq=64, Hkv=8, seed=2),
    dict(name="bf16_g7", dtype="bf16", seqlens=[300, 128, 1], Hq=28, Hkv=4, seed=3),
    dict(name="fp16_g1_mha", dtype="fp16", seqlens=[700, 64], Hq=8, Hkv=8, seed=4),
    dict(name="bf16_g4_qhalf", dtype="bf16", seqlens=[2048, 1500], Hq=32, Hkv=8, seed=5, q_std=0.5),
    dict(name="fp16_cfg1", dtype="fp16", config=1, seed=0),
]


# Append cases: lengths before the append (0, page boundaries), seqlen_new =
# seqlen_q new tokens, causal and not; G * sq <= 16 takes the tensor-core
# path, G = 7 with 3 tokens the CUDA-core one.
APPEND_SPECS = [
    dict(name="app_bf16_g4_s1", dtype="bf16", seqlens=[0, 255, 256, 1000], Hq=32, Hkv=8, seed=11, sq=1, causal=False),
    dict(name="app_fp16_g8_s2_causal", dtype="fp16", seqlens=[1, 254, 511, 64], Hq=64, Hkv=8, seed=12, sq=2, causal=True),
    dict(name="app_bf16_g4_s4_causal", dtype="bf16", seqlens=[0, 3, 300, 767], Hq=32, Hkv=8, seed=13, sq=4, causal=True),
    dict(name="app_bf16_g7_s3", dtype="bf16", seqlens=[128, 2000, 5], Hq=28, Hkv=4, seed=14, sq=3, causal=False),
]


def build_append_case(spec: dict):
    """(DecodeCase with pages for L + sq keys, CPU tensors incl. q [B, sq, Hq, D], k, v)."""
    sq = spec["sq"]
    alloc = [L + sq for L in spec["seqlens"]]
    c = cases.custom_case(spec["name"], DTYPES[spec["dtype"]], alloc, spec["Hq"], spec["Hkv"],
                          D=128, page=256, seed=spec["seed"])
    t = cases.materialize(c, "cpu", seed=spec["seed"])
    g = torch.Generator().manual_seed(spec["seed"] + 100)
    dt = DTYPES[spec["dtype"]]
    t["q"] = torch.randn((c.B, sq, c.Hq, c.D), generator=g, dtype=dt)
    t["k_new"] = torch.randn((c.B, sq, c.Hkv, c.D), generator=g, dtype=dt)
    t["v_new"] = torch.randn((c.B, sq, c.Hkv, c.D), generator=g, dtype=dt)
    t["cache_seqlens"] = torch.tensor(spec["seqlens"], dtype=torch.int32)
    return c, t


def build_case(spec: dict):
    """(DecodeCase, CPU tensors) for one spec; identical on every machine."""
    if "config" in spec:
        c = cases.config_case(spec["config"], seed=spec["seed"])
    else:
        c = cases.custom_case(spec["name"], DTYPES[spec["dtype"]], spec["seqlens"], spec["Hq"],
                              spec["Hkv"], D=128, page=256, seed=spec["seed"],
                              q_std=spec.get("q_std", 1.0))
    t = cases.materialize(c, "cpu", seed=spec["seed"])
    return c, t


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--append", action="store_true")
    args = ap.parse_args()
    from flash_attn import __version__ as fa_version
    from flash_attn.flash_attn_interface import flash_attn_with_kvcache

    os.makedirs(args.out, exist_ok=True)
    if args.append:
        arrays = {}
        for spec in APPEND_SPECS:
            c, t = build_append_case(spec)
            dev = {k: v.cuda() for k, v in t.items()}
            bt = dev["block_table"].clamp(min=0)
            out, lse = flash_attn_with_kvcache(
                dev["q"], dev["k_cache"], dev["v_cache"], dev["k_new"], dev["v_new"],
                cache_seqlens=dev["cache_seqlens"], cache_batch_idx=None, block_table=bt,
                softmax_scale=c.softmax_scale, causal=spec["causal"], window_size=(-1, -1),
                rotary_interleaved=False, alibi_slopes=None, num_splits=0, return_softmax_lse=True)
            torch.cuda.synchronize()
            arrays[spec["name"] + "_out"] = out.float().cpu().numpy()
            arrays[spec["name"] + "_lse"] = lse.float().reshape(c.B, c.Hq, spec["sq"]).cpu().numpy()
            print(spec["name"], tuple(out.shape), float(out.float().abs().max()))
        np.savez_compressed(os.path.join(args.out, "fa_golden_append.npz"), **arrays)
        meta = dict(kind="append", npz="fa_golden_append.npz",
                    generator="tests/golden/make_golden.py --append", flash_attn=fa_version,
                    torch=torch.__version__, device=torch.cuda.get_device_name(0),
                    cases=APPEND_SPECS)
        with open(os.path.join(args.out, "fa_golden_append.json"), "w") as f:
            json.dump(meta, f, indent=1)
        return
    arrays = {}
    for spec in CASE_SPECS:
        c, t = build_case(spec)
        dev = {k: v.cuda() for k, v in t.items()}
        bt = dev["block_table"].clamp(min=0)  # unused entries -> page 0 (never read)
        out, lse = flash_attn_with_kvcache(
            dev["q"], dev["k_cache"], dev["v_cache"], None, None,
            cache_seqlens=dev["cache_seqlens"], cache_batch_idx=None, block_table=bt,
            softmax_scale=c.softmax_scale, causal=False, window_size=(-1, -1),
            rotary_interleaved=False, alibi_slopes=None, num_splits=0, return_softmax_lse=True)
        torch.cuda.synchronize()
        arrays[spec["name"] + "_out"] = out.float().cpu().numpy()
        arrays[spec["name"] + "_lse"] = lse.float().reshape(c.B, c.Hq).cpu().numpy()
        print(spec["name"], tuple(out.shape), float(out.float().abs().max()))
    np.savez_compressed(os.path.join(args.out, "fa_golden.npz"), **arrays)
    meta = dict(npz="fa_golden.npz", generator="tests/golden/make_golden.py",
                flash_attn=fa_version, torch=torch.__version__,
                device=torch.cuda.get_device_name(0), cases=CASE_SPECS)
    with open(os.path.join(args.out, "fa_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)


if __name__ == "__main__":
    main()
