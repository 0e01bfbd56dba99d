"""CPU oracle for paged-KV GQA decode attention.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py may import this module, and
only as the checker or as the timed CPU baseline.  The operator itself never
calls it: there is no CPU fallback.

What it restates: the reference's decode semantics for one query token,
    s_t   = scale * q . k_t              for t < cache_seqlens[b]
    O     = sum_t softmax(s)_t v_t,      LSE = ln sum_t exp(s_t)
with k_t / v_t found through the page table (page = block_table[b, t // bs],
row t % bs, KV head h // (Hq / Hkv)), following
  - the math of the reference kernels: QK dot and scale
    (submission-oj/best_flashattn_kvcache_decode.cu:286-287, :398-400),
    softmax/merge (:541-578, :838-953), split combine (:956-1037);
  - the page-table gather (best :266-271, :741-742) and GQA head mapping
    (best :250, :653);
  - edge rules: length <= 0 gives O = 0 (best :256-260, :422-430) and
    LSE = -inf, length 1 returns the single V row (best :273-284, :443-460);
  - the numpy restatement in submission-oj/diagnostics/diag_integrated.py:48-57.
The reference's own oracle is flash_attn_with_kvcache
(scripts/evaluate_flashattn_submission.py:232-247; flash_attn 2.6.3 on its
box, 2.8.3 here), a CUDA-only library; tests/golden/ holds its outputs on
seeded inputs, against which this oracle is pinned.
"""
from __future__ import annotations

import math

import torch


def decode_reference(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                     softmax_scale: float | None = None, rows=None,
                     compute_dtype: torch.dtype = torch.float32, causal: bool = False):
    """Vectorised oracle (torch on CPU).

    q [B, sq, Hq, D]; k_cache/v_cache [num_blocks, page, Hkv, D];
    cache_seqlens [B]; block_table [B, max_blocks].
    Returns (out [B, sq, Hq, D], lse [B, Hq] for sq = 1 else [B, Hq, sq]) in
    compute_dtype; rows not in `rows` (when given) are left zero / -inf.
    causal: query token i sits at position L - sq + i and sees keys up to it
    (the bottom-right convention of flash_attn_with_kvcache, which the
    reference's run_kernel carries as its `causal` argument, best :1200).
    """
    q = q.cpu()
    B, sq, Hq, D = q.shape
    _, page, Hkv, _ = k_cache.shape
    G = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    seqlens = cache_seqlens.cpu().tolist()
    bt = block_table.cpu()
    out = torch.zeros((B, sq, Hq, D), dtype=compute_dtype)
    lse = torch.full((B, Hq, sq), float("-inf"), dtype=compute_dtype)
    for b in (range(B) if rows is None else rows):
        L = max(0, int(seqlens[b]))
        if L == 0:
            continue
        n_pages = (L + page - 1) // page
        pages = bt[b, :n_pages].long()
        K = k_cache[pages.to(k_cache.device)].cpu().reshape(n_pages * page, Hkv, D)[:L].to(compute_dtype)
        V = v_cache[pages.to(v_cache.device)].cpu().reshape(n_pages * page, Hkv, D)[:L].to(compute_dtype)
        for i in range(sq):
            vis = L - (sq - 1 - i) if causal else L
            if vis <= 0:
                continue
            qb = q[b, i].to(compute_dtype).reshape(Hkv, G, D)
            s = torch.einsum("hgd,lhd->hgl", qb, K[:vis]) * scale
            m = s.amax(dim=-1, keepdim=True)
            e = torch.exp(s - m)
            den = e.sum(dim=-1, keepdim=True)
            o = torch.einsum("hgl,lhd->hgd", e / den, V[:vis])
            out[b, i] = o.reshape(Hq, D)
            lse[b, :, i] = (m + torch.log(den)).reshape(Hq)
    return out, (lse[:, :, 0] if sq == 1 else lse)


def decode_reference_loops(q, k_cache, v_cache, cache_seqlens, block_table,
                           softmax_scale: float | None = None):
    """Independent scalar restatement in float64 pure-Python loops (small cases only)."""
    qf = q.double().tolist()
    kf = k_cache.double().tolist()
    vf = v_cache.double().tolist()
    B, Hq, D = len(qf), len(qf[0][0]), len(qf[0][0][0])
    page, Hkv = len(kf[0]), len(kf[0][0])
    G = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    out = [[[0.0] * D for _ in range(Hq)] for _ in range(B)]
    lse = [[float("-inf")] * Hq for _ in range(B)]
    for b in range(B):
        L = max(0, int(cache_seqlens[b]))
        for h in range(Hq):
            kvh = h // G
            scores, vals = [], []
            for t in range(L):
                pg = int(block_table[b][t // page])
                krow = kf[pg][t % page][kvh]
                scores.append(scale * sum(qf[b][0][h][d] * krow[d] for d in range(D)))
                vals.append(vf[pg][t % page][kvh])
            if L == 0:
                continue
            m = max(scores)
            w = [math.exp(s - m) for s in scores]
            tot = sum(w)
            lse[b][h] = m + math.log(tot)
            out[b][h] = [sum(w[t] * vals[t][d] for t in range(L)) / tot for d in range(D)]
    return (torch.tensor(out, dtype=torch.float64).reshape(B, 1, Hq, D),
            torch.tensor(lse, dtype=torch.float64))


def append_reference(k_cache: torch.Tensor, v_cache: torch.Tensor, k_new: torch.Tensor,
                     v_new: torch.Tensor, cache_seqlens: torch.Tensor, block_table: torch.Tensor):
    """Cache update of flash_attn_with_kvcache(k=k_new, v=v_new) on CPU copies.

    Row t of sequence b goes to position max(L_b, 0) + t: page
    block_table[b, pos // page], row pos % page (the same gather the reference
    reads through, best :266-271).  A position past the table or a page id
    outside the pool is skipped.  Returns (k_cache', v_cache', attended
    lengths max(L_b, 0) + seqlen_new).  The reference evaluator passes
    k = v = None (evaluate_flashattn_submission.py:233-239), so this restates
    the documented flash_attn behaviour, pinned by tests/golden/ outputs.
    """
    kc = k_cache.cpu().clone()
    vc = v_cache.cpu().clone()
    kn, vn = k_new.cpu(), v_new.cpu()
    B, sn = kn.shape[0], kn.shape[1]
    nb, page = kc.shape[0], kc.shape[1]
    bt = block_table.cpu()
    stride = bt.shape[1]
    lens = cache_seqlens.cpu().clamp(min=0)
    for b in range(B):
        for t in range(sn):
            pos = int(lens[b]) + t
            if pos // page >= stride:
                continue
            pg = int(bt[b, pos // page])
            if pg < 0 or pg >= nb:
                continue
            kc[pg, pos % page] = kn[b, t]
            vc[pg, pos % page] = vn[b, t]
    return kc, vc, (lens + sn).to(torch.int32)


def quantize_e4m3(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """e4m3 (float8_e4m3fn) of x / scale[h] for x [..., Hkv, D], scale [Hkv]:
    fp32 division, round to nearest even, saturated at +-448 (the FP8 cache
    format of the operator's fd_append_kv_paged_fp8; the reference has no FP8
    path)."""
    q = x.cpu().float() / scale.cpu().float()[:, None]
    return q.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def dequantize_e4m3(c: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 values of an e4m3 cache [..., Hkv, D] with per-KV-head scales."""
    return c.cpu().float() * scale.cpu().float()[:, None]


def append_reference_e4m3(k_cache, v_cache, k_new, v_new, k_scale, v_scale, cache_seqlens,
                          block_table):
    """append_reference for an e4m3 cache: new rows are quantised first."""
    kq = quantize_e4m3(k_new, k_scale).view(torch.uint8)
    vq = quantize_e4m3(v_new, v_scale).view(torch.uint8)
    kc, vc, lens = append_reference(k_cache.cpu().view(torch.uint8), v_cache.cpu().view(torch.uint8),
                                    kq, vq, cache_seqlens, block_table)
    return kc.view(torch.float8_e4m3fn), vc.view(torch.float8_e4m3fn), lens


def merge_partials(part_o: torch.Tensor, part_lse: torch.Tensor):
    """Merge normalised partials over disjoint KV ranges (natural-log LSE).

    Restates the reference's combine (best :956-1037): weights
    exp(lse_j - max lse), parts with lse = -inf weigh zero.
    """
    po = part_o.double()
    pl = part_lse.double()
    mx = pl.amax(dim=0)
    mx_safe = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
    w = torch.where(torch.isinf(pl), torch.zeros_like(pl), torch.exp(pl - mx_safe))
    den = w.sum(dim=0)
    out = (w.unsqueeze(-1) * torch.nan_to_num(po)).sum(dim=0) / den.clamp(min=1e-300).unsqueeze(-1)
    out = torch.where(den.unsqueeze(-1) > 0, out, torch.zeros_like(out))
    lse = torch.where(den > 0, mx_safe + torch.log(den.clamp(min=1e-300)), torch.full_like(den, float("-inf")))
    return out, lse
