"""Host-side model of the device scheduler in csrc/fd_decode_sm100.cu.

The kernel decides its split on the device from cache_seqlens; this module
computes the same partition on the host so tests can check its invariants
(every tile covered once, partial slots unique, balanced ranges) and the
bench can report split statistics.  It replaces the reference's
choose_splits table (submission-oj/best_flashattn_kvcache_decode.cu:1039-1076)
and its per-split page ranges (:664-671).
"""
from __future__ import annotations

from dataclasses import dataclass

TILE_TOKENS = 128
MAX_BATCH_PER_LAUNCH = 1024


@dataclass(frozen=True)
class Segment:
    cta: int
    b: int
    kvh: int
    pair: int
    tile0: int
    ntiles: int
    nseg: int
    cfirst: int

    @property
    def slot(self) -> int:
        return self.cta + self.pair


def tiles_of(length: int, max_len: int | None = None) -> int:
    L = max(0, int(length))
    if max_len is not None:
        L = min(L, max_len)
    return (L + TILE_TOKENS - 1) // TILE_TOKENS if L > 0 else 1


def cta_of(w: int, total: int, grid: int) -> int:
    """Largest c with floor(total * c / grid) <= w."""
    return ((w + 1) * grid + total - 1) // total - 1


def grid_size(batch: int, hkv: int, num_sms: int, tiles_bound: int) -> int:
    return min(num_sms, batch * hkv * tiles_bound)


def segments(seqlens, hkv: int, grid: int, max_len: int | None = None) -> list[Segment]:
    """All segments of all CTAs, in CTA order then work order."""
    n = [tiles_of(L, max_len) for L in seqlens]
    prefix = [0]
    for x in n:
        prefix.append(prefix[-1] + x)
    total = hkv * prefix[-1]
    grid = min(grid, total)  # the kernel never splits over more CTAs than tiles
    out: list[Segment] = []
    for c in range(grid):
        w, w_end = total * c // grid, total * (c + 1) // grid
        while w < w_end:
            # largest b with hkv * prefix[b] <= w
            lo, hi = 0, len(n) - 1
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if hkv * prefix[mid] <= w:
                    lo = mid
                else:
                    hi = mid - 1
            b = lo
            r = w - hkv * prefix[b]
            kvh, tile0 = divmod(r, n[b])
            pair_start = w - tile0
            pair_end = pair_start + n[b]
            seg_end = min(w_end, pair_end)
            c0, c1 = cta_of(pair_start, total, grid), cta_of(pair_end - 1, total, grid)
            out.append(Segment(c, b, kvh, b * hkv + kvh, tile0, seg_end - w, c1 - c0 + 1, c0))
            w = seg_end
    return out


def split_stats(seqlens, hkv: int, grid: int) -> dict:
    segs = segments(seqlens, hkv, grid)
    split_pairs = {s.pair for s in segs if s.nseg > 1}
    per_cta = [0] * grid
    for s in segs:
        per_cta[s.cta] += s.ntiles
    return dict(segments=len(segs), pairs=len(seqlens) * hkv, split_pairs=len(split_pairs),
                tiles_total=sum(per_cta), tiles_per_cta_max=max(per_cta),
                tiles_per_cta_min=min(per_cta))
