"""Host-side model of the device scheduler in csrc/fd_decode_sm100.cu.

The kernel decides its split on the device from cache_seqlens; this module
computes the same partition on the host so tests can check its invariants
(every tile covered once, partial slots unique, no empty CTA inside a pair's
span) and the bench can report split statistics.  It replaces the
reference's choose_splits table
(submission-oj/best_flashattn_kvcache_decode.cu:1039-1076) and its per-split
page ranges (:664-671).

Cost model (integer units, a full 128-token tile's K/V bytes = 8): a tile
adds ``tile_fixed``; a sequence's partial last tile costs its 16-token boxes
instead of 8; every (sequence, KV head) pair adds ``seg``, raised where
needed so that no pair costs less than ``floor`` (the pair's ``lead``: its
first tile starts at the pair's start, tile j >= 1 at start + lead + j *
full).  Pairs are laid end to end (b-major, then KV head) and CTA c takes the
tiles whose start cost is in [C*c/G, C*(c+1)/G).
"""
from __future__ import annotations

from dataclasses import dataclass

TILE_TOKENS = 128
MAX_BATCH_PER_LAUNCH = 512
FULL_TILE = 8
DEFAULT_TILE_FIXED = 2
DEFAULT_SEG = 12
DEFAULT_FLOOR = 40
# e4m3 caches (half the bytes per tile for the same fixed work, plus the
# in-kernel query split per pair): the kernel's defaults for that path
E4M3_TILE_FIXED = 8
E4M3_SEG = 48
E4M3_FLOOR = 0
# pair-aligned split: one whole pair per CTA when B * Hkv <= grid and no
# sequence has more than this many tiles
DEFAULT_ALIGN_TILES = 16


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


def tiles_cost(length: int, tile_fixed: int = DEFAULT_TILE_FIXED) -> int:
    L = max(0, int(length))
    n_full, rem = divmod(L, TILE_TOKENS)
    tail = ((rem + 15) // 16 + tile_fixed) if (rem > 0 or L == 0) else 0
    return n_full * (FULL_TILE + tile_fixed) + tail


def lead(length: int, tile_fixed: int = DEFAULT_TILE_FIXED, seg: int = DEFAULT_SEG,
         floor: int = DEFAULT_FLOOR) -> int:
    return max(seg, floor - tiles_cost(length, tile_fixed))


def pair_cost(length: int, tile_fixed: int = DEFAULT_TILE_FIXED, seg: int = DEFAULT_SEG,
              floor: int = DEFAULT_FLOOR) -> int:
    return lead(length, tile_fixed, seg, floor) + tiles_cost(length, tile_fixed)


def segments(seqlens, hkv: int, grid: int, max_len: int | None = None,
             tile_fixed: int = DEFAULT_TILE_FIXED, seg: int = DEFAULT_SEG,
             align_tiles: int = 0, floor: int = DEFAULT_FLOOR) -> list[Segment]:
    """All segments of all CTAs, in CTA order then work order (kernel's split).

    align_tiles > 0: with m = ceil(B * Hkv / grid) pairs per CTA, when no
    sequence has more than align_tiles // m tiles, every pair costs the same
    (max lead + align_tiles full tiles + 1) and CTA c takes exactly the whole
    pairs [m c, m (c + 1))."""
    lens = [min(max(0, int(L)), max_len) if max_len is not None else max(0, int(L)) for L in seqlens]
    full = FULL_TILE + tile_fixed
    npairs = len(lens) * hkv
    m = -(-npairs // grid)
    aligned = align_tiles // m > 0 and all(tiles_of(L) <= align_tiles // m for L in lens)
    max_lead = max(seg, floor)
    k_aligned = max_lead + align_tiles * full + 1
    leads = [lead(L, tile_fixed, seg, floor) for L in lens]
    prefix = [0]
    for L in lens:
        prefix.append(prefix[-1] + (k_aligned if aligned else pair_cost(L, tile_fixed, seg, floor)))
    total = hkv * prefix[-1]
    grid = -(-npairs // m) if aligned else max(1, min(grid, total // (max_lead + full + 1)))

    def range_start(c):
        if aligned:
            return k_aligned * min(m * c, npairs)
        return total * c // grid

    def cta_of(s):
        return ((s + 1) * grid + total - 1) // total - 1

    def pair_start(pair):
        b, kvh = divmod(pair, hkv)
        return hkv * prefix[b] + kvh * (prefix[b + 1] - prefix[b])

    def tile_start(cp, ld, j):
        return cp if j == 0 else cp + ld + j * full

    def make(c, pair, j0, e1):
        b, kvh = divmod(pair, hkv)
        n = tiles_of(lens[b])
        ld = leads[b]
        cp = pair_start(pair)
        if j0 >= n or tile_start(cp, ld, j0) >= e1:
            return None
        x = e1 - cp - ld
        jmax = -(-x // full) - 1 if x > 0 else 0
        jmax = min(jmax, n - 1)
        c0 = cta_of(cp)
        return Segment(c, b, kvh, pair, j0, jmax - j0 + 1, cta_of(tile_start(cp, ld, n - 1)) - c0 + 1, c0)

    out: list[Segment] = []
    for c in range(grid):
        e0, e1 = range_start(c), range_start(c + 1)
        lo, hi = 0, len(lens) - 1
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if hkv * prefix[mid] <= e0:
                lo = mid
            else:
                hi = mid - 1
        pc = prefix[lo + 1] - prefix[lo]
        kvh = min(hkv - 1, (e0 - hkv * prefix[lo]) // pc)
        pair = lo * hkv + kvh
        cp = pair_start(pair)
        j0 = 0
        if e0 > cp:
            x = e0 - cp - leads[lo]
            j0 = max(1, -(-x // full)) if x > 0 else 1
        s = make(c, pair, j0, e1)
        if s is None and pair + 1 < npairs:
            s = make(c, pair + 1, 0, e1)
        while s is not None:
            out.append(s)
            if s.tile0 + s.ntiles < tiles_of(lens[s.b]) or s.pair + 1 >= npairs:
                break
            s = make(c, s.pair + 1, 0, e1)
    return out


def grid_size(batch: int, hkv: int, num_sms: int, tiles_bound: int) -> int:
    return min(num_sms, batch * hkv * tiles_bound)


def split_stats(seqlens, hkv: int, grid: int, **kw) -> dict:
    segs = segments(seqlens, hkv, grid, **kw)
    ctas = max(s.cta for s in segs) + 1
    split_pairs = {s.pair for s in segs if s.nseg > 1}
    per_cta = [0] * ctas
    seg_cta = [0] * ctas
    for s in segs:
        per_cta[s.cta] += s.ntiles
        seg_cta[s.cta] += 1
    return dict(segments=len(segs), pairs=len(seqlens) * hkv, split_pairs=len(split_pairs),
                ctas=ctas, tiles_total=sum(per_cta), tiles_per_cta_max=max(per_cta),
                tiles_per_cta_min=min(per_cta), segments_per_cta_max=max(seg_cta))
