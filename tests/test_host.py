"""CPU checks of the host-side logic: workload layouts and the split scheduler
model (the same partition the kernel computes on the device)."""
import math

import pytest
import torch

from flashdecode import cases, schedule


def test_config2_matches_baseline_sizes():
    c = cases.config_case(2)
    assert (c.B, c.Hq, c.Hkv, c.D, c.page, c.dtype) == (64, 32, 8, 128, 256, torch.bfloat16)
    assert torch.all(c.seqlens == 4096)
    assert c.num_blocks == 1024
    assert sorted(c.block_table.flatten().tolist()) == list(range(1024))
    assert c.kv_bytes() == 1_073_741_824
    assert c.algorithmic_bytes() == 1_074_802_944
    assert c.flops() == 4 * 64 * 4096 * 32 * 128


@pytest.mark.parametrize("idx", [1, 3, 5])
def test_random_layouts_use_every_page_once(idx):
    c = cases.config_case(idx)
    used = c.block_table[c.block_table >= 0]
    assert used.numel() == c.num_blocks
    assert torch.equal(used.sort().values, torch.arange(c.num_blocks, dtype=torch.int32))
    n = (c.seqlens + c.page - 1) // c.page
    for b in range(c.B):
        assert torch.all(c.block_table[b, : n[b]] >= 0)
        assert torch.all(c.block_table[b, n[b]:] == -1)


def test_length_distributions():
    c1, c3, c5 = cases.config_case(1), cases.config_case(3), cases.config_case(5)
    assert c1.seqlens.min() >= 1 and c1.seqlens.max() <= 2048
    assert c3.seqlens.min() >= 16 and c3.seqlens.max() <= 32768
    assert c3.seqlens.float().log().std() > 1.0  # log-uniform spread
    assert c5.seqlens.min() >= 512 and c5.seqlens.max() <= 8192
    assert (c5.Hq, c5.Hkv, c5.page, c5.dtype) == (28, 4, 16, torch.float16)
    c4 = cases.config_case(4)
    assert c4.kv_bytes() == 2_147_483_648 and c4.q_std == 0.5


def test_contest_layout_formula():
    c = cases.contest_case(16, 141, 4)
    assert c.num_blocks == 16 * math.ceil(141 / 16)
    assert c.block_table.shape == (16, 9)
    assert c.seqlens[0] == 141 and c.seqlens[1] == 1
    assert c.seqlens[5] == 1 + ((5 * 9973 + 141 // 3) % 140)


def test_materialize_is_deterministic_on_cpu():
    c = cases.custom_case("det", torch.bfloat16, [10, 3], 8, 2, page=16)
    a, b = cases.materialize(c, "cpu", seed=3), cases.materialize(c, "cpu", seed=3)
    assert all(torch.equal(a[k], b[k]) for k in a)


def test_subset_case_compacts_pool():
    c = cases.config_case(3)
    rows = [5, 17, 100]
    s = cases.subset_case(c, rows)
    assert s.B == 3 and torch.equal(s.seqlens, c.seqlens[rows])
    assert s.num_blocks == int(((c.seqlens[rows] + 255) // 256).sum())


@pytest.mark.parametrize("world", [2, 4, 8])
def test_lpt_partition_balances_skew(world):
    c = cases.config_case(3)
    shards = cases.lpt_partition(c.seqlens.tolist(), world)
    assert sorted(sum(shards, [])) == list(range(c.B))
    loads = [int(c.seqlens[s].sum()) for s in shards]
    assert max(loads) - min(loads) <= int(c.seqlens.max())


@pytest.mark.parametrize("seqlens,hkv,grid", [
    ([4096] * 64, 8, 148), ([1, 0, 5000, 300, 128, 129], 4, 148), ([262144] * 2, 8, 148),
    ([0], 1, 1), ([7, 9], 2, 3), (list(range(0, 3000, 37)), 8, 148),
    ([300, 7], 8, 148), ([1, 127, 128, 129, 300, 0, 1000, 2049], 4, 148),
    ([1, 127, 128, 129, 300, 0, 1000, 2049], 1, 148),
])
@pytest.mark.parametrize("weights", ["16-bit", "e4m3", "no-floor", "high-floor"])
@pytest.mark.parametrize("align", [0, schedule.DEFAULT_ALIGN_TILES, 64])
def test_schedule_covers_every_tile_once(seqlens, hkv, grid, weights, align):
    kw = {"16-bit": {}, "e4m3": dict(tile_fixed=schedule.E4M3_TILE_FIXED, seg=schedule.E4M3_SEG,
                                     floor=schedule.E4M3_FLOOR),
          # no floor, and one far above a few tiles' cost
          "no-floor": dict(seg=12, floor=0), "high-floor": dict(seg=18, floor=300)}[weights]
    kw["align_tiles"] = align
    segs = schedule.segments(seqlens, hkv, grid, **kw)
    seen = {}
    for s in segs:
        for t in range(s.tile0, s.tile0 + s.ntiles):
            key = (s.pair, t)
            assert key not in seen
            seen[key] = s.cta
    want = {(b * hkv + h, t) for b, L in enumerate(seqlens) for h in range(hkv)
            for t in range(schedule.tiles_of(L))}
    assert set(seen) == want
    # partial slots c + pair are unique and below grid + pairs
    slots = [s.slot for s in segs if s.nseg > 1]
    assert len(slots) == len(set(slots))
    assert all(0 <= x < grid + len(seqlens) * hkv for x in slots)
    # segment count of a pair equals its nseg, and they are numbered from cfirst
    by_pair = {}
    for s in segs:
        by_pair.setdefault(s.pair, []).append(s)
    for pair, ss in by_pair.items():
        assert len(ss) == ss[0].nseg
        assert [s.cta for s in ss] == list(range(ss[0].cfirst, ss[0].cfirst + ss[0].nseg))


@pytest.mark.parametrize("seqlens,hkv", [([1, 2, 300, 0], 8), ([17] * 16, 4), ([141] * 16, 4),
                                         ([512, 1, 7], 8)])
def test_pair_aligned_split_takes_whole_pairs(seqlens, hkv):
    """Few short pairs: one whole pair per CTA, nothing split or merged."""
    segs = schedule.segments(seqlens, hkv, 148, align_tiles=schedule.DEFAULT_ALIGN_TILES)
    assert [s.cta for s in segs] == list(range(len(seqlens) * hkv))
    assert [s.pair for s in segs] == list(range(len(seqlens) * hkv))
    assert all(s.nseg == 1 and s.tile0 == 0 and s.ntiles == schedule.tiles_of(seqlens[s.b])
               for s in segs)
    # a longer sequence goes back to the cost split
    assert any(s.nseg > 1 for s in schedule.segments([5000] + seqlens, hkv, 148,
                                                     align_tiles=schedule.DEFAULT_ALIGN_TILES))


@pytest.mark.parametrize("seqlens,hkv,m", [([8] * 64, 4, 2), ([362] * 32, 8, 2), ([100] * 300, 4, 9)])
def test_pair_aligned_split_several_pairs_per_cta(seqlens, hkv, m):
    """More pairs than CTAs: m = ceil(pairs / 148) whole pairs per CTA while
    m pairs stay within the tile budget; otherwise the cost split."""
    segs = schedule.segments(seqlens, hkv, 148, align_tiles=schedule.DEFAULT_ALIGN_TILES)
    per_cta_tiles = m * schedule.tiles_of(seqlens[0])
    if per_cta_tiles <= schedule.DEFAULT_ALIGN_TILES:
        assert all(s.nseg == 1 and s.cta == s.pair // m for s in segs)
        assert max(s.cta for s in segs) + 1 == -(-len(seqlens) * hkv // m)
    else:
        assert any(s.nseg > 1 for s in segs)


def test_cost_floor_raises_short_pairs_only():
    """A pair never costs less than the floor; pairs above it keep seg."""
    for L in [0, 1, 127, 128, 129, 300, 1000, 5000]:
        base = schedule.pair_cost(L, seg=12, floor=0)
        raised = schedule.pair_cost(L, seg=12, floor=40)
        assert raised == max(base, 40)
        assert schedule.lead(L, seg=12, floor=40) >= 12
    assert schedule.pair_cost(5000, seg=12, floor=40) == schedule.pair_cost(5000, seg=12, floor=0)
    assert schedule.pair_cost(1, seg=12, floor=0) < 40 == schedule.pair_cost(1, seg=12, floor=40)


def test_cost_floor_caps_pairs_per_cta_on_skewed_shards():
    """Config 3 split over 8 ranks: with the per-pair cost alone some CTAs
    take up to 17 short pairs (the slowest shard measured on a B200 was the
    one with 17); the floor spreads them to at most 8 per CTA without
    changing the tiles a CTA streams by more than one."""
    from flashdecode import dist as fdist
    c = cases.config_case(3)
    worst_seg_only = 0
    for rank in range(8):
        sh = fdist.batch_shard(c, rank, 8)[0]
        sl = sh.seqlens.tolist()
        seg_only = schedule.split_stats(sl, sh.Hkv, 148, floor=0, align_tiles=16)
        floored = schedule.split_stats(sl, sh.Hkv, 148, align_tiles=16)
        worst_seg_only = max(worst_seg_only, seg_only["segments_per_cta_max"])
        assert floored["segments_per_cta_max"] <= 8
        assert floored["tiles_per_cta_max"] <= seg_only["tiles_per_cta_max"] + 1
    assert worst_seg_only >= 16


def _cta_costs(seqlens, hkv, grid):
    full = schedule.FULL_TILE + schedule.DEFAULT_TILE_FIXED
    costs = {}
    for s in schedule.segments(seqlens, hkv, grid):
        L = max(0, int(seqlens[s.b]))
        c = schedule.lead(L) if s.tile0 == 0 else 0
        for j in range(s.tile0, s.tile0 + s.ntiles):
            rem = L - j * schedule.TILE_TOKENS
            c += full if rem >= schedule.TILE_TOKENS else (rem + 15) // 16 + schedule.DEFAULT_TILE_FIXED
        costs[s.cta] = costs.get(s.cta, 0) + c
    return costs


@pytest.mark.parametrize("idx", [2, 3, 5])
def test_schedule_balances_estimated_cost(idx):
    c = cases.config_case(idx)
    costs = _cta_costs(c.seqlens.tolist(), c.Hkv, 148)
    assert len(costs) == 148
    item = (max(schedule.DEFAULT_SEG, schedule.DEFAULT_FLOOR) + schedule.FULL_TILE
            + schedule.DEFAULT_TILE_FIXED)
    assert max(costs.values()) - min(costs.values()) <= 2 * item


def test_schedule_is_balanced_on_config2():
    st = schedule.split_stats([4096] * 64, 8, 148)
    assert st["tiles_total"] == 64 * 8 * 32
    assert st["tiles_per_cta_max"] - st["tiles_per_cta_min"] <= 2


def test_head_shard_slices_heads_and_decodes_the_same_rows():
    """KV-head sharding: the ranks' KV-head ranges partition the heads, and
    decoding a rank's head slice (oracle) gives exactly the matching query
    heads of the full decode."""
    from flashdecode import dist as fdist
    from oracle.decode_ref import decode_reference
    c = cases.custom_case("hs", torch.float32, [37, 0, 200], 8, 4, D=16, page=8, seed=4)
    t = cases.materialize(c, "cpu", seed=4)
    full_o, full_l = decode_reference(t["q"], t["k_cache"], t["v_cache"], t["cache_seqlens"],
                                      t["block_table"], softmax_scale=c.softmax_scale)
    world = 2
    covered = []
    for rank in range(world):
        local, (q0, q1) = fdist.head_shard(c, rank, world)
        h0, h1 = fdist.head_range(c.Hkv, rank, world)
        covered += list(range(h0, h1))
        assert local.Hkv == h1 - h0 and local.Hq == q1 - q0 == (h1 - h0) * (c.Hq // c.Hkv)
        o, l = decode_reference(t["q"][:, :, q0:q1], t["k_cache"][:, :, h0:h1],
                                t["v_cache"][:, :, h0:h1], local.seqlens, local.block_table,
                                softmax_scale=local.softmax_scale)
        assert torch.equal(o, full_o[:, :, q0:q1])
        assert torch.equal(l, full_l[:, q0:q1])
    assert covered == list(range(c.Hkv))
    with pytest.raises(ValueError):
        fdist.head_range(6, 0, 4)


def test_cost_defaults_match_the_host_library():
    """The mirror's cost weights are the ones fd_api.cu launches with."""
    import re
    from pathlib import Path
    src = (Path(__file__).resolve().parent.parent / "flashatte-hand_b200" / "csrc" / "fd_api.cu").read_text()
    got = {m.group(1): int(m.group(2))
           for m in re.finditer(r"constexpr int (kDefaultCost\w+) = (\d+);", src)}
    assert got == {"kDefaultCostTile": schedule.DEFAULT_TILE_FIXED, "kDefaultCostSeg": schedule.DEFAULT_SEG,
                   "kDefaultCostTile8": schedule.E4M3_TILE_FIXED, "kDefaultCostSeg8": schedule.E4M3_SEG,
                   "kDefaultCostFloor": schedule.DEFAULT_FLOOR, "kDefaultCostFloor8": schedule.E4M3_FLOOR}
    align = re.search(r"constexpr int kDefaultAlignTiles = (\d+);", src)
    assert int(align.group(1)) == schedule.DEFAULT_ALIGN_TILES
