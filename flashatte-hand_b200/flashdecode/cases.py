"""Seeded synthetic decode workloads.

* ``config_case(i)`` builds the five workloads this operator is measured on
  (i = 1..5): shapes, dtypes and length distributions as listed in
  ``CONFIGS`` below.  Sequence lengths and page tables are drawn on the CPU
  from a fixed seed, so every machine builds the same layout; the bulk K/V/q
  tensors are drawn on the target device by ``materialize``.
* ``contest_case(B, L, Hkv)`` rebuilds the reference evaluator's contest
  layout (scripts/evaluate_flashattn_submission.py:105-151, :359-389):
  Hq = 32, D = 128, page 16, num_blocks = B * ceil(L / 16),
  block_table = randperm(num_blocks).reshape(B, -1), row 0 has length L,
  row 1 length 1, row b >= 2 length 1 + ((b * 9973 + L // 3) % (L - 1)).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

CONFIGS = {
    1: dict(name="cfg1_fp16_b4_l2048_cpu", dtype=torch.float16, B=4, Hq=32, Hkv=8, D=128, page=256,
            lengths=("uniform", 1, 2048), q_std=1.0),
    2: dict(name="cfg2_llama3_8b_b64_l4096", dtype=torch.bfloat16, B=64, Hq=32, Hkv=8, D=128,
            page=256, lengths=("fixed", 4096), q_std=1.0),
    3: dict(name="cfg3_skew_b128_hq64", dtype=torch.bfloat16, B=128, Hq=64, Hkv=8, D=128, page=256,
            lengths=("loguniform", 16, 32768), q_std=1.0),
    4: dict(name="cfg4_long_b2_l262144", dtype=torch.bfloat16, B=2, Hq=32, Hkv=8, D=128, page=256,
            lengths=("fixed", 262144), q_std=0.5),
    5: dict(name="cfg5_g7_page16_b256", dtype=torch.float16, B=256, Hq=28, Hkv=4, D=128, page=16,
            lengths=("uniform", 512, 8192), q_std=1.0),
}


@dataclass
class DecodeCase:
    name: str
    dtype: torch.dtype
    B: int
    Hq: int
    Hkv: int
    D: int
    page: int
    seqlens: torch.Tensor          # [B] int32, CPU
    block_table: torch.Tensor      # [B, max_blocks] int32, CPU, -1 = unused
    num_blocks: int
    q_std: float = 1.0
    softmax_scale: float = field(default=0.0)

    def __post_init__(self):
        if not self.softmax_scale:
            self.softmax_scale = 1.0 / math.sqrt(self.D)

    @property
    def group(self) -> int:
        return self.Hq // self.Hkv

    def kv_bytes(self) -> int:
        """K and V bytes the decode must read (each cached token, each KV head, once)."""
        es = torch.empty((), dtype=self.dtype).element_size()
        return int(self.seqlens.clamp(min=0).sum()) * self.Hkv * self.D * 2 * es

    def algorithmic_bytes(self, with_lse: bool = True) -> int:
        """KV + q + out + LSE + the block_table entries read + cache_seqlens."""
        es = torch.empty((), dtype=self.dtype).element_size()
        pages = int(((self.seqlens.clamp(min=0) + self.page - 1) // self.page).sum())
        qo = 2 * self.B * self.Hq * self.D * es
        return self.kv_bytes() + qo + (4 * self.B * self.Hq if with_lse else 0) + 4 * pages + 4 * self.B

    def flops(self) -> int:
        return 4 * int(self.seqlens.clamp(min=0).sum()) * self.Hq * self.D


def _pack_pages(seqlens: torch.Tensor, page: int, gen: torch.Generator, pool_extra: int = 0):
    """Random permutation of a pool of sum(ceil(L/page)) pages dealt out in order."""
    n = ((seqlens.clamp(min=0) + page - 1) // page).to(torch.int64)
    n = torch.where(seqlens > 0, n, torch.zeros_like(n))
    num_blocks = int(n.sum()) + pool_extra
    num_blocks = max(num_blocks, 1)
    perm = torch.randperm(num_blocks, generator=gen).to(torch.int32)
    max_blocks = max(int(n.max()), 1)
    bt = torch.full((len(seqlens), max_blocks), -1, dtype=torch.int32)
    off = 0
    for b, nb in enumerate(n.tolist()):
        bt[b, :nb] = perm[off:off + nb]
        off += nb
    return bt, num_blocks


def config_case(idx: int, seed: int = 0) -> DecodeCase:
    c = CONFIGS[idx]
    g = torch.Generator().manual_seed(seed)
    kind = c["lengths"]
    B = c["B"]
    if kind[0] == "fixed":
        seqlens = torch.full((B,), kind[1], dtype=torch.int32)
    elif kind[0] == "uniform":
        seqlens = torch.randint(kind[1], kind[2] + 1, (B,), generator=g, dtype=torch.int64).to(torch.int32)
    else:
        lo, hi = math.log(kind[1]), math.log(kind[2])
        u = torch.rand((B,), generator=g, dtype=torch.float64)
        seqlens = torch.exp(lo + (hi - lo) * u).round().clamp(kind[1], kind[2]).to(torch.int32)
    bt, num_blocks = _pack_pages(seqlens, c["page"], g)
    return DecodeCase(name=c["name"], dtype=c["dtype"], B=B, Hq=c["Hq"], Hkv=c["Hkv"], D=c["D"],
                      page=c["page"], seqlens=seqlens, block_table=bt, num_blocks=num_blocks,
                      q_std=c["q_std"])


def custom_case(name: str, dtype: torch.dtype, seqlens, Hq: int, Hkv: int, D: int = 128,
                page: int = 256, seed: int = 0, q_std: float = 1.0, pool_extra: int = 0,
                pad_blocks: int = 0) -> DecodeCase:
    g = torch.Generator().manual_seed(seed)
    sl = torch.as_tensor(seqlens, dtype=torch.int32)
    bt, num_blocks = _pack_pages(sl, page, g, pool_extra)
    if pad_blocks:
        bt = torch.cat([bt, torch.full((bt.shape[0], pad_blocks), -1, dtype=torch.int32)], dim=1)
    return DecodeCase(name=name, dtype=dtype, B=len(sl), Hq=Hq, Hkv=Hkv, D=D, page=page,
                      seqlens=sl, block_table=bt, num_blocks=num_blocks, q_std=q_std)


def contest_case(batch: int, seqlen: int, kv_heads: int, seed: int = 0) -> DecodeCase:
    page = 16
    blocks_per_batch = math.ceil(seqlen / page)
    num_blocks = batch * blocks_per_batch
    g = torch.Generator().manual_seed(seed)
    bt = torch.randperm(num_blocks, generator=g).to(torch.int32).reshape(batch, -1)
    vals = []
    for b in range(batch):
        if b == 0:
            vals.append(seqlen)
        elif b == 1:
            vals.append(1)
        else:
            span = max(1, seqlen - 1)
            vals.append(1 + ((b * 9973 + seqlen // 3) % span))
    return DecodeCase(name=f"contest_b{batch}_l{seqlen}_hkv{kv_heads}", dtype=torch.bfloat16,
                      B=batch, Hq=32, Hkv=kv_heads, D=128, page=page,
                      seqlens=torch.tensor(vals, dtype=torch.int32), block_table=bt,
                      num_blocks=num_blocks)


# (B, L, Hkv) rows of the reference's contest profile (evaluate_flashattn_submission.py:359-389).
CONTEST_SHAPES = [(4, 1, 8), (4, 2, 8), (16, 17, 4), (64, 8, 4), (16, 141, 4), (32, 362, 8),
                  (64, 2048, 4), (16, 4096, 4), (32, 4096, 8), (1, 8192, 4), (16, 12251, 4),
                  (8, 32768, 8), (1, 58966, 8), (1, 61519, 4)]


def materialize(case: DecodeCase, device, seed: int = 0) -> dict:
    """Draw q, K, V ~ N(0, 1) (q ~ N(0, q_std)) on `device` from `seed`."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    shape_kv = (case.num_blocks, case.page, case.Hkv, case.D)
    q = torch.randn((case.B, 1, case.Hq, case.D), generator=g, device=dev, dtype=case.dtype)
    if case.q_std != 1.0:
        q.mul_(case.q_std)
    k = torch.randn(shape_kv, generator=g, device=dev, dtype=case.dtype)
    v = torch.randn(shape_kv, generator=g, device=dev, dtype=case.dtype)
    return dict(q=q, k_cache=k, v_cache=v, cache_seqlens=case.seqlens.to(dev),
                block_table=case.block_table.to(dev))


def materialize_e4m3(case: DecodeCase, device, seed: int = 0) -> dict:
    """materialize() with an e4m3 K/V cache: the N(0, 1) K and V are stored as
    e4m3(x / scale[h]) with per-KV-head scales in [1/64, 1/32) (so the values
    use most of the e4m3 range); q stays case.dtype.  Adds k_scale, v_scale."""
    t = materialize(case, device, seed=seed)
    dev = torch.device(device)
    g = torch.Generator().manual_seed(seed + 2)
    ks = (1.0 + torch.rand(case.Hkv, generator=g)) / 64.0
    vs = (1.0 + torch.rand(case.Hkv, generator=g)) / 64.0
    t["k_scale"], t["v_scale"] = ks.to(dev), vs.to(dev)
    for name, sc in (("k_cache", t["k_scale"]), ("v_cache", t["v_scale"])):
        x = t[name]
        t[name] = (x.float() / sc[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
        del x
    return t


def lpt_partition(seqlens, world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of sequences to `world` shards."""
    order = sorted(range(len(seqlens)), key=lambda b: (-int(seqlens[b]), b))
    loads = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for b in order:
        r = min(range(world), key=lambda i: (loads[i], i))
        shards[r].append(b)
        loads[r] += max(int(seqlens[b]), 1)
    return [sorted(s) for s in shards]


def subset_case(case: DecodeCase, rows: list[int], name: str | None = None) -> DecodeCase:
    """The sequences `rows` of `case` with their own compacted page pool."""
    sl = case.seqlens[rows].clone()
    bt_old = case.block_table[rows]
    used = bt_old[bt_old >= 0].unique(sorted=True)
    remap = torch.full((case.num_blocks,), -1, dtype=torch.int32)
    remap[used.long()] = torch.arange(len(used), dtype=torch.int32)
    bt = torch.where(bt_old >= 0, remap[bt_old.clamp(min=0).long()], bt_old)
    return DecodeCase(name=name or f"{case.name}_sub{len(rows)}", dtype=case.dtype, B=len(rows),
                      Hq=case.Hq, Hkv=case.Hkv, D=case.D, page=case.page, seqlens=sl,
                      block_table=bt.contiguous(), num_blocks=max(len(used), 1), q_std=case.q_std,
                      softmax_scale=case.softmax_scale)
