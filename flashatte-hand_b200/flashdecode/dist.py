"""Multi-GPU partitioning of the decode inside one node (one process per GPU).

The reference has no multi-GPU code; its only decomposition is intra-GPU
split-KV (submission-oj/best_flashattn_kvcache_decode.cu:1381-1425).  Two
partitions are provided here:

* batch sharding (``batch_shard``): each rank owns whole sequences and their
  KV pages, chosen longest-first (LPT) so skewed length mixes balance.  No
  collective is on the data path; every rank writes its own output rows.
* KV-head sharding (``head_shard``): each rank owns Hkv / world KV heads of
  every sequence and the query heads that read them, and holds only those
  heads' pages; no collective, every rank writes its own output heads.  The
  natural choice for a small batch of long sequences when Hkv >= world.
* cross-GPU split-KV (``kv_split_case``): each rank owns a contiguous page
  range of every sequence and decodes it to a normalised fp32 partial
  (O, LSE) per output row; the ranks' partials are merged with LSE weights.
  That is the reference's split/combine (best :595-1037) with the splits
  placed on different GPUs.  ``PeerSplitKVDecode`` is the product path: the
  decode kernel itself stores its partial into every rank's exchange buffer
  over NVLink (peer mappings of buffers swapped as IPC handles) and a merge
  kernel on each rank waits for all ranks' flags.  ``SplitKVDecode`` runs the
  same protocol through a collective (all-gather of packed [O | LSE] blocks,
  B*Hq*(D+1) floats per rank) with injectable decode/merge steps; the CPU
  tests drive it over gloo.
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as tdist

from . import cases as _cases
from ._lib import FD_DTYPE_BF16, FD_DTYPE_FP16, FD_DTYPE_FP32, check, load_library


def batch_shard(case: _cases.DecodeCase, rank: int, world: int):
    """(sub-case of the sequences rank owns, their global row indices)."""
    rows = _cases.lpt_partition(case.seqlens.tolist(), world)[rank]
    if not rows:
        raise ValueError(f"rank {rank} of {world} owns no sequence (batch {case.B})")
    return _cases.subset_case(case, rows, name=f"{case.name}_shard{rank}of{world}"), rows


def head_range(num_heads_k: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads [h0, h1) of `rank`: contiguous, equal shares (Hkv % world == 0)."""
    if num_heads_k % world != 0:
        raise ValueError(f"{num_heads_k} KV heads do not split over {world} ranks")
    per = num_heads_k // world
    return rank * per, (rank + 1) * per


def head_shard(case: _cases.DecodeCase, rank: int, world: int):
    """(local case with Hkv / world KV heads and Hq / world query heads, the
    global query-head range [q0, q1) it serves).  Sequences, lengths and the
    page table are unchanged; the local cache holds only this rank's heads."""
    h0, h1 = head_range(case.Hkv, rank, world)
    group = case.Hq // case.Hkv
    local = _cases.DecodeCase(name=f"{case.name}_heads{rank}of{world}", dtype=case.dtype, B=case.B,
                              Hq=(h1 - h0) * group, Hkv=h1 - h0, D=case.D, page=case.page,
                              seqlens=case.seqlens.clone(), block_table=case.block_table.clone(),
                              num_blocks=case.num_blocks, q_std=case.q_std,
                              softmax_scale=case.softmax_scale)
    return local, (h0 * group, h1 * group)


def kv_page_range(n_pages: int, rank: int, world: int) -> tuple[int, int]:
    return n_pages * rank // world, n_pages * (rank + 1) // world


def kv_split_case(case: _cases.DecodeCase, rank: int, world: int):
    """Local view of rank's page range of every sequence.

    Returns (local case with its own compact page pool, page_map) where
    page_map[i] is the global page id of local page i.
    """
    page = case.page
    sl_local, rows_pages = [], []
    for b in range(case.B):
        L = max(int(case.seqlens[b]), 0)
        n = math.ceil(L / page)
        p0, p1 = kv_page_range(n, rank, world)
        sl_local.append(max(0, min(L, p1 * page) - p0 * page))
        rows_pages.append(case.block_table[b, p0:p1].tolist())
    page_map = [pg for r in rows_pages for pg in r]
    width = max(1, max(len(r) for r in rows_pages))
    bt = torch.full((case.B, width), -1, dtype=torch.int32)
    off = 0
    for b, r in enumerate(rows_pages):
        bt[b, : len(r)] = torch.arange(off, off + len(r), dtype=torch.int32)
        off += len(r)
    local = _cases.DecodeCase(name=f"{case.name}_kv{rank}of{world}", dtype=case.dtype, B=case.B,
                              Hq=case.Hq, Hkv=case.Hkv, D=case.D, page=page,
                              seqlens=torch.tensor(sl_local, dtype=torch.int32), block_table=bt,
                              num_blocks=max(len(page_map), 1), q_std=case.q_std,
                              softmax_scale=case.softmax_scale)
    return local, torch.tensor(page_map, dtype=torch.int64)


def _default_decode(q, k, v, seqlens, bt, scale, out_o, out_lse):
    from .ops import flash_decode
    flash_decode(q, k, v, seqlens, bt, softmax_scale=scale, out=out_o, out_dtype=torch.float32,
                 lse=out_lse)


def _default_combine(part_o, part_lse, out_dtype):
    from .ops import combine_lse
    return combine_lse(part_o, part_lse, out_dtype=out_dtype, return_lse=True)


class SplitKVDecode:
    """Cross-GPU split-KV decode step: local partial -> all-gather -> combine.

    ``decode_fn`` / ``combine_fn`` default to the CUDA operator; tests on CPU
    ranks pass stand-ins to exercise the exchange protocol without a GPU.
    """

    def __init__(self, B: int, Hq: int, D: int, out_dtype: torch.dtype, device,
                 group=None, decode_fn=None, combine_fn=None):
        self.B, self.Hq, self.D = B, Hq, D
        self.rows = B * Hq
        self.block = self.rows * D + self.rows
        self.group = group
        self.world = tdist.get_world_size(group)
        self.out_dtype = out_dtype
        self.send = torch.empty(self.block, dtype=torch.float32, device=device)
        self.recv = torch.empty(self.world * self.block, dtype=torch.float32, device=device)
        self.decode_fn = decode_fn or _default_decode
        self.combine_fn = combine_fn or _default_combine
        self._flat = tdist.get_backend(group) == "nccl"

    def __call__(self, q, k_local, v_local, seqlens_local, bt_local, softmax_scale: float):
        o_view = self.send[: self.rows * self.D].view(self.B, 1, self.Hq, self.D)
        l_view = self.send[self.rows * self.D:].view(self.B, self.Hq)
        self.decode_fn(q, k_local, v_local, seqlens_local, bt_local, softmax_scale, o_view, l_view)
        if self._flat:
            tdist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        else:
            tdist.all_gather(list(self.recv.view(self.world, self.block).unbind(0)), self.send,
                             group=self.group)
        parts = self.recv.view(self.world, self.block)
        part_o = parts[:, : self.rows * self.D].view(self.world, self.rows, self.D)
        part_l = parts[:, self.rows * self.D:]
        out, lse = self.combine_fn(part_o, part_l, self.out_dtype)
        return out.view(self.B, 1, self.Hq, self.D), lse.view(self.B, self.Hq)


_DT = {torch.bfloat16: FD_DTYPE_BF16, torch.float16: FD_DTYPE_FP16, torch.float32: FD_DTYPE_FP32}


class PeerSplitKVDecode:
    """Cross-GPU split-KV decode step over peer memory (one process per GPU).

    Set-up (collective, every rank): allocate this rank's exchange buffer,
    swap IPC handles over the process group, map the peers' buffers.  Each
    call then launches two kernels on the current stream: the decode kernel,
    which writes this rank's partial for every output row into every rank's
    buffer and flags it, and the merge kernel, which waits for all ranks'
    flags and writes the full result on every rank.  Every rank must make the
    same sequence of calls.
    """

    def __init__(self, B: int, Hq: int, D: int, out_dtype: torch.dtype, device, group=None,
                 seqlen_q: int = 1):
        self.lib = load_library()
        self.B, self.Hq, self.D, self.sq = B, Hq, D, seqlen_q
        self.out_dtype = out_dtype
        self.device = torch.device(device)
        self.group = group
        self.world = tdist.get_world_size(group)
        self.rank = tdist.get_rank(group)
        size = self.lib.fd_xgpu_buffer_size(B, seqlen_q, Hq, self.world)
        if size == 0:
            raise ValueError("unsupported exchange shape")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            check(self.lib.fd_xgpu_alloc(size, ctypes.byref(own), handle))
        self._own = own.value
        handles = [None] * self.world
        tdist.all_gather_object(handles, handle.raw, group=group)
        ptrs, self._opened = [], []
        with torch.cuda.device(self.device):
            for j, h in enumerate(handles):
                if j == self.rank:
                    ptrs.append(self._own)
                    continue
                p = ctypes.c_void_p()
                check(self.lib.fd_xgpu_open(h, ctypes.byref(p)))
                ptrs.append(p.value)
                self._opened.append(p.value)
        self.xbufs = (ctypes.c_void_p * self.world)(*ptrs)
        self.step = 0
        tdist.barrier(group=group)

    def __call__(self, q, k_local, v_local, seqlens_local, bt_local, softmax_scale: float,
                 causal: bool = False, out=None, lse=None, k_scale=None, v_scale=None):
        """One step.  e4m3 caches (torch.float8_e4m3fn) take fp32 per-KV-head
        k_scale / v_scale [Hkv], as flashdecode.flash_decode does."""
        B, sq, Hq, D = q.shape
        if out is None:
            out = torch.empty((B, sq, Hq, D), dtype=self.out_dtype, device=q.device)
        if lse is None:
            lse = torch.empty((B, Hq) if sq == 1 else (B, Hq, sq), dtype=torch.float32,
                              device=q.device)
        st = torch.cuda.current_stream(q.device)
        nb, page, Hkv, _ = k_local.shape
        with torch.cuda.device(q.device):
            if k_local.dtype == torch.float8_e4m3fn:
                if k_scale is None or v_scale is None:
                    raise ValueError("e4m3 caches need k_scale and v_scale")
                status = self.lib.fd_decode_paged_fp8_xgpu(
                    q.data_ptr(), k_local.data_ptr(), v_local.data_ptr(), k_scale.data_ptr(),
                    v_scale.data_ptr(), seqlens_local.data_ptr(), bt_local.data_ptr(),
                    bt_local.shape[1], B, sq, Hq, Hkv, D, page, nb, _DT[q.dtype],
                    _DT[self.out_dtype], float(softmax_scale), 1 if causal else 0, 0, self.rank,
                    self.world, self.xbufs, self.step, out.data_ptr(), lse.data_ptr(), None, 0,
                    st.cuda_stream)
            else:
                status = self.lib.fd_decode_paged_xgpu(
                    q.data_ptr(), k_local.data_ptr(), v_local.data_ptr(), seqlens_local.data_ptr(),
                    bt_local.data_ptr(), bt_local.shape[1], B, sq, Hq, Hkv, D, page, nb, _DT[q.dtype],
                    _DT[self.out_dtype], float(softmax_scale), 1 if causal else 0, 0, self.rank,
                    self.world, self.xbufs, self.step, out.data_ptr(), lse.data_ptr(), None, 0,
                    st.cuda_stream)
        check(status)
        self.step += 1
        return out, lse

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective)."""
        torch.cuda.synchronize(self.device)
        tdist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                check(self.lib.fd_xgpu_close(p))
            self._opened = []
        tdist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            if self._own:
                check(self.lib.fd_xgpu_free(self._own))
                self._own = None
