"""Torch-facing host API of the paged-KV GQA decode operator.

``run_kernel`` mirrors the reference binding ``run_kernel_torch``
(scripts/evaluate_flashattn_submission.py:46-78): same argument names and
order, tensors in, pointers forwarded to the C ABI, nothing returned, and
arguments the operator rejects are ignored silently exactly as the reference
does (``last_error()`` tells why).

``flash_decode`` is the extended call with the ``flash_attn_with_kvcache``
argument vocabulary the reference's evaluator uses for its oracle
(evaluate_flashattn_submission.py:232-247): q, k_cache, v_cache,
cache_seqlens, block_table, softmax_scale, return_softmax_lse.  It runs on
the tensors' device and current stream and raises on any error.
"""
from __future__ import annotations

import contextlib
import math

import torch

from ._lib import (FD_DTYPE_BF16, FD_DTYPE_FP16, FD_DTYPE_FP32, FlashDecodeError, check,
                   load_library)

_DTYPES = {torch.bfloat16: FD_DTYPE_BF16, torch.float16: FD_DTYPE_FP16}
_OUT_DTYPES = {torch.bfloat16: FD_DTYPE_BF16, torch.float16: FD_DTYPE_FP16, torch.float32: FD_DTYPE_FP32}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(stream, dev: torch.device) -> int:
    """cudaStream_t of `stream`, or of the current stream of `dev` (read
    without building a Stream object when torch offers that)."""
    if stream is not None:
        return stream.cuda_stream
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _on_device(dev: torch.device):
    """Context that makes `dev` current, or nothing when it already is (the
    device switch costs more than the rest of a small call)."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("flashdecode runs on CUDA tensors only (no CPU path)")


def run_kernel(q, k_cache_paged, v_cache_paged, output, cache_seqlens, block_table, batch_size,
               seqlen_k, seqlen_q, num_heads, num_heads_k, headdim, page_block_size, num_blocks,
               causal) -> None:
    """Reference operator surface: bf16, scale 1/sqrt(headdim), default stream."""
    lib = load_library()
    lib.run_kernel(_ptr(q), _ptr(k_cache_paged), _ptr(v_cache_paged), _ptr(output),
                   _ptr(cache_seqlens), _ptr(block_table), int(batch_size), int(seqlen_k),
                   int(seqlen_q), int(num_heads), int(num_heads_k), int(headdim),
                   int(page_block_size), int(num_blocks), int(causal))


def last_error() -> tuple[int, str]:
    """(status, message) of the last C-ABI call on this thread."""
    lib = load_library()
    return int(lib.fd_last_error()), lib.fd_last_error_message().decode()


def device_status() -> int:
    """Read and clear the device error word of the library-owned workspace."""
    return int(load_library().fd_device_status())


def workspace_size(batch_size: int, num_heads: int, num_heads_k: int, headdim: int = 128,
                   seqlen_q: int = 1) -> int:
    return int(load_library().fd_decode_workspace_size_mq(batch_size, seqlen_q, num_heads,
                                                          num_heads_k, headdim))


def flash_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                 softmax_scale: float | None = None, return_softmax_lse: bool = False,
                 out: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                 max_seqlen_k: int | None = None, workspace: torch.Tensor | None = None,
                 stream: torch.cuda.Stream | None = None, lse: torch.Tensor | None = None,
                 causal: bool = False, k: torch.Tensor | None = None,
                 v: torch.Tensor | None = None, k_scale: torch.Tensor | None = None,
                 v_scale: torch.Tensor | None = None):
    """Paged decode attention for seqlen_q >= 1 query tokens per sequence.

    q [B, sq, Hq, D]; k_cache/v_cache [num_blocks, page, Hkv, D];
    cache_seqlens [B] int32; block_table [B, max_blocks] int32.
    Returns out [B, sq, Hq, D] (and lse fp32 natural log: [B, Hq] for sq = 1,
    else [B, Hq, sq]).  causal: query token i sits at position L - sq + i
    (L = attended keys) and sees keys up to it.  `out` and `lse` may be
    given as preallocated contiguous buffers; passing `lse` implies
    return_softmax_lse.

    k / v [B, seqlen_new, Hkv, D] (optional, together): as in
    flash_attn_with_kvcache, they are first written into the cache at
    positions cache_seqlens[b] .. cache_seqlens[b] + seqlen_new - 1, then
    attention runs over L = cache_seqlens[b] + seqlen_new keys;
    cache_seqlens itself is left unchanged.

    FP8 cache: k_cache / v_cache of dtype torch.float8_e4m3fn with k_scale /
    v_scale fp32 [Hkv] (the attended key is k_cache * k_scale[h]); q stays
    bf16 or fp16 and k / v, when given, are 16-bit rows quantised into the
    cache.  Head dim 128, seqlen_q * (Hq / Hkv) <= 16, pages of a multiple
    of 16 tokens.
    """
    call = _prepare(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                    return_softmax_lse, out, out_dtype, max_seqlen_k, workspace, lse, causal, k, v,
                    k_scale, v_scale)
    with _on_device(q.device):
        check(call.fn(*call.args, _stream_handle(stream, q.device)))
    return (call.out, call.lse) if call.return_lse else call.out


class _Call:
    """One validated C call: entry point, its arguments up to the stream, and
    the output tensors it writes."""

    __slots__ = ("fn", "args", "out", "lse", "return_lse")

    def __init__(self, fn, args, out, lse, return_lse):
        self.fn, self.args, self.out, self.lse, self.return_lse = fn, args, out, lse, return_lse


def _prepare(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, return_softmax_lse,
             out, out_dtype, max_seqlen_k, workspace, lse, causal, k, v, k_scale, v_scale) -> _Call:
    """Check the arguments of flash_decode, allocate the outputs it was not
    given and bind the C entry point that serves them."""
    lib = load_library()
    _require_cuda(q, k_cache, v_cache, cache_seqlens, block_table)
    if q.dim() != 4:
        raise ValueError(f"q must be [B, seqlen_q, Hq, D], got {tuple(q.shape)}")
    kv8 = k_cache.dtype == torch.float8_e4m3fn
    if q.dtype not in _DTYPES or v_cache.dtype != k_cache.dtype or (not kv8 and k_cache.dtype != q.dtype):
        raise ValueError("q, k_cache, v_cache must share dtype bf16 or fp16 (or e4m3 caches)")
    if kv8:
        _check_scales(k_scale, v_scale, k_cache.shape[2])
    elif k_scale is not None or v_scale is not None:
        raise ValueError("k_scale / v_scale apply to float8_e4m3fn caches only")
    if cache_seqlens.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("cache_seqlens and block_table must be int32")
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("cache_seqlens", cache_seqlens), ("block_table", block_table)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    B, sq, Hq, D = q.shape
    num_blocks, page, Hkv, Dk = k_cache.shape
    if tuple(v_cache.shape) != tuple(k_cache.shape) or Dk != D:
        raise ValueError("k_cache/v_cache shape mismatch")
    if block_table.dim() != 2 or block_table.shape[0] != B or cache_seqlens.shape != (B,):
        raise ValueError("block_table must be [B, max_blocks] and cache_seqlens [B]")
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    odt = q.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((B, sq, Hq, D), dtype=odt, device=q.device)
    elif out.dtype != odt or tuple(out.shape) != (B, sq, Hq, D) or not out.is_contiguous():
        raise ValueError("out has the wrong shape, dtype or layout")
    lse_shape = (B, Hq) if sq == 1 else (B, Hq, sq)
    if lse is not None:
        if lse.dtype != torch.float32 or lse.numel() != B * Hq * sq or not lse.is_contiguous():
            raise ValueError(f"lse must be a contiguous fp32 {lse_shape} tensor")
        return_softmax_lse = True
    elif return_softmax_lse:
        lse = torch.empty(lse_shape, dtype=torch.float32, device=q.device)
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    if (k is None) != (v is None):
        raise ValueError("k and v must be given together")
    causal_i = 1 if causal else 0
    max_len = int(max_seqlen_k or 0)
    if kv8:
        if k is not None:
            _check_new_kv(k, v, k_cache, B, q.dtype)
        args = (_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k_scale), _ptr(v_scale), _ptr(k),
                _ptr(v), 0 if k is None else k.shape[1], _ptr(out), _ptr(lse), _ptr(cache_seqlens),
                _ptr(block_table), int(block_table.shape[1]), B, sq, Hq, Hkv, D, page, num_blocks,
                _DTYPES[q.dtype], _OUT_DTYPES[odt], scale, causal_i, max_len, ws_ptr, ws_bytes)
        return _Call(lib.fd_decode_paged_fp8, args, out, lse, return_softmax_lse)
    if k is not None:
        _check_new_kv(k, v, k_cache, B)
        args = (_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(k), _ptr(v), _ptr(out), _ptr(lse),
                _ptr(cache_seqlens), _ptr(block_table), int(block_table.shape[1]), B, sq,
                k.shape[1], Hq, Hkv, D, page, num_blocks, _DTYPES[q.dtype], _OUT_DTYPES[odt],
                scale, causal_i, max_len, ws_ptr, ws_bytes)
        return _Call(lib.fd_decode_paged_kvappend, args, out, lse, return_softmax_lse)
    args = (_ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), _ptr(lse), _ptr(cache_seqlens),
            _ptr(block_table), int(block_table.shape[1]), B, sq, Hq, Hkv, D, page, num_blocks,
            _DTYPES[q.dtype], _OUT_DTYPES[odt], scale, causal_i, max_len, ws_ptr, ws_bytes)
    return _Call(lib.fd_decode_paged_mq, args, out, lse, return_softmax_lse)


class DecodePlan:
    """flash_decode bound to fixed tensors and checked once.

    A serving loop writes each step's query, lengths and page table into the
    same buffers; binding them once leaves a single C call per step (no
    argument checks, no output allocation: about a third of flash_decode's
    host time).  Takes flash_decode's arguments; the outputs are allocated
    once (or given) and overwritten by every call.  The bound tensors must
    stay alive and keep their storage, as for a captured CUDA graph: build a
    new plan when one of them is reallocated.

        plan = DecodePlan(q, k_cache, v_cache, cache_seqlens, block_table,
                          return_softmax_lse=True)
        out, lse = plan()          # on the current stream, or plan(stream)
    """

    def __init__(self, q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale=None,
                 return_softmax_lse=False, out=None, out_dtype=None, max_seqlen_k=None,
                 workspace=None, lse=None, causal=False, k=None, v=None, k_scale=None,
                 v_scale=None):
        self._call = _prepare(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                              return_softmax_lse, out, out_dtype, max_seqlen_k, workspace, lse,
                              causal, k, v, k_scale, v_scale)
        self._device = q.device
        self._keep = (q, k_cache, v_cache, cache_seqlens, block_table, workspace, k, v, k_scale,
                      v_scale)

    @property
    def out(self) -> torch.Tensor:
        return self._call.out

    @property
    def lse(self) -> torch.Tensor | None:
        return self._call.lse

    def __call__(self, stream: torch.cuda.Stream | None = None):
        c = self._call
        with _on_device(self._device):
            check(c.fn(*c.args, _stream_handle(stream, self._device)))
        return (c.out, c.lse) if c.return_lse else c.out


def _check_scales(k_scale, v_scale, Hkv: int) -> None:
    for name, sc in (("k_scale", k_scale), ("v_scale", v_scale)):
        if sc is None:
            raise ValueError(f"{name} [Hkv] fp32 is required with a float8_e4m3fn cache")
        _require_cuda(sc)
        if sc.dtype != torch.float32 or sc.shape != (Hkv,) or not sc.is_contiguous():
            raise ValueError(f"{name} must be a contiguous fp32 [{Hkv}] tensor")


def _check_new_kv(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, B: int,
                  new_dtype: torch.dtype | None = None) -> None:
    _require_cuda(k, v)
    if k.dim() != 4 or tuple(v.shape) != tuple(k.shape):
        raise ValueError("k and v must both be [B, seqlen_new, Hkv, D]")
    if k.shape[0] != B or k.shape[2] != k_cache.shape[2] or k.shape[3] != k_cache.shape[3]:
        raise ValueError("k / v shape does not match the batch and cache heads")
    want = k_cache.dtype if new_dtype is None else new_dtype
    if k.dtype != want or v.dtype != want:
        raise ValueError(f"k / v must be {want}")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("k and v must be contiguous")


def append_kv(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              cache_seqlens: torch.Tensor, block_table: torch.Tensor,
              stream: torch.cuda.Stream | None = None, k_scale: torch.Tensor | None = None,
              v_scale: torch.Tensor | None = None) -> None:
    """Write k / v [B, seqlen_new, Hkv, D] into the paged cache at positions
    cache_seqlens[b] + t (the cache update of flash_attn_with_kvcache).  For
    float8_e4m3fn caches k / v are 16-bit and stored as e4m3(x / scale[h])
    with the fp32 [Hkv] k_scale / v_scale."""
    lib = load_library()
    _require_cuda(k_cache, v_cache, cache_seqlens, block_table)
    if cache_seqlens.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("cache_seqlens and block_table must be int32")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous() and block_table.is_contiguous()):
        raise ValueError("caches and block_table must be contiguous")
    kv8 = k_cache.dtype == torch.float8_e4m3fn
    if (k_cache.dtype not in _DTYPES and not kv8) or v_cache.dtype != k_cache.dtype \
            or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError("k_cache/v_cache must be bf16, fp16 or float8_e4m3fn with equal shapes")
    B = block_table.shape[0]
    num_blocks, page, Hkv, D = k_cache.shape
    st = stream if stream is not None else torch.cuda.current_stream(k.device)
    if kv8:
        _check_scales(k_scale, v_scale, Hkv)
        if k.dtype not in _DTYPES:
            raise ValueError("k / v must be bf16 or fp16")
        _check_new_kv(k, v, k_cache, B, k.dtype)
        with torch.cuda.device(k.device):
            status = lib.fd_append_kv_paged_fp8(
                _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(k_scale), _ptr(v_scale),
                _ptr(cache_seqlens), _ptr(block_table), int(block_table.shape[1]), B, k.shape[1],
                Hkv, D, page, num_blocks, _DTYPES[k.dtype], st.cuda_stream)
        check(status)
        return
    _check_new_kv(k, v, k_cache, B)
    with torch.cuda.device(k.device):
        status = lib.fd_append_kv_paged(
            _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(cache_seqlens), _ptr(block_table),
            int(block_table.shape[1]), B, k.shape[1], Hkv, D, page, num_blocks, _DTYPES[k.dtype],
            st.cuda_stream)
    check(status)


def combine_lse(part_o: torch.Tensor, part_lse: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
                return_lse: bool = False, stream: torch.cuda.Stream | None = None):
    """Merge partial results over disjoint KV ranges.

    part_o [n, rows, D] fp32 (normalised), part_lse [n, rows] fp32 natural log.
    Each part must be contiguous; the parts themselves may be strided (views
    into one gathered buffer of per-part [O | LSE] blocks).
    Returns out [rows, D] (and lse [rows]).
    """
    lib = load_library()
    _require_cuda(part_o, part_lse)
    if part_o.dtype != torch.float32 or part_lse.dtype != torch.float32:
        raise ValueError("partials must be fp32")
    n, rows, D = part_o.shape
    if part_o.stride()[1:] != (D, 1):
        part_o = part_o.contiguous()
    if part_lse.stride(1) != 1:
        part_lse = part_lse.contiguous()
    out = torch.empty((rows, D), dtype=out_dtype, device=part_o.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=part_o.device) if return_lse else None
    st = stream if stream is not None else torch.cuda.current_stream(part_o.device)
    with torch.cuda.device(part_o.device):
        status = lib.fd_combine_lse(_ptr(part_o), part_o.stride(0), _ptr(part_lse), part_lse.stride(0),
                                    n, rows, D, _ptr(out), _OUT_DTYPES[out_dtype], _ptr(lse),
                                    st.cuda_stream)
    check(status)
    return (out, lse) if return_lse else out


__all__ = ["run_kernel", "flash_decode", "DecodePlan", "append_kv", "combine_lse", "last_error",
           "device_status", "workspace_size", "FlashDecodeError"]
