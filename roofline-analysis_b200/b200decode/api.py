"""Python host layer: the decodebench-facing decode() / decode_mla() calls.

Signatures follow the reference's closest call surface,
flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, block_table)
(decodebench/flashattn_kvcache_kernel.py:161-169), returning (out, lse) like
FA4's interface, and trtllm_batch_decode_with_kv_cache_mla for MLA
(decodebench/trtllm_mla_kernel.py:115-132).  Every call enqueues on the
current torch stream and never synchronises.  Errors surface as ValueError
(bad shapes/dtypes, as the reference adapters raise, e.g.
flashmla_kernel.py:45-46) or B2DError (a RuntimeError) for library codes.
"""
from __future__ import annotations

import ctypes as C
import threading
from typing import Optional, Tuple

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.B2D_BF16, torch.float16: _lib.B2D_FP16,
       torch.float8_e4m3fn: _lib.B2D_FP8_E4M3}


class B2DError(RuntimeError):
    def __init__(self, code: int, where: str):
        msg = _lib.load().b2d_error_string(code).decode()
        super().__init__(f"{where}: b2d status {code}: {msg}")
        self.code = code


def library_path() -> str:
    return str(_lib.LIB_PATH)


class DecodeWorkspace:
    """Caller-owned device scratch for split partials.  Its head is the
    library's workspace header (status word and split-merge arrival
    counters), which must be zero before first use: buffers are allocated
    with torch.zeros.  Grows on demand.

    The default workspaces are one per (device, stream): two decodes
    enqueued on different streams never share partials.  A workspace is
    allocated, and re-allocated when it grows, on the stream it serves, so
    torch's caching allocator recycles the old buffer only in that stream's
    order (after the last decode that read it)."""

    def __init__(self, device: torch.device, nbytes: int = 0, stream=None):
        self.device = torch.device(device)
        self.stream = stream
        self.buf = self._alloc(max(nbytes, 1 << 20))

    def _alloc(self, n: int) -> torch.Tensor:
        if self.stream is None:
            return torch.zeros(n, dtype=torch.uint8, device=self.device)
        with torch.cuda.stream(self.stream):
            return torch.zeros(n, dtype=torch.uint8, device=self.device)

    def ensure(self, nbytes: int) -> "DecodeWorkspace":
        if self.buf.numel() < nbytes:
            self.buf = self._alloc(int(nbytes * 1.25) + 4096)
        return self

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    @property
    def nbytes(self) -> int:
        return self.buf.numel()


_ws_lock = threading.Lock()
_ws: dict = {}


def _default_ws(device: torch.device, stream=None) -> DecodeWorkspace:
    """The default workspace of (device, stream); stream defaults to the
    device's current torch stream."""
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if stream is None:
        stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _ws_lock:
        if key not in _ws:
            _ws[key] = DecodeWorkspace(device, stream=stream)
        return _ws[key]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check(code: int, where: str) -> None:
    if code != 0:
        raise B2DError(code, where)


def _layout_strides(cache: torch.Tensor, kv_layout: str):
    """(stride_page, stride_tok, stride_head, page_size, num_kv_heads)."""
    if kv_layout == "NHD":   # [pages, P, Hkv, D]
        return cache.stride(0), cache.stride(1), cache.stride(2), cache.shape[1], cache.shape[2]
    if kv_layout == "HND":   # [pages, Hkv, P, D]
        return cache.stride(0), cache.stride(2), cache.stride(1), cache.shape[2], cache.shape[1]
    raise ValueError(f"kv_layout must be 'NHD' or 'HND', got {kv_layout!r}")


def _gqa_args(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, k_scale, v_scale,
              out, lse, kv_layout, num_ctas) -> _lib.GqaArgs:
    if q.dim() == 4:
        if q.shape[1] != 1:
            raise ValueError("decode takes one query token per sequence (q [B, 1, Hq, D])")
        q = q[:, 0]
    if q.dim() != 3:
        raise ValueError(f"q must be [B, Hq, D] or [B, 1, Hq, D], got {tuple(q.shape)}")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"q dtype must be bf16 or fp16, got {q.dtype}")
    vllm = kv_layout == "vllm"
    if vllm:
        # vLLM paged_attention (decodebench/vllm_paged_kernel.py:102-123):
        # K [blocks, Hkv, D/x, P, x] with x * elem = 16 bytes, V [blocks, Hkv, D, P]
        if k_cache.dim() != 5 or v_cache.dim() != 4:
            raise ValueError("kv_layout='vllm' takes K [blocks, Hkv, D/x, P, x] and V [blocks, Hkv, D, P]")
        nb, hkv_, dx, page_, x = k_cache.shape
        if x * k_cache.element_size() != 16 or tuple(v_cache.shape) != (nb, hkv_, dx * x, page_):
            raise ValueError("vLLM cache shapes do not match (x must be 16 bytes of elements)")
        if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
            raise ValueError("kv_layout='vllm' needs contiguous caches")
    elif k_cache.dim() != 4 or v_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache must be matching 4-D paged caches")
    if k_cache.dtype != v_cache.dtype or k_cache.dtype not in (q.dtype, torch.float8_e4m3fn):
        raise ValueError(f"cache dtype {k_cache.dtype} must equal q's {q.dtype} or be float8_e4m3fn")
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1 or v_cache.stride(-1) != 1:
        raise ValueError("the head_dim axis must be contiguous")
    for t, n in ((cache_seqlens, "cache_seqlens"), (block_table, "block_table")):
        if t.dtype != torch.int32:
            raise ValueError(f"{n} must be int32")
    if block_table.dim() != 2 or block_table.stride(1) != 1:
        raise ValueError("block_table must be [B, max_pages] with contiguous rows")
    bsz, hq, d = q.shape
    if vllm:
        ks_p, ks_t, ks_h, page, hkv = k_cache.stride(0), x, k_cache.stride(1), page_, hkv_
        vs_p, vs_t, vs_h = v_cache.stride(0), 1, v_cache.stride(1)
        if dx * x != d:
            raise ValueError("head_dim mismatch between q and the caches")
    else:
        ks_p, ks_t, ks_h, page, hkv = _layout_strides(k_cache, kv_layout)
        vs_p, vs_t, vs_h, _, _ = _layout_strides(v_cache, kv_layout)
        if k_cache.shape[-1] != d:
            raise ValueError("head_dim mismatch between q and the caches")
    if hq % hkv:
        raise ValueError(f"num_q_heads {hq} must be a multiple of num_kv_heads {hkv}")
    if cache_seqlens.shape != (bsz,) or block_table.shape[0] != bsz:
        raise ValueError("cache_seqlens / block_table batch mismatch")
    fp8 = k_cache.dtype == torch.float8_e4m3fn
    for s, n in ((k_scale, "k_scale"), (v_scale, "v_scale")):
        if s is not None and (s.dtype != torch.float32 or s.numel() != hkv):
            raise ValueError(f"{n} must be fp32 with num_kv_heads elements")
    a = _lib.GqaArgs()
    a.q, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.k_stride_page, a.k_stride_tok, a.k_stride_head = ks_p, ks_t, ks_h
    a.v_stride_page, a.v_stride_tok, a.v_stride_head = vs_p, vs_t, vs_h
    a.num_pages = k_cache.shape[0]
    a.cache_seqlens, a.block_table = cache_seqlens.data_ptr(), block_table.data_ptr()
    a.block_table_stride = block_table.stride(0)
    a.k_scale = _ptr(k_scale) if fp8 else None
    a.v_scale = _ptr(v_scale) if fp8 else None
    a.out, a.out_stride_b, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse = _ptr(lse)
    a.lse_stride_b = lse.stride(0) if lse is not None else 0
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = bsz, hq, hkv, d
    a.page_size, a.max_pages_per_seq = page, block_table.shape[1]
    a.q_dtype, a.kv_dtype = _DT[q.dtype], _DT[k_cache.dtype]
    a.softmax_scale = float(softmax_scale)
    a.num_ctas = int(num_ctas or 0)
    a.kv_layout = _lib.B2D_KV_VLLM if vllm else _lib.B2D_KV_STRIDED
    return a


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
           cache_seqlens: torch.Tensor, block_table: torch.Tensor,
           softmax_scale: Optional[float] = None, *, k_scale: Optional[torch.Tensor] = None,
           v_scale: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           lse: Optional[torch.Tensor] = None, kv_layout: str = "NHD",
           num_ctas: Optional[int] = None, workspace: Optional[DecodeWorkspace] = None,
           flags: int = 0, wait_limit_us: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Paged GQA/MHA/MQA decode for one query token per sequence.

    q: [B, Hq, D] or [B, 1, Hq, D] (bf16/fp16).  k_cache, v_cache:
    [num_pages, P, Hkv, D] ("NHD") or [num_pages, Hkv, P, D] ("HND"), in q's
    dtype or float8_e4m3fn with fp32 per-KV-head k_scale/v_scale; or vLLM's
    own layout ("vllm", 16-bit caches, P % 16 == 0): k_cache [blocks, Hkv,
    D/8, P, 8], v_cache [blocks, Hkv, D, P].
    cache_seqlens: int32 [B]; block_table: int32 [B, max_pages].
    softmax_scale defaults to 1/sqrt(D).  Returns out (shape of q, q's dtype)
    and lse [B, Hq] fp32 (natural log).  `flags` (B2D_FLAG_*) exists for
    timing the split-KV and combine kernels separately and for testing;
    `wait_limit_us` bounds every in-kernel wait (0 = the 2 s default).
    """
    if not q.is_cuda:
        raise RuntimeError("b200decode.decode needs CUDA tensors (there is no CPU path)")
    lib = _lib.load()
    q3 = q[:, 0] if q.dim() == 4 else q
    if softmax_scale is None:
        softmax_scale = q3.shape[-1] ** -0.5
    if out is None:
        out = torch.empty_like(q)
    out3 = out[:, 0] if out.dim() == 4 else out
    if lse is None:
        lse = torch.empty(q3.shape[0], q3.shape[1], dtype=torch.float32, device=q.device)
    a = _gqa_args(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale, k_scale,
                  v_scale, out3, lse, kv_layout, num_ctas)
    a.flags = int(flags)
    a.wait_limit_us = int(wait_limit_us)
    ws = workspace or _default_ws(q.device)
    need = C.c_size_t(0)
    _check(lib.b2d_gqa_workspace_bytes(C.byref(a), C.byref(need)), "b2d_gqa_workspace_bytes")
    ws.ensure(need.value)
    a.workspace, a.workspace_bytes = ws.ptr, ws.nbytes
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _check(lib.b2d_decode_gqa(C.byref(a), C.c_void_p(stream)), "b2d_decode_gqa")
    return out, lse


class GqaDecoder:
    """Plan once, run many times: the plan()/run() split of FlashInfer's
    BatchDecodeWithPagedKVCacheWrapper (decodebench/flashinfer_kernel.py:
    88-116), so a decode loop pays the argument checks and workspace sizing
    once.  Tensors are bound by address: refill q / cache_seqlens /
    block_table / the caches in place between runs (shapes fixed).

    run() enqueues one decode on the current stream and returns (out, lse).
    capture() records run() into a CUDA graph; replay() launches it.  The
    decoder's workspace is bound at construction (the default one of the
    stream current then): run it on that stream, or pass `workspace`.
    """

    def __init__(self, q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale=None, *,
                 k_scale=None, v_scale=None, out=None, lse=None, kv_layout="NHD",
                 num_ctas=None, workspace=None, flags=0):
        if not q.is_cuda:
            raise RuntimeError("GqaDecoder needs CUDA tensors (there is no CPU path)")
        self._lib = _lib.load()
        q3 = q[:, 0] if q.dim() == 4 else q
        if softmax_scale is None:
            softmax_scale = q3.shape[-1] ** -0.5
        self.out = torch.empty_like(q) if out is None else out
        out3 = self.out[:, 0] if self.out.dim() == 4 else self.out
        self.lse = (torch.empty(q3.shape[0], q3.shape[1], dtype=torch.float32, device=q.device)
                    if lse is None else lse)
        self._args = _gqa_args(q, k_cache, v_cache, cache_seqlens, block_table, softmax_scale,
                               k_scale, v_scale, out3, self.lse, kv_layout, num_ctas)
        self._args.flags = int(flags)
        self._keep = (q, k_cache, v_cache, cache_seqlens, block_table, k_scale, v_scale)
        self.ws = workspace or _default_ws(q.device)
        need = C.c_size_t(0)
        _check(self._lib.b2d_gqa_workspace_bytes(C.byref(self._args), C.byref(need)),
               "b2d_gqa_workspace_bytes")
        self.ws.ensure(need.value)
        self._ws_buf = self.ws.buf   # pin the buffer this plan points at
        self._args.workspace, self._args.workspace_bytes = self.ws.ptr, self.ws.nbytes
        self._argp = C.byref(self._args)
        self._fn = self._lib.b2d_decode_gqa
        self.device = q.device
        self._graph = None

    def run(self):
        rc = self._fn(self._argp, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        if rc:
            raise B2DError(rc, "b2d_decode_gqa")
        return self.out, self.lse

    def launches_per_run(self) -> int:
        """Kernel launches one run() enqueues (split-KV kernel, plus the
        combine kernel when the merge is not done in-kernel)."""
        n = C.c_int32(0)
        _check(self._lib.b2d_gqa_launch_count(self._argp, C.byref(n)), "b2d_gqa_launch_count")
        return n.value

    def capture(self):
        """Record one run() into a CUDA graph (after a warm-up run, which does
        the one-time per-device set-up outside the capture)."""
        self.run()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.run()
        self._graph = g
        return self

    def replay(self):
        self._graph.replay()
        return self.out, self.lse


def gqa_plan(q, k_cache, v_cache, cache_seqlens, block_table, kv_layout="NHD", num_ctas=None):
    """(num_ctas, chunk_tokens, kv_heads_per_cta) the kernel would use."""
    lib = _lib.load()
    q3 = q[:, 0] if q.dim() == 4 else q
    a = _gqa_args(q, k_cache, v_cache, cache_seqlens, block_table, 1.0, None, None, q3, None,
                  kv_layout, num_ctas)
    n, t, hk = C.c_int32(), C.c_int32(), C.c_int32()
    _check(lib.b2d_gqa_plan(C.byref(a), C.byref(n), C.byref(t), C.byref(hk)), "b2d_gqa_plan")
    return n.value, t.value, hk.value


def decode_mla(q: torch.Tensor, kv_cache: torch.Tensor, cache_seqlens: torch.Tensor,
               block_table: torch.Tensor, softmax_scale: Optional[float] = None, *,
               head_dim_v: int = 512, out: Optional[torch.Tensor] = None,
               lse: Optional[torch.Tensor] = None, num_ctas: Optional[int] = None,
               workspace: Optional[DecodeWorkspace] = None, flags: int = 0):
    """Absorbed-MLA decode: q [B, H, 576] (or [B, 1, H, 576]) bf16, kv_cache
    [num_pages, P, 576] (or [num_pages, P, 1, 576]) bf16.  Scores use all 576
    columns, V is the first head_dim_v.  softmax_scale defaults to 1/sqrt(192)
    (qk_nope 128 + qk_rope 64, decodebench/trtllm_mla_kernel.py:20-21).
    Returns out [B, H, head_dim_v] bf16 and lse [B, H] fp32."""
    if not q.is_cuda:
        raise RuntimeError("b200decode.decode_mla needs CUDA tensors (there is no CPU path)")
    lib = _lib.load()
    q3 = q[:, 0] if q.dim() == 4 else q
    kv = kv_cache[:, :, 0] if kv_cache.dim() == 4 else kv_cache
    if q3.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16:
        raise ValueError("decode_mla takes bf16 q and kv_cache")
    if kv.dim() != 3 or kv.shape[-1] != q3.shape[-1] or kv.stride(-1) != 1 or q3.stride(-1) != 1:
        raise ValueError("kv_cache must be [num_pages, P, D_qk] with contiguous rows")
    if cache_seqlens.dtype != torch.int32 or block_table.dtype != torch.int32:
        raise ValueError("cache_seqlens and block_table must be int32")
    if softmax_scale is None:
        softmax_scale = 192 ** -0.5
    bsz, h, dqk = q3.shape
    if out is None:
        out = torch.empty(bsz, h, head_dim_v, dtype=q3.dtype, device=q.device)
    if lse is None:
        lse = torch.empty(bsz, h, dtype=torch.float32, device=q.device)
    a = _lib.MlaArgs()
    a.q, a.q_stride_b, a.q_stride_h = q3.data_ptr(), q3.stride(0), q3.stride(1)
    a.kv_cache, a.kv_stride_page, a.kv_stride_tok = kv.data_ptr(), kv.stride(0), kv.stride(1)
    a.num_pages = kv.shape[0]
    a.cache_seqlens, a.block_table = cache_seqlens.data_ptr(), block_table.data_ptr()
    a.block_table_stride = block_table.stride(0)
    a.out, a.out_stride_b, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.lse_stride_b = lse.data_ptr(), lse.stride(0)
    a.batch, a.num_heads, a.head_dim_qk, a.head_dim_v = bsz, h, dqk, head_dim_v
    a.page_size, a.max_pages_per_seq = kv.shape[1], block_table.shape[1]
    a.dtype, a.softmax_scale = _lib.B2D_BF16, float(softmax_scale)
    a.num_ctas = int(num_ctas or 0)
    a.flags = int(flags)
    ws = workspace or _default_ws(q.device)
    need = C.c_size_t(0)
    _check(lib.b2d_mla_workspace_bytes(C.byref(a), C.byref(need)), "b2d_mla_workspace_bytes")
    ws.ensure(need.value)
    a.workspace, a.workspace_bytes = ws.ptr, ws.nbytes
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _check(lib.b2d_decode_mla(C.byref(a), C.c_void_p(stream)), "b2d_decode_mla")
    return out, lse


def append_kv(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
              slot_mapping: torch.Tensor, *, k_scale: Optional[torch.Tensor] = None,
              v_scale: Optional[torch.Tensor] = None, kv_layout: str = "NHD",
              bad_slots: Optional[torch.Tensor] = None) -> None:
    """Write new tokens' K/V rows into the paged caches (vLLM's
    reshape_and_cache, decodebench/vllm_paged_kernel.py:160-172).

    key, value: [T, Hkv, D] bf16/fp16; slot_mapping: int64 [T] with slot =
    page * P + offset (negative = skip).  Caches in the source dtype, or
    float8_e4m3fn: stored value = e4m3(x / scale[head]) (round-to-nearest-even,
    saturated).  kv_layout "NHD", "HND" or "vllm" (paged_attention's K
    [blocks, Hkv, D/8, P, 8] and V [blocks, Hkv, D, P], 16-bit caches).
    bad_slots: optional int32 [1] counter of out-of-range slots."""
    if not key.is_cuda:
        raise RuntimeError("append_kv needs CUDA tensors (there is no CPU path)")
    lib = _lib.load()
    if key.shape != value.shape or key.dim() != 3 or key.dtype != value.dtype:
        raise ValueError("key and value must be matching [T, Hkv, D] tensors")
    if key.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("key/value must be bf16 or fp16")
    if key.stride(-1) != 1 or value.stride() != key.stride():
        raise ValueError("key and value need the same strides and a contiguous head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (key.shape[0],):
        raise ValueError("slot_mapping must be int64 [T]")
    if k_cache.dtype != v_cache.dtype or k_cache.dtype not in (key.dtype, torch.float8_e4m3fn):
        raise ValueError("caches must be in the source dtype or float8_e4m3fn")
    vllm = kv_layout == "vllm"
    if vllm:   # K [blocks, Hkv, D/8, P, 8], V [blocks, Hkv, D, P] (16-bit caches)
        if (k_cache.dim() != 5 or v_cache.dim() != 4 or k_cache.shape[-1] * k_cache.element_size() != 16
                or not (k_cache.is_contiguous() and v_cache.is_contiguous())):
            raise ValueError("kv_layout='vllm' takes contiguous K [blocks, Hkv, D/x, P, x] and V [blocks, Hkv, D, P]")
        nb, hkv, dx, page, x = k_cache.shape
        if tuple(v_cache.shape) != (nb, hkv, dx * x, page) or dx * x != key.shape[2] or hkv != key.shape[1]:
            raise ValueError("vLLM cache shapes do not match key")
        ks_p, ks_t, ks_h = k_cache.stride(0), x, k_cache.stride(1)
        vs_p, vs_t, vs_h = v_cache.stride(0), 1, v_cache.stride(1)
    else:
        ks_p, ks_t, ks_h, page, hkv = _layout_strides(k_cache, kv_layout)
        vs_p, vs_t, vs_h, _, _ = _layout_strides(v_cache, kv_layout)
        if hkv != key.shape[1] or k_cache.shape[-1] != key.shape[2]:
            raise ValueError("cache heads / head_dim do not match key")
    a = _lib.AppendArgs()
    a.key, a.value = key.data_ptr(), value.data_ptr()
    a.src_stride_t, a.src_stride_h = key.stride(0), key.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.k_stride_page, a.k_stride_tok, a.k_stride_head = ks_p, ks_t, ks_h
    a.v_stride_page, a.v_stride_tok, a.v_stride_head = vs_p, vs_t, vs_h
    a.num_pages = k_cache.shape[0]
    a.slot_mapping = slot_mapping.data_ptr()
    fp8 = k_cache.dtype == torch.float8_e4m3fn
    a.k_scale = _ptr(k_scale) if fp8 else None
    a.v_scale = _ptr(v_scale) if fp8 else None
    a.bad_slots = _ptr(bad_slots)
    a.num_tokens, a.num_kv_heads, a.head_dim, a.page_size = key.shape[0], hkv, key.shape[2], page
    a.src_dtype, a.cache_dtype = _DT[key.dtype], _DT[k_cache.dtype]
    a.kv_layout = _lib.B2D_KV_VLLM if vllm else _lib.B2D_KV_STRIDED
    stream = torch.cuda.current_stream(key.device).cuda_stream
    _check(lib.b2d_append_kv(C.byref(a), C.c_void_p(stream)), "b2d_append_kv")


def check_device_status(workspace: Optional[DecodeWorkspace] = None, device=None,
                        clear: bool = True) -> None:
    """Synchronise and raise B2DError if a kernel recorded a timeout or an
    out-of-range page id in a workspace status word.  Without `workspace`,
    every default workspace of the device (one per stream used) is read."""
    lib = _lib.load()
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if workspace is not None:
        spaces = [workspace]
    else:
        _default_ws(device)   # at least the current stream's
        with _ws_lock:
            spaces = [w for (idx, _), w in _ws.items() if idx == device.index]
    stream = torch.cuda.current_stream(device).cuda_stream
    torch.cuda.synchronize(device)
    for ws in spaces:
        _check(lib.b2d_check_device_status(C.c_void_p(ws.ptr), int(clear), C.c_void_p(stream)),
               "device status")
