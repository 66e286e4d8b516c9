"""b2d_decode_gqa_static_scratch — the decode entry point for callers that
cannot allocate device memory (an inference plugin whose enqueue step may not
allocate, a serving loop that reserved all free HBM for its KV cache), so
cannot hand the library a workspace.  It keeps its scratch in a fixed 16 MiB
device array inside the library.

Called here through the C ABI (ctypes, b2d_gqa_args) and compared with the
regular b2d_decode_gqa on two calls in a row with different inputs, so a
result that depended on what the previous call left in the shared array
would show.  This file is named to be collected last."""
import ctypes as C

import pytest
import torch

import b200decode
from b200decode import _lib
from b200decode import workloads as W
from b200decode.api import _default_ws, _gqa_args
from helpers import LSE_ATOL, OUT_ATOL, OUT_RTOL

pytestmark = pytest.mark.gpu


def _args_for(x, out, lse):
    return _gqa_args(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"], x["block_table"],
                     x["softmax_scale"], x["k_scale"], x["v_scale"], out, lse, "NHD", None)


def _close(a, b, atol, rtol):
    a, b = a.float(), b.float()
    return bool(((a - b).abs() <= atol + rtol * b.abs()).all())


def test_static_scratch_matches_regular_entry_point(cuda):
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    cases = [
        W.CFG2_GQA_PAGED.scaled(batch=16, seed=11),                      # split rows + combine
        W.CFG5_FP8.scaled(batch=8, seqlen_lo=1, seqlen_hi=3000, seed=12),  # different shape/dtype
    ]
    for w in cases:
        x = W.make_gqa_inputs(w, cuda)
        ref_out, ref_lse = b200decode.decode(x["q"], x["k_cache"], x["v_cache"],
                                             x["cache_seqlens"], x["block_table"],
                                             x["softmax_scale"], k_scale=x["k_scale"],
                                             v_scale=x["v_scale"])
        out = torch.full_like(x["q"], float("nan"))
        lse = torch.full(ref_lse.shape, float("nan"), device=cuda)
        a = _args_for(x, out, lse)
        rc = lib.b2d_decode_gqa_static_scratch(C.byref(a), stream)
        assert rc == 0, lib.b2d_error_string(rc)
        torch.cuda.synchronize()
        assert _close(out, ref_out, OUT_ATOL, OUT_RTOL)
        assert _close(lse, ref_lse, LSE_ATOL, 0.0)
        # nothing went wrong on the device during the call
        assert lib.b2d_static_scratch_check_status(1, stream) == 0


def test_static_scratch_reports_device_errors(cuda):
    """A block-table entry out of range is clamped to page 0 by the kernel
    and recorded in the scratch array's status word; the static-scratch
    status call reports it once, clears it, and the next call is clean."""
    lib = _lib.load()
    stream = C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    x = W.make_gqa_inputs(W.CFG2_GQA_PAGED.scaled(batch=4, seqlen_lo=40, seqlen_hi=200, seed=13),
                          cuda)
    out = torch.empty_like(x["q"])
    lse = torch.empty(x["q"].shape[:2], dtype=torch.float32, device=cuda)
    good = x["block_table"].clone()
    x["block_table"][1, 0] = x["k_cache"].shape[0] + 5
    a = _args_for(x, out, lse)
    assert lib.b2d_decode_gqa_static_scratch(C.byref(a), stream) == 0
    assert lib.b2d_static_scratch_check_status(1, stream) == -7   # B2D_ERR_DEVICE_BOUNDS
    assert lib.b2d_static_scratch_check_status(1, stream) == 0    # cleared
    x["block_table"].copy_(good)
    assert lib.b2d_decode_gqa_static_scratch(C.byref(a), stream) == 0
    assert lib.b2d_static_scratch_check_status(1, stream) == 0


def test_static_scratch_rejects_too_large(cuda):
    lib = _lib.load()
    # 4096 sequences x 32 heads x 129 floats of partials is far above 16 MiB
    a = _lib.GqaArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = 2048, 32, 8, 128
    a.page_size, a.max_pages_per_seq = 16, 8
    a.q_dtype = a.kv_dtype = _lib.B2D_BF16
    a.num_ctas = 296
    n = C.c_size_t(0)
    assert lib.b2d_gqa_workspace_bytes(C.byref(a), C.byref(n)) == 0 and n.value > 16 << 20
    assert lib.b2d_decode_gqa_static_scratch(C.byref(a), None) == -8  # B2D_ERR_TOO_LARGE
