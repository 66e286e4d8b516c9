"""The C-ABI library: loads, exports every declared symbol, validates
arguments on the host (no GPU needed for any call made here)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from b200decode import _lib

REPO = Path(__file__).resolve().parent.parent


def _declared():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        names |= set(re.findall(r"\b(b2d_[a-z0-9_]+)\s*\(", h.read_text()))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (b2d_\w+)", out))
    assert declared <= exported, f"missing: {declared - exported}"
    for name in declared:
        assert hasattr(lib, name)
    assert set(_lib.EXPORTED) <= declared


def test_error_strings_and_version():
    lib = _lib.load()
    assert lib.b2d_error_string(0) == b"ok"
    for code in range(-1, -9, -1):
        assert lib.b2d_error_string(code) != b"unknown b2d status"
    assert b"sm_100a" in lib.b2d_version()


def _args(**kw):
    a = _lib.GqaArgs()
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = 64, 32, 8, 128
    a.page_size, a.max_pages_per_seq = 16, 512
    a.q_dtype, a.kv_dtype = _lib.B2D_BF16, _lib.B2D_BF16
    a.num_ctas = 296
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_query_and_plan_on_host():
    lib = _lib.load()
    n = C.c_size_t(0)
    assert lib.b2d_gqa_workspace_bytes(C.byref(_args()), C.byref(n)) == 0
    nc, t, hk = C.c_int32(), C.c_int32(), C.c_int32()
    assert lib.b2d_gqa_plan(C.byref(_args()), C.byref(nc), C.byref(t), C.byref(hk)) == 0
    # status + row table + (rows + ctas) * (query heads per row) * (D + 1) floats
    rows, heads_per_row = 64 * (8 // hk.value), 4 * hk.value
    assert n.value >= (rows + 296) * heads_per_row * 129 * 4
    assert nc.value == 296 and 16 % t.value == 0 and 8 % hk.value == 0
    # page size 48: chunks still divide a page
    assert lib.b2d_gqa_plan(C.byref(_args(page_size=48)), C.byref(nc), C.byref(t), C.byref(hk)) == 0
    assert 48 % t.value == 0
    # GQA group 8 and MQA group 32 are planned too
    for hq in (64, 8 * 32):
        assert lib.b2d_gqa_plan(C.byref(_args(num_q_heads=hq)), C.byref(nc), C.byref(t),
                                C.byref(hk)) == 0


def test_tile_width_plan():
    """KV heads per tile: whole token rows (8 heads) for 16-bit caches, 4 for
    fp8, narrower when the block table bounds the problem to fewer chunks
    than about two per CTA (host-only plan, no GPU)."""
    lib = _lib.load()
    nc, t, hk = C.c_int32(), C.c_int32(), C.c_int32()

    def plan(**kw):
        assert lib.b2d_gqa_plan(C.byref(_args(**kw)), C.byref(nc), C.byref(t), C.byref(hk)) == 0
        return hk.value

    assert plan() == 8                                      # B=64 x 8192 tokens, bf16
    assert plan(kv_dtype=_lib.B2D_FP8_E4M3) == 4
    small = plan(batch=1, max_pages_per_seq=256)            # B=1, 4096 tokens
    assert small < 8 and 8 % small == 0
    assert plan(batch=1, max_pages_per_seq=8192) == 8       # B=1, 128k tokens: plenty of chunks


@pytest.mark.parametrize("kw,code", [
    (dict(head_dim=96), -2),                 # unsupported head_dim
    (dict(head_dim=192, kv_dtype=_lib.B2D_FP8_E4M3), -2),  # fp8 needs head_dim % 128 == 0
    (dict(head_dim=192, page_size=8), -2),   # 192 only on the tensor-core path (page % 16)
    (dict(kv_layout=_lib.B2D_KV_VLLM, kv_dtype=_lib.B2D_FP8_E4M3), -2),  # vLLM layout: 16-bit
    (dict(kv_layout=_lib.B2D_KV_VLLM, page_size=8), -2),                # ... and page % 16
    (dict(kv_layout=7), -1),                 # unknown layout
    (dict(num_q_heads=30), -1),              # not a multiple of num_kv_heads
    (dict(q_dtype=_lib.B2D_FP8_E4M3), -2),   # q must be 16-bit
    (dict(kv_dtype=_lib.B2D_FP16), -2),      # cache must match q or be fp8
    (dict(num_q_heads=8 * 64), -2),          # group 64 not built
    (dict(page_size=0), -1),
])
def test_host_validation_rejects(kw, code):
    lib = _lib.load()
    n = C.c_size_t(0)
    assert lib.b2d_gqa_workspace_bytes(C.byref(_args(**kw)), C.byref(n)) == code


def test_head_dim_192_is_planned_for_16bit_caches():
    lib = _lib.load()
    n = C.c_size_t(0)
    for page in (16, 64):
        assert lib.b2d_gqa_workspace_bytes(C.byref(_args(head_dim=192, page_size=page)),
                                           C.byref(n)) == 0
        assert n.value > 0


def test_decode_rejects_null_pointers_before_touching_a_gpu():
    lib = _lib.load()
    assert lib.b2d_decode_gqa(C.byref(_args()), None) == -1
    assert lib.b2d_decode_gqa(None, None) == -1
    assert lib.b2d_decode_gqa(C.byref(_args(batch=0)), None) == 0  # no-op


def test_python_layer_refuses_cpu_tensors():
    import torch
    import b200decode
    q = torch.zeros(1, 4, 64, dtype=torch.bfloat16)
    kc = torch.zeros(1, 16, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        b200decode.decode(q, kc, kc, torch.ones(1, dtype=torch.int32),
                          torch.zeros(1, 1, dtype=torch.int32))


def _mla_args(**kw):
    a = _lib.MlaArgs()
    a.batch, a.num_heads, a.head_dim_qk, a.head_dim_v = 128, 128, 576, 512
    a.page_size, a.max_pages_per_seq, a.dtype = 64, 256, _lib.B2D_BF16
    a.num_ctas = 148
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_mla_workspace_and_validation_on_host():
    """Workspace sizing and argument checks of the MLA entry points run on the
    host (no GPU): partials for (rows + CTA pairs) segments x 128 heads x 512."""
    lib = _lib.load()
    n = C.c_size_t(0)
    assert lib.b2d_mla_workspace_bytes(C.byref(_mla_args()), C.byref(n)) == 0
    assert n.value >= (128 + 74) * 128 * 512 * 4
    for kw, code in ((dict(num_heads=64), -2), (dict(head_dim_qk=512), -2),
                     (dict(dtype=_lib.B2D_FP16), -2), (dict(page_size=16), -2),
                     (dict(page_size=0), -1), (dict(batch=-1), -1)):
        assert lib.b2d_mla_workspace_bytes(C.byref(_mla_args(**kw)), C.byref(n)) == code, kw
    assert lib.b2d_decode_mla(C.byref(_mla_args()), None) == -1      # null pointers
    assert lib.b2d_decode_mla(C.byref(_mla_args(batch=0)), None) == 0  # nothing to do


def test_append_validation_on_host():
    lib = _lib.load()
    a = _lib.AppendArgs()
    a.num_tokens, a.num_kv_heads, a.head_dim, a.page_size = 4, 8, 128, 16
    a.src_dtype, a.cache_dtype = _lib.B2D_BF16, _lib.B2D_BF16
    assert lib.b2d_append_kv(C.byref(a), None) == -1                  # null pointers
    a.head_dim = 96
    assert lib.b2d_append_kv(C.byref(a), None) == -2                  # head_dim not built
    a.head_dim, a.cache_dtype = 128, _lib.B2D_FP16
    assert lib.b2d_append_kv(C.byref(a), None) == -2                  # cache must match or be fp8
    a.cache_dtype, a.kv_layout = _lib.B2D_FP8_E4M3, _lib.B2D_KV_VLLM
    assert lib.b2d_append_kv(C.byref(a), None) == -2                  # vLLM layout: 16-bit only
    a.kv_layout, a.num_tokens = _lib.B2D_KV_STRIDED, 0
    assert lib.b2d_append_kv(C.byref(a), None) == 0                   # nothing to append


def test_header_is_plain_c_and_links(tmp_path):
    """include/b2d_decode.h compiles as C99 (what cgo / JNI / other FFI hosts
    include) and a C program links against libb2d.so and calls host-only
    entry points."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    src = tmp_path / "probe.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "b2d_decode.h"
int main(void) {
  b2d_gqa_args a;
  size_t n = 0;
  int32_t ctas = 0, t = 0, hk = 0;
  memset(&a, 0, sizeof a);
  a.batch = 64; a.num_q_heads = 32; a.num_kv_heads = 8; a.head_dim = 128;
  a.page_size = 16; a.max_pages_per_seq = 512; a.q_dtype = B2D_BF16; a.kv_dtype = B2D_BF16;
  a.num_ctas = 296; a.kv_layout = B2D_KV_STRIDED;
  if (b2d_gqa_workspace_bytes(&a, &n) != B2D_OK || n == 0) return 1;
  if (b2d_gqa_plan(&a, &ctas, &t, &hk) != B2D_OK || ctas != 296) return 2;
  if (b2d_decode_gqa(&a, NULL) != B2D_ERR_INVALID_ARG) return 3;   /* null pointers */
  printf("%s %s\n", b2d_version(), b2d_error_string(B2D_ERR_UNSUPPORTED));
  return 0;
}
''')
    lib = _lib.LIB_PATH
    exe = tmp_path / "probe"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{REPO / 'include'}", str(src),
                        f"-L{lib.parent}", "-lb2d", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stderr)
    assert "sm_100a" in r.stdout
