"""GPU parity of the KV-cache append kernel (b2d_append_kv) against the CPU
oracle, bit for bit, plus an append -> decode round trip."""
import numpy as np
import pytest
import torch

import b200decode
from b200decode import workloads as W
from helpers import assert_parity, oracle_gqa, to_oracle
from oracle import decode_ref as R

pytestmark = pytest.mark.gpu


def _plus_zero(codes: np.ndarray) -> np.ndarray:
    """e4m3 codes with -0 (0x80) written as +0 (0x00)."""
    return np.where(codes == 0x80, 0, codes).astype(np.uint8)


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_append_matches_oracle(cuda, fp8, layout):
    g = torch.Generator(device=cuda).manual_seed(0)
    T, H, D, P, pages = 37, 4, 128, 16, 8
    key = (torch.randn(T, H, D, generator=g, device=cuda) * 2).to(torch.bfloat16)
    val = (torch.randn(T, H, D, generator=g, device=cuda) * 2).to(torch.bfloat16)
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    shape = (pages, P, H, D) if layout == "NHD" else (pages, H, P, D)
    kc = torch.zeros(shape, dtype=dt, device=cuda)
    vc = torch.zeros(shape, dtype=dt, device=cuda)
    slots = torch.randperm(pages * P, generator=torch.Generator().manual_seed(1))[:T].to(cuda)
    slots[3] = -1
    slots[5] = pages * P + 4          # out of range: skipped and counted
    ks = torch.tensor([0.02, 0.05, 0.1, 0.5], device=cuda) if fp8 else None
    vs = torch.tensor([0.03, 0.07, 0.2, 1.0], device=cuda) if fp8 else None
    bad = torch.zeros(1, dtype=torch.int32, device=cuda)
    b200decode.append_kv(key, val, kc, vc, slots, k_scale=ks, v_scale=vs, kv_layout=layout,
                         bad_slots=bad)
    torch.cuda.synchronize()
    assert int(bad.item()) == 1
    for cache, src, sc in ((kc, key, ks), (vc, val, vs)):
        got = cache if layout == "NHD" else cache.permute(0, 2, 1, 3)
        got = got.contiguous()
        ref = np.zeros(tuple(got.shape), dtype=np.uint8 if fp8 else np.float64)
        R.append_kv(ref, to_oracle(src).astype(np.float32), slots.cpu().numpy(), P,
                    None if sc is None else sc.cpu().numpy(), fp8=fp8)
        if fp8:
            # bit for bit, up to the sign of zero (0x80 vs 0x00: both decode to 0)
            np.testing.assert_array_equal(_plus_zero(got.view(torch.uint8).cpu().numpy()),
                                          _plus_zero(ref))
        else:
            np.testing.assert_array_equal(to_oracle(got), ref)


def test_append_then_decode_round_trip(cuda):
    """Filling an FP8 cache token by token through append_kv gives the same
    decode as the cache the workload generator quantised directly."""
    w = W.CFG5_FP8.scaled(batch=3, seqlen_lo=20, seqlen_hi=90)
    x = W.make_gqa_inputs(w, cuda)
    page = w.page_size
    kc = torch.zeros_like(x["k_cache"])
    vc = torch.zeros_like(x["v_cache"])
    for b in range(w.batch):
        L = int(x["cache_seqlens"][b])
        pages = x["block_table"][b, : (L + page - 1) // page].long()
        slots = (pages[:, None] * page + torch.arange(page, device=cuda)[None]).reshape(-1)[:L]
        # dequantised source rows (exactly representable: the append re-quantises them)
        krow = (x["k_cache"][pages].reshape(-1, w.num_kv_heads, w.head_dim)[:L].float()
                * x["k_scale"][None, :, None]).to(torch.bfloat16)
        vrow = (x["v_cache"][pages].reshape(-1, w.num_kv_heads, w.head_dim)[:L].float()
                * x["v_scale"][None, :, None]).to(torch.bfloat16)
        b200decode.append_kv(krow, vrow, kc, vc, slots.to(torch.int64), k_scale=x["k_scale"],
                             v_scale=x["v_scale"])
    torch.cuda.synchronize()
    y = dict(x, k_cache=kc, v_cache=vc)
    out, lse = b200decode.decode(y["q"], kc, vc, y["cache_seqlens"], y["block_table"],
                                 y["softmax_scale"], k_scale=y["k_scale"], v_scale=y["v_scale"])
    torch.cuda.synchronize()
    assert_parity(out, lse, *oracle_gqa(y))
    ref_out, ref_lse = b200decode.decode(x["q"], x["k_cache"], x["v_cache"], x["cache_seqlens"],
                                         x["block_table"], x["softmax_scale"], k_scale=x["k_scale"],
                                         v_scale=x["v_scale"])
    torch.cuda.synchronize()
    assert (out.float() - ref_out.float()).abs().max().item() < 2e-2


def test_append_vllm_layout_bit_exact_and_round_trip(cuda):
    """reshape_and_cache into vLLM paged_attention's own layout (K [blocks,
    Hkv, D/8, P, 8], V [blocks, Hkv, D, P]) writes the same values as the NHD
    oracle, and decoding those caches with kv_layout="vllm" matches."""
    g = torch.Generator(device=cuda).manual_seed(2)
    T, H, D, P, pages = 45, 2, 128, 16, 6
    key = torch.randn(T, H, D, generator=g, device=cuda).to(torch.bfloat16)
    val = torch.randn(T, H, D, generator=g, device=cuda).to(torch.bfloat16)
    kc = torch.zeros(pages, H, D // 8, P, 8, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros(pages, H, D, P, dtype=torch.bfloat16, device=cuda)
    slots = torch.randperm(pages * P, generator=torch.Generator().manual_seed(3))[:T].to(cuda)
    slots[7] = -1
    b200decode.append_kv(key, val, kc, vc, slots, kv_layout="vllm")
    torch.cuda.synchronize()
    k_nhd = kc.permute(0, 3, 1, 2, 4).reshape(pages, P, H, D)
    v_nhd = vc.permute(0, 3, 1, 2)
    for got, src in ((k_nhd, key), (v_nhd, val)):
        ref = np.zeros((pages, P, H, D))
        R.append_kv(ref, to_oracle(src).astype(np.float32), slots.cpu().numpy(), P)
        np.testing.assert_array_equal(to_oracle(got.contiguous()), ref)
    # decode one sequence over every written slot, in slot order
    used = torch.sort(slots[slots >= 0]).values
    L = int(used.numel())
    bt_pages = torch.unique(used // P)
    assert bt_pages.numel() <= pages
    # a sequence whose pages are all pages (identity), length = pages * P,
    # with unwritten slots zero: decode both layouts and compare
    q = torch.randn(1, 4 * H, D, generator=g, device=cuda).to(torch.bfloat16)
    bt = torch.arange(pages, dtype=torch.int32, device=cuda)[None]
    sl = torch.tensor([pages * P], dtype=torch.int32, device=cuda)
    o1, l1 = b200decode.decode(q, kc, vc, sl, bt, kv_layout="vllm")
    o2, l2 = b200decode.decode(q, k_nhd.contiguous(), v_nhd.contiguous(), sl, bt)
    torch.cuda.synchronize()
    assert L == T - 1
    torch.testing.assert_close(o1.float(), o2.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(l1, l2, atol=1e-3, rtol=0)
