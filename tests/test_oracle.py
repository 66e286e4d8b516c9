"""The CPU oracle, pinned against the reference's own split-KV contract and
its decode call (fixtures made by tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import decode_ref as R

GOLD = Path(__file__).resolve().parent / "golden"


def test_split_merge_matches_reference_contract():
    z = np.load(GOLD / "split_merge_bh3_s129_d128.npz")
    q, k, v = (z[n].astype(np.float64) for n in ("q", "k", "v"))
    scale = float(z["scale"])
    assert int(z["payload_floats"]) == 128 + 2  # leader_reduce_payload_floats(128)
    for cs in (2, 4):
        m, l, o = R.split_partials(q[:, 0], k, v, cs, scale)
        np.testing.assert_allclose(m, z[f"m_{cs}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(l, z[f"l_{cs}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(o, z[f"o_{cs}"], rtol=1e-5, atol=1e-4)
        out, _ = R.merge_partials(m, l, o)
        np.testing.assert_allclose(out, z[f"merged_{cs}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(out, z[f"split_ref_{cs}"][:, 0], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(out, z["dense_out"][:, 0], rtol=1e-5, atol=1e-5)
    for i in range(q.shape[0]):
        o1, l1 = R.dense_decode(q[i], k[i:i + 1], v[i:i + 1], scale)
        np.testing.assert_allclose(o1[0], z["dense_out"][i, 0], rtol=1e-5, atol=1e-5)
        m, l, o = R.split_partials(q[i:i + 1, 0], k[i:i + 1], v[i:i + 1], 3, scale)
        _, lse = R.merge_partials(m, l, o)
        np.testing.assert_allclose(lse[0], l1[0], rtol=0, atol=1e-10)


def test_paged_oracle_matches_reference_sdpa_call():
    z = np.load(GOLD / "sdpa_paged_gqa.npz")
    q = R.bf16_bits_to_f64(z["q_bits"].view(np.uint16))
    k = R.bf16_bits_to_f64(z["k_bits"].view(np.uint16))
    v = R.bf16_bits_to_f64(z["v_bits"].view(np.uint16))
    out, lse = R.paged_decode(q, k, v, z["seqlens"], z["block_table"], float(z["scale"]))
    np.testing.assert_allclose(out, z["out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse, z["lse"], rtol=0, atol=1e-5)


def test_mla_oracle_matches_reference_sdpa_call():
    """The absorbed-MLA oracle against the fixture whose geometry (576-wide
    latent rows, V = first 512 columns, scale 1/sqrt(192)) comes from the
    reference's TRTLLMMLADecodeShape and whose answer is its SDPA call."""
    z = np.load(GOLD / "sdpa_paged_mla.npz")
    q = R.bf16_bits_to_f64(z["q_bits"].view(np.uint16))
    kv = R.bf16_bits_to_f64(z["kv_bits"].view(np.uint16))
    out, lse = R.paged_decode_mla(q, kv, z["seqlens"], z["block_table"], float(z["scale"]),
                                  head_dim_v=int(z["head_dim_v"]))
    np.testing.assert_allclose(out, z["out"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse, z["lse"], rtol=0, atol=1e-5)


def test_e4m3_table_matches_definition_and_torch():
    codes = np.arange(256, dtype=np.uint8)
    tab = R.e4m3_bits_to_f64(codes)
    t = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).to(torch.float64).numpy()
    fin = np.isfinite(t)
    assert np.array_equal(np.isnan(tab), np.isnan(t))
    np.testing.assert_array_equal(tab[fin], t[fin])
    assert np.nanmax(tab) == 448.0 and tab[1] == 2.0 ** -9
    x = np.random.default_rng(0).normal(size=4096) * 30
    bits = R.f64_to_e4m3_bits(x)
    tb = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(bits, tb)


def test_bf16_and_f16_bit_conversions():
    x = torch.randn(1000)
    for dt, fn in ((torch.bfloat16, R.bf16_bits_to_f64), (torch.float16, R.f16_bits_to_f64)):
        t = x.to(dt)
        bits = t.view(torch.int16).numpy().view(np.uint16)
        np.testing.assert_array_equal(fn(bits), t.double().numpy())


@pytest.mark.parametrize("lens", [[0, 1, 16, 17], [5], [31, 64]])
def test_paged_oracle_edges(lens):
    rng = np.random.default_rng(1)
    page, hq, hkv, d = 16, 4, 2, 64
    npg = [(l + page - 1) // page for l in lens]
    total = max(1, sum(npg))
    perm = rng.permutation(total)
    bt = np.zeros((len(lens), max(1, max(npg))), dtype=np.int32)
    off = 0
    for i, n in enumerate(npg):
        bt[i, :n] = perm[off:off + n]
        off += n
    q = rng.normal(size=(len(lens), hq, d))
    kc = rng.normal(size=(total, page, hkv, d))
    vc = rng.normal(size=(total, page, hkv, d))
    out, lse = R.paged_decode(q, kc, vc, np.array(lens), bt, 0.125)
    for b, l in enumerate(lens):
        if l == 0:
            assert np.all(out[b] == 0) and np.all(np.isneginf(lse[b]))
            continue
        k = R.gather_pages(kc, bt[b], l, page)
        v = R.gather_pages(vc, bt[b], l, page)
        kk = np.repeat(k, hq // hkv, axis=0)
        vv = np.repeat(v, hq // hkv, axis=0)
        for n in (1, 2, 4):   # any split count merges back to the unsplit result
            m, ll, o = R.split_partials(q[b], kk, vv, n, 0.125)
            mo, ml = R.merge_partials(m, ll, o)
            np.testing.assert_allclose(mo, out[b], rtol=1e-12, atol=1e-12)
            np.testing.assert_allclose(ml, lse[b], rtol=1e-12, atol=1e-12)


def test_sdpa_cpu_path_matches_oracle():
    from oracle.sdpa_cpu import gather_dense, sdpa_decode
    from b200decode import workloads as W
    w = W.CFG2_GQA_PAGED.scaled(batch=3, seqlen_lo=5, seqlen_hi=70)
    x = W.make_gqa_inputs(w, "cpu")
    dense = gather_dense(x["k_cache"], x["v_cache"], x["cache_seqlens"], x["block_table"],
                         dtype=torch.float32)
    out = sdpa_decode(x["q"].float(), dense, w.softmax_scale)
    f = lambda t: t.float().double().numpy()
    ref, _ = R.paged_decode(f(x["q"]), f(x["k_cache"]), f(x["v_cache"]),
                            x["cache_seqlens"].numpy(), x["block_table"].numpy(), w.softmax_scale)
    np.testing.assert_allclose(out.double().numpy(), ref, rtol=1e-4, atol=1e-5)


def test_fp8_workload_dequantises_to_unit_scale_values():
    """Config 5 stores e4m3(N(0,1)/scale): dequantised values are ~N(0,1)."""
    from b200decode import workloads as W
    from helpers import to_oracle
    x = W.make_gqa_inputs(W.CFG5_FP8.scaled(batch=2, seqlen_lo=64, seqlen_hi=64), "cpu")
    k = to_oracle(x["k_cache"]) * x["k_scale"].double().numpy()[None, None, :, None]
    assert 0.9 < k.std() < 1.1
    assert float(x["k_scale"].min()) >= 0.01 and float(x["k_scale"].max()) <= 0.1


def test_append_oracle_quantises_like_torch_and_skips_slots():
    rng = np.random.default_rng(3)
    cache = np.zeros((4, 16, 2, 64), dtype=np.uint8)
    rows = rng.normal(size=(5, 2, 64)).astype(np.float32) * 3
    scale = np.array([0.05, 0.2], dtype=np.float32)
    slots = np.array([0, 17, -1, 63, 64])
    bad = R.append_kv(cache, rows, slots, 16, scale, fp8=True)
    assert bad == 1
    want = (torch.from_numpy(rows) * (1 / torch.from_numpy(scale))[None, :, None]).to(
        torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(cache[0, 0], want[0])
    np.testing.assert_array_equal(cache[1, 1], want[1])
    np.testing.assert_array_equal(cache[3, 15], want[3])
    assert not cache[0, 2].any()   # slot 2 untouched by the skipped token


def test_e4m3_rounding_corners():
    """Round-to-nearest-even at exact midpoints, subnormals and signed zero
    match torch's float8_e4m3fn cast; magnitudes beyond 448 saturate to 448
    (the append kernel's satfinite conversion)."""
    pos = np.unique(R.E4M3_TABLE[np.isfinite(R.E4M3_TABLE) & (R.E4M3_TABLE >= 0)])
    mids = (pos[:-1] + pos[1:]) / 2                       # exact ties
    sub = np.linspace(2.0 ** -10, 2.0 ** -6, 97)          # subnormal range and its edge
    x = np.concatenate([mids, -mids, sub, -sub, [0.0, -0.0, 447.9, -447.9]])
    bits = R.f64_to_e4m3_bits(x)
    tb = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(bits, tb)
    # every tie went to the even code (last mantissa bit 0)
    assert not (R.f64_to_e4m3_bits(mids) & 1).any()
    sat = R.f64_to_e4m3_bits(np.array([448.0, 449.0, 1e4, -1e4]))
    np.testing.assert_array_equal(R.e4m3_bits_to_f64(sat), [448.0, 448.0, 448.0, -448.0])


def test_streamed_oracle_matches_whole_cache_oracle():
    """The chunked oracle used on full-size caches (only the pages a chunk of
    sequences uses, renumbered) gives the same result as the oracle over the
    whole cache, including a zero-length sequence."""
    import torch
    from b200decode import workloads as W
    from helpers import oracle_gqa, oracle_gqa_streamed
    w = W.CFG5_FP8.scaled(batch=7, seqlen_lo=0, seqlen_hi=300, seed=4)
    sl = torch.tensor([0, 1, 16, 17, 299, 150, 3])
    x = W.make_gqa_inputs(w, "cpu", seqlens=sl)
    o1, l1 = oracle_gqa(x)
    o2, l2 = oracle_gqa_streamed(x, chunk=3)
    np.testing.assert_array_equal(o1, o2)
    np.testing.assert_array_equal(l1, l2)
