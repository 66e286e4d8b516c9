"""The reference's own decode entry points (cluster_decode_forward /
cluster_decode_split_forward, cute_attention/cluster_decode/) served by this
library: same config record, same input checks and messages, and outputs
matching the CPU oracle."""
import numpy as np
import pytest
import torch

from b200decode import cluster_decode as CD
from helpers import assert_parity, to_oracle
from oracle import decode_ref as R


def _qkv(b, h, s, d=128, dtype=torch.bfloat16, device="cpu", seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(b, h, 1, d, generator=g).to(dtype).to(device)
    k = torch.randn(b, h, s, d, generator=g).to(dtype).to(device)
    v = torch.randn(b, h, s, d, generator=g).to(dtype).to(device)
    return q, k, v


@pytest.mark.parametrize("mutate,msg", [
    (lambda q, k, v: (q[0], k, v), "Expected q, k, v to have shape"),
    (lambda q, k, v: (q, k[:1], v), "same batch size"),
    (lambda q, k, v: (q, k[:, :1], v[:, :1]), "only supports MHA"),
    (lambda q, k, v: (q.expand(-1, -1, 2, -1), k, v), "q_len=1"),
    (lambda q, k, v: (q[..., :64], k[..., :64], v), "same head_dim"),
    (lambda q, k, v: (q[..., :64], k[..., :64], v[..., :64]), "head_dim=128"),
    (lambda q, k, v: (q, k, v), "CUDA tensors only"),
])
def test_checks_and_messages_match_the_reference(mutate, msg):
    q, k, v = _qkv(2, 4, 20)
    with pytest.raises(ValueError, match=msg):
        CD.cluster_decode_forward(*mutate(q, k, v))


def test_config_record():
    c = CD.ClusterDecodeConfig()
    assert (c.softmax_scale, c.num_threads, c.cluster_size) == (None, 128, 2)
    assert abs(c.resolve_scale(128) - 128 ** -0.5) < 1e-12
    assert CD.ClusterDecodeConfig(softmax_scale=0.3).resolve_scale(128) == 0.3
    q, k, v = _qkv(1, 2, 8)
    with pytest.raises(ValueError, match="cluster_size 2 or 4"):
        CD.cluster_decode_forward(q, k, v, CD.ClusterDecodeConfig(cluster_size=3))


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,s,dtype", [(2, 4, 300, torch.bfloat16), (3, 8, 512, torch.float16),
                                         (1, 16, 2048, torch.float16), (4, 2, 17, torch.bfloat16)])
@pytest.mark.parametrize("fn", ["cluster_decode_forward", "cluster_decode_split_forward"])
def test_outputs_match_oracle(cuda, b, h, s, dtype, fn):
    q, k, v = _qkv(b, h, s, dtype=dtype, device=cuda, seed=s)
    cfg = CD.ClusterDecodeConfig(softmax_scale=0.07 if s == 17 else None)
    o = getattr(CD, fn)(q, k, v, cfg)
    torch.cuda.synchronize()
    assert o.shape == (b, h, 1, 128) and o.dtype == dtype
    scale = cfg.resolve_scale(128)
    ref = np.stack([R.dense_decode(to_oracle(q[i, :, 0]), to_oracle(k[i]), to_oracle(v[i]), scale)[0]
                    for i in range(b)])
    err = np.abs(to_oracle(o[:, :, 0]) - ref)
    assert (err <= 2e-2 + 1e-2 * np.abs(ref)).all(), err.max()
