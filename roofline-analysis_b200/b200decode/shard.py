"""Multi-GPU decode: one process per GPU, torch.distributed (NCCL) plumbing.

The reference has no multi-GPU code (decodebench runs one process on one
GPU).  Decode shards without any data-path exchange in two ways:

* DP (batch-sharded): rank r owns a subset of the sequences, together with
  their pages and block-table rows.  Sequences are assigned greedily,
  longest first, to the least-loaded rank, because uniform-random lengths
  make a plain B/N cut unbalanced.  No collective runs inside a step.
* TP (KV-head-sharded): rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and the
  matching query heads of every sequence.  After the local decode one NCCL
  all_gather_into_tensor of a packed (out, lse) buffer assembles the full
  heads (HeadGather; gather_heads is the allocating one-off form).

The helpers that decide placement are pure functions (tested on CPU); the
gather needs an initialised process group (NCCL on GPUs, gloo on CPU tests).
"""
from __future__ import annotations

from typing import List, Sequence

import torch
import torch.distributed as dist


def balance_sequences(seqlens: Sequence[int], world: int) -> List[List[int]]:
    """Greedy longest-processing-time assignment of sequences to ranks.
    Returns per-rank sorted index lists (every index exactly once)."""
    order = sorted(range(len(seqlens)), key=lambda i: (-int(seqlens[i]), i))
    load = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        out[r].append(i)
        load[r] += int(seqlens[i])
    return [sorted(x) for x in out]


def head_shard(num_q_heads: int, num_kv_heads: int, world: int, rank: int):
    """(q_head_slice, kv_head_slice) rank `rank` owns under TP."""
    if num_kv_heads % world:
        raise ValueError(f"num_kv_heads {num_kv_heads} not divisible by world size {world}")
    kv_per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    kv = slice(rank * kv_per, (rank + 1) * kv_per)
    return slice(kv.start * g, kv.stop * g), kv


def gather_heads(out_local: torch.Tensor, lse_local: torch.Tensor, group=None):
    """All-gather head-sharded [B, Hq/N, D] outputs and [B, Hq/N] lse into
    full [B, Hq, D] / [B, Hq] (rank order = head order)."""
    world = dist.get_world_size(group)
    b, hl, d = out_local.shape
    buf_o = torch.empty(world * b, hl, d, dtype=out_local.dtype, device=out_local.device)
    buf_l = torch.empty(world * b, hl, dtype=lse_local.dtype, device=lse_local.device)
    dist.all_gather_into_tensor(buf_o, out_local.contiguous(), group=group)
    dist.all_gather_into_tensor(buf_l, lse_local.contiguous(), group=group)
    out = buf_o.view(world, b, hl, d).permute(1, 0, 2, 3).reshape(b, world * hl, d)
    lse = buf_l.view(world, b, hl).permute(1, 0, 2).reshape(b, world * hl)
    return out, lse


def slice_gqa_inputs_by_heads(x: dict, world: int, rank: int) -> dict:
    """TP: keep this rank's KV heads (cache copies) and query heads."""
    hq, hkv = x["q"].shape[1], x["k_cache"].shape[2]
    qs, ks = head_shard(hq, hkv, world, rank)
    y = dict(x)
    y["q"] = x["q"][:, qs].contiguous()
    y["k_cache"] = x["k_cache"][:, :, ks].contiguous()
    y["v_cache"] = x["v_cache"][:, :, ks].contiguous()
    if x.get("k_scale") is not None:
        y["k_scale"] = x["k_scale"][ks].contiguous()
        y["v_scale"] = x["v_scale"][ks].contiguous()
    return y


def slice_gqa_inputs_by_batch(x: dict, rows: Sequence[int], seed: int = 0) -> dict:
    """DP: keep sequences `rows`; their pages are re-packed into a local pool
    so each rank stores only its own sequences' pages, at a seeded random
    permutation of the local page ids (as the whole-batch pool is)."""
    dev = x["q"].device
    rows_t = torch.as_tensor(list(rows), dtype=torch.long, device=dev)
    page = x["k_cache"].shape[1]
    sl = x["cache_seqlens"][rows_t]
    bt = x["block_table"][rows_t]
    lens = sl.tolist()
    npg = [(l + page - 1) // page for l in lens]
    if sum(npg):
        used = torch.cat([bt[i, :n].long() for i, n in enumerate(npg) if n])
    else:
        used = torch.zeros(1, dtype=torch.long, device=dev)
    gen = torch.Generator().manual_seed(seed)
    perm = torch.randperm(used.numel(), generator=gen).to(dev)
    new_bt = torch.zeros(len(lens), max(1, max(npg) if npg else 1), dtype=torch.int32, device=dev)
    off = 0
    for i, n in enumerate(npg):
        new_bt[i, :n] = perm[off:off + n].to(torch.int32)
        off += n
    src = used[torch.argsort(perm)]   # local page perm[j] holds global page used[j]
    y = dict(x)
    y["q"] = x["q"][rows_t].contiguous()
    y["k_cache"] = x["k_cache"][src].contiguous()
    y["v_cache"] = x["v_cache"][src].contiguous()
    y["cache_seqlens"] = sl.contiguous()
    y["block_table"] = new_bt
    return y


class HeadGather:
    """TP output assembly with preallocated, packed buffers.

    The local decode writes out [B, Hq/N, D] and lse [B, Hq/N] straight into
    one send buffer (`out_local`, `lse_local` are views of it), so a step is
    ONE all_gather_into_tensor into a preallocated receive buffer followed by
    one copy of each output into head order: rank r's heads are
    [r*Hq/N, (r+1)*Hq/N).  Nothing is allocated per step."""

    def __init__(self, batch: int, local_heads: int, head_dim: int, dtype: torch.dtype,
                 device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        b, hl, d = batch, local_heads, head_dim
        es = torch.empty(0, dtype=dtype).element_size()
        self.ob = b * hl * d * es
        self.lb = b * hl * 4
        self.nbytes = (self.ob + self.lb + 15) // 16 * 16
        self.send = torch.zeros(self.nbytes, dtype=torch.uint8, device=device)
        self.out_local = self.send[: self.ob].view(dtype).view(b, hl, d)
        self.lse_local = self.send[self.ob: self.ob + self.lb].view(torch.float32).view(b, hl)
        self.recv = torch.zeros(self.world * self.nbytes, dtype=torch.uint8, device=device)
        self.out = torch.empty(b, self.world * hl, d, dtype=dtype, device=device)
        self.lse = torch.empty(b, self.world * hl, dtype=torch.float32, device=device)
        self._shape = (b, hl, d, dtype)

    def gather(self):
        b, hl, d, dtype = self._shape
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        r = self.recv.view(self.world, self.nbytes)
        ro = r[:, : self.ob].view(dtype).view(self.world, b, hl, d)
        rl = r[:, self.ob: self.ob + self.lb].view(torch.float32).view(self.world, b, hl)
        self.out.view(b, self.world, hl, d).copy_(ro.permute(1, 0, 2, 3))
        self.lse.view(b, self.world, hl).copy_(rl.permute(1, 0, 2))
        return self.out, self.lse
