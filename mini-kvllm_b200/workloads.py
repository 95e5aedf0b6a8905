"""Seeded synthetic workloads with the shapes of the BASELINE configurations.

The reference measures on no public dataset; these builders make the inputs its
benchmark configurations describe (shapes, value distributions, page permutations),
directly on the target device:

  config 1  decode, fp32: B=4, H=16, KVH=8, D=128, block_size=16, ctx ~ U[64, 512]
  config 2  append microbench: 4096 new tokens = 16 prefill chunks x 128 tokens +
            2048 single decode tokens, KVH=8, D=128, bf16 N(0,1) with 0.1% outliers x20,
            into a 64k-slot cache (block_size 256), bf16 and FP8 E4M3
  config 3  decode, bf16, Qwen3-8B attention: H=32, KVH=8, D=128, block_size=256,
            B=256, ctx ~ U[1024, 8192]
  config 4  decode, FP8 E4M3 per-tensor: H=32, KVH=8, D=128, block_size=256, B=64,
            ctx = 32768 for every sequence

Pages are assigned by a random permutation of the physical blocks; each sequence's
table covers exactly ceil(ctx / block_size) pages and is -1 padded to the widest
table (max_num_blocks). Sharded variants keep the full batch and lengths and take
the KV heads [r*KVH/N, (r+1)*KVH/N) of rank r with their query heads.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass
class DecodeWorkload:
    name: str
    query: torch.Tensor          # (B, H_local, D)
    k_cache: torch.Tensor        # (NB, BS, KVH_local, D)
    v_cache: torch.Tensor
    block_tables: torch.Tensor   # (B, max_blocks) int32
    context_lens: torch.Tensor   # (B,) int64
    num_heads: int               # local (per rank)
    num_kv_heads: int            # local
    head_dim: int
    block_size: int
    scale: float
    k_scale: Optional[torch.Tensor] = None  # (1,) fp32 for FP8 caches
    v_scale: Optional[torch.Tensor] = None
    # the step's new token per sequence (appended before the decode, as the engine does)
    new_k: Optional[torch.Tensor] = None    # (B, KVH_local, D), query dtype
    new_v: Optional[torch.Tensor] = None
    slot_mapping: Optional[torch.Tensor] = None  # (B,) int64, slot of position ctx-1
    meta: dict = field(default_factory=dict)

    @property
    def fp8(self) -> bool:
        return self.k_cache.dtype == torch.float8_e4m3fn

    def kv_bytes(self) -> int:
        """Algorithmic K+V cache bytes one decode reads: sum(ctx) * KVH * D * elem * 2."""
        tokens = int(self.context_lens.clamp(max=self.block_tables.shape[1] * self.block_size).sum())
        return tokens * self.num_kv_heads * self.head_dim * self.k_cache.element_size() * 2

    def decode_bytes(self) -> int:
        """Algorithmic bytes of one decode: K/V reads + q read + out write + tables."""
        q = self.query.numel() * self.query.element_size()
        return self.kv_bytes() + 2 * q + self.block_tables.numel() * 4 + self.context_lens.numel() * 8

    def append_bytes(self) -> int:
        """Algorithmic bytes of the step's append: read new K/V, write them into the pages."""
        if self.new_k is None:
            return 0
        n = self.new_k.numel()
        return 2 * n * self.new_k.element_size() + 2 * n * self.k_cache.element_size() + \
            self.slot_mapping.numel() * 8


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _tables(lens, block_size, device, gen_cpu):
    need = [(n + block_size - 1) // block_size for n in lens]
    nb = sum(need)
    perm = torch.randperm(nb, generator=gen_cpu)
    width = max(need) if need else 0
    bt = torch.full((len(lens), width), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].to(torch.int32)
        pos += k
    return bt.to(device), nb


def _fill_normal(t: torch.Tensor, gen, chunk_elems: int = 1 << 28, outliers: float = 0.0,
                 scale_fp8: Optional[float] = None):
    """Fills t with N(0,1) (optionally x20 outliers, optionally quantised to e4m3 with
    the given scale) chunk by chunk, to bound temporary memory."""
    flat = t.view(-1)
    for s in range(0, flat.numel(), chunk_elems):
        e = min(flat.numel(), s + chunk_elems)
        x = torch.randn(e - s, generator=gen, device=t.device, dtype=torch.float32)
        if outliers > 0:
            m = torch.rand(e - s, generator=gen, device=t.device) < outliers
            x = torch.where(m, x * 20.0, x)
        if scale_fp8 is not None:
            x = (x.to(torch.bfloat16).float() / scale_fp8).clamp(-448.0, 448.0)
            flat[s:e] = x.to(torch.float8_e4m3fn)
        else:
            flat[s:e] = x.to(t.dtype)


def decode_workload(name: str, batch: int, num_heads: int, num_kv_heads: int, head_dim: int,
                    block_size: int, lens, dtype=torch.bfloat16, fp8: bool = False,
                    device="cuda", seed: int = 0, rank: int = 0, world_size: int = 1,
                    with_append: bool = True) -> DecodeWorkload:
    """Decode workload for rank `rank` of `world_size` (KV-head sharding)."""
    gen_cpu = torch.Generator().manual_seed(seed)
    lens = [int(x) for x in lens]
    assert len(lens) == batch
    bt, nb = _tables(lens, block_size, device, gen_cpu)
    h_loc = num_heads // world_size
    kvh_loc = num_kv_heads // world_size
    gen = _gen(device, seed * 1000 + 17 + rank)
    q = torch.empty(batch, h_loc, head_dim, dtype=dtype, device=device)
    _fill_normal(q, gen)
    cache_dtype = torch.float8_e4m3fn if fp8 else dtype
    kc = torch.empty(nb, block_size, kvh_loc, head_dim, dtype=cache_dtype, device=device)
    vc = torch.empty_like(kc)
    ks = vs = None
    if fp8:
        # per-tensor scales as calibrated from N(0,1) bf16 data: amax over 2^24 draws / 448
        probe = torch.randn(1 << 24, generator=gen, device=device).to(torch.bfloat16)
        s = float((probe.abs().amax().float() * (1.0 / 448.0)).to(torch.bfloat16))
        ks = torch.tensor([s], dtype=torch.float32, device=device)
        vs = torch.tensor([s], dtype=torch.float32, device=device)
        _fill_normal(kc, gen, scale_fp8=s)
        _fill_normal(vc, gen, scale_fp8=s)
    else:
        _fill_normal(kc, gen)
        _fill_normal(vc, gen)
    cl = torch.tensor(lens, dtype=torch.int64, device=device)
    w = DecodeWorkload(name, q, kc, vc, bt, cl, h_loc, kvh_loc, head_dim, block_size,
                       1.0 / math.sqrt(head_dim), ks, vs,
                       meta=dict(batch=batch, num_heads=num_heads, num_kv_heads=num_kv_heads,
                                 rank=rank, world_size=world_size, seed=seed))
    if with_append:
        nk = torch.empty(batch, kvh_loc, head_dim, dtype=dtype, device=device)
        nv = torch.empty_like(nk)
        _fill_normal(nk, gen)
        _fill_normal(nv, gen)
        bt_cpu = bt.cpu()
        slots = [int(bt_cpu[b, (n - 1) // block_size]) * block_size + (n - 1) % block_size if n > 0 else -1
                 for b, n in enumerate(lens)]
        w.new_k, w.new_v = nk, nv
        w.slot_mapping = torch.tensor(slots, dtype=torch.int64, device=device)
    return w


def config1(device="cuda", seed=0, **kw) -> DecodeWorkload:
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(64, 513, (4,), generator=g).tolist()
    return decode_workload("config1", 4, 16, 8, 128, 16, lens, dtype=torch.float32,
                           device=device, seed=seed, **kw)


def config3(device="cuda", seed=0, batch=256, **kw) -> DecodeWorkload:
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1024, 8193, (batch,), generator=g).tolist()
    return decode_workload("config3", batch, 32, 8, 128, 256, lens, dtype=torch.bfloat16,
                           device=device, seed=seed, **kw)


def config4(device="cuda", seed=0, batch=64, ctx=32768, **kw) -> DecodeWorkload:
    return decode_workload("config4", batch, 32, 8, 128, 256, [ctx] * batch,
                           dtype=torch.bfloat16, fp8=True, device=device, seed=seed, **kw)


@dataclass
class AppendWorkload:
    key: torch.Tensor            # (T, KVH, D) bf16
    value: torch.Tensor
    slot_mapping: torch.Tensor   # (T,) int64
    num_blocks: int
    block_size: int

    def bytes(self, cache_elem: int) -> int:
        n = self.key.numel()
        return 2 * n * self.key.element_size() + 2 * n * cache_elem + self.slot_mapping.numel() * 8


def config2(device="cuda", seed=0) -> AppendWorkload:
    """4096 new tokens: 16 prefill chunks of 128 consecutive slots (half a 256-slot page
    each, on distinct pages) and 2048 single decode tokens on random slots of other
    pages, in a 65536-slot cache (256 blocks of 256)."""
    T_chunk, n_chunks, n_single, BS, NB, KVH, D = 128, 16, 2048, 256, 256, 8, 128
    g = torch.Generator().manual_seed(seed)
    pages = torch.randperm(NB, generator=g)
    chunk_pages, other = pages[:n_chunks], pages[n_chunks:]
    slots = []
    for p in chunk_pages.tolist():
        off = int(torch.randint(0, 2, (1,), generator=g)) * T_chunk
        slots.extend(range(p * BS + off, p * BS + off + T_chunk))
    pool = (other[:, None] * BS + torch.arange(BS)[None, :]).reshape(-1)
    pick = pool[torch.randperm(pool.numel(), generator=g)[:n_single]]
    slots.extend(pick.tolist())
    T = len(slots)
    gen = _gen(device, seed * 1000 + 29)
    key = torch.empty(T, KVH, D, dtype=torch.bfloat16, device=device)
    value = torch.empty_like(key)
    _fill_normal(key, gen, outliers=0.001)
    _fill_normal(value, gen, outliers=0.001)
    return AppendWorkload(key, value, torch.tensor(slots, dtype=torch.int64, device=device), NB, BS)
