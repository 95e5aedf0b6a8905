"""Host side of the paged KV cache around the kernels: the cache allocation and
per-layer binding of ModelRunner.allocate_kv_cache, the per-step decode metadata of
ModelRunner.prepare_decode, and the tensor-parallel KV-head split.

Reference (heart1128/mini-kvllm, src/myvllm/engine/model_runner.py):
  allocate_kv_cache   204-395  one zeros(2, L, NB, BS, KVH/world, D) tensor; fp8 caches are
                               float8_e4m3fn and int8 caches int8 (247-252); per-tensor
                               scales ones(2, L, 1) fp32 (324-329); per-(token, head) scales
                               ones(2, L, NB, BS, KVH/world) fp32 (330-338); layer l gets
                               views [0, l] / [1, l] (376-395)
  prepare_decode      631-671  context_lens = len(seq) (includes the new token),
                               (decode_metadata restates it; DecodeMetadataBuilder
                               computes it with one copy and one kernel per step)
                               slot = block_table[-1] * BS + last_block_num_tokens - 1,
                               block_tables padded with -1 to the longest table; int64
                               slots and lengths, int32 tables
  KV-head sharding    215      each rank holds num_kv_heads // world_size heads, and the
                               matching num_heads // world_size query heads
                               (models/qwen3.py:27-33)
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, Optional, Sequence

import torch

PER_TOKEN_HEAD = ("fp8_per_token_head", "int8_per_token_head")
QUANTIZED = ("fp8_per_tensor",) + PER_TOKEN_HEAD
KV_CACHE_DTYPES = ("auto",) + QUANTIZED


@dataclass
class KVCache:
    kv: torch.Tensor                      # (2, L, NB, BS, KVH, D)
    k_scale: Optional[torch.Tensor]       # (L, 1) or (L, NB, BS, KVH) fp32 views, or None
    v_scale: Optional[torch.Tensor]
    kv_cache_dtype: str
    block_size: int

    def layer(self, l: int):
        """(k_cache, v_cache, k_scale, v_scale) of layer l."""
        ks = self.k_scale[l] if self.k_scale is not None else None
        vs = self.v_scale[l] if self.v_scale is not None else None
        return self.kv[0, l], self.kv[1, l], ks, vs


def allocate_kv_cache(num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                      head_dim: int, kv_cache_dtype: str = "auto",
                      default_dtype: torch.dtype = torch.bfloat16,
                      device: torch.device | str = "cuda") -> KVCache:
    """One zero-initialised (2, L, NB, BS, KVH, D) cache (model_runner.py:311-314).
    'fp8_per_tensor': float8_e4m3fn pages and (2, L, 1) float32 scales at the calibration
    sentinel 1.0 (324-329). 'fp8_per_token_head' / 'int8_per_token_head': float8_e4m3fn /
    int8 pages and one float32 scale per (page, row, kv head), (2, L, NB, BS, KVH), set to
    1.0 (330-338); the append writes each row's scale."""
    if kv_cache_dtype not in KV_CACHE_DTYPES:
        raise NotImplementedError(f"kv_cache_dtype {kv_cache_dtype!r} is not implemented")
    if kv_cache_dtype == "int8_per_token_head":
        data_dtype = torch.int8
    elif kv_cache_dtype in QUANTIZED:
        data_dtype = torch.float8_e4m3fn
    else:
        data_dtype = default_dtype
    kv = torch.zeros(2, num_layers, num_blocks, block_size, num_kv_heads, head_dim,
                     dtype=data_dtype, device=device)
    ks = vs = None
    if kv_cache_dtype == "fp8_per_tensor":
        buf = torch.ones(2, num_layers, 1, dtype=torch.float32, device=device)
        ks, vs = buf[0], buf[1]
    elif kv_cache_dtype in PER_TOKEN_HEAD:
        buf = torch.ones(2, num_layers, num_blocks, block_size, num_kv_heads, dtype=torch.float32,
                         device=device)
        ks, vs = buf[0], buf[1]
    return KVCache(kv, ks, vs, kv_cache_dtype, block_size)


def bind_kv_cache(modules: Iterable[torch.nn.Module], cache: KVCache) -> int:
    """Injects per-layer cache views (and scales) into every module that has k_cache and
    v_cache attributes, in module order (model_runner.py:376-395). Returns the count."""
    layer = 0
    for m in modules:
        if hasattr(m, "k_cache") and hasattr(m, "v_cache"):
            k, v, ks, vs = cache.layer(layer)
            m.k_cache, m.v_cache = k, v
            m.kv_cache_dtype = cache.kv_cache_dtype
            if ks is not None:
                m.k_scale, m.v_scale = ks, vs
            layer += 1
    return layer


@dataclass
class DecodeMetadata:
    slot_mapping: torch.Tensor   # (B,) int64
    context_lens: torch.Tensor   # (B,) int64
    block_tables: torch.Tensor   # (B, max_blocks) int32, -1 padded


def decode_metadata(block_tables: Sequence[Sequence[int]], seq_lens: Sequence[int],
                    block_size: int, device: torch.device | str = "cuda",
                    pin_memory: bool = False) -> DecodeMetadata:
    """Per-step decode metadata of prepare_decode (model_runner.py:631-671): seq_lens are
    the sequence lengths including the token being decoded; each slot is the last
    token's position inside the last block of the sequence's table."""
    if len(block_tables) != len(seq_lens):
        raise ValueError("one block table per sequence is required")
    slots, lens = [], []
    for bt, n in zip(block_tables, seq_lens):
        if n <= 0 or len(bt) < (n + block_size - 1) // block_size:
            raise ValueError(f"sequence of length {n} needs {(n + block_size - 1) // block_size} blocks, has {len(bt)}")
        last_block_tokens = n - (len(bt) - 1) * block_size
        slots.append(bt[-1] * block_size + last_block_tokens - 1)
        lens.append(n)
    width = max((len(bt) for bt in block_tables), default=0)
    padded = [list(bt) + [-1] * (width - len(bt)) for bt in block_tables]
    pin = pin_memory and torch.cuda.is_available()
    def to(t):
        return t.pin_memory().to(device, non_blocking=True) if pin else t.to(device)
    return DecodeMetadata(
        slot_mapping=to(torch.tensor(slots, dtype=torch.int64)),
        context_lens=to(torch.tensor(lens, dtype=torch.int64)),
        block_tables=to(torch.tensor(padded, dtype=torch.int32).reshape(len(padded), width)))


class DecodeMetadataBuilder:
    """Decode metadata with one host-to-device copy and one kernel per step, instead of
    prepare_decode's per-sequence Python loops and three host tensors
    (model_runner.py:631-671).

    Block tables live in a host mirror indexed by a persistent sequence slot. The block
    manager reports only their changes: `set_table` when a sequence takes a slot,
    `append` when it takes a block. Each step then packs [lengths | tables] into a pinned
    buffer, copies it once, and `mkv_decode_metadata` derives the int64 slot mapping and
    context lengths on the device. The table width is max_blocks, fixed, so every step
    has the same shapes (capturable decode graphs). Two pinned buffers alternate, each
    reused only after its previous copy has completed. The returned tensors are
    overwritten by the next step."""

    def __init__(self, max_seqs: int, max_blocks: int, block_size: int,
                 device: torch.device | str = "cuda"):
        import numpy as np
        from .. import _lib
        self._np, self._lib_mod = np, _lib
        self._lib = _lib.load()
        self.max_seqs, self.max_blocks, self.block_size = max_seqs, max_blocks, block_size
        self.device = torch.device(device)
        n = max_seqs * (1 + max_blocks)
        self._host = [torch.empty(n, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._host_np = [h.numpy() for h in self._host]
        self._copied = [None, None]
        self._k = 0
        self._tables = np.full((max_seqs, max_blocks), -1, dtype=np.int32)
        self._nblocks = np.zeros(max_seqs, dtype=np.int64)
        self._packed = torch.empty(n, dtype=torch.int32, device=self.device)
        self._slots = torch.empty(max_seqs, dtype=torch.int64, device=self.device)
        self._lens = torch.empty(max_seqs, dtype=torch.int64, device=self.device)

    def set_table(self, seq: int, table: Sequence[int]) -> None:
        if len(table) > self.max_blocks:
            raise ValueError(f"a table of {len(table)} blocks exceeds max_blocks {self.max_blocks}")
        row = self._tables[seq]
        row[:] = -1
        row[:len(table)] = table
        self._nblocks[seq] = len(table)

    def append(self, seq: int, block: int) -> None:
        n = int(self._nblocks[seq])
        if n >= self.max_blocks:
            raise ValueError(f"sequence slot {seq} already holds max_blocks {self.max_blocks}")
        self._tables[seq, n] = block
        self._nblocks[seq] = n + 1

    def step(self, seqs: Sequence[int], seq_lens: Sequence[int]) -> DecodeMetadata:
        """Metadata of one decode step over sequence slots `seqs` (batch order), with
        lengths including the token being decoded."""
        np = self._np
        B, W = len(seqs), self.max_blocks
        if B > self.max_seqs or len(seq_lens) != B:
            raise ValueError("one length per sequence, at most max_seqs sequences")
        k = self._k
        if self._copied[k] is not None:
            self._copied[k].synchronize()  # the copy that last read this buffer is done
        hv = self._host_np[k]
        idx = np.asarray(seqs, dtype=np.int64)
        hv[:B] = seq_lens
        hv[B:B + B * W].reshape(B, W)[:] = self._tables[idx]
        stream = torch.cuda.current_stream(self.device)
        self._packed[:B * (1 + W)].copy_(self._host[k][:B * (1 + W)], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._copied[k] = ev
        self._k ^= 1
        st = self._lib.mkv_decode_metadata(self._packed.data_ptr(), B, W, self.block_size,
                                           self._slots.data_ptr(), self._lens.data_ptr(),
                                           stream.cuda_stream)
        self._lib_mod.check("mkv_decode_metadata", st)
        return DecodeMetadata(slot_mapping=self._slots[:B], context_lens=self._lens[:B],
                              block_tables=self._packed[B:B + B * W].view(B, W))


def kv_head_shard(num_heads: int, num_kv_heads: int, rank: int, world_size: int):
    """(query-head range, kv-head range) owned by `rank` under tensor parallelism: KV heads
    split evenly (model_runner.py:215) with their GQA query heads (qwen3.py:27-33)."""
    if num_kv_heads % world_size or num_heads % world_size or num_heads % num_kv_heads:
        raise ValueError(f"cannot split {num_heads} query / {num_kv_heads} kv heads over {world_size} ranks")
    kvh = num_kv_heads // world_size
    h = num_heads // world_size
    return range(rank * h, (rank + 1) * h), range(rank * kvh, (rank + 1) * kvh)
