"""Forward-pass context: the paging metadata the model runner hands to every
attention layer of one step.

Mirrors the reference's global-context contract (heart1128/mini-kvllm,
src/myvllm/utils/context.py:25-47 for the fields, 94-124 for get/reset/set), so a
model runner written against the reference fills it the same way:
  slot_mapping  (num_tokens,)          int64, cache slot of each new token (-1 = skip)
  context_lens  (num_seqs,)            int64, tokens visible to each decode query,
                                       including the one being appended
  block_tables  (num_seqs, max_blocks) int32, physical page of each logical block, -1 padded
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional


@dataclass
class MixedAttentionSplit:
    """Decode/prefill partition of a mixed batch (context.py:10-21 in the reference)."""

    decode_token_indices: list
    decode_seq_indices: list
    prefill_token_indices: list
    prefill_seq_indices: list
    prefill_cu_seqlens_q: list
    decode_token_indices_tensor: Optional[Any] = None
    decode_seq_indices_tensor: Optional[Any] = None
    prefill_token_indices_tensor: Optional[Any] = None
    prefill_seq_indices_tensor: Optional[Any] = None
    prefill_cu_seqlens_q_tensor: Optional[Any] = None


@dataclass
class Context:
    is_prefill: bool = False
    cu_seqlens_q: Optional[Any] = None
    cu_seqlens_k: Optional[Any] = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: Optional[Any] = None
    context_lens: Optional[Any] = None
    block_tables: Optional[Any] = None
    positions: Optional[Any] = None
    query_lens: Optional[Any] = None
    is_decode: Optional[Any] = None
    mixed_attention_split: Optional[MixedAttentionSplit] = None
    is_full_prefill: bool = False
    residual_slots: Optional[Any] = None
    residual_lens: Optional[Any] = None


def split_mixed_decode_prefill_metadata(cu_seqlens_q, query_lens, is_decode) -> MixedAttentionSplit:
    """Partitions a mixed batch's token and sequence indices into decode and prefill
    parts (reference context.py:55-88): decode sequences contribute their token indices
    and sequence index; prefill sequences also extend a cumulative q-length list."""

    def as_list(values):
        return list(values.tolist()) if hasattr(values, "tolist") else list(values)

    cu_q = as_list(cu_seqlens_q)
    q_lens = as_list(query_lens)
    flags = [bool(v) for v in as_list(is_decode)]
    out = MixedAttentionSplit([], [], [], [], [0])
    for seq_idx, (q_len, dec) in enumerate(zip(q_lens, flags)):
        tokens = range(cu_q[seq_idx], cu_q[seq_idx + 1])
        if dec:
            out.decode_token_indices.extend(tokens)
            out.decode_seq_indices.append(seq_idx)
        else:
            out.prefill_token_indices.extend(tokens)
            out.prefill_seq_indices.append(seq_idx)
            out.prefill_cu_seqlens_q.append(out.prefill_cu_seqlens_q[-1] + q_len)
    return out


_context = Context()


def get_context() -> Context:
    return _context


def reset_context() -> None:
    global _context
    _context = Context()


def set_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0, max_seqlen_k=0,
                slot_mapping=None, context_lens=None, block_tables=None, positions=None,
                query_lens=None, is_decode=None, mixed_attention_split=None,
                is_full_prefill=False, residual_slots=None, residual_lens=None) -> None:
    global _context
    _context = Context(
        is_prefill=is_prefill, cu_seqlens_q=cu_seqlens_q, cu_seqlens_k=cu_seqlens_k,
        max_seqlen_q=max_seqlen_q, max_seqlen_k=max_seqlen_k, slot_mapping=slot_mapping,
        context_lens=context_lens, block_tables=block_tables, positions=positions,
        query_lens=query_lens, is_decode=is_decode, mixed_attention_split=mixed_attention_split,
        is_full_prefill=is_full_prefill, residual_slots=residual_slots, residual_lens=residual_lens)
