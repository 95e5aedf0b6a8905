"""CPU restatement of mini-kvllm's paged KV-cache hot path — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the checker;
the product (libmkv.so and its Python wrappers) never calls it.

Every function cites the reference code it restates (heart1128/mini-kvllm; paths
relative to that repository). All functions take and return CPU torch tensors.
"""
from __future__ import annotations

import numpy as np
import torch

FP8_E4M3_MAX = 448.0  # attention.py:113


# ------------------------------------------------------------------------------ append
def store_kvcache_ref(key, value, k_cache, v_cache, slot_mapping, block_size):
    """src/myvllm/layers/attention.py:7-64 (kernel) and 67-108 (wrapper):
    cache.view(-1, KVH, D)[slot] = x[t] for every token whose slot is not -1.
    block_size only fixes the (block, offset) split of a slot, which the flat view
    already encodes. Stores convert to the cache dtype (tl.store semantics)."""
    num_tokens, num_kv_heads, head_dim = key.shape
    assert k_cache.shape == v_cache.shape
    slots = slot_mapping.reshape(-1).long()
    keep = slots != -1
    kflat = k_cache.view(-1, num_kv_heads, head_dim)
    vflat = v_cache.view(-1, num_kv_heads, head_dim)
    kflat[slots[keep]] = key[keep].to(k_cache.dtype)
    vflat[slots[keep]] = value[keep].to(v_cache.dtype)


def fp8_scale_ref(x: torch.Tensor) -> float:
    """The per-tensor scale of attention.py:318-323,
        scale = x.abs().amax().clamp(min=1e-8) / FP8_E4M3_MAX,
    evaluated with torch's CUDA semantics for a tensor of x.dtype: the clamp bound is
    first converted to x.dtype (NaN passes through), and dividing by a Python scalar
    multiplies by the float32 reciprocal; the result is rounded to x.dtype and read
    back exactly by .item()/.fill_ into the float32 scale. (For bf16 inputs the true
    quotient rounds to the same bf16 value for every input, so CPU and CUDA agree.)"""
    a = x.abs().amax()
    lo = torch.tensor(1e-8, dtype=x.dtype)
    a = torch.where(torch.isnan(a), a, torch.maximum(a, lo))
    inv = torch.tensor(1.0, dtype=torch.float32) / torch.tensor(FP8_E4M3_MAX, dtype=torch.float32)
    return float((a.float() * inv).to(x.dtype))


def quantize_fp8_ref(x: torch.Tensor, scale: float) -> torch.Tensor:
    """attention.py:166-167 and 188-191: q = clamp(float32(x) / scale, -448, 448) cast
    to float8_e4m3fn (round to nearest even). The quotient is the correctly rounded
    float32 division. tl.maximum/tl.minimum return the non-NaN operand, so a NaN
    quotient becomes -448 (maximum(NaN, -448) = -448)."""
    q = x.float() / torch.tensor(scale, dtype=torch.float32)
    q = torch.where(torch.isnan(q), torch.full_like(q, -FP8_E4M3_MAX), q)
    q = q.clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX)
    return q.to(torch.float8_e4m3fn)


def store_kvcache_fp8_ref(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping,
                          block_size):
    """attention.py:281-333, per-tensor mode: calibrate each scale from this batch while
    it still holds the sentinel 1.0 (315-323; the K scale first, then V), then quantise
    with the (possibly just calibrated) scales and scatter like store_kvcache."""
    if float(k_scale.reshape(-1)[0]) == 1.0:
        k_scale.fill_(fp8_scale_ref(key))
    if float(v_scale.reshape(-1)[0]) == 1.0:
        v_scale.fill_(fp8_scale_ref(value))
    kq = quantize_fp8_ref(key, float(k_scale.reshape(-1)[0]))
    vq = quantize_fp8_ref(value, float(v_scale.reshape(-1)[0]))
    store_kvcache_ref(kq, vq, k_cache, v_cache, slot_mapping, block_size)


INT8_MAX, INT8_MIN = 127.0, -128.0  # attention.py:114-115


def per_token_head_scales_ref(x: torch.Tensor, mode: str) -> torch.Tensor:
    """Per-(token, kv head) scales of the dynamic quantisers, float32, shape x.shape[:-1]:
      fp8:  attention.py:170-175  amax = max|x| over head_dim; scale = amax / 448 when
            amax > 0, else 1.0 (a NaN amax also gives 1.0: NaN > 0 is false);
      int8: attention.py:231-234  scale = maximum(amax / 127, 1e-6) (tl.maximum keeps the
            non-NaN operand, so a NaN amax gives 1e-6).
    Divisions are the correctly rounded float32 quotient."""
    a = x.float().abs().amax(dim=-1)
    if mode == "fp8":
        q = a / torch.tensor(FP8_E4M3_MAX, dtype=torch.float32)
        return torch.where(a > 0, q, torch.ones_like(q))
    q = a / torch.tensor(INT8_MAX, dtype=torch.float32)
    lo = torch.tensor(1e-6, dtype=torch.float32)
    return torch.where(torch.isnan(q), lo, torch.maximum(q, lo))


def quantize_int8_ref(x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """attention.py:240-247: q = x * (1 / scale) in float32 (reciprocal first, as written),
    rounded half away from zero by adding +-0.5 and truncating toward zero on the int8
    store, after clamping to [-128, 127]. `scale` broadcasts over head_dim. tl.clamp
    keeps the non-NaN bound (min(max(x, lo), hi) without NaN propagation), so a NaN
    element stores -128."""
    inv = torch.tensor(1.0, dtype=torch.float32) / scale.float()
    q = x.float() * inv.unsqueeze(-1)
    q = torch.where(q >= 0, q + 0.5, q - 0.5)
    q = torch.where(torch.isnan(q), torch.full_like(q, INT8_MIN), q)
    q = q.clamp(INT8_MIN, INT8_MAX)
    return torch.trunc(q).to(torch.int8)


def store_kvcache_quant_per_token_head_ref(key, value, k_cache, v_cache, k_scales, v_scales,
                                           slot_mapping, block_size, mode):
    """store_kvcache_fp8 with kv_cache_dtype 'fp8_per_token_head' (attention.py:118-191 with
    PER_TOKEN_HEAD=1, wrapper 281-333) and store_kvcache_int8 (attention.py:195-278): each
    (token, kv head) row gets its own scale, written to k_scales/v_scales (num_blocks,
    block_size, num_kv_heads) at the token's slot, and is quantised with it (FP8:
    clamp(x / scale) -> e4m3 as in quantize_fp8_ref; INT8: quantize_int8_ref)."""
    num_tokens, num_kv_heads, head_dim = key.shape
    slots = slot_mapping.reshape(-1).long()
    keep = slots != -1
    for x, cache, scales in ((key, k_cache, k_scales), (value, v_cache, v_scales)):
        sc = per_token_head_scales_ref(x, mode)  # (T, KVH)
        if mode == "fp8":
            q = x.float() / sc.unsqueeze(-1)
            q = torch.where(torch.isnan(q), torch.full_like(q, -FP8_E4M3_MAX), q)
            q = q.clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn)
        else:
            q = quantize_int8_ref(x, sc)
        cache.view(-1, num_kv_heads, head_dim)[slots[keep]] = q[keep].view(cache.dtype)
        scales.view(-1, num_kv_heads)[slots[keep]] = sc[keep]


def e4m3_encode_reference(x: np.ndarray) -> np.ndarray:
    """Independent float32 -> E4M3 (OCP 'fn' variant) byte encoder, written from the
    format definition, used to pin torch's conversion: 1 sign bit, 4 exponent bits
    (bias 7), 3 mantissa bits, no infinities, S.1111.111 = NaN, largest finite 448,
    subnormals m * 2^-9. Round to nearest, ties to even; magnitudes beyond 448 saturate
    to 448 (the 'satfinite' behaviour; the quantiser clamps before converting)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    out = np.zeros(x.shape, dtype=np.uint8)
    mant, ex = np.frexp(a)  # a = mant * 2^ex, mant in [0.5, 1)
    e = ex.astype(np.int64) - 1  # a in [2^e, 2^(e+1))
    sub = a < 2.0 ** -6
    # subnormal: m * 2^-9, m may round up to 8 = smallest normal (exponent field 1)
    m_sub = np.rint(a / 2.0 ** -9).astype(np.int64)
    # normal: (1 + m/8) * 2^e
    with np.errstate(over="ignore", invalid="ignore"):
        m_nrm = np.rint((a / np.exp2(e.astype(np.float64)) - 1.0) * 8.0).astype(np.int64)
    carry = m_nrm == 8
    e_n = e + carry
    m_n = np.where(carry, 0, m_nrm)
    field = e_n + 7
    code_n = (field << 3) | m_n
    code = np.where(sub, m_sub, code_n)
    code = np.where(code > 0x7E, 0x7E, code)  # saturate to 448
    out = (code.astype(np.uint8) | sign)
    out = np.where(np.isnan(x), sign | 0x7F, out).astype(np.uint8)
    return out


# ------------------------------------------------------------------------------ decode
def decode_torch_optimized(q, k_cache, v_cache, block_tables, context_lens, scale, num_heads,
                           num_kv_heads, head_dim, block_size):
    """benchmark_decoding.py:145-198 ("optimized PyTorch" paged decode): gather each
    sequence's pages into a zero-padded (B, max_ctx, KVH, D) tensor (blocks with id -1
    dropped), repeat K/V over the GQA group, scores = q K^T * scale with positions >=
    context_len masked to -inf, softmax, times V. Runs in the input dtype."""
    batch = q.shape[0]
    dtype = q.dtype
    max_ctx = int(context_lens.max().item())
    kp = torch.zeros(batch, max_ctx, num_kv_heads, head_dim, dtype=dtype)
    vp = torch.zeros(batch, max_ctx, num_kv_heads, head_dim, dtype=dtype)
    for i in range(batch):
        n = int(context_lens[i].item())
        nblk = (n + block_size - 1) // block_size
        blocks = block_tables[i, :nblk]
        blocks = blocks[blocks != -1].long()
        if blocks.numel() > 0:
            kp[i, :n] = k_cache[blocks].reshape(-1, num_kv_heads, head_dim)[:n]
            vp[i, :n] = v_cache[blocks].reshape(-1, num_kv_heads, head_dim)[:n]
    if num_kv_heads != num_heads:
        rep = num_heads // num_kv_heads
        kp = kp.repeat_interleave(rep, dim=2)
        vp = vp.repeat_interleave(rep, dim=2)
    qh = q.unsqueeze(2)
    kp = kp.transpose(1, 2)
    vp = vp.transpose(1, 2)
    scores = torch.matmul(qh, kp.transpose(-2, -1)) * scale
    mask = torch.arange(max_ctx)[None, :] < context_lens[:, None]
    scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, vp).squeeze(2)


def paged_decode_ref(query, k_cache, v_cache, block_tables, context_lens, scale, num_heads,
                     num_kv_heads, head_dim, block_size, k_scale=None, v_scale=None,
                     compute_dtype=torch.float64, k_scales=None, v_scales=None):
    """Token-level restatement of paged_attention_decode_kernel (attention.py:517-646)
    and, with k_scale/v_scale, paged_attention_decode_fp8_kernel with PER_TOKEN_HEAD=0
    (attention.py:953-1121), evaluated in `compute_dtype`:
      * kv head of query head h is h // (num_heads // num_kv_heads) (541, 996);
      * token t < context_len is visible when its logical block t // block_size is
        < max_num_blocks (581, 1040) and its page block_tables[b, t // block_size]
        is not -1 (586, 1045); invisible tokens carry no weight;
      * FP8 values are dequantised as float(x) * scale (1051-1062, 1098-1107); with
        per-token scales k_scales/v_scales (num_blocks, block_size, num_kv_heads) an
        FP8 or INT8 value at (page, row, kv head) is float(x) * scales[page, row, head]
        (per_token_head modes: 1054-1062, 1098-1107 and the tile kernel 1124-1210);
      * out = sum_t softmax(scale * q.k_t) v_t; a sequence with no visible token gives
        0/0 = NaN, like the kernel's acc / l_i with l_i = 0 (642, 1119).
    Returns (B, H, D) in compute_dtype."""
    batch = query.shape[0]
    group = num_heads // num_kv_heads
    max_blocks = block_tables.shape[1]
    num_blocks = k_cache.shape[0]
    kc = k_cache.to(compute_dtype)
    vc = v_cache.to(compute_dtype)
    if k_scale is not None:
        kc = kc * float(k_scale.reshape(-1)[0])
        vc = vc * float(v_scale.reshape(-1)[0])
    if k_scales is not None:
        kc = kc * k_scales.to(compute_dtype).unsqueeze(-1)
        vc = vc * v_scales.to(compute_dtype).unsqueeze(-1)
    out = torch.empty(batch, num_heads, head_dim, dtype=compute_dtype)
    for b in range(batch):
        n = max(0, min(int(context_lens[b]), max_blocks * block_size))
        t = torch.arange(n)
        blk = block_tables[b, t // block_size].long() if n > 0 else torch.zeros(0, dtype=torch.long)
        ok = (blk >= 0) & (blk < num_blocks)
        t, blk = t[ok], blk[ok]
        if t.numel() == 0:
            out[b] = float("nan")
            continue
        K = kc[blk, t % block_size]  # (n, KVH, D)
        V = vc[blk, t % block_size]
        q = query[b].to(compute_dtype).view(num_kv_heads, group, head_dim)
        s = torch.einsum("hgd,thd->hgt", q, K) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgt,thd->hgd", p, V).reshape(num_heads, head_dim)
    return out


# ------------------------------------------------------------------- contiguous prefill
def varlen_prefill_ref(query, key, value, cu_seqlens, scale, num_heads, num_kv_heads,
                       compute_dtype=torch.float64):
    """flash_attention_prefill (attention.py:446-516) and flash_attention_varlen_kernel
    (336-443): sequence b owns rows [cu_seqlens[b], cu_seqlens[b+1]) of query / key /
    value; row m of the sequence attends to the sequence's rows 0..m (mask_causal,
    :392-393) with kv head h // (num_heads // num_kv_heads) (:357), softmax(scale q.k) v.
    Returns (total_tokens, num_heads, head_dim) in compute_dtype."""
    total, _, head_dim = query.shape
    group = num_heads // num_kv_heads
    out = torch.empty(total, num_heads, head_dim, dtype=compute_dtype)
    cu = [int(x) for x in cu_seqlens.reshape(-1).tolist()]
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        n = e - s
        if n <= 0:
            continue
        q = query[s:e].to(compute_dtype).view(n, num_kv_heads, group, head_dim)
        k = key[s:e].to(compute_dtype)
        v = value[s:e].to(compute_dtype)
        sc = torch.einsum("mhgd,thd->hgmt", q, k) * scale
        causal = torch.arange(n)[None, :] <= torch.arange(n)[:, None]  # t <= m
        sc = sc.masked_fill(~causal, float("-inf"))
        p = torch.softmax(sc, dim=-1)
        out[s:e] = torch.einsum("hgmt,thd->mhgd", p, v).reshape(n, num_heads, head_dim)
    return out


# ------------------------------------------------------------------- prefill / extend
def paged_prefill_ref(query, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q,
                      positions, scale, num_heads, num_kv_heads, block_size, k_scale=None,
                      v_scale=None, k_scales=None, v_scales=None, compute_dtype=torch.float64):
    """Chunked-prefill / extend attention over the paged cache, restating
    paged_attention_prefill_torch (attention.py:649-701) and the kernel
    paged_attention_prefill_kernel (attention.py:704-849): query token q of sequence b
    (q in [cu_seqlens_q[b], cu_seqlens_q[b+1])) at absolute position positions[q] sees
    the cached tokens t < min(context_lens[b], positions[q] + 1) (749), gathered through
    block_tables[b, t // block_size]; a -1 page is skipped (792-796). GQA kv head
    h // (H / KVH). With per-tensor k_scale/v_scale or per-(page, row, kv head)
    k_scales/v_scales the 8-bit pages are dequantised as float(x) * scale, as the decode
    kernels do (the reference has no quantised prefill; its TODO,
    docs/chunked_prefill_todo.md:23-30, asks for exactly this). A query that sees no
    token gives 0/0 = NaN. Returns (total_q, H, D) in compute_dtype."""
    total_q, _, head_dim = query.shape
    group = num_heads // num_kv_heads
    num_blocks = k_cache.shape[0]
    max_blocks = block_tables.shape[1]
    kc = k_cache.to(compute_dtype)
    vc = v_cache.to(compute_dtype)
    if k_scale is not None:
        kc = kc * float(k_scale.reshape(-1)[0])
        vc = vc * float(v_scale.reshape(-1)[0])
    if k_scales is not None:
        kc = kc * k_scales.to(compute_dtype).unsqueeze(-1)
        vc = vc * v_scales.to(compute_dtype).unsqueeze(-1)
    out = torch.empty(total_q, num_heads, head_dim, dtype=compute_dtype)
    cu = cu_seqlens_q.reshape(-1).tolist()
    for b in range(len(cu) - 1):
        ctx = int(context_lens[b])
        for q in range(cu[b], cu[b + 1]):
            n = max(0, min(ctx, int(positions[q]) + 1, max_blocks * block_size))
            t = torch.arange(n)
            blk = block_tables[b, t // block_size].long() if n > 0 else torch.zeros(0, dtype=torch.long)
            ok = (blk >= 0) & (blk < num_blocks)
            t, blk = t[ok], blk[ok]
            if t.numel() == 0:
                out[q] = float("nan")
                continue
            K = kc[blk, t % block_size]  # (n, KVH, D)
            V = vc[blk, t % block_size]
            qv = query[q].to(compute_dtype).view(num_kv_heads, group, head_dim)
            s = torch.einsum("hgd,thd->hgt", qv, K) * scale
            p = torch.softmax(s, dim=-1)
            out[q] = torch.einsum("hgt,thd->hgd", p, V).reshape(num_heads, head_dim)
    return out


def allreduce_residual_rmsnorm_ref(partials, residual, weight, eps, dtype=torch.bfloat16):
    """The tensor-parallel all-reduce of RowParallelLinear.forward (linear.py:222-225)
    followed by LayerNorm.residual_rms_forward (layernorm.py:25-27):
      x = sum of the ranks' partials (rounded to dtype, as the all-reduced tensor is);
      s = x + residual (a dtype add: rounded); out = s / sqrt(mean(s^2) + eps) * weight,
    the normalisation in fp32 with one final rounding, as the reference's torch.compile'd
    rms_forward computes it on the GPU. partials: (N, T, H); residual may be None.
    Returns (out, s) in dtype."""
    x = partials[0].float()
    for i in range(1, partials.shape[0]):  # rank order, one fp32 add at a time
        x = x + partials[i].float()
    if partials.shape[0] > 1:
        x = x.to(dtype).float()
    s = x if residual is None else (x + residual.float()).to(dtype).float()
    out = s / torch.sqrt(s.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
    return out.to(dtype), s.to(dtype)
