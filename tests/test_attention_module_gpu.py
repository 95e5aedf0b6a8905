"""`Attention.forward` on a mixed batch (attention.py:1617-1807): the step's K/V are
appended, decode rows go through the decode kernels and prefill rows through the paged
prefill, each over the same cache (attention.py:1711-1760). Checked against the oracle's
paged prefill over the post-append cache, a decode row being a one-token chunk.

Tolerance: bf16 queries, atol 2e-2 / rtol 1e-2."""
import math

import pytest
import torch

from conftest import mkv_module
from oracle import paged_prefill_ref

pytestmark = pytest.mark.gpu
attn_mod = mkv_module("layers.attention")
ctx_mod = mkv_module("utils.context")

H, KVH, D, BS = 16, 4, 128, 16


def build(mode, seed=0):
    g = torch.Generator().manual_seed(seed)
    # (context after this step, new tokens this step, decode?)
    seqs = [(70, 1, True), (300, 37, False), (5, 1, True), (200, 200, False), (129, 1, True)]
    need = [(c + BS - 1) // BS for c, _, _ in seqs]
    nb = sum(need) + 4
    perm = torch.randperm(nb, generator=g)
    bt = torch.full((len(seqs), max(need)), -1, dtype=torch.int32)
    pos = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[pos:pos + k].int()
        pos += k
    raw = torch.randn(2, nb, BS, KVH, D, generator=g)
    if mode == "auto":
        kc, vc = raw[0].bfloat16(), raw[1].bfloat16()
        ks = vs = None
    elif mode == "fp8_per_tensor":
        kc, vc = (raw[0] * 40).to(torch.float8_e4m3fn), (raw[1] * 40).to(torch.float8_e4m3fn)
        ks, vs = torch.tensor([0.05]), torch.tensor([0.04])  # not the 1.0 sentinel: no calibration
    else:
        kc = (raw[0] * 40).round().clamp(-127, 127).to(torch.int8)
        vc = (raw[1] * 40).round().clamp(-127, 127).to(torch.int8)
        ks = torch.rand(nb, BS, KVH, generator=g) * 0.04 + 0.002
        vs = torch.rand(nb, BS, KVH, generator=g) * 0.04 + 0.002
    q_lens = [n for _, n, _ in seqs]
    cu = [0]
    for n in q_lens:
        cu.append(cu[-1] + n)
    positions = torch.cat([torch.arange(c - n, c) for c, n, _ in seqs])
    slots = torch.cat([bt[b, positions[cu[b]:cu[b + 1]] // BS].long() * BS + positions[cu[b]:cu[b + 1]] % BS
                       for b in range(len(seqs))])
    T = cu[-1]
    q = torch.randn(T, H, D, generator=g).bfloat16()
    k = torch.randn(T, KVH, D, generator=g).bfloat16()
    v = torch.randn(T, KVH, D, generator=g).bfloat16()
    return dict(seqs=seqs, bt=bt, kc=kc, vc=vc, ks=ks, vs=vs, cu=cu, q_lens=q_lens,
                positions=positions, slots=slots, q=q, k=k, v=v)


@pytest.mark.parametrize("mode", ["auto", "fp8_per_tensor", "int8_per_token_head"])
def test_mixed_batch_forward_matches_oracle(mode):
    c = build(mode)
    dev = torch.device("cuda")
    layer = attn_mod.Attention(H, D, num_kv_heads=KVH, block_size=BS)
    layer.k_cache, layer.v_cache = c["kc"].to(dev), c["vc"].to(dev)
    layer.kv_cache_dtype = mode
    if c["ks"] is not None:
        layer.k_scale, layer.v_scale = c["ks"].to(dev), c["vs"].to(dev)
    is_dec = [d for _, _, d in c["seqs"]]
    split = ctx_mod.split_mixed_decode_prefill_metadata(c["cu"], c["q_lens"], is_dec)
    as_t = lambda x, dt=torch.int64: torch.tensor(x, dtype=dt, device=dev)
    split.decode_token_indices_tensor = as_t(split.decode_token_indices)
    split.decode_seq_indices_tensor = as_t(split.decode_seq_indices)
    split.prefill_token_indices_tensor = as_t(split.prefill_token_indices)
    split.prefill_seq_indices_tensor = as_t(split.prefill_seq_indices)
    split.prefill_cu_seqlens_q_tensor = as_t(split.prefill_cu_seqlens_q, torch.int32)
    cl = torch.tensor([ctx for ctx, _, _ in c["seqs"]], dtype=torch.int64)
    ctx_mod.set_context(True, cu_seqlens_q=as_t(c["cu"], torch.int32), slot_mapping=c["slots"].to(dev),
                        context_lens=cl.to(dev), block_tables=c["bt"].to(dev),
                        positions=c["positions"].to(dev), query_lens=as_t(c["q_lens"]),
                        is_decode=torch.tensor(is_dec, device=dev), mixed_attention_split=split)
    try:
        out = layer(c["q"].to(dev), c["k"].to(dev), c["v"].to(dev))
        torch.cuda.synchronize()
    finally:
        ctx_mod.reset_context()
    assert out.shape == (c["q"].shape[0], H * D)
    # the oracle attends over the cache as the step left it (the append is checked
    # bit-exact elsewhere)
    kc, vc = layer.k_cache.cpu(), layer.v_cache.cpu()
    scale = 1.0 / math.sqrt(D)
    cu = torch.tensor(c["cu"], dtype=torch.int32)
    if mode == "auto":
        ref = paged_prefill_ref(c["q"], kc, vc, c["bt"], cl, cu, c["positions"], scale, H, KVH, BS)
    elif mode == "fp8_per_tensor":
        ref = paged_prefill_ref(c["q"], kc, vc, c["bt"], cl, cu, c["positions"], scale, H, KVH, BS,
                                k_scale=layer.k_scale.cpu(), v_scale=layer.v_scale.cpu())
    else:
        ref = paged_prefill_ref(c["q"], kc, vc, c["bt"], cl, cu, c["positions"], scale, H, KVH, BS,
                                k_scales=layer.k_scale.cpu(), v_scales=layer.v_scale.cpu())
    diff = (out.cpu().double().view_as(ref) - ref).abs()
    assert bool((diff <= 2e-2 + 1e-2 * ref.abs()).all()), f"max abs err {float(diff.max()):.3e}"
    # decode rows equal a decode call over the same cache
    di = split.decode_token_indices_tensor
    ds = split.decode_seq_indices_tensor
    if mode == "auto":
        dec = attn_mod.paged_attention_decode(c["q"].to(dev)[di], layer.k_cache, layer.v_cache,
                                              c["bt"].to(dev)[ds], cl.to(dev)[ds], scale, H, KVH, D, BS)
    else:
        dec = attn_mod.paged_attention_decode_quantized(c["q"].to(dev)[di], layer.k_cache, layer.v_cache,
                                                        layer.k_scale, layer.v_scale, c["bt"].to(dev)[ds],
                                                        cl.to(dev)[ds], scale, H, KVH, D, BS, mode)
    assert torch.equal(out[di].view(-1, H, D), dec)
