"""Host-side logic without a GPU: forward context, decode metadata, KV-cache layout,
KV-head sharding (with a 2-rank gloo group), and the workload builders' metadata."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import mkv_module

ctx_mod = mkv_module("utils.context")
kv = mkv_module("engine.kv_cache")


def test_context_roundtrip():
    ctx_mod.set_context(False, slot_mapping=torch.tensor([3]), context_lens=torch.tensor([4]),
                        block_tables=torch.tensor([[0]]))
    c = ctx_mod.get_context()
    assert not c.is_prefill and int(c.slot_mapping[0]) == 3 and int(c.context_lens[0]) == 4
    ctx_mod.reset_context()
    assert ctx_mod.get_context().slot_mapping is None


def test_mixed_split_metadata():
    # reference context.py:55-88: decode seqs 0 and 2, prefill seq 1 with 3 tokens
    s = ctx_mod.split_mixed_decode_prefill_metadata([0, 1, 4, 5], [1, 3, 1], [True, False, True])
    assert s.decode_token_indices == [0, 4] and s.decode_seq_indices == [0, 2]
    assert s.prefill_token_indices == [1, 2, 3] and s.prefill_seq_indices == [1]
    assert s.prefill_cu_seqlens_q == [0, 3]


def test_decode_metadata_matches_prepare_decode():
    # model_runner.py:631-671 with block_size 4: lengths include the new token
    m = kv.decode_metadata([[7, 2, 9], [5], [1, 3]], [9, 4, 5], 4, device="cpu")
    assert m.slot_mapping.tolist() == [9 * 4 + 0, 5 * 4 + 3, 3 * 4 + 0]
    assert m.context_lens.tolist() == [9, 4, 5] and m.context_lens.dtype == torch.int64
    assert m.block_tables.tolist() == [[7, 2, 9], [5, -1, -1], [1, 3, -1]]
    assert m.block_tables.dtype == torch.int32
    with pytest.raises(ValueError):
        kv.decode_metadata([[1]], [5], 4, device="cpu")


def test_allocate_and_bind_kv_cache():
    attn_mod = mkv_module("layers.attention")
    layers = torch.nn.ModuleList([attn_mod.Attention(4, 16, num_kv_heads=2, block_size=4)
                                  for _ in range(3)])
    cache = kv.allocate_kv_cache(3, 5, 4, 2, 16, "fp8_per_tensor", device="cpu")
    assert cache.kv.shape == (2, 3, 5, 4, 2, 16) and cache.kv.dtype == torch.float8_e4m3fn
    assert kv.bind_kv_cache(layers.modules(), cache) == 3
    assert layers[1].k_cache.data_ptr() == cache.kv[0, 1].data_ptr()
    assert float(layers[2].v_scale[0]) == 1.0 and layers[0].kv_cache_dtype == "fp8_per_tensor"
    with pytest.raises(NotImplementedError):
        kv.allocate_kv_cache(1, 1, 4, 1, 16, "kivi_4bit", device="cpu")


@pytest.mark.parametrize("mode,dtype", [("fp8_per_token_head", torch.float8_e4m3fn),
                                        ("int8_per_token_head", torch.int8)])
def test_allocate_per_token_head_scales(mode, dtype):
    """Per-(token, head) modes: (2, L, NB, BS, KVH) float32 scales at 1.0 beside the 8-bit
    pages, and layer l's (NB, BS, KVH) views bound to the l-th attention module
    (model_runner.py:330-338, 376-395)."""
    attn_mod = mkv_module("layers.attention")
    layers = torch.nn.ModuleList([attn_mod.Attention(4, 16, num_kv_heads=2, block_size=4)
                                  for _ in range(3)])
    cache = kv.allocate_kv_cache(3, 5, 4, 2, 16, mode, device="cpu")
    assert cache.kv.shape == (2, 3, 5, 4, 2, 16) and cache.kv.dtype == dtype
    assert cache.k_scale.shape == (3, 5, 4, 2) and cache.k_scale.dtype == torch.float32
    assert bool((cache.k_scale == 1).all()) and bool((cache.v_scale == 1).all())
    assert kv.bind_kv_cache(layers.modules(), cache) == 3
    assert layers[2].k_scale.shape == (5, 4, 2) and layers[2].k_scale.is_contiguous()
    assert layers[1].v_scale.data_ptr() == cache.v_scale[1].data_ptr()
    assert layers[0].kv_cache_dtype == mode


def test_kv_head_shard_ranges():
    owned_q, owned_kv = set(), set()
    for r in range(4):
        qh, kvh = kv.kv_head_shard(32, 8, r, 4)
        assert all(h // 4 in kvh for h in qh)  # every query head's kv head is local
        owned_q |= set(qh)
        owned_kv |= set(kvh)
    assert owned_q == set(range(32)) and owned_kv == set(range(8))
    with pytest.raises(ValueError):
        kv.kv_head_shard(32, 8, 0, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    kvm = mkv_module("engine.kv_cache")
    qh, kvh = kvm.kv_head_shard(16, 8, rank, world)
    # each rank reports its heads and a per-rank "time"; the job aggregates like bench.py:
    # total work = sum over ranks, elapsed = max over ranks
    heads = torch.zeros(16)
    heads[list(qh)] = 1
    dist.all_reduce(heads)
    t = torch.tensor([1.0 + rank])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out[rank] = (heads.tolist(), float(t))
    dist.destroy_process_group()


def test_kv_head_sharding_two_ranks_gloo():
    port = _free_port()
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.start_processes(_shard_worker, args=(2, port, out), nprocs=2, start_method="spawn")
        for r in range(2):
            heads, t = out[r]
            assert heads == [1.0] * 16  # every query head owned exactly once
            assert t == 2.0


def test_engine_harness_sequence_state_for_workers():
    """The config-5 harness's fix for the reference's tensor-parallel workers: a Sequence
    that crosses the runner's shared-memory RPC (pickle) keeps block_size, and the
    worker's last-block token count (the decode slot of model_runner.py:639) equals rank
    0's at every length, page boundaries included. Uses the reference's own Sequence;
    skipped when the reference is not installed."""
    import importlib
    import pickle

    from conftest import REPO
    if not os.path.isdir(os.path.join(REPO, "baseline", "_ref", "myvllm")):
        pytest.skip("reference not installed in baseline/_ref")
    be = importlib.import_module("mini-kvllm_b200.bench_engine")
    from myvllm.engine.sequence import Sequence
    bs = 16
    seq = Sequence(token_ids=list(range(37)), block_size=bs)
    with pytest.raises(AttributeError):  # the unmodified round trip loses block_size
        getattr(pickle.loads(pickle.dumps(seq)), "block_size")
    be.sequence_state_for_workers(bs)
    for n_out in range(0, 3 * bs):
        if n_out:
            seq.append_token(1000 + n_out)
        rank0 = len(seq.token_ids[seq.num_tokens // bs * bs:])  # sequence.py:80-82 on rank 0
        worker = pickle.loads(pickle.dumps(seq))
        assert worker.block_size == bs
        assert worker.num_tokens == seq.num_tokens
        assert seq.last_block_num_tokens == rank0
        assert worker.last_block_num_tokens == rank0
