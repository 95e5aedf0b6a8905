"""DecodeMetadataBuilder (one copy + `mkv_decode_metadata` per step) against
decode_metadata, the restatement of ModelRunner.prepare_decode (model_runner.py:631-671):
slot mapping, context lengths and block tables bit-exact, over incremental appends and
a shuffled batch order."""
import random

import pytest
import torch

from conftest import mkv_module

pytestmark = pytest.mark.gpu
kvc = mkv_module("engine.kv_cache")


def _expect(tables, lens, bs):
    ref = kvc.decode_metadata(tables, lens, bs, device="cuda")
    return ref.slot_mapping.cpu(), ref.context_lens.cpu(), ref.block_tables.cpu()


@pytest.mark.parametrize("bs", [16, 256])
def test_builder_matches_prepare_decode(bs):
    rng = random.Random(bs)
    S, W = 40, 24
    b = kvc.DecodeMetadataBuilder(max_seqs=S, max_blocks=W, block_size=bs)
    lens, tables = {}, {}
    free = list(range(10_000))
    rng.shuffle(free)
    for s in range(S):
        n = rng.randint(1, bs * 8)
        tables[s] = [free.pop() for _ in range((n + bs - 1) // bs)]
        lens[s] = n
        b.set_table(s, tables[s])
    for step in range(12):
        order = list(range(S))
        rng.shuffle(order)
        order = order[: rng.randint(1, S)]
        md = b.step(order, [lens[s] for s in order])
        slots, ctx, bt = _expect([tables[s] for s in order], [lens[s] for s in order], bs)
        torch.cuda.synchronize()
        assert torch.equal(md.slot_mapping.cpu(), slots)
        assert torch.equal(md.context_lens.cpu(), ctx)
        got = md.block_tables.cpu()
        assert torch.equal(got[:, : bt.shape[1]], bt)
        assert bool((got[:, bt.shape[1]:] == -1).all())
        # every sequence decodes one token; a full last block takes a new one
        for s in range(S):
            if lens[s] % bs == 0 and len(tables[s]) < W:
                blk = free.pop()
                tables[s].append(blk)
                b.append(s, blk)
            if lens[s] < len(tables[s]) * bs:
                lens[s] += 1


def test_missing_page_gives_skip_slot():
    b = kvc.DecodeMetadataBuilder(max_seqs=2, max_blocks=4, block_size=16)
    b.set_table(0, [5, -1])
    b.set_table(1, [7])
    md = b.step([0, 1], [20, 3])
    torch.cuda.synchronize()
    assert md.slot_mapping.cpu().tolist() == [-1, 7 * 16 + 2]
    assert md.context_lens.cpu().tolist() == [20, 3]
