"""Host-side logic that needs no GPU: row sharding, workload generators,
API argument validation (no CPU fallback), and the tier/cluster choice
arithmetic mirrored from fw_capi.cu."""
import numpy as np
import pytest
import torch

from fwloss_b200 import FWLoss, familywise_loss, workloads
from fwloss_b200.distributed import shard_rows


@pytest.mark.parametrize("B,W", [(4096, 1), (4096, 8), (8192, 8), (10, 3), (7, 8), (0, 2)])
def test_shard_rows_partitions(B, W):
    spans = [shard_rows(B, r, W) for r in range(W)]
    assert spans[0][0] == 0 and spans[-1][1] == B
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_workloads_are_deterministic_and_shaped():
    for name, rows in (("cfg0", None), ("cfg1", 64), ("cfg2", 4), ("cfg3", 128), ("cfg4", 3)):
        z1, y1 = workloads.make(name, rows=rows)
        z2, y2 = workloads.make(name, rows=rows)
        B, C = workloads.CONFIGS[name]
        assert z1.shape == (rows or B, C) and z1.dtype == torch.float32 and y1.dtype == torch.int64
        assert torch.equal(z1, z2) and torch.equal(y1, y2)
        assert int(y1.min()) >= 0 and int(y1.max()) < C


def test_cfg3_has_levels_and_signed_zeros():
    z, _ = workloads.make("cfg3", rows=512)
    vals = set(np.unique(z.numpy()).tolist())
    assert vals <= {-3.5, -2.5, -1.5, -0.5, 0.0, 0.5, 1.5, 2.5, 3.5}
    neg0 = torch.signbit(z) & (z == 0)
    assert neg0.any() and ((z == 0) & ~torch.signbit(z)).any()


def test_cfg4_blocks_compose():
    a, ya = workloads.make_cfg4_rows(0, 2048, C=64)
    b, yb = workloads.make_cfg4_rows(1024, 2048, C=64)
    assert torch.equal(a[1024:], b) and torch.equal(ya[1024:], yb)


def test_cpu_tensors_are_rejected():
    with pytest.raises(TypeError):
        familywise_loss(torch.randn(3, 4), torch.zeros(3, dtype=torch.long))
    with pytest.raises(ValueError):
        familywise_loss(torch.randn(3, 4), torch.zeros(3, dtype=torch.long), reduction="max")
    with pytest.raises(ValueError):
        FWLoss(4, reduction="avg")


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("B,C", [(8192, 128256), (300, 20000), (64, 5000), (4096, 1000)])
def test_vocab_parallel_chunk_lists(world, fused, B, C):
    """The chunk list every rank derives for the vocabulary-parallel LM head:
    the same number of chunks per rank (the all-gathers need equal shapes),
    within the combined solve's limits, starting on 256-column tiles of each
    rank's own weight rows (fused kernel), covering [0, C) in order."""
    from fwloss_b200.lm_head import FUSED_TILE
    from fwloss_b200.sharded import even_col_start
    from fwloss_b200.vocab_parallel import (LIST_CAP, MAX_CHUNKS, chunks_per_rank, global_chunk_starts,
                                            local_chunk_starts)

    K = 16
    if C // world < 1 or K * world > LIST_CAP:
        pytest.skip("shape outside the supported range")
    cs = even_col_start(C, world)
    n = chunks_per_rank(world, B, cs, K, fused, 148)
    assert 1 <= n and n * world <= MAX_CHUNKS and n * world * K <= LIST_CAP
    for q in range(world):
        loc = local_chunk_starts(cs[q + 1] - cs[q], n, fused)
        assert len(loc) - 1 == n and loc[0] == 0 and loc[-1] == cs[q + 1] - cs[q]
        assert all(b > a for a, b in zip(loc, loc[1:]))
        if fused:
            assert all(c % FUSED_TILE == 0 for c in loc[:-1])
    g = global_chunk_starts(cs, n, fused)
    assert len(g) == world * n + 1 and g[0] == 0 and g[-1] == C
    assert all(b > a for a, b in zip(g, g[1:]))
    assert set(cs[:-1]) <= set(g)
