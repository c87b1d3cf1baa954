"""CPU oracle for the fused collectives' schedules (nuvla_forge_b200/parallel/emulate.py)."""

import random

import numpy as np
import pytest

from nuvla_forge_b200.parallel import emulate as em


def _ref_sum(srcs, scale):
    return sum(em.bf16_round(s) for s in srcs) * np.float32(scale)


@pytest.mark.parametrize("world,n,ctas", [(2, 16, 1), (2, 8 * 2 * 1000, 48), (4, 8 * 4 * 131, 7),
                                          (8, 8 * 8 * 999, 132), (3, 8 * 3 * 5, 16)])
def test_two_shot_allreduce_schedule(world, n, ctas):
    rng = np.random.default_rng(n + world)
    srcs = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    outs = em.two_shot_allreduce(srcs, ctas, 1.0 / world)
    ref = em.bf16_round(_ref_sum(srcs, 1.0 / world))
    for o in outs:
        np.testing.assert_allclose(o, ref, rtol=0, atol=1e-6)


@pytest.mark.parametrize("world,n,ctas,chunk", [(2, 8 * 2 * 100, 3, 7), (4, 8 * 4 * 64, 5, 4), (8, 8 * 8 * 40, 4, 3),
                                                (3, 8 * 3 * 10, 16, 1)])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_pipelined_allreduce_random_interleavings(world, n, ctas, chunk, seed):
    """Three back-to-back launches, ranks and CTAs interleaved at random: no deadlock, no stale read."""
    rng = np.random.default_rng(seed + world)
    launches = [[rng.standard_normal(n).astype(np.float32) for _ in range(world)] for _ in range(3)]
    outs = em.pipelined_allreduce(launches, ctas, chunk, 1.0 / world, seed=seed)
    for srcs, got in zip(launches, outs):
        ref = em.bf16_round(_ref_sum(srcs, 1.0 / world))
        for o in got:
            np.testing.assert_allclose(o, ref, rtol=0, atol=1e-6)


@pytest.mark.parametrize("world,n,ctas", [(2, 64, 3), (8, 8 * 8 * 77, 16)])
def test_one_shot_allreduce_schedule(world, n, ctas):
    rng = np.random.default_rng(world)
    srcs = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    outs = em.one_shot_allreduce(srcs, ctas, 0.5)
    ref = _ref_sum(srcs, 0.5)
    for o in outs:
        np.testing.assert_allclose(o, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("world,n,ctas", [(2, 8 * 2 * 100, 32), (4, 8 * 4 * 1001, 32), (8, 8 * 8 * 50, 200)])
def test_reduce_scatter_push_schedule(world, n, ctas):
    rng = np.random.default_rng(world * n)
    srcs = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    shards = em.reduce_scatter_push(srcs, ctas, 1.0 / world)
    ref = _ref_sum(srcs, 1.0 / world)
    sv = n // world
    for r, s in enumerate(shards):
        np.testing.assert_allclose(s, ref[r * sv:(r + 1) * sv], rtol=1e-6, atol=1e-6)


def test_bf16_round_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(em.bf16_round(x), want)


def test_ag_gemm_schedule_covers_unit_once_weight_first():
    rng = random.Random(1)
    for _ in range(60):
        world = rng.choice([1, 2, 4, 8])
        shard = 16 * rng.randint(1, 40000)
        total = shard * world
        lo = 16 * rng.randint(0, total // 64)
        wb = 16 * rng.randint(1, max(1, (total - lo) // 32))
        w0 = lo + 16 * rng.randint(0, (total - lo - wb) // 16)
        grid = rng.choice([1, 7, 148])
        for order in (em.ORDER_FLAT, em.ORDER_OWN_FIRST, em.ORDER_PEERS_FIRST, em.ORDER_INTERLEAVED):
            for rank in range(world):
                per_cta = em.ag_gemm_schedule(shard, world, rank, lo, total, w0, wb, grid, order)
                pieces = sorted(p for cta in per_cta for p in cta)
                pos = lo
                for q, f0, f1 in pieces:
                    assert f0 == pos, (order, rank, "gap or overlap")
                    assert q * shard <= f0 < f1 <= (q + 1) * shard
                    pos = f1
                assert pos == total
                if order != em.ORDER_FLAT:
                    # every CTA issues all its W-overlapping chunks before any other chunk
                    for cta in per_cta:
                        seen_rest = False
                        for q, f0, f1 in cta:
                            overlaps_w = f0 < w0 + wb and f1 > w0
                            assert not (overlaps_w and seen_rest)
                            seen_rest |= not overlaps_w
