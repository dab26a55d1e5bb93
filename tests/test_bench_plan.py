"""Host logic of bench.py's multi-GPU partitioning (no GPU): every (KV-head
group, request) unit of the global step is served by exactly one rank, the
8-rank request halves of cfg5 carry equal history, and the cfg5 step cycle
rewrites rejected MTP positions within the pages it allocates."""
import numpy as np
import pytest

import bench


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_plan_covers_every_unit_once(world):
    seen = {}
    for rank in range(world):
        p = bench.shard_plan(world, rank, 8)
        for g in range(p.g0, p.g1):
            for r in range(p.r0, p.r1):
                assert (g, r) not in seen
                seen[(g, r)] = rank
    assert set(seen) == {(g, r) for g in range(bench.GROUPS) for r in range(8)}


def test_shard_plan_rejects_uneven_worlds():
    for world in (3, 6):
        with pytest.raises(SystemExit):
            bench.shard_plan(world, 0, 8)


def test_pairs_at_eight_ranks():
    plans = [bench.shard_plan(8, r, 8) for r in range(8)]
    for p in plans:
        assert p.splits == 2 and len(p.pair) == 2
        assert all(plans[q].g0 == p.g0 for q in p.pair)
    assert [p.split for p in plans] == [0, 1] * 4


def test_cfg5_request_halves_are_balanced():
    prefixes, _ = bench.cfg5_schedule()
    plans = [bench.shard_plan(8, r, 8) for r in range(2)]
    (a0, a1), (b0, b1) = (bench.cfg5_requests(prefixes, p) for p in plans)
    assert a0 == 0 and a1 == b0 and b1 == len(prefixes)
    h0, h1 = sum(prefixes[a0:a1]), sum(prefixes[b0:b1])
    assert abs(h0 - h1) <= max(prefixes)
    assert bench.cfg5_requests(prefixes, bench.shard_plan(4, 0, 8)) == (0, len(prefixes))


def test_cfg5_schedule_rewrites_rejected_positions():
    prefixes, steps = bench.cfg5_schedule()
    assert len(prefixes) == 64 and len(steps) >= 3
    base0 = steps[0][0]
    assert base0 == prefixes
    for (base, lengths), (nxt, _) in zip(steps, steps[1:]):
        for b, ln, b2 in zip(base, lengths, nxt):
            assert 1 <= ln <= 4
            assert b + 1 <= b2 <= b + ln  # 1..len accepted: the next step starts inside the rejected tail
    for base, lengths in steps:
        # within the 16 tokens of page headroom the cfg5 caches are built with
        assert all(b + ln <= p + 16 for b, ln, p in zip(base, lengths, prefixes))
    assert any(b2 < b + ln for (base, lengths), (nxt, _) in zip(steps, steps[1:])
               for b, ln, b2 in zip(base, lengths, nxt)), "no step rewrites a rejected position"


def test_shifted_table_and_page_shards():
    torch = pytest.importorskip("torch")
    from oscar_b200.shards import page_shards

    bt = torch.arange(2 * 200, dtype=torch.int32).reshape(2, 200)
    lo, hi = page_shards(24576, 128, 2)[1]
    assert (lo, hi) == (12288, 24576)
    t = bench.shifted_table(torch, bt, lo // 128)
    assert torch.equal(t[:, :104], bt[:, 96:])
    assert int(t[:, 104:].abs().sum()) == 0
    assert np.array_equal(t[1, :3].numpy(), [296, 297, 298])
