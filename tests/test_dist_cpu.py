"""The N > 1 host path on CPU with world_size-2 gloo process groups: the
sequence-shard exchange and merge equals one pass over the whole history,
and step timings reduce to the slowest rank.  No GPU is used."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oscar_oracle as orc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    return dist


def _case():
    """One cache-only query (sees every history key), 2048 history tokens, INT2 caches by the oracle store."""
    from oscar_b200.synthetic import make_case

    case = make_case([2048], [1], fresh=False, window=False, seed=5)
    k8 = case.kc.view(torch.uint8).numpy().copy()
    v8 = case.vc.view(torch.uint8).numpy().copy()
    orc.store(case.old_k.numpy(), case.old_v.numpy(), k8, v8, case.slots.numpy())
    return case, k8, v8


def _shard_worker(rank, world, port, result):
    dist = _init(rank, world, port)
    from oscar_b200 import shards

    case, k8, v8 = _case()
    bs = case.kc.shape[1]
    lo, hi = shards.page_shards(2048, bs, world)[rank]
    bt = case.bt.numpy()[:, lo // bs: -(-hi // bs)].copy()
    q = case.q.float().numpy()
    out, lse = orc.streaming_attention(q, None, None, k8, v8, bt, [0, 1], [hi - lo], case.scale, None, dtype="bf16")
    outs, lses = shards.exchange_partials(torch.from_numpy(out), torch.from_numpy(lse))

    def merge(o, l, p, pl):
        ov, lv = o.numpy(), l.numpy()
        orc.merge_slab(ov, lv, p.numpy(), pl.numpy(), 0)

    mo, ml = shards.merge_partials(outs, lses, merge)
    if rank == 0:
        whole, whole_lse = orc.streaming_attention(q, None, None, k8, v8, case.bt.numpy(), [0, 1], [2048], case.scale,
                                                   None, dtype="bf16")
        result["err_out"] = float(np.abs(mo.numpy() - whole).max())
        result["err_lse"] = float(np.abs(ml.numpy() - whole_lse).max())
    dist.destroy_process_group()


def _max_worker(rank, world, port, result):
    dist = _init(rank, world, port)
    from oscar_b200 import shards

    result[f"max{rank}"] = shards.max_over_ranks(1.5 + rank)
    dist.destroy_process_group()


def _spawn(fn, world=2):
    port = _free_port()
    with mp.Manager() as m:
        result = m.dict()
        mp.start_processes(fn, args=(world, port, result), nprocs=world, join=True, start_method="spawn")
        return dict(result)


def test_page_shards_cover_the_history_once():
    from oscar_b200.shards import page_shards

    for prefix, bs, world in ((2048, 128, 2), (3000, 128, 4), (100, 16, 8), (0, 128, 2)):
        sh = page_shards(prefix, bs, world)
        assert len(sh) == world
        assert sh[0][0] == 0 and sh[-1][1] == prefix
        for (a, b), (c, _) in zip(sh, sh[1:]):
            assert b == c and a % bs == 0 and a <= b
    with pytest.raises(ValueError):
        page_shards(10, 0, 2)


def test_sequence_shards_exchanged_over_gloo_merge_to_one_pass():
    r = _spawn(_shard_worker)
    assert r["err_out"] < 2e-5 and r["err_lse"] < 2e-5, r


def test_step_time_is_the_slowest_ranks():
    r = _spawn(_max_worker)
    assert r["max0"] == r["max1"] == 2.5
