"""Split-KV history shards (the multi-GPU exchange's math on one GPU).

A request's paged history is cut at a page boundary into a head shard
[0, h0) and a tail shard [h0, prefix).  The owner computes the head shard
together with the causal current chunk (``slab_attention`` with
seq = h0 + q_len), the other rank the tail shard alone
(``slab_attention_shard`` over the block-table row shifted by h0 pages);
``merge_slab`` combines the two partials.  The result must equal the
single-pass ``slab_attention`` over the whole history and the oracle
(the sequential slab merge of kernels/slab_attention.py:458-475 and
merge_slab :341-373).
"""
import numpy as np
import pytest
import torch

from gpu_helpers import LSE_TOL, OUT_TOL, need_gpu
from oracle import oscar_oracle as orc

pytestmark = pytest.mark.gpu

BS = 128


def shard_split(prefixes, mode):
    """Page-aligned split point of each request's history."""
    if mode == "half":
        return [(p // 2) // BS * BS for p in prefixes]
    return [p // BS * BS for p in prefixes]  # "floor": tail shorter than a page (or empty)


def shifted_table(bt, h0):
    """Block-table rows that start at page h0[r] / BS (zero padded)."""
    out = torch.zeros_like(bt)
    for r, h in enumerate(h0):
        k = h // BS
        out[r, :bt.shape[1] - k] = bt[r, k:]
    return out


@pytest.mark.parametrize("path", ["auto", "decode"])
@pytest.mark.parametrize("mode", ["half", "floor"])
def test_two_history_shards_merge_to_the_single_pass(path, mode):
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, make_case

    dev = need_gpu()
    prefixes, lengths = [3000, 2560, 700, 130, 0], [4, 1, 2, 3, 2]
    case = make_case(prefixes, lengths, hk=2, group=6, seed=4242, device=dev)
    fill_caches(case)
    h0 = shard_split(prefixes, mode)
    kernels.set_attention_path(path)
    try:
        full_o, full_l = kernels.slab_attention(case.q, case.k_new, case.v_new, case.kc, case.vc, case.bt, case.qsl,
                                                case.seqs, case.scale, case.stage)
        head_o, head_l = kernels.slab_attention(case.q, case.k_new, case.v_new, case.kc, case.vc, case.bt, case.qsl,
                                                [h + n for h, n in zip(h0, lengths)], case.scale, case.stage)
        tail_o, tail_l = kernels.slab_attention_shard(case.q, case.kc, case.vc, shifted_table(case.bt, h0), case.qsl,
                                                      [p - h for p, h in zip(prefixes, h0)], case.scale, case.stage)
        kernels.merge_slab(head_o, head_l, tail_o, tail_l, 0, None)
        assert kernels.device_error(dev) == 0
    finally:
        kernels.set_attention_path("auto")
    np.testing.assert_allclose(head_o.cpu().numpy(), full_o.cpu().numpy(), **OUT_TOL)
    np.testing.assert_allclose(head_l.cpu().numpy(), full_l.cpu().numpy(), **LSE_TOL)
    # and against the oracle over the same bytes
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    stage = tuple(t.cpu().numpy() for t in case.stage)
    want_o, want_l = orc.streaming_attention(f(case.q), f(case.k_new), f(case.v_new),
                                             case.kc.view(torch.uint8).cpu().numpy(),
                                             case.vc.view(torch.uint8).cpu().numpy(), case.bt.cpu().numpy(), case.qsl,
                                             case.seqs, case.scale, stage)
    np.testing.assert_allclose(head_o.cpu().numpy(), want_o, **OUT_TOL)
    np.testing.assert_allclose(head_l.cpu().numpy(), want_l, **LSE_TOL)


def test_tail_shard_alone_matches_the_oracle_over_its_pages():
    """The tail shard is plain attention over its pages with every key visible."""
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, make_case

    dev = need_gpu()
    prefixes, lengths = [2048, 1000], [4, 4]
    case = make_case(prefixes, lengths, hk=1, group=6, seed=99, device=dev)
    fill_caches(case)
    h0 = [1024, 512]
    tail = [p - h for p, h in zip(prefixes, h0)]
    bt_t = shifted_table(case.bt, h0)
    o, lse = kernels.slab_attention_shard(case.q, case.kc, case.vc, bt_t, case.qsl, tail, case.scale, case.stage)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    # the oracle's cache-only form with q_len extra visible positions: every
    # query row sees keys [0, tail + i] of which only [0, tail) exist -- so
    # evaluate it one query row at a time with seq = tail (all keys visible)
    k8, v8 = case.kc.view(torch.uint8).cpu().numpy(), case.vc.view(torch.uint8).cpu().numpy()
    stage = tuple(t.cpu().numpy() for t in case.stage)
    q = f(case.q)
    for r in range(2):
        for t in range(case.qsl[r], case.qsl[r + 1]):
            wo, wl = orc.streaming_attention(q[t:t + 1], None, None, k8, v8, bt_t[r:r + 1].cpu().numpy(), [0, 1],
                                             [tail[r]], case.scale, stage)
            np.testing.assert_allclose(o[t].cpu().numpy(), wo[0], **OUT_TOL)
            np.testing.assert_allclose(lse[t].cpu().numpy(), wl[0], **LSE_TOL)


def test_shard_rejects_layouts_off_the_decode_kernels():
    from oscar_b200 import kernels
    from oscar_b200.synthetic import make_case

    dev = need_gpu()
    case = make_case([256], [8], hk=1, group=6, seed=5, device=dev)  # 48 query rows per KV head
    with pytest.raises(ValueError, match="decode kernels"):
        kernels.slab_attention_shard(case.q, case.kc, case.vc, case.bt, case.qsl, [256], case.scale, case.stage)
