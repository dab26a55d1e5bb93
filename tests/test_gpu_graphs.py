"""CUDA-graph replay of the backend forward gives the eager forward's output
and leaves the same staging window (graph-safe staging write)."""
from types import SimpleNamespace as NS

import pytest
import torch

from gpu_helpers import need_gpu

pytestmark = pytest.mark.gpu


def _layer_setup(dev, seed):
    from oscar_b200 import synthetic
    from oscar_b200.backend import OscarAttentionBackendImpl

    impl = OscarAttentionBackendImpl.create(6, 1, 256)
    cfg = impl._oscar
    cfg.sink_tokens, cfg.recent_tokens, cfg.staging_tokens = 128, 256, 4096
    cfg.window_enabled = True
    case = synthetic.make_case([3000, 1000], [4, 4], hk=1, group=6, seed=seed, device=dev)
    synthetic.fill_caches(case)
    g = torch.Generator(device=dev).manual_seed(seed)
    rk = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
    rv = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
    layer = NS(layer_name="model.layers.0.self_attn.attn", _oscar_rots=(rk, rv))
    cache = (case.kc, case.vc)
    slots = []
    for r, (p, n) in enumerate(zip([3000, 1000], [4, 4])):
        pos = torch.arange(p, p + n, device=dev)
        slots.append(case.bt[r, pos // 128].long() * 128 + pos % 128)
    md = NS(num_actual_tokens=8, slot_mapping=torch.cat(slots), query_start_loc_cpu=torch.tensor(case.qsl),
            seq_lens_list=case.seqs, block_tables=case.bt,
            query_start_loc=torch.tensor(case.qsl, dtype=torch.int32, device=dev),
            seq_lens=torch.tensor(case.seqs, dtype=torch.int32, device=dev))
    return impl, layer, case, cache, md


def test_graph_replay_matches_eager_forward():
    from oscar_b200.graphs import GraphedForward

    dev = need_gpu()
    impl, layer, case, cache, md = _layer_setup(dev, 31)
    out = torch.empty(8, 6 * 256, dtype=torch.bfloat16, device=dev)
    gf = GraphedForward(impl, layer, case.q, case.k_new, case.v_new, cache, md, out)
    # new inputs written into the static tensors, then replayed
    q2, k2, v2 = torch.randn_like(case.q.float()).bfloat16(), torch.randn_like(case.k_new.float()).bfloat16(), \
        torch.randn_like(case.v_new.float()).bfloat16()
    case.q.copy_(q2)
    case.k_new.copy_(k2)
    case.v_new.copy_(v2)
    got = gf.replay().clone()
    want = torch.empty_like(out)
    impl.forward(layer, case.q, case.k_new, case.v_new, cache, md, output=want)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), want.float(), atol=0, rtol=0)


def test_graph_replay_leaves_staging_window_as_eager_forward():
    """Graph capture runs the graph-safe staging write (scratch cleared per
    call); after the same number of forwards the window matches the eager one."""
    from oscar_b200.graphs import GraphedForward

    dev = need_gpu()
    impl_g, layer_g, case_g, cache_g, md_g = _layer_setup(dev, 41)
    impl_e, layer_e, case_e, cache_e, md_e = _layer_setup(dev, 41)
    out = torch.empty(8, 6 * 256, dtype=torch.bfloat16, device=dev)
    gf = GraphedForward(impl_g, layer_g, case_g.q, case_g.k_new, case_g.v_new, cache_g, md_g, out)
    for t in range(2):
        impl_e.forward(layer_e, case_e.q, case_e.k_new, case_e.v_new, cache_e, md_e, output=torch.empty_like(out))
    want = torch.empty_like(out)
    impl_e.forward(layer_e, case_e.q, case_e.k_new, case_e.v_new, cache_e, md_e, output=want)
    got = gf.replay().clone()
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), want.float(), atol=0, rtol=0)
    assert torch.equal(layer_g._oscar_slot_owner, layer_e._oscar_slot_owner)
    assert torch.equal(layer_g._oscar_stage_k, layer_e._oscar_stage_k)


def test_graphed_sequence_of_layers_matches_eager_forwards():
    """Two layers captured in one graph (layer A, layer B, layer A again): the
    replay gives each eager forward's output, in order, with the second A step
    seeing the staging window the first one left."""
    from oscar_b200.graphs import GraphedSequence

    dev = need_gpu()
    impl_a, layer_a, case_a, cache_a, md_a = _layer_setup(dev, 51)
    impl_b, layer_b, case_b, cache_b, md_b = _layer_setup(dev, 52)
    ea = _layer_setup(dev, 51)
    eb = _layer_setup(dev, 52)
    outs = [torch.empty(8, 6 * 256, dtype=torch.bfloat16, device=dev) for _ in range(3)]
    seq = GraphedSequence([(impl_a, layer_a, case_a.q, case_a.k_new, case_a.v_new, cache_a, md_a, outs[0]),
                           (impl_b, layer_b, case_b.q, case_b.k_new, case_b.v_new, cache_b, md_b, outs[1]),
                           (impl_a, layer_a, case_a.q, case_a.k_new, case_a.v_new, cache_a, md_a, outs[2])])
    # the capture's warm-up ran one eager forward per distinct layer
    for impl, layer, case, cache, md in (ea, eb):
        impl.forward(layer, case.q, case.k_new, case.v_new, cache, md, output=torch.empty_like(outs[0]))
    seq.replay()
    want = [torch.empty_like(outs[0]) for _ in range(3)]
    for w, (impl, layer, case, cache, md) in zip(want, (ea, eb, ea)):
        impl.forward(layer, case.q, case.k_new, case.v_new, cache, md, output=w)
    torch.cuda.synchronize()
    for g, w in zip(outs, want):
        torch.testing.assert_close(g.float(), w.float(), atol=0, rtol=0)
    assert torch.equal(layer_a._oscar_slot_owner, ea[1]._oscar_slot_owner)
