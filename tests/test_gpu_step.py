"""The native decode layer step (oscar_decode_layer_step) against the
per-kernel forward of the same step: outputs, INT2 cache bytes and the
staging arena bit-identical, over three steps with MTP-reject rewrites, with
q / k / v as strided views of one fused QKV buffer and padded output rows."""
from types import SimpleNamespace as NS

import pytest
import torch

from gpu_helpers import need_gpu

pytestmark = pytest.mark.gpu


def make_impl(hq, hk, d):
    from oscar_b200.backend import OscarAttentionBackendImpl

    impl = OscarAttentionBackendImpl.create(hq, hk, d)
    cfg = impl._oscar
    cfg.sink_tokens, cfg.recent_tokens, cfg.staging_tokens = 128, 256, 2048
    cfg.k_clip_ratio, cfg.v_clip_ratio = 0.96, 0.92
    cfg.window_enabled = True
    return impl


def clone_state(case, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    rk = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
    rv = torch.linalg.qr(torch.randn(256, 256, generator=g, device=dev)).Q.contiguous()
    layer = NS(layer_name="model.layers.5.self_attn.attn", _oscar_rots=(rk, rv))
    return layer, (case.kc.clone(), case.vc.clone())


@pytest.mark.parametrize("rot_path", ["auto", "tensor"])
@pytest.mark.parametrize("fused_qkv", [False, True])
def test_native_step_equals_per_kernel_forward(fused_qkv, rot_path):
    """With rot_path "tensor" the rotations run on the tcgen05 kernel, whose
    row-heads addressing (strided q / k / v, the output's token stride) the
    native step uses and the per-kernel path does not."""
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, make_case

    dev = need_gpu()
    kernels.set_rotation_path(rot_path)
    try:
        _run_native_vs_per_kernel(dev, fused_qkv)
    finally:
        kernels.set_rotation_path("auto")


def _run_native_vs_per_kernel(dev, fused_qkv):
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, make_case

    hq, hk, d = 12, 2, 256
    prefixes = [3000, 700, 129, 2048]
    lengths = [4, 1, 3, 2]
    case = make_case(prefixes, lengths, hk=hk, group=hq // hk, seed=21, device=dev, staging_tokens=2048)
    fill_caches(case)
    impls, layers, caches = [], [], []
    for native in (True, False):
        impl = make_impl(hq, hk, d)
        impl._oscar_native_step = native
        layer, cache = clone_state(case, dev, 3)
        impl._set_caches(cache)
        impl._ensure_staging(layer, cache)
        for dst, src in zip((layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner), case.stage):
            dst.copy_(src)
        impls.append(impl)
        layers.append(layer)
        caches.append(cache)
    gen = torch.Generator(device=dev).manual_seed(8)
    base = list(prefixes)
    for step in range(3):
        qsl = [0]
        for ln in lengths:
            qsl.append(qsl[-1] + ln)
        n = qsl[-1]
        seqs = [b + ln for b, ln in zip(base, lengths)]
        pos = [(r, b + i) for r, (b, ln) in enumerate(zip(base, lengths)) for i in range(ln)]
        bt = case.bt
        slots = torch.tensor([int(bt[r, p // 128]) * 128 + p % 128 for r, p in pos], dtype=torch.int64, device=dev)
        if fused_qkv:
            qkv = torch.randn(n, (hq + 2 * hk) * d, generator=gen, device=dev).bfloat16()
            q, k, v = qkv[:, :hq * d], qkv[:, hq * d:(hq + hk) * d], qkv[:, (hq + hk) * d:]
        else:
            q = torch.randn(n, hq, d, generator=gen, device=dev).bfloat16()
            k = torch.randn(n, hk, d, generator=gen, device=dev).bfloat16()
            v = torch.randn(n, hk, d, generator=gen, device=dev).bfloat16()
        md = NS(num_actual_tokens=n, slot_mapping=slots, query_start_loc_cpu=torch.tensor(qsl), seq_lens_list=seqs,
                block_tables=bt, query_start_loc=torch.tensor(qsl, dtype=torch.int32, device=dev),
                seq_lens=torch.tensor(seqs, dtype=torch.int32, device=dev))
        outs = []
        for impl, layer, cache in zip(impls, layers, caches):
            out = torch.full((n + 3, hq * d), 7.0, dtype=torch.bfloat16, device=dev)  # 3 padded rows
            impl.forward(layer, q, k, v, cache, md, output=out)
            outs.append(out)
        torch.cuda.synchronize(dev)
        assert impls[0]._oscar_stats["writes"] == step + 1
        assert torch.equal(outs[0], outs[1]), f"step {step}: outputs differ"
        assert int(outs[0][n:].abs().sum()) == 0
        for a, b in zip(caches[0], caches[1]):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), f"step {step}: cache bytes differ"
        for name in ("_oscar_stage_k", "_oscar_stage_v", "_oscar_slot_owner"):
            assert torch.equal(getattr(layers[0], name), getattr(layers[1], name)), f"step {step}: {name} differs"
        # MTP verification accepts 1..len tokens; the next step rewrites the rest
        base = [b + max(1, ln - 1) for b, ln in zip(base, lengths)]
        lengths = [1 + (ln + step) % 4 for ln in lengths]
    assert kernels.device_error(dev) == 0


def test_native_step_declines_prefix_free_requests():
    from oscar_b200.synthetic import make_case

    dev = need_gpu()
    case = make_case([0, 300], [5, 2], hk=1, group=6, seed=4, device=dev)
    impl = make_impl(6, 1, 256)
    layer, cache = clone_state(case, dev, 5)
    impl._set_caches(cache)
    n = 7
    md = NS(num_actual_tokens=n, slot_mapping=torch.arange(n, device=dev), query_start_loc_cpu=torch.tensor([0, 5, 7]),
            seq_lens_list=[5, 302], block_tables=case.bt,
            query_start_loc=torch.tensor([0, 5, 7], dtype=torch.int32, device=dev),
            seq_lens=torch.tensor([5, 302], dtype=torch.int32, device=dev))
    out = torch.empty(n, 6 * 256, dtype=torch.bfloat16, device=dev)
    assert not impl._native_step(layer, case.q, case.k_new, case.v_new, md, out)
