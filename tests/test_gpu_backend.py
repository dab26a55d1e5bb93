"""Full OSCAR layer steps through the B200 backend impl on the GPU.

* the reference backend's own outputs for a prefill -> MTP -> cache-only
  sequence with QR rotations, clip 0.96/0.92 and sink/recent windows (golden);
* the lifecycle known answers of tests/test_streaming_backend.py:68-205
  (cache-only rewrite 3.0, MTP reject 45/8 and 75/9, recycled pages -3/-4,
  cached long prefill 1.0, mixed prefix-free batch)."""
from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

from gpu_helpers import need_gpu
from oracle import oscar_oracle as orc

pytestmark = pytest.mark.gpu


def make_impl(hq, hk, d, *, sink, recent, staging, k_clip=0.0, v_clip=0.0, window=True):
    from oscar_b200.backend import OscarAttentionBackendImpl

    impl = OscarAttentionBackendImpl.create(hq, hk, d)
    impl._oscar.sink_tokens, impl._oscar.recent_tokens, impl._oscar.staging_tokens = sink, recent, staging
    impl._oscar.k_clip_ratio, impl._oscar.v_clip_ratio = k_clip, v_clip
    impl._oscar.window_enabled = window
    return impl


def meta(dev, slots, ends, seqs, bt):
    return NS(num_actual_tokens=len(slots), slot_mapping=torch.tensor(slots, dtype=torch.int64, device=dev),
              query_start_loc_cpu=torch.tensor([0] + list(ends)), actual_seq_lengths_q=list(ends),
              seq_lens_list=list(seqs), block_tables=torch.tensor(bt, dtype=torch.int32, device=dev))


def test_golden_layer_sequence_matches_reference_backend(golden):
    dev = need_gpu()
    c = golden("backend")
    d, hk, hq, bs, nb = (int(c[k]) for k in ("d", "hk", "hq", "bs", "nb"))
    impl = make_impl(hq, hk, d, sink=int(c["sink"]), recent=int(c["recent"]), staging=int(c["staging"]),
                     k_clip=float(c["k_clip"]), v_clip=float(c["v_clip"]))
    layer = NS(layer_name="model.layers.0.self_attn.attn",
               _oscar_rots=(torch.from_numpy(c["rk"]).to(dev), torch.from_numpy(c["rv"]).to(dev)))
    cache = torch.zeros(2, nb, bs, hk, d, dtype=torch.int8, device=dev)
    bt = c["bt"].tolist()
    for i in range(2):
        q = torch.from_numpy(c[f"s{i}_q"]).to(dev).bfloat16()
        k = torch.from_numpy(c[f"s{i}_k"]).to(dev).bfloat16()
        v = torch.from_numpy(c[f"s{i}_v"]).to(dev).bfloat16()
        qsl = c[f"s{i}_qsl"].tolist()
        md = meta(dev, c[f"s{i}_slots"].tolist(), qsl[1:], c[f"s{i}_seqs"].tolist(), bt)
        out = impl.forward(layer, q, k, v, cache, md, output=torch.empty(q.shape[0], hq * d, dtype=torch.bfloat16,
                                                                          device=dev))
        np.testing.assert_allclose(out.float().cpu().numpy(), c[f"s{i}_out"], atol=3e-2, rtol=3e-2)
    # state after two steps: owners exact, staged fp32 within GEMM rounding, codes nearly all identical
    assert np.array_equal(layer._oscar_slot_owner.cpu().numpy(), c["owner"])
    np.testing.assert_allclose(layer._oscar_stage_k.cpu().numpy(), c["stage_k"], atol=2e-4, rtol=1e-4)
    np.testing.assert_allclose(layer._oscar_stage_v.cpu().numpy(), c["stage_v"], atol=2e-4, rtol=1e-4)
    k8 = cache[0].view(torch.uint8).cpu().numpy()
    same = (k8 == c["k8"]).mean()
    assert same > 0.995, same  # rotation GEMMs differ in the last ulp only at rounding ties of the codes
    q = torch.from_numpy(c["s2_q"]).to(dev).bfloat16()
    md = meta(dev, [-1, -1], [1, 2], c["s2_seqs"].tolist(), bt)
    out = impl.forward(layer, q, None, None, cache, md, output=torch.empty(2, hq * d, dtype=torch.bfloat16, device=dev))
    np.testing.assert_allclose(out.float().cpu().numpy(), c["s2_out"], atol=3e-2, rtol=3e-2)


def fixture(dev, window=True, dtype=torch.bfloat16):
    """tests/test_backend.py:27-40 geometry: D=64, Hk=1, Hq=2, bs=4, 8 blocks, sink/recent 4, staging 8."""
    impl = make_impl(2, 1, 64, sink=4, recent=4, staging=8, window=window)
    layer = NS(layer_name="model.layers.0.self_attn.attn")
    cache = [torch.zeros(8, 4, 1, 64, dtype=dtype, device=dev) for _ in range(2)]
    impl._set_caches(cache)
    return impl, layer, cache


def test_cache_only_update_invalidates_old_window():
    dev = need_gpu()
    impl, layer, cache = fixture(dev)
    old = torch.ones(4, 1, 64, device=dev)
    impl.do_kv_cache_update(layer, old, old, cache, torch.arange(4, device=dev))
    impl._ensure_staging(layer, cache)
    impl._staging_write(layer, old, old, meta(dev, [0, 1, 2, 3], [4], [4], [[0, 1, 2, 3]]))
    assert layer._oscar_slot_owner[0, 1].item() == 0
    rep = torch.full((1, 1, 64), 9.0, device=dev)
    impl.do_kv_cache_update(layer, rep, rep, cache, torch.tensor([1], device=dev))
    assert layer._oscar_slot_owner[0, 1].item() == -1 and layer._oscar_slot_owner[0, 0].item() == 0
    md = meta(dev, [], [1], [4], [[0, 1, 2, 3]])
    md.num_actual_tokens = 1
    q = torch.zeros(1, 2, 64, device=dev)
    out = impl.forward(layer, q, None, None, cache, md, output=torch.empty_like(q))
    torch.testing.assert_close(out, torch.full_like(out, 3.0))  # mean(1, 9, 1, 1)


def test_rejected_mtp_tail_and_recycled_blocks_cannot_leak():
    dev = need_gpu()
    impl, layer, cache = fixture(dev)
    bt = [[0, 1, 2, 3]]
    oldv = torch.arange(6, device=dev).float()[:, None, None].expand(6, 1, 64).contiguous()
    oldk = torch.zeros_like(oldv)
    impl.do_kv_cache_update(layer, oldk, oldv, cache, torch.arange(6, device=dev))
    impl._ensure_staging(layer, cache)
    impl._staging_write(layer, oldk, oldv, meta(dev, list(range(6)), [6], [6], bt))
    firstv = torch.tensor([10.0, 100.0, 1000.0, 10000.0], device=dev)[:, None, None].expand(4, 1, 64)
    impl.forward(layer, torch.zeros(4, 2, 64, device=dev), torch.zeros_like(firstv), firstv, cache,
                 meta(dev, [6, 7, 8, 9], [4], [10], bt), output=torch.empty(4, 2, 64, device=dev))
    secondv = torch.tensor([20.0, 30.0], device=dev)[:, None, None].expand(2, 1, 64)
    out = impl.forward(layer, torch.zeros(2, 2, 64, device=dev), torch.zeros_like(secondv), secondv, cache,
                       meta(dev, [7, 8], [2], [9], bt), output=torch.empty(2, 2, 64, device=dev))
    torch.testing.assert_close(out[0], torch.full_like(out[0], 45 / 8))
    torch.testing.assert_close(out[1], torch.full_like(out[1], 75 / 9))
    newv = torch.full((4, 1, 64), -3.0, device=dev)
    out = impl.forward(layer, torch.zeros(4, 2, 64, device=dev), torch.zeros_like(newv), newv, cache,
                       meta(dev, [0, 1, 2, 3], [4], [4], bt), output=torch.empty(4, 2, 64, device=dev))
    torch.testing.assert_close(out, torch.full_like(out, -3.0))
    tail = torch.full((1, 1, 64), -8.0, device=dev)
    out = impl.forward(layer, torch.zeros(1, 2, 64, device=dev), torch.zeros_like(tail), tail, cache,
                       meta(dev, [4], [1], [5], bt), output=torch.empty(1, 2, 64, device=dev))
    torch.testing.assert_close(out, torch.full_like(out, -4.0))


def test_cached_long_prefill_is_also_streaming():
    dev = need_gpu()
    impl, layer, cache = fixture(dev, window=False)
    old = torch.ones(4, 1, 64, device=dev)
    impl.do_kv_cache_update(layer, old, old, cache, torch.arange(4, device=dev))
    q = torch.zeros(20, 2, 64, device=dev)
    new = torch.ones(20, 1, 64, device=dev)
    md = meta(dev, list(range(4, 24)), [20], [24], [[0, 1, 2, 3, 4, 5]])
    out = impl.forward(layer, q, new, new, cache, md, output=torch.empty_like(q))
    torch.testing.assert_close(out, torch.ones_like(out))


def test_mixed_prefix_free_prefill_and_cached_request():
    dev = need_gpu()
    impl, layer, cache = fixture(dev, window=False)
    old = torch.ones(6, 1, 64, device=dev)
    impl.do_kv_cache_update(layer, old, old, cache, torch.tensor([24, 25, 26, 27, 28, 29], device=dev))
    q = torch.zeros(21, 2, 64, device=dev)
    cur = torch.ones(21, 1, 64, device=dev)
    md = meta(dev, list(range(17)) + [30, 31, 20, 21], [17, 21], [17, 10], [[0, 1, 2, 3, 4], [6, 7, 5, 0, 0]])
    out = impl.forward(layer, q, cur, cur, cache, md, output=torch.empty_like(q))
    torch.testing.assert_close(out, torch.ones_like(out))


@pytest.mark.parametrize("window", [False, True])
def test_rotated_mixed_batch_with_padding_matches_oracle(window):
    """tests/test_streaming_backend.py:24-65 shape: rotations, fp16, a padding
    request and two padding tokens; expected from the oracle in rotated space."""
    dev = need_gpu()
    torch.manual_seed(0)
    impl, layer, cache = fixture(dev, window=window, dtype=torch.float16)
    rk, rv = [torch.linalg.qr(torch.randn(64, 64)).Q for _ in range(2)]
    layer._oscar_rots = (rk.to(dev), rv.to(dev))
    oldk, oldv = [torch.randn(9, 1, 64) for _ in range(2)]
    slots = [16, 17, 18, 19, 4, 5, 0, 1, 2]
    impl.do_kv_cache_update(layer, oldk.to(dev), oldv.to(dev), cache, torch.tensor(slots, device=dev))
    if window:
        impl._ensure_staging(layer, cache)
        impl._staging_write(layer, oldk.to(dev), oldv.to(dev), meta(dev, slots, [6, 9], [6, 3], [[4, 1, 6]]))
    q, k, v = [torch.randn(7, h, 64).half() for h in (2, 1, 1)]
    bt = [[4, 1, 6], [0, 0, 0], [0, 0, 0]]
    md = meta(dev, [6, 7, 24, 25, 3], [4, 5, 7], [10, 4, 0], bt)
    out = impl.forward(layer, q.to(dev), k.to(dev), v.to(dev), [t for t in cache], md,
                       output=torch.empty(7, 128, dtype=torch.float16, device=dev))
    # oracle: same caches (read back), rotated queries, fp16
    k8 = cache[0].view(torch.uint8).cpu().numpy()
    v8 = cache[1].view(torch.uint8).cpu().numpy()
    stage = None
    if window:
        stage = tuple(t.cpu().numpy() for t in (layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner))
    rq = orc.round_f16(q[:5].float().numpy() @ rk.numpy())
    rkn = orc.round_f16(k[:5].float().numpy() @ rk.numpy())
    rvn = orc.round_f16(v[:5].float().numpy() @ rv.numpy())
    o, _ = orc.streaming_attention(rq, rkn, rvn, k8, v8, np.asarray(bt[:2], np.int32), [0, 4, 5], [10, 4], 64**-0.5,
                                   stage, dtype="f16")
    want = o @ rv.t().numpy()
    np.testing.assert_allclose(out[:5].float().cpu().numpy().reshape(5, 2, 64), want, atol=1e-2, rtol=1e-2)
    assert torch.count_nonzero(out[5:]) == 0
