"""Parity at the benchmarked configurations (4 and 5).

* cfg3 exactly as bench.py runs it (8 x 24576 history + 4 MTP tokens, Hq 6 /
  Hk 1, clip 0.96 / 0.92, sink 128 / recent 256, QR rotations): two layer
  steps through ``backend.forward`` (eager, then a ``GraphedForward``
  replay) against the oracle's layer step, the INT2 codes of the written
  slots bit-exact given the GPU's rotated fp32 rows, and the attention pass
  alone (out and LSE) at full size;
* cfg4 at full size (15360 new tokens on 9256 tokens of INT2 history, Hq 24 /
  Hk 4), with and without the continuation pre-pass, checked on sampled
  query tiles (first, middle, last);
* cfg5 (64 requests with lognormal histories, Hq 24 / Hk 4) over three
  steps with interleaved MTP-reject tail rewrites, the pattern of the
  reference's tests/test_streaming_backend.py:89-145.
"""
from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

from gpu_helpers import LSE_TOL, OUT_TOL, need_gpu
from oracle import oscar_oracle as orc

pytestmark = pytest.mark.gpu

# the layer output is the attention output rotated back (@ R_v^T, fp32) and cast to
# bf16: the tolerance of the reference-backend layer golden (test_gpu_backend.py);
# the attention itself is held to the north-star 2e-2 / 1e-3 in rotated space
LAYER_TOL = dict(atol=3e-2, rtol=3e-2)


class OracleLayer:
    """The reference backend's FULL-layer step on the CPU: rotate new K/V, clip
    and INT2-store them, staging write of the unclipped rotated rows, rotated
    attention over the paged history and the causal chunk, output @ R_v^T
    (backend.py:151-198, :513-555, :334-393)."""

    def __init__(self, k8, v8, stage, rk, rv, *, bs, hk, d, sink, recent, staging, k_clip, v_clip):
        self.k8, self.v8 = k8, v8
        self.rk, self.rv = rk, rv
        self.hk, self.d, self.clip = hk, d, (k_clip, v_clip)
        self.st = orc.Staging(bs, hk, d, sink, recent, staging)
        sk, sv, owner = stage
        assert self.st.stage_k.shape == sk.shape
        self.st.stage_k[:], self.st.stage_v[:], self.st.owner[:] = sk, sv, owner

    def step(self, q, k, v, slots, qsl, seqs, bt, scale, rows=None):
        n = k.shape[0]
        hq = q.shape[1]
        k = k.reshape(n, self.hk, self.d)
        v = v.reshape(n, self.hk, self.d)
        kr, vr = (k @ self.rk).astype(np.float32), (v @ self.rv).astype(np.float32)
        orc.store(orc.clip_only(kr, self.clip[0]), orc.clip_only(vr, self.clip[1]), self.k8, self.v8, slots)
        self.st.write(k, v, self.rk, self.rv, slots, qsl, seqs, n)
        qr = orc.round_bf16(q @ self.rk)
        out, lse = orc.streaming_attention(qr, orc.round_bf16(kr), orc.round_bf16(vr), self.k8, self.v8, bt, qsl, seqs,
                                           scale, self.st.tuple(), rows=rows)
        final = orc.round_bf16(out @ self.rv.T).reshape(q.shape[0], hq * self.d)
        return final, out, lse


def qr_rotation(seed, d, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.linalg.qr(torch.randn(d, d, generator=g, device=dev)).Q.contiguous()


def make_impl(hq, hk, d, *, sink, recent, staging, k_clip, v_clip):
    from oscar_b200.backend import OscarAttentionBackendImpl

    impl = OscarAttentionBackendImpl.create(hq, hk, d)
    cfg = impl._oscar
    cfg.sink_tokens, cfg.recent_tokens, cfg.staging_tokens = sink, recent, staging
    cfg.k_clip_ratio, cfg.v_clip_ratio = k_clip, v_clip
    cfg.window_enabled = True
    return impl


def layer_setup(case, dev, *, hq, hk, d, k_clip, v_clip, seed):
    """GPU impl + layer (rotations, staging arena copied from the case) and the
    oracle over byte copies of the same caches and arena."""
    rk, rv = qr_rotation(seed, d, dev), qr_rotation(seed + 1, d, dev)
    impl = make_impl(hq, hk, d, sink=128, recent=256, staging=8192, k_clip=k_clip, v_clip=v_clip)
    layer = NS(layer_name="model.layers.0.self_attn.attn", _oscar_rots=(rk, rv))
    cache = (case.kc, case.vc)
    impl._set_caches(cache)
    impl._ensure_staging(layer, cache)
    sk, sv, owner = case.stage
    layer._oscar_stage_k.copy_(sk)
    layer._oscar_stage_v.copy_(sv)
    layer._oscar_slot_owner.copy_(owner)
    oracle = OracleLayer(case.kc.view(torch.uint8).cpu().numpy(), case.vc.view(torch.uint8).cpu().numpy(),
                         tuple(t.cpu().numpy() for t in case.stage), rk.cpu().numpy(), rv.cpu().numpy(),
                         bs=128, hk=hk, d=d, sink=128, recent=256, staging=8192, k_clip=k_clip, v_clip=v_clip)
    return impl, layer, cache, oracle


def step_meta(dev, slots, qsl, seqs, bt):
    return NS(num_actual_tokens=len(slots), slot_mapping=torch.as_tensor(slots, dtype=torch.int64, device=dev),
              query_start_loc_cpu=torch.tensor(qsl), seq_lens_list=list(seqs), block_tables=bt,
              query_start_loc=torch.tensor(qsl, dtype=torch.int32, device=dev),
              seq_lens=torch.tensor(seqs, dtype=torch.int32, device=dev))


def slots_of(bt, positions):
    """Cache slots of (request, position) pairs through the block table."""
    bt = bt.cpu()
    return [int(bt[r, p // 128]) * 128 + p % 128 for r, p in positions]


def assert_codes_match(impl, layer, key, value, slots, cache):
    """The written slots' bytes equal the oracle quantisation of the GPU's own
    rotated fp32 rows (clip included): bit-exact given identical rotated input.
    Only the last write of each slot counts (duplicates keep the last)."""
    n = len(slots)
    k_rot, v_rot = impl._rotate_step(layer, key, value, n)[:2]
    want = orc.make_slot_bytes(orc.clip_only(k_rot.cpu().numpy(), impl._oscar.k_clip_ratio),
                               orc.clip_only(v_rot.cpu().numpy(), impl._oscar.v_clip_ratio))
    last = {s_: i for i, s_ in enumerate(slots) if s_ >= 0}
    idx = np.asarray(list(last.values()))
    sl = np.asarray(list(last.keys()))
    gk = cache[0].view(torch.uint8).cpu().numpy()[sl // 128, sl % 128]
    gv = cache[1].view(torch.uint8).cpu().numpy()[sl // 128, sl % 128]
    assert np.array_equal(gk[..., 0:8], want[idx, :, 0:8])
    assert np.array_equal(gk[..., 32:96], want[idx, :, 32:96])
    assert np.array_equal(gv[..., 0:64], want[idx, :, 96:160])


def test_cfg3_bench_workload_layer_steps_and_graph_replay():
    """bench.py's workload: eager step, then a captured step replayed, both
    against the oracle's layer step; the attention pass alone (out and LSE)."""
    from oscar_b200 import kernels
    from oscar_b200.graphs import GraphedForward
    from oscar_b200.synthetic import fill_caches, make_case

    dev = need_gpu()
    prefixes, lengths = [24576] * 8, [4] * 8
    case = make_case(prefixes, lengths, hk=1, group=6, seed=1000, device=dev)
    fill_caches(case)
    impl, layer, cache, oracle = layer_setup(case, dev, hq=6, hk=1, d=256, k_clip=0.96, v_clip=0.92, seed=7)
    slots = slots_of(case.bt, [(r, p + i) for r, p in enumerate(prefixes) for i in range(4)])
    bt_np = case.bt.cpu().numpy()
    md = step_meta(dev, slots, case.qsl, case.seqs, case.bt)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    # step 1: eager forward
    q, k, v = case.q.clone(), case.k_new.clone(), case.v_new.clone()
    out = torch.empty(q.shape[0], 6 * 256, dtype=torch.bfloat16, device=dev)
    impl.forward(layer, q, k, v, cache, md, output=out)
    want, _, _ = oracle.step(f(q), f(k), f(v), np.asarray(slots), case.qsl, case.seqs, bt_np, case.scale)
    np.testing.assert_allclose(f(out), want, **LAYER_TOL)
    assert_codes_match(impl, layer, k, v, slots, cache)
    assert np.array_equal(layer._oscar_slot_owner.cpu().numpy(), oracle.st.owner)
    # step 2: the same MTP slots rewritten with new values, replayed from a CUDA graph
    g = torch.Generator(device=dev).manual_seed(99)
    q.copy_(torch.randn(q.shape, generator=g, device=dev))
    k.copy_(torch.randn(k.shape, generator=g, device=dev))
    v.copy_(torch.randn(v.shape, generator=g, device=dev))
    graph = GraphedForward(impl, layer, q, k, v, cache, md, out)
    graph.replay()
    want2, o_rot, lse_rot = oracle.step(f(q), f(k), f(v), np.asarray(slots), case.qsl, case.seqs, bt_np, case.scale)
    np.testing.assert_allclose(f(out), want2, **LAYER_TOL)
    assert_codes_match(impl, layer, k, v, slots, cache)
    assert np.array_equal(layer._oscar_slot_owner.cpu().numpy(), oracle.st.owner)
    # the attention pass alone on the step's rotated inputs: rotated-space out and LSE
    rk, rv = layer._oscar_rots
    qr = (q.float() @ rk).bfloat16()
    kr = (k.float().view(-1, 256) @ rk).view(k.shape).bfloat16()
    vr = (v.float().view(-1, 256) @ rv).view(v.shape).bfloat16()
    stage = (layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner)
    o, lse = kernels.slab_attention(qr, kr, vr, cache[0], cache[1], case.bt, case.qsl, case.seqs, case.scale, stage)
    np.testing.assert_allclose(o.cpu().numpy(), o_rot, **OUT_TOL)
    np.testing.assert_allclose(lse.cpu().numpy(), lse_rot, **LSE_TOL)
    assert kernels.device_error(dev) == 0


@pytest.mark.parametrize("prepass", [True, False])
def test_cfg4_full_size_continuation_sampled_tiles(prepass):
    """15360 new tokens on 9256 tokens of INT2 history, Hq 24 / Hk 4: the first,
    a middle and the last 32-row query tile of the chunk (every head)."""
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, make_case

    dev = need_gpu()
    case = make_case([9256], [15360], hk=4, group=6, seed=31, device=dev)
    fill_caches(case)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    rows = [(0, 32), (7680, 7712), (15328, 15360)]
    want, want_lse = orc.streaming_attention(f(case.q), f(case.k_new), f(case.v_new),
                                             case.kc.view(torch.uint8).cpu().numpy(),
                                             case.vc.view(torch.uint8).cpu().numpy(), case.bt.cpu().numpy(), case.qsl,
                                             case.seqs, case.scale, tuple(t.cpu().numpy() for t in case.stage),
                                             rows=rows)
    ws = kernels.DEFAULT_WORKSPACE_BYTES if prepass else 0  # 0: every CTA dequantises its own tiles
    out, lse = kernels.slab_attention(*case.args(), workspace_bytes=ws)
    out, lse = out.cpu().numpy(), lse.cpu().numpy()
    for r0, r1 in rows:
        np.testing.assert_allclose(out[r0:r1], want[r0:r1], **OUT_TOL)
        np.testing.assert_allclose(lse[r0:r1], want_lse[r0:r1], **LSE_TOL)
    assert kernels.device_error(dev) == 0


def test_cfg5_mixed_batch_mtp_reject_rewrites():
    """64 requests (lognormal histories, median 4096, clipped 1024-32768), Hq 24 /
    Hk 4: three layer steps of 1-4 MTP tokens each; after every step a random
    number of the request's tokens is accepted and the next step rewrites the
    rejected positions' slots (tests/test_streaming_backend.py:89-145)."""
    from oscar_b200 import kernels
    from oscar_b200.synthetic import fill_caches, lognormal_lengths, make_case

    dev = need_gpu()
    prefixes = lognormal_lengths(64, 5)
    lengths = [1 + (i * 7) % 4 for i in range(64)]
    case = make_case(prefixes, lengths, hk=4, group=6, seed=55, device=dev, compact=True, headroom=16)
    fill_caches(case)
    impl, layer, cache, oracle = layer_setup(case, dev, hq=24, hk=4, d=256, k_clip=0.96, v_clip=0.92, seed=11)
    bt_np = case.bt.cpu().numpy()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    rng = np.random.default_rng(3)
    gen = torch.Generator(device=dev).manual_seed(17)
    base = list(prefixes)  # accepted tokens of each request
    q, k, v = case.q, case.k_new, case.v_new
    for step in range(3):
        if step:
            lengths = [int(x) for x in rng.integers(1, 5, len(base))]
            n = sum(lengths)
            q = torch.randn(n, 24, 256, generator=gen, device=dev).bfloat16()
            k = torch.randn(n, 4, 256, generator=gen, device=dev).bfloat16()
            v = torch.randn(n, 4, 256, generator=gen, device=dev).bfloat16()
        qsl = [0]
        for ln in lengths:
            qsl.append(qsl[-1] + ln)
        seqs = [b + ln for b, ln in zip(base, lengths)]
        slots = slots_of(case.bt, [(r, b + i) for r, (b, ln) in enumerate(zip(base, lengths)) for i in range(ln)])
        md = step_meta(dev, slots, qsl, seqs, case.bt)
        out = torch.empty(q.shape[0], 24 * 256, dtype=torch.bfloat16, device=dev)
        impl.forward(layer, q, k, v, cache, md, output=out)
        want, o_rot, lse_rot = oracle.step(f(q), f(k), f(v), np.asarray(slots), qsl, seqs, bt_np, case.scale)
        np.testing.assert_allclose(f(out), want, **LAYER_TOL)
        assert np.array_equal(layer._oscar_slot_owner.cpu().numpy(), oracle.st.owner)
        assert_codes_match(impl, layer, k, v, slots, cache)
        # the attention pass alone on the step's rotated inputs (rotated space)
        rk, rv = layer._oscar_rots
        qr = (q.float() @ rk).bfloat16()
        kr = (k.float() @ rk).bfloat16()
        vr = (v.float() @ rv).bfloat16()
        stage = (layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner)
        o, lse = kernels.slab_attention(qr, kr, vr, cache[0], cache[1], case.bt, qsl, seqs, case.scale, stage)
        np.testing.assert_allclose(o.cpu().numpy(), o_rot, **OUT_TOL)
        np.testing.assert_allclose(lse.cpu().numpy(), lse_rot, **LSE_TOL)
        # MTP verification: 1..len tokens of each request are accepted; the rest is rewritten next step
        base = [b + int(rng.integers(1, ln + 1)) for b, ln in zip(base, lengths)]
