"""Streaming attention (K2/K3 + split combine) and the K4 merge on the GPU vs
the reference's own outputs (golden) and the oracle on seeded synthetic cases.
Tolerances: output 2e-2 abs/rel, LSE 1e-3 abs/rel."""
import numpy as np
import pytest
import torch

from gpu_helpers import LSE_TOL, OUT_TOL, cache_from_bytes, case_to_device, case_to_oracle, need_gpu
from oracle import oscar_oracle as orc
from oscar_b200.synthetic import make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["auto", "decode", "tile"])
def attn_path(request):
    """Run a test under every attention kernel family: "auto" (the tensor-core
    decode kernel where eligible), the mma.sync decode kernel and the general
    tile kernel."""
    from oscar_b200 import kernels

    need_gpu()
    kernels.set_attention_path(request.param)
    yield request.param
    kernels.set_attention_path("auto")

ATTN_CASES = ["mixed_d256", "mtp_hk2_d256", "nowin_d256", "cache_only_multi", "cache_only_empty", "cached_prefill",
              "legacy_hk2_d64_f16", "hk4_d128_f16", "f32_query_d64"]
DT = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def assert_attention_close(out, lse, want_out, want_lse):
    out, lse = out.cpu().numpy(), lse.cpu().numpy()
    assert np.array_equal(np.isneginf(lse), np.isneginf(want_lse))
    np.testing.assert_allclose(out, want_out, **OUT_TOL)
    fin = np.isfinite(want_lse)
    np.testing.assert_allclose(lse[fin], want_lse[fin], **LSE_TOL)


@pytest.mark.parametrize("name", ATTN_CASES)
def test_attention_matches_reference_golden(golden, name, attn_path):
    from oscar_b200 import kernels

    dev = need_gpu()
    c = golden(f"attn_{name}")
    qdt = DT[str(c["qdtype"])]
    d = c["q"].shape[-1]
    t = lambda a: torch.from_numpy(a).to(dev)  # noqa: E731
    q = t(c["q"]).to(qdt)
    k = v = None
    if int(c["has_new"]):
        k, v = t(c["k_new"]).to(qdt), t(c["v_new"]).to(qdt)
    stage = (t(c["stage_k"]), t(c["stage_v"]), t(c["owner"])) if int(c["has_stage"]) else None
    kc, vc = cache_from_bytes(c["k8"], d, dev), cache_from_bytes(c["v8"], d, dev)
    out, lse = kernels.slab_attention(q, k, v, kc, vc, t(c["bt"]), c["qsl"].tolist(), c["seqs"].tolist(),
                                      float(c["scale"]), stage)
    assert_attention_close(out, lse, c["out"], c["lse"])
    assert kernels.device_error(dev) == 0


SYNTH = [
    # (prefixes, lengths, options)
    ([8192], [4], dict()),
    ([3000, 17, 1500, 0, 640], [4, 1, 3, 2, 4], dict()),
    ([2049, 700], [4, 4], dict(hk=2)),
    ([1900, 300], [3, 2], dict(hk=4, group=6, d=128, bs=32)),
    ([1200], [4], dict(window=False, outliers=False)),
    ([1000, 5, 300], [7, 9, 1], dict(fresh=False)),          # cache-only, right-aligned causal
    ([400], [300], dict(hk=2, group=6)),                     # continuation (q-blocks, causal)
    ([0, 0], [200, 33], dict(hk=1, group=6, window=False)),  # prefix-free prefill
    ([2500, 0, 130], [120, 90, 200], dict(hk=2, group=6, dtype=torch.float16)),  # 128-row q-blocks, fp16
    ([3000], [600], dict(hk=2, group=6, seed=5)),            # 128-row q-blocks, staged sink/recent
    ([700, 90], [120, 40], dict(hk=1, group=6, bs=32)),    # 128-row q-blocks over 32-token pages
    ([2000], [300], dict(hk=2, group=6, fresh=False)),      # cache-only, 128-row q-blocks (pre-pass tiles)
    ([777], [5], dict(dtype=torch.float16, d=64, bs=16)),
    ([513], [4], dict(cache_dtype=torch.bfloat16, hk=2)),    # legacy bf16 geometry
    ([300, 200], [2, 3], dict(group=8, hk=2, d=64, bs=8)),
]


@pytest.mark.parametrize("prefixes,lengths,opts", SYNTH)
def test_attention_matches_oracle_on_synthetic_cases(prefixes, lengths, opts, attn_path):
    from oscar_b200 import kernels

    dev = need_gpu()
    opts = dict(opts)
    bs = opts.pop("bs", 128)
    case = make_case(prefixes, lengths, bs=bs, **opts)
    args, dt = case_to_oracle(case)
    want_out, want_lse = orc.streaming_attention(*args, dtype=dt)
    out, lse = kernels.slab_attention(*case_to_device(case, args[3], args[4], dev))
    assert_attention_close(out, lse, want_out, want_lse)


def test_split_kv_is_invisible_and_workspace_optional(attn_path):
    """Any workspace size (0 = no split partials) gives the oracle's answer;
    LSE is split-invariant to fp32 rounding (P.V rounds P to fp16 per split)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([5000, 2500], [4, 4], hk=2)
    args, dt = case_to_oracle(case)
    want_out, want_lse = orc.streaming_attention(*args, dtype=dt)
    dargs = case_to_device(case, args[3], args[4], dev)
    full, full_lse = kernels.slab_attention(*dargs)
    assert_attention_close(full, full_lse, want_out, want_lse)
    for ws in (0, 300_000):
        o, l = kernels.slab_attention(*dargs, workspace_bytes=ws)
        assert_attention_close(o, l, want_out, want_lse)
        torch.testing.assert_close(l, full_lse, atol=2e-5, rtol=2e-5)


def test_full_size_24k_mtp_matches_oracle(attn_path):
    """BASELINE config 2 at full size (1 x 24576 history + 4-token MTP)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([24576], [4])
    args, dt = case_to_oracle(case)
    want_out, want_lse = orc.streaming_attention(*args, dtype=dt)
    out, lse = kernels.slab_attention(*case_to_device(case, args[3], args[4], dev))
    assert_attention_close(out, lse, want_out, want_lse)


def test_empty_queries_and_nan_propagation(attn_path):
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([0, 40], [3, 2], fresh=False, d=64, bs=8)
    args, _ = case_to_oracle(case)
    dargs = list(case_to_device(case, args[3], args[4], dev))
    out, lse = kernels.slab_attention(*dargs)
    assert torch.count_nonzero(out[:3]) == 0 and torch.isneginf(lse[:3]).all()
    q = dargs[0].clone()
    q[3, 0, 0] = float("nan")
    dargs[0] = q
    out, lse = kernels.slab_attention(*dargs)
    assert torch.isnan(out[3, 0]).all() and torch.isnan(lse[3, 0])


def test_layout_errors_raise_value_error():
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([20], [3], d=64, bs=8)
    args, _ = case_to_oracle(case)
    q, k, v, kc, vc, bt, qsl, seqs, scale, stage = case_to_device(case, args[3], args[4], dev)
    with pytest.raises(ValueError, match="query layout"):
        kernels.slab_attention(q, k, v, kc, vc, bt, [0, 2], seqs, scale, stage)
    with pytest.raises(ValueError, match="cover its query chunk"):
        kernels.slab_attention(q, k, v, kc, vc, bt, qsl, [2], scale, stage)
    with pytest.raises(ValueError, match="together"):
        kernels.slab_attention(q, k, None, kc, vc, bt, qsl, seqs, scale, stage)
    with pytest.raises(ValueError, match="Block table cannot cover"):
        kernels.slab_attention(q, k, v, kc, vc, bt[:, :1], qsl, [100], scale, stage)
    with pytest.raises(ValueError, match="staging geometry"):
        kernels.slab_attention(q, k, v, kc, vc, bt, qsl, seqs, scale, (stage[0][:1], stage[1], stage[2]))


@pytest.mark.parametrize("kind", ["contig", "contig2", "indexed"])
def test_merge_matches_reference_edge_cases(golden, kind):
    """tests/test_slab_attention.py:220-259 data: -inf, +-1000, NaN."""
    from oscar_b200 import kernels

    dev = need_gpu()
    c = golden("merge")
    out = torch.from_numpy(c["out"]).to(dev)
    lse = torch.from_numpy(c["lse"]).to(dev)
    part = torch.from_numpy(c["part"]).to(dev).half()
    ids = c[f"{kind}_ids"]
    kernels.merge_slab(out, lse, part, torch.from_numpy(c["part_lse"]).to(dev), int(c[f"{kind}_start"]),
                       torch.from_numpy(ids).to(dev) if ids.size else None)
    np.testing.assert_allclose(out.cpu().numpy(), c[f"{kind}_out"], rtol=2e-6, atol=2e-6, equal_nan=True)
    np.testing.assert_allclose(lse.cpu().numpy(), c[f"{kind}_lse"], rtol=2e-6, atol=2e-6, equal_nan=True)


def test_merge_of_sequence_shards_equals_whole(attn_path):
    """Two split-KV sequence shards (page-aligned halves of the history, as a
    2-GPU split would hold them) merged with K4 equal one pass over all keys."""
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([3072], [1], fresh=False, window=False)  # 1 cache-only query sees all 3072 keys
    args, _ = case_to_oracle(case)
    q, _, _, kc, vc, bt, qsl, seqs, scale, _ = case_to_device(case, args[3], args[4], dev)
    whole, whole_lse = kernels.slab_attention(q, None, None, kc, vc, bt, [0, 1], [3072], scale)
    a_out, a_lse = kernels.slab_attention(q, None, None, kc, vc, bt[:, :12].contiguous(), [0, 1], [1536], scale)
    b_out, b_lse = kernels.slab_attention(q, None, None, kc, vc, bt[:, 12:].contiguous(), [0, 1], [1536], scale)
    kernels.merge_slab(a_out, a_lse, b_out, b_lse, 0, None)
    torch.testing.assert_close(a_out, whole, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(a_lse, whole_lse, atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("frac", [0.02, 0.3])
def test_scattered_staged_positions_match_oracle(frac, attn_path):
    """Staged positions anywhere in the history (not only sink / recent
    windows): every one is masked in its split's INT2 stages and attended
    once from its fp32 row, by whichever CTA the kernel assigns it to."""
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case([5000, 3000, 700], [4, 2, 3], hk=2, seed=23)
    sk, sv, owner = case.stage
    rows, bs = owner.shape
    g = torch.Generator().manual_seed(int(frac * 1000))
    offset = 0
    for r, prefix in enumerate([5000, 3000, 700]):
        pos = torch.nonzero(torch.rand(prefix, generator=g) < frac).flatten()
        blk = case.bt[r, pos // bs].long()
        row, col = blk % rows, pos % bs
        owner[row, col] = blk
        sk[row, col] = case.old_k[offset + pos]
        sv[row, col] = case.old_v[offset + pos]
        offset += prefix
    args, dt = case_to_oracle(case)
    want_out, want_lse = orc.streaming_attention(*args, dtype=dt)
    out, lse = kernels.slab_attention(*case_to_device(case, args[3], args[4], dev))
    assert_attention_close(out, lse, want_out, want_lse)
    assert kernels.device_error(dev) == 0


@pytest.mark.parametrize("prefixes,lengths", [([3000], [600]), ([2500, 0, 130], [120, 90, 200])])
def test_continuation_prepass_and_per_cta_dequant_agree(prefixes, lengths):
    """128-row q-blocks at head dim 256: with room in the workspace the keys'
    tiles are written once by a pre-pass and fetched by bulk copy; without it
    each CTA dequantises its own tiles.  Both give the oracle's answer."""
    from oscar_b200 import kernels

    dev = need_gpu()
    case = make_case(prefixes, lengths, hk=2, group=6, seed=41)
    args, dt = case_to_oracle(case)
    want_out, want_lse = orc.streaming_attention(*args, dtype=dt)
    dargs = case_to_device(case, args[3], args[4], dev)
    full, full_lse = kernels.slab_attention(*dargs)
    assert_attention_close(full, full_lse, want_out, want_lse)
    own, own_lse = kernels.slab_attention(*dargs, workspace_bytes=0)
    assert_attention_close(own, own_lse, want_out, want_lse)
    # the two runs plan different KV splits: LSE agrees to fp32 rounding, outputs to the
    # fp16 rounding of P within each split
    torch.testing.assert_close(own_lse, full_lse, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(own, full, **OUT_TOL)
    assert kernels.device_error(dev) == 0
