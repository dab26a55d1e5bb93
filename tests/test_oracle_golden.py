"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py runs oscar_ascend's torch CPU path)."""
import numpy as np
import pytest

from oracle import oscar_oracle as orc

STORE_CASES = ["d256_hk1_int8", "d64_hk2_bf16", "const_d64", "d256_hk4_bf16vals", "d32_hk2_bf16", "ties_d64", "dup_slot_d64"]
ATTN_CASES = ["mixed_d256", "mtp_hk2_d256", "nowin_d256", "cache_only_multi", "cache_only_empty", "cached_prefill",
              "legacy_hk2_d64_f16", "hk4_d128_f16", "f32_query_d64"]


@pytest.mark.parametrize("name", STORE_CASES)
def test_oracle_store_bytes_match_reference(golden, name):
    c = golden(name)
    k8, v8 = c["k8_before"].copy(), c["v8_before"].copy()
    orc.store(c["k_rot"], c["v_rot"], k8, v8, c["slots"])
    assert np.array_equal(k8, c["k8_after"])
    assert np.array_equal(v8, c["v8_after"])


def test_oracle_ties_use_floor_plus_half(golden):
    # x - zero = 0.5 * scale exactly -> floor(0.5 + 0.5) = 1 (torch.round would give 0)
    packed, scale, zero = orc.quantize(np.array([[0.0, 3.0, 0.5, 1.5]], np.float32))
    assert scale[0, 0] == 1.0 and zero[0, 0] == 0.0
    assert list(orc.unpack(packed, 4)[0]) == [0, 3, 1, 2]


@pytest.mark.parametrize("ratio", [0, 50, 92, 96, 100])
def test_oracle_rotate_clip(golden, ratio):
    c = golden("clip")
    y = orc.rotate_clip(c["x"], c["rot"], ratio / 100.0)
    np.testing.assert_allclose(y, c[f"y_{ratio}"], rtol=2e-6, atol=2e-6)


def test_oracle_staging_sequence(golden):
    c = golden("staging")
    st = orc.Staging(int(c["bs"]), 1, 64, 4, int(c["recent"]), 8)
    assert st.rows == int(c["rows"]) and st.sink_eff == int(c["sink_eff"])
    for i in range(int(c["nsteps"])):
        slots = c[f"s{i}_slots"]
        if int(c[f"s{i}_kind"]) == 1:
            st.invalidate(slots)
        else:
            st.write(c[f"s{i}_k"], c[f"s{i}_v"], c["rk"], c["rv"], slots,
                     c[f"s{i}_qsl"].tolist(), c[f"s{i}_seqs"].tolist(), len(slots))
        assert np.array_equal(st.owner, c[f"s{i}_owner"]), i
        np.testing.assert_allclose(st.stage_k, c[f"s{i}_stage_k"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(st.stage_v, c[f"s{i}_stage_v"], rtol=1e-5, atol=1e-6)


def attn_args(c):
    has_new = bool(c["has_new"])
    stage = (c["stage_k"], c["stage_v"], c["owner"]) if int(c["has_stage"]) else None
    dt = {"bfloat16": "bf16", "float16": "f16", "float32": "f32"}[str(c["qdtype"])]
    return (c["q"], c["k_new"] if has_new else None, c["v_new"] if has_new else None, c["k8"], c["v8"],
            c["bt"], c["qsl"].tolist(), c["seqs"].tolist(), float(c["scale"]), stage), dt


@pytest.mark.parametrize("name", ATTN_CASES)
def test_oracle_streaming_attention_matches_reference(golden, name):
    c = golden(f"attn_{name}")
    args, dt = attn_args(c)
    out, lse = orc.streaming_attention(*args, dtype=dt)
    np.testing.assert_allclose(out, c["out"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(lse, c["lse"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("kind", ["contig", "contig2", "indexed"])
def test_oracle_merge_edge_cases(golden, kind):
    c = golden("merge")
    out, lse = c["out"].copy(), c["lse"].copy()
    ids = c[f"{kind}_ids"]
    orc.merge_slab(out, lse, c["part"], c["part_lse"], int(c[f"{kind}_start"]), ids if ids.size else None)
    np.testing.assert_allclose(out, c[f"{kind}_out"], rtol=2e-6, atol=2e-6, equal_nan=True)
    np.testing.assert_allclose(lse, c[f"{kind}_lse"], rtol=2e-6, atol=2e-6, equal_nan=True)


def test_oracle_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, np.inf, 3.0e38], np.float32)
    r = orc.round_bf16(x)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 -> 1 + 2^-6
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.015625)
    assert r[3] == -2.5 and np.isinf(r[4])
