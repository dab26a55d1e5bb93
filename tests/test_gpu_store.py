"""K1 store and K5 staging on the GPU vs the reference (golden) and the oracle.
Codes and scale/zero bytes must be bit-exact for identical rotated fp32 input."""
import numpy as np
import pytest
import torch

from gpu_helpers import cache_bytes, cache_from_bytes, need_gpu
from oracle import oscar_oracle as orc

pytestmark = pytest.mark.gpu

STORE_CASES = ["d256_hk1_int8", "d64_hk2_bf16", "const_d64", "d256_hk4_bf16vals", "d32_hk2_bf16", "ties_d64"]


@pytest.mark.parametrize("name", STORE_CASES)
def test_store_bytes_bit_exact_vs_reference(golden, name):
    from oscar_b200 import kernels

    dev = need_gpu()
    c = golden(name)
    d = c["k_rot"].shape[-1]
    kc = cache_from_bytes(c["k8_before"], d, dev)
    vc = cache_from_bytes(c["v8_before"], d, dev)
    kernels.oscar_store(torch.from_numpy(c["k_rot"]).to(dev), torch.from_numpy(c["v_rot"]).to(dev), kc, vc,
                        torch.from_numpy(c["slots"]).to(dev))
    assert np.array_equal(cache_bytes(kc), c["k8_after"])
    assert np.array_equal(cache_bytes(vc), c["v8_after"])
    assert kernels.device_error(dev) == 0


@pytest.mark.parametrize("kclip,vclip", [(0.96, 0.92), (0.5, 1.0), (0.0, 0.96)])
@pytest.mark.parametrize("d,hk", [(256, 1), (256, 4), (128, 2), (64, 2), (36, 1)])
def test_store_with_clip_bit_exact_vs_oracle(d, hk, kclip, vclip):
    """Clip (backend.py:140-146) + quantize + pack at random slots, vs the oracle."""
    from oscar_b200 import kernels

    dev = need_gpu()
    rng = np.random.default_rng(d * 7 + hk)
    n, bs, nb = 300, 16, 40
    k = rng.standard_normal((n, hk, d)).astype(np.float32)
    v = rng.standard_normal((n, hk, d)).astype(np.float32) * 3
    k[..., :: max(1, d // 4)] *= 20
    slots = rng.permutation(nb * bs)[:n].astype(np.int64)
    slots[::17] = -1
    slot_bytes = d if d % 64 == 0 else 2 * d
    if slot_bytes < 32 + d // 4:
        slot_bytes = 2 * d
    k8 = rng.integers(0, 256, (nb, bs, hk, slot_bytes), dtype=np.uint8)
    v8 = rng.integers(0, 256, (nb, bs, hk, slot_bytes), dtype=np.uint8)
    ek, ev = k8.copy(), v8.copy()
    orc.store(orc.clip_only(k, kclip), orc.clip_only(v, vclip), ek, ev, slots)
    kc = torch.from_numpy(k8).to(dev)
    vc = torch.from_numpy(v8).to(dev)
    kernels.oscar_store(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), kc, vc,
                        torch.from_numpy(slots).to(dev), kclip, vclip)
    assert np.array_equal(kc.cpu().numpy(), ek)
    assert np.array_equal(vc.cpu().numpy(), ev)


@pytest.mark.parametrize("d", [256, 64])
def test_store_clip_with_tied_magnitudes_at_the_top_vs_oracle(d):
    """Clip thresholds near the top of |x| are selected by a warp tournament;
    ties at the top (the same |x| in several lanes, and twice in one lane, of
    either sign) must count with their multiplicity, at every rank around the
    tied run."""
    from oscar_b200 import kernels

    dev = need_gpu()
    rng = np.random.default_rng(90 + d)
    rows = []
    for t in range(24):
        x = rng.standard_normal(d).astype(np.float32)
        top = rng.choice(d, size=9, replace=False)
        x[top[:5]] = 3.0
        x[top[5:]] = -3.0
        x[(top[0] // 4) * 4 + (top[0] + 1) % 4] = -3.0  # a second copy in the lane holding top[0]
        if t % 3 == 1:
            x[top[:2]] = 7.5  # a tied run above the first one
        if t % 3 == 2:
            x[:] = np.float32(-2.0)  # every |x| equal
        rows.append(x)
    k = np.stack(rows)[:, None, :]
    v = -k
    n, bs, nb = k.shape[0], 16, 4
    slots = np.arange(n, dtype=np.int64)
    for ratio in (0.96, 0.95, 0.962, 0.97, 0.99, 0.92, 0.88):
        k8 = np.zeros((nb, bs, 1, d), dtype=np.uint8)
        v8 = np.zeros_like(k8)
        ek, ev = k8.copy(), v8.copy()
        orc.store(orc.clip_only(k, ratio), orc.clip_only(v, ratio), ek, ev, slots)
        kc = torch.from_numpy(k8).to(dev)
        vc = torch.from_numpy(v8).to(dev)
        kernels.oscar_store(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), kc, vc,
                            torch.from_numpy(slots).to(dev), ratio, ratio)
        assert np.array_equal(kc.cpu().numpy(), ek), ratio
        assert np.array_equal(vc.cpu().numpy(), ev), ratio


def test_store_clip_golden_rotate_clip(golden):
    """Rotated input from the reference's _rotate_clip: the kernel's in-kernel
    clip of the unclipped rotation equals storing the reference's clipped rows."""
    from oscar_b200 import kernels

    dev = need_gpu()
    c = golden("clip")
    y0 = (c["x"] @ c["rot"]).astype(np.float32)  # rotation as computed by the reference (fp32)
    n, hk, d = c["x"].shape
    nb, bs = 4, 8
    slots = np.arange(n, dtype=np.int64)
    for ratio in (50, 92, 96):
        y_ref = c[f"y_{ratio}"]
        # identical rotated input: feed the reference's unclipped rotation (ratio 0)
        y_unclipped = c["y_0"]
        ek = np.zeros((nb, bs, hk, d), np.uint8)
        ev = np.zeros_like(ek)
        orc.store(y_ref, y_ref, ek, ev, slots)
        kc = torch.zeros(nb, bs, hk, d, dtype=torch.int8, device=dev)
        vc = torch.zeros_like(kc)
        t = torch.from_numpy(y_unclipped).to(dev)
        kernels.oscar_store(t, t, kc, vc, torch.from_numpy(slots).to(dev), ratio / 100, ratio / 100)
        assert np.array_equal(cache_bytes(kc), ek), ratio
        assert np.array_equal(cache_bytes(vc), ev), ratio
    assert y0.shape == c["y_0"].shape


def test_store_large_random_bit_exact():
    """65536 vectors of D=256 (fp32 inputs spanning many exponents)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    g = torch.Generator(device="cpu").manual_seed(3)
    n, hk, d, bs = 16384, 4, 256, 128
    k = torch.randn(n, hk, d, generator=g) * torch.exp(torch.randn(n, hk, 1, generator=g) * 3)
    v = torch.randn(n, hk, d, generator=g) + torch.randn(n, hk, 1, generator=g) * 50
    nb = n // bs + 2
    slots = torch.randperm(nb * bs, generator=g)[:n]
    ek = np.zeros((nb, bs, hk, d), np.uint8)
    ev = np.zeros_like(ek)
    orc.store(k.numpy(), v.numpy(), ek, ev, slots.numpy())
    kc = torch.zeros(nb, bs, hk, d, dtype=torch.int8, device=dev)
    vc = torch.zeros_like(kc)
    kernels.oscar_store(k.to(dev), v.to(dev), kc, vc, slots.to(dev))
    assert np.array_equal(cache_bytes(kc), ek)
    assert np.array_equal(cache_bytes(vc), ev)


@pytest.mark.parametrize("hk,dtype", [(1, torch.int8), (2, torch.bfloat16), (4, torch.int8)])
def test_negative_slots_are_noops_and_out_of_range_is_flagged(hk, dtype):
    """tests/test_backend.py:56-74 on the device, plus the bounds latch."""
    from oscar_b200 import kernels

    dev = need_gpu()
    cache = [torch.zeros(8, 4, hk, 64, dtype=dtype, device=dev) for _ in range(2)]
    k, v = torch.randn(3, hk, 64, device=dev), torch.randn(3, hk, 64, device=dev)
    before = [t.clone() for t in cache]
    kernels.oscar_store(k, v, *cache, torch.tensor([-1, 2, -1], device=dev))
    expected = [t.clone() for t in before]
    kernels.oscar_store(k[1:2], v[1:2], *expected, torch.tensor([2], device=dev))
    assert all(torch.equal(a.view(torch.uint8), b.view(torch.uint8)) for a, b in zip(cache, expected))
    before = [t.clone() for t in cache]
    kernels.oscar_store(k, v, *cache, torch.full((3,), -1, device=dev))
    assert all(torch.equal(a.view(torch.uint8), b.view(torch.uint8)) for a, b in zip(cache, before))
    assert kernels.device_error(dev) == 0
    kernels.oscar_store(k[:1], v[:1], *cache, torch.tensor([8 * 4 + 3], device=dev))  # block 8 of 8
    assert all(torch.equal(a.view(torch.uint8), b.view(torch.uint8)) for a, b in zip(cache, before))
    assert kernels.device_error(dev) & 1


def test_staging_sequence_matches_reference(golden):
    """Seat hashing, last-writer-wins collisions, padding request, negative
    slots, direct-update invalidation (backend.py:172-176, :513-555)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    c = golden("staging")
    rows, bs = int(c["rows"]), int(c["bs"])
    sk = torch.zeros(rows, bs, 1, 64, device=dev)
    sv = torch.zeros_like(sk)
    owner = torch.full((rows, bs), -1, dtype=torch.int64, device=dev)
    winner = torch.zeros(rows * bs, dtype=torch.int64, device=dev)
    epoch = 0
    for i in range(int(c["nsteps"])):
        slots = torch.from_numpy(c[f"s{i}_slots"]).to(dev)
        if int(c[f"s{i}_kind"]) == 1:
            kernels.staging_invalidate(slots, owner, bs)
        else:
            n = slots.numel()
            krot = torch.from_numpy((c[f"s{i}_k"].reshape(n, 64) @ c["rk"]).reshape(n, 1, 64).astype(np.float32))
            vrot = torch.from_numpy((c[f"s{i}_v"].reshape(n, 64) @ c["rv"]).reshape(n, 1, 64).astype(np.float32))
            epoch += 1
            qsl = torch.from_numpy(c[f"s{i}_qsl"].astype(np.int32)).to(dev)
            seqs = torch.from_numpy(c[f"s{i}_seqs"].astype(np.int32)).to(dev)
            kernels.staging_write(krot.to(dev), vrot.to(dev), slots, qsl, seqs, int(c["sink_eff"]), int(c["recent"]),
                                  sk, sv, owner, winner, epoch)
        assert np.array_equal(owner.cpu().numpy(), c[f"s{i}_owner"]), i
        np.testing.assert_allclose(sk.cpu().numpy(), c[f"s{i}_stage_k"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(sv.cpu().numpy(), c[f"s{i}_stage_v"], rtol=1e-5, atol=1e-6)


def test_staging_collisions_at_scale_match_oracle():
    """Many tokens hashing onto few seats across repeated calls (epoch reuse)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    rng = np.random.default_rng(11)
    bs, hk, d = 16, 2, 64
    st = orc.Staging(bs, hk, d, 32, 48, 64)
    sk = torch.zeros(st.rows, bs, hk, d, device=dev)
    sv = torch.zeros_like(sk)
    owner = torch.full((st.rows, bs), -1, dtype=torch.int64, device=dev)
    winner = torch.zeros(st.rows * bs, dtype=torch.int64, device=dev)
    eye = np.eye(d, dtype=np.float32)
    for step in range(6):
        lens = rng.integers(1, 200, size=5)
        qsl = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        seqs = (lens + rng.integers(0, 400, size=5)).astype(np.int64)
        n = int(qsl[-1])
        slots = rng.integers(-1, 200 * bs, size=n).astype(np.int64)
        k = rng.standard_normal((n, hk, d)).astype(np.float32)
        v = rng.standard_normal((n, hk, d)).astype(np.float32)
        st.write(k, v, eye, eye, slots, qsl.tolist(), seqs.tolist(), n)
        kernels.staging_write(torch.from_numpy(k).to(dev), torch.from_numpy(v).to(dev), torch.from_numpy(slots).to(dev),
                              torch.from_numpy(qsl.astype(np.int32)).to(dev),
                              torch.from_numpy(seqs.astype(np.int32)).to(dev), st.sink_eff, st.recent, sk, sv, owner,
                              winner, step + 1)
        assert np.array_equal(owner.cpu().numpy(), st.owner), step
        assert np.array_equal(sk.cpu().numpy(), st.stage_k), step
        assert np.array_equal(sv.cpu().numpy(), st.stage_v), step


def test_store_rounding_boundaries_bit_exact():
    """Values placed on and a few ulps around every rounding boundary
    (x - zero) / scale = k + 0.5 of their vector: the codes must follow the
    reference's correctly rounded fp32 division exactly."""
    from oscar_b200 import kernels

    dev = need_gpu()
    rng = np.random.default_rng(11)
    n, d, bs = 512, 256, 16
    x = np.zeros((n, 1, d), np.float32)
    for i in range(n):
        lo = np.float32(rng.normal() * 10 ** rng.uniform(-3, 3))
        hi = np.float32(lo + abs(rng.normal()) * 10 ** rng.uniform(-3, 3) + 1e-3)
        row = np.full(d, lo, np.float32)
        row[1] = hi
        scale, zero = orc.vector_scales(row[None])
        s, z = np.float32(scale[0, 0]), np.float32(zero[0, 0])
        vals = []
        for k in range(3):
            c = np.float32(np.float64(z) + np.float64(s) * (k + 0.5))
            for step in range(-4, 5):
                v = c
                for _ in range(abs(step)):
                    v = np.nextafter(v, np.float32(np.inf) if step > 0 else np.float32(-np.inf))
                vals.append(v)
        vals = np.clip(np.array(vals, np.float32), lo, hi)
        row[2:2 + len(vals)] = vals
        x[i, 0] = row
    nb = n // bs + 1
    slots = np.arange(n)
    ek = np.zeros((nb, bs, 1, d), np.uint8)
    ev = np.zeros_like(ek)
    orc.store(x, x, ek, ev, slots)
    kc = torch.zeros(nb, bs, 1, d, dtype=torch.int8, device=dev)
    vc = torch.zeros_like(kc)
    t = torch.from_numpy(x).to(dev)
    kernels.oscar_store(t, t, kc, vc, torch.from_numpy(slots).to(dev))
    assert np.array_equal(cache_bytes(kc), ek)
    assert np.array_equal(cache_bytes(vc), ev)
