"""The staging-window write for callers that cannot allocate device memory.

`oscar_staging_write_noalloc` keeps its seat-winner scratch in a static device
array inside the library instead of taking caller-allocated scratch, for
engines that have handed all device memory to the KV cache or hosts that
forbid allocations after start-up.  It is checked through the C ABI against
the regular `oscar_staging_write` on two calls in a row over the same arena:
the second call lands on the same seats with lower token indices, so winners
left in the shared array by the first call would win if the array were not
cleared between calls.

This file is collected last so that a stop-at-first-failure run has already
run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BS, ROWS, HK, D = 16, 32, 2, 64
SINK_EFF, RECENT = 16, 48


def _arena(dev):
    sk = torch.zeros(ROWS, BS, HK, D, device=dev)
    return sk, torch.zeros_like(sk), torch.full((ROWS, BS), -1, dtype=torch.int64, device=dev)


def _call_inputs(rng, lengths, extra, dev):
    n = int(sum(lengths))
    qsl = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    seqs = (np.asarray(lengths) + np.asarray(extra)).astype(np.int32)
    slots = rng.integers(0, 2 * ROWS * BS, size=n).astype(np.int64)  # blocks b and b + ROWS share seats
    slots[rng.random(n) < 0.1] = -1
    k = torch.from_numpy(rng.standard_normal((n, HK, D)).astype(np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((n, HK, D)).astype(np.float32)).to(dev)
    return (k, v, torch.from_numpy(slots).to(dev), torch.from_numpy(qsl).to(dev), torch.from_numpy(seqs).to(dev),
            len(lengths))


def test_noalloc_staging_write_matches_regular_entry_point_on_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from oscar_b200 import _native, kernels

    dev = torch.device("cuda", 0)
    lib = _native.lib()
    rng = np.random.default_rng(2026)
    ref_arena, na_arena = _arena(dev), _arena(dev)
    winner = torch.zeros(ROWS * BS, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    calls = [([100, 120, 80], [500, 10, 300]), ([25, 15], [7, 900])]
    for epoch, (lengths, extra) in enumerate(calls, start=1):
        k, v, slots, qsl, seqs, nreq = _call_inputs(rng, lengths, extra, dev)
        kernels.staging_write(k, v, slots, qsl, seqs, SINK_EFF, RECENT, *ref_arena, winner, epoch)
        sk, sv, owner = na_arena
        st = lib.oscar_staging_write_noalloc(
            k.data_ptr(), v.data_ptr(), k.shape[0], HK, D, slots.data_ptr(), qsl.data_ptr(), seqs.data_ptr(), nreq,
            SINK_EFF, RECENT, sk.data_ptr(), sv.data_ptr(), owner.data_ptr(), ROWS, BS, ctypes.c_void_p(stream))
        _native.check(st)
        torch.cuda.synchronize(dev)
        assert torch.equal(na_arena[2], ref_arena[2]), f"owner tags differ after call {epoch}"
        assert torch.equal(na_arena[0], ref_arena[0]), f"staged K differs after call {epoch}"
        assert torch.equal(na_arena[1], ref_arena[1]), f"staged V differs after call {epoch}"
        assert int((na_arena[2] >= 0).sum()) > 0
    assert kernels.device_error(dev) == 0


def test_noalloc_rejects_arenas_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from oscar_b200 import _native

    lib = _native.lib()
    dummy = torch.zeros(16, device="cuda")
    p = dummy.data_ptr()
    st = lib.oscar_staging_write_noalloc(p, p, 1, 1, 4, p, p, p, 1, 0, 0, p, p, p, 1024, 128, None)
    assert st == _native.ERR_INVALID
    assert b"exceed the built-in scratch" in lib.oscar_last_error()
