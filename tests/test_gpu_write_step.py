"""The fused write step (store + staging write in one launch) leaves exactly
the bytes of the separate store and staging-write kernels: colliding seats
(the later token wins), negative slots, padding tokens after the last
request."""
import pytest
import torch

from gpu_helpers import need_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,hk,reqs", [(7, 1, [3, 4]), (64, 2, [16, 16, 16, 10]), (256, 1, [100, 100, 50])])
def test_write_step_equals_store_then_staging_write(n, hk, reqs):
    from oscar_b200 import kernels

    dev = need_gpu()
    g = torch.Generator(device="cpu").manual_seed(n + hk)
    d, bs, blocks, rows = 256, 16, 64, 6
    k = (torch.randn(n, hk, d, generator=g) * 3).to(dev)
    v = torch.randn(n, hk, d, generator=g).to(dev)
    # unique slots (a step never writes one slot twice) over 64 blocks but only
    # rows x bs = 96 staging seats: seats collide; the later token must win
    slots = torch.randperm((blocks - rows) * bs, generator=g)[:n]
    slots[n - 1] = slots[0] % bs + ((slots[0] // bs) % rows + rows * 9) * bs  # one sure collision
    assert len(set(slots.tolist())) == n
    seats = (slots // bs % rows) * bs + slots % bs
    assert len(set(seats.tolist())) < n
    slots[1::9] = -1                      # skipped tokens
    slots = slots.to(dev)
    qsl = [0]
    for r in reqs:
        qsl.append(qsl[-1] + r)           # tokens after qsl[-1] are padding
    seqs = [qsl[i + 1] - qsl[i] + 40 * (i + 1) for i in range(len(reqs))]
    qsl_d = torch.tensor(qsl, dtype=torch.int32, device=dev)
    seqs_d = torch.tensor(seqs, dtype=torch.int32, device=dev)

    def fresh():
        kc = torch.zeros(blocks, bs, hk, d, dtype=torch.int8, device=dev)
        vc = torch.zeros_like(kc)
        sk = torch.zeros(rows, bs, hk, d, device=dev)
        sv = torch.zeros_like(sk)
        owner = torch.full((rows, bs), -1, dtype=torch.int64, device=dev)
        owner[0, :4] = 7                  # stale tags that the step must overwrite or keep
        return kc, vc, sk, sv, owner

    a = fresh()
    kernels.oscar_store(k, v, a[0], a[1], slots, 0.9, 0.5)
    winner = torch.zeros(rows * bs, dtype=torch.int64, device=dev)
    kernels.staging_write(k, v, slots, qsl_d, seqs_d, 16, 24, a[2], a[3], a[4], winner, 1)
    b = fresh()
    kernels.write_step(k, v, b[0], b[1], slots, 0.9, 0.5, qsl_d, seqs_d, 16, 24, b[2], b[3], b[4])
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    assert kernels.device_error(dev) == 0


def test_write_step_rejects_large_batches():
    from oscar_b200 import kernels

    dev = need_gpu()
    n = kernels.WRITE_STEP_MAX_TOKENS + 1
    k = torch.zeros(n, 1, 64, device=dev)
    kc = torch.zeros(4, 16, 1, 64, dtype=torch.int8, device=dev)
    with pytest.raises(Exception):
        kernels.write_step(k, k, kc, kc.clone(), torch.zeros(n, dtype=torch.int64, device=dev), 0.0, 0.0,
                           torch.tensor([0, n], dtype=torch.int32, device=dev),
                           torch.tensor([n], dtype=torch.int32, device=dev), 0, 8,
                           torch.zeros(4, 16, 1, 64, device=dev), torch.zeros(4, 16, 1, 64, device=dev),
                           torch.full((4, 16), -1, dtype=torch.int64, device=dev))
