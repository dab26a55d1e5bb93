"""The per-layer rotation kernels (x @ R and x @ R^T) against torch's fp64
product, for every dtype pair the backend uses and strided outputs: the fp32
FMA kernel of 16-row tiles, the tcgen05 kind::tf32 kernel with split
precision and the register-tiled FMA kernel of 128-row tiles (each test runs
on all three, through the process-wide rotation path; D 64 always takes the
16-row kernel on the last)."""
import pytest
import torch

from gpu_helpers import need_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["fma", "tensor", "fma_big"], autouse=True)
def rot_path(request):
    from oscar_b200 import kernels

    need_gpu()
    kernels.set_rotation_path(request.param)
    yield request.param
    kernels.set_rotation_path("auto")


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("xdt,odt", [(torch.bfloat16, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.float16, torch.float16), (torch.float32, torch.bfloat16)])
@pytest.mark.parametrize("transpose", [False, True])
def test_rotate_rows_matches_fp64_product(d, xdt, odt, transpose):
    from oscar_b200 import kernels

    dev = need_gpu()
    g = torch.Generator(device="cpu").manual_seed(d + (7 if transpose else 0))
    rot = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    x = torch.randn(37, 3, d, generator=g).to(dev, xdt)  # 111 rows: not a multiple of the 16-row tile
    out, f32 = kernels.rotate_rows(x, rot, transpose=transpose, out=torch.empty(37, 3, d, dtype=odt, device=dev),
                                   out_f32=torch.empty(37, 3, d, dtype=torch.float32, device=dev))
    r = rot.double().t() if transpose else rot.double()
    want = (x.double().reshape(-1, d) @ r).reshape(37, 3, d)
    torch.testing.assert_close(f32.double(), want, atol=2e-5, rtol=2e-5)
    # both outputs come from the same fp32 accumulator: out is its round-to-nearest cast
    torch.testing.assert_close(out, f32.to(odt), atol=0, rtol=0)


def test_rotate_rows_into_strided_rows_of_a_wider_output():
    from oscar_b200 import kernels

    dev = need_gpu()
    d = 256
    rot = torch.linalg.qr(torch.randn(d, d, dtype=torch.float64)).Q.float().to(dev)
    x = torch.randn(10, 6, d, device=dev)
    wide = torch.zeros(12, 6 * d, dtype=torch.bfloat16, device=dev)
    kernels.rotate_rows(x, rot, transpose=True, out=wide[:10].view(10, 6, d))
    want = (x.reshape(-1, d) @ rot.t()).reshape(10, 6 * d).bfloat16()
    torch.testing.assert_close(wide[:10].float(), want.float(), atol=1e-2, rtol=1e-2)
    assert torch.count_nonzero(wide[10:]) == 0


@pytest.mark.parametrize("d", [64, 256])
def test_rotate_rows_many_one_launch_matches_separate_products(d):
    from oscar_b200 import kernels

    dev = need_gpu()
    g = torch.Generator(device="cpu").manual_seed(d)
    rk = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    rv = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    q = torch.randn(5, 6, d, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(5, 1, d, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(5, 1, d, generator=g).to(dev, torch.bfloat16)
    q_lo, k_lo, v_lo = (torch.empty_like(t) for t in (q, k, v))
    k32, v32 = (torch.empty(t.shape, dtype=torch.float32, device=dev) for t in (k, v))
    kernels.rotate_rows_many([(k, rk, k_lo, k32), (v, rv, v_lo, v32), (q, rk, q_lo, None)])
    for x, r, lo, f32 in ((k, rk, k_lo, k32), (v, rv, v_lo, v32), (q, rk, q_lo, None)):
        want = (x.double().reshape(-1, d) @ r.double()).reshape(x.shape)
        if f32 is not None:
            torch.testing.assert_close(f32.double(), want, atol=2e-5, rtol=2e-5)
            torch.testing.assert_close(lo, f32.to(lo.dtype), atol=0, rtol=0)
        torch.testing.assert_close(lo.double(), want.to(lo.dtype).double(), atol=1e-2, rtol=1e-2)


def test_rotation_output_used_as_the_next_rotation_matrix():
    """The kernel loads rotation matrices before waiting for the launch in front
    of it; a matrix that launch just wrote (here: R1 @ R2 computed by the
    library, then used to rotate) must be read after it is complete."""
    from oscar_b200 import kernels

    dev = need_gpu()
    d = 256
    g = torch.Generator(device="cpu").manual_seed(11)
    r1 = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    r2 = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    x = torch.randn(64, d, generator=g).to(dev)
    for _ in range(3):
        prod = torch.full((d, d), float("nan"), device=dev)
        kernels.rotate_rows(r1, r2, out=prod)  # prod = r1 @ r2, written by this launch
        out = torch.empty(64, d, device=dev)
        kernels.rotate_rows(x, prod, out=out)  # reads prod as its rotation right after
        want = x.double() @ (r1.double() @ r2.double())
        torch.testing.assert_close(out.double(), want, atol=5e-5, rtol=5e-5)


@pytest.mark.parametrize("d", [256, 128])
@pytest.mark.parametrize("n", [3001, 1201])
@pytest.mark.parametrize("xdt,odt", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.bfloat16)])
def test_rotate_many_rows(xdt, odt, n, d, rot_path):
    """n tokens x 6 heads (18006 rows in 128-row tiles, 7206 in 64-row tiles,
    a partial last tile each) from a strided view of one buffer (the row-heads
    layout reaches the tensor-core kernel through the layer step,
    tests/test_gpu_step.py)."""
    from oscar_b200 import kernels

    dev = need_gpu()
    heads = 6
    g = torch.Generator(device="cpu").manual_seed(5)
    rot = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64)).Q.float().to(dev)
    buf = torch.randn(n, (heads + 2) * d, generator=g).to(dev, xdt)
    x = buf[:, :heads * d].reshape(n, heads, d)
    out = torch.empty(n, heads, d, dtype=odt, device=dev)
    f32 = torch.empty(n, heads, d, dtype=torch.float32, device=dev)
    kernels.rotate_rows(x, rot, out=out, out_f32=f32)
    want = (x.double().reshape(-1, d) @ rot.double()).reshape(n, heads, d)
    torch.testing.assert_close(f32.double(), want, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(out, f32.to(odt), atol=0, rtol=0)
    assert kernels.device_error(dev) == 0
