"""Shared helpers for the -m gpu parity tests (oracle on CPU, kernels on cuda:0)."""
import numpy as np
import pytest
import torch

from oracle import oscar_oracle as orc

OUT_TOL = dict(atol=2e-2, rtol=2e-2)     # north-star tolerance for bf16 attention output
LSE_TOL = dict(atol=1e-3, rtol=1e-3)     # north-star tolerance for LSE


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def cache_from_bytes(b: np.ndarray, d: int, device) -> torch.Tensor:
    """uint8 [nb, bs, hk, slot_bytes] -> int8 (slot == D) or bf16 (slot == 2D) cache."""
    t = torch.from_numpy(np.ascontiguousarray(b)).to(device)
    if b.shape[-1] == d:
        return t.view(torch.int8)
    assert b.shape[-1] == 2 * d
    return t.view(torch.bfloat16)


def cache_bytes(c: torch.Tensor) -> np.ndarray:
    return c.contiguous().view(torch.uint8).cpu().numpy()


def case_to_oracle(case):
    """synthetic.Case (CPU tensors) -> oracle arguments with caches filled by the oracle store."""
    k8 = case.kc.view(torch.uint8).numpy().copy()
    v8 = case.vc.view(torch.uint8).numpy().copy()
    orc.store(case.old_k.numpy(), case.old_v.numpy(), k8, v8, case.slots.numpy())
    stage = None
    if case.stage is not None:
        stage = tuple(t.numpy() for t in case.stage)
    f = lambda t: None if t is None else t.float().numpy()  # noqa: E731
    dt = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[case.q.dtype]
    return (f(case.q), f(case.k_new), f(case.v_new), k8, v8, case.bt.numpy(), case.qsl, case.seqs, case.scale,
            stage), dt


def case_to_device(case, k8, v8, device):
    d = case.q.shape[-1]
    g = lambda t: None if t is None else t.to(device)  # noqa: E731
    stage = None if case.stage is None else tuple(t.to(device) for t in case.stage)
    return (g(case.q), g(case.k_new), g(case.v_new), cache_from_bytes(k8, d, device), cache_from_bytes(v8, d, device),
            g(case.bt), case.qsl, case.seqs, case.scale, stage)
