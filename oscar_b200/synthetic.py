"""Seeded synthetic workloads for the OSCAR hot path (tests and bench).

Follows the case construction of delivery/probe_streaming.py:31-81
(make_case): history K/V ~ N(0, 1) (optionally with four outlier channels
x20), written into 128-token pages through randomly permuted block tables;
sink/recent tokens also live unquantized in an fp32 staging arena with owner
tags; queries and the current chunk are bf16.  Values are generated in the
rotated space (identity rotation), exactly as the reference probe does.

``BASELINE_CONFIGS`` holds the five workloads of the benchmark definition.
The reference measures on no public dataset; these seeded inputs stand in.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

OUTLIER_CHANNELS = (3, 77, 150, 201)


@dataclass
class Case:
    q: torch.Tensor
    k_new: torch.Tensor | None
    v_new: torch.Tensor | None
    kc: torch.Tensor
    vc: torch.Tensor
    bt: torch.Tensor
    qsl: list
    seqs: list
    scale: float
    stage: tuple | None
    old_k: torch.Tensor          # [sum(prefixes), hk, d] fp32 history values (rotated space)
    old_v: torch.Tensor
    slots: torch.Tensor          # [sum(prefixes)] int64 cache slots of the history
    meta: dict = field(default_factory=dict)

    def args(self):
        """Positional arguments of slab_attention / streaming_attention_ref."""
        return (self.q, self.k_new, self.v_new, self.kc, self.vc, self.bt, self.qsl, self.seqs, self.scale, self.stage)


def _outliers(x: torch.Tensor, factor: float = 20.0) -> torch.Tensor:
    for c in OUTLIER_CHANNELS:
        if c < x.shape[-1]:
            x[..., c] *= factor
    return x


def make_case(prefixes, lengths, *, hk=1, group=6, d=256, dtype=torch.bfloat16, cache_dtype=torch.int8, bs=128,
              window=True, fresh=True, seed=117, outliers=True, sink=128, recent=256, staging_tokens=8192,
              device="cpu", extra_blocks=0, compact=False, headroom=0) -> Case:
    """Build one case.  Caches are allocated zeroed; fill them with
    :func:`fill_caches` (device kernel) or with the CPU oracle in tests.
    ``compact`` allocates only the pages the requests use (plus ``headroom``
    tokens of growth each) instead of a full-width block table per request;
    unused block-table entries are 0."""
    gen = torch.Generator(device=device).manual_seed(seed)
    hq = hk * group
    seqs = [p + n if fresh else p for p, n in zip(prefixes, lengths)]
    width = max(16, math.ceil((max(seqs, default=0) + headroom) / bs / 16) * 16)
    if compact:
        need = [math.ceil((s_ + headroom) / bs) for s_ in seqs]
        blocks = sum(need) + extra_blocks
        perm = torch.randperm(blocks, generator=gen, device=device).to(torch.int32)
        bt = torch.zeros(len(seqs), width, dtype=torch.int32, device=device)
        off = 0
        for r, n_ in enumerate(need):
            bt[r, :n_] = perm[off:off + n_]
            off += n_
    else:
        blocks = len(seqs) * width + extra_blocks
        perm = torch.randperm(blocks, generator=gen, device=device)
        bt = perm[: len(seqs) * width].reshape(len(seqs), width).to(torch.int32)
    kc = torch.zeros(blocks, bs, hk, d, dtype=cache_dtype, device=device)
    vc = torch.zeros_like(kc)
    qsl, slots = [0], []
    for req, (prefix, n) in enumerate(zip(prefixes, lengths)):
        pos = torch.arange(prefix, device=device)
        slots.append(bt[req, pos // bs].long() * bs + pos % bs)
        qsl.append(qsl[-1] + n)
    total = sum(prefixes)
    old_k = torch.randn(total, hk, d, generator=gen, device=device)
    old_v = torch.randn(total, hk, d, generator=gen, device=device)
    if outliers:
        old_k, old_v = _outliers(old_k), _outliers(old_v)
    q = torch.randn(qsl[-1], hq, d, generator=gen, device=device).to(dtype)
    k_new = v_new = None
    if fresh:
        k_new = torch.randn(qsl[-1], hk, d, generator=gen, device=device)
        v_new = torch.randn(qsl[-1], hk, d, generator=gen, device=device)
        if outliers:
            k_new, v_new = _outliers(k_new), _outliers(v_new)
        k_new, v_new = k_new.to(dtype), v_new.to(dtype)
    stage = None
    if window:
        sink_eff = (sink // bs) * bs
        rows = max(math.ceil(staging_tokens / bs), (sink_eff // bs) + (recent + bs - 1) // bs + 3)
        sk = torch.zeros(rows, bs, hk, d, device=device)
        sv = torch.zeros_like(sk)
        owner = torch.full((rows, bs), -1, dtype=torch.int64, device=device)
        offset = 0
        for req, prefix in enumerate(prefixes):
            tail0 = max(sink_eff, prefix - recent)
            retained = torch.cat([torch.arange(min(sink_eff, prefix), device=device),
                                  torch.arange(min(tail0, prefix), prefix, device=device)])
            if retained.numel():
                blk = bt[req, retained // bs].long()
                row, col = blk % rows, retained % bs
                owner[row, col] = blk
                sk[row, col] = old_k[offset + retained]
                sv[row, col] = old_v[offset + retained]
            offset += prefix
        stage = (sk, sv, owner)
    slot_t = torch.cat(slots) if slots else torch.zeros(0, dtype=torch.int64, device=device)
    return Case(q, k_new, v_new, kc, vc, bt, qsl, seqs, d**-0.5, stage, old_k, old_v, slot_t,
                meta=dict(hk=hk, hq=hq, d=d, bs=bs, blocks=blocks))


def fill_caches(case: Case, chunk_tokens: int = 1 << 16) -> None:
    """Write the history into the paged caches with the device store kernel."""
    from .kernels import oscar_store

    n = case.slots.numel()
    for a in range(0, n, chunk_tokens):
        b = min(n, a + chunk_tokens)
        oscar_store(case.old_k[a:b], case.old_v[a:b], case.kc, case.vc, case.slots[a:b])


def lognormal_lengths(n: int, seed: int, median: int = 4096, sigma: float = 1.0, lo: int = 1024, hi: int = 32768):
    rng = np.random.default_rng(seed)
    x = np.exp(rng.normal(math.log(median), sigma, n))
    return [int(v) for v in np.clip(x, lo, hi)]


# BASELINE.json configs (name -> make_case keyword arguments)
BASELINE_CONFIGS = {
    "cfg1_mtp_8k": dict(prefixes=[8192], lengths=[4], hk=1, group=6),
    "cfg2_mtp_24k": dict(prefixes=[24576], lengths=[4], hk=1, group=6),
    "cfg3_mtp_8x24k": dict(prefixes=[24576] * 8, lengths=[4] * 8, hk=1, group=6),
    "cfg4_continuation": dict(prefixes=[9256], lengths=[15360], hk=4, group=6),
    "cfg5_mixed_64": dict(prefixes=lognormal_lengths(64, 5), lengths=[1 + (i * 7) % 4 for i in range(64)], hk=4,
                          group=6),
}


def attention_flops(prefixes, lengths, hq: int, d: int) -> float:
    """Algorithmic FLOPs of one slab attention pass: 4 Hq D per (query, key)
    pair, over each request's history (N x C) and causal current chunk
    (N (N + 1) / 2)."""
    pairs = sum(n * c + n * (n + 1) // 2 for c, n in zip(prefixes, lengths))
    return 4.0 * hq * d * pairs
