"""Generate golden vectors by running the reference implementation itself.

Runs ONLY in the build container (the reference tree is not present on GPU
boxes).  The reference is the pure-Python ``oscar_ascend`` package; its torch
CPU path (``OSCAR_ASCEND_USE_TRITON=0``) is the parity oracle for this build.
``vllm``, ``vllm_ascend`` and ``torch_npu`` are masked in ``sys.modules`` so the
reference selects its CPU placeholders (oscar_ascend/backend.py:68-85).

Usage:  python tests/golden/make_golden.py REFERENCE_ROOT   (or OSCAR_REFERENCE=...)
Writes ``tests/golden/*.npz``; the committed fixtures are what the tests read.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path
from types import SimpleNamespace as NS

import numpy as np

HERE = Path(__file__).resolve().parent


def _import_reference(root: str):
    for name in ("vllm", "vllm_ascend", "torch_npu"):
        sys.modules[name] = None
    sys.dont_write_bytecode = True
    sys.path.insert(0, root)
    import torch  # noqa: F401

    import oscar_ascend.backend as backend
    import oscar_ascend.format as fmt
    import oscar_ascend.kernels.slab_attention as slab
    import oscar_ascend.kernels.store_kernel as store
    import oscar_ascend.kernels.streaming_attention as stream

    return NS(backend=backend, fmt=fmt, slab=slab, store=store, stream=stream)


def f32(t):
    return t.detach().float().cpu().numpy().astype(np.float32)


def u8(t):
    return t.detach().contiguous().view(__import__("torch").uint8).cpu().numpy().copy()


def outliers(x, channels=(3, 77, 150, 201), factor=20.0):
    d = x.shape[-1]
    for c in channels:
        if c < d:
            x[..., c] *= factor
    return x


# ---------------------------------------------------------------------------
def gen_store(ref, torch):
    cases = {}
    g = torch.Generator().manual_seed(2024)

    def run(name, k, v, slots, nb, bs, hk, d, cache_dtype):
        kc = torch.zeros(nb, bs, hk, d, dtype=cache_dtype)
        vc = torch.zeros_like(kc)
        # random garbage everywhere: pins that untouched bytes (pad, other slots) survive
        kc.view(torch.uint8).copy_(torch.randint(0, 256, kc.view(torch.uint8).shape, generator=g, dtype=torch.uint8))
        vc.view(torch.uint8).copy_(torch.randint(0, 256, vc.view(torch.uint8).shape, generator=g, dtype=torch.uint8))
        k8_before, v8_before = u8(kc), u8(vc)
        ref.store.oscar_store_ref(k, v, kc, vc, torch.tensor(slots, dtype=torch.int64))
        cases[name] = dict(
            k_rot=f32(k), v_rot=f32(v), slots=np.asarray(slots, np.int64),
            k8_before=k8_before, v8_before=v8_before, k8_after=u8(kc), v8_after=u8(vc),
            slot_bytes=np.int64(k8_before.shape[-1]),
        )

    # 1. D=256, Hk=1, int8 packed x2 geometry, outlier channels, two negative slots
    n, hk, d, bs, nb = 40, 1, 256, 16, 6
    k = outliers(torch.randn(n, hk, d, generator=g) * 1.5)
    v = outliers(torch.randn(n, hk, d, generator=g))
    slots = torch.randperm(nb * bs, generator=g)[:n].tolist()
    slots[5] = -1
    slots[17] = -1
    run("d256_hk1_int8", k, v, slots, nb, bs, hk, d, torch.int8)
    # 2. D=64, Hk=2, bf16 legacy geometry (512 B-per-head equivalent: 2*D bytes)
    n, hk, d, bs, nb = 12, 2, 64, 4, 8
    k = torch.randn(n, hk, d, generator=g) * 1.5
    v = torch.randn(n, hk, d, generator=g) * 1.5
    slots = [3, -1, 7, 8, 30, 31, 0, 1, 2, -1, 12, 13]
    run("d64_hk2_bf16", k, v, slots, nb, bs, hk, d, torch.bfloat16)
    # 3. constant vectors (tests/test_backend.py:153-162 values)
    vals = torch.tensor([0.0, 1.0, -1.25, 1e-7])
    k = vals[:, None, None].expand(4, 1, 64).contiguous()
    v = (-vals)[:, None, None].expand(4, 1, 64).contiguous()
    run("const_d64", k, v, [0, 1, 2, 3], 2, 4, 1, 64, torch.int8)
    # 4. D=256, Hk=4, bf16-valued inputs
    n, hk, d, bs, nb = 9, 4, 256, 8, 3
    k = torch.randn(n, hk, d, generator=g).bfloat16().float()
    v = torch.randn(n, hk, d, generator=g).bfloat16().float()
    run("d256_hk4_bf16vals", k, v, list(range(5, 14)), nb, bs, hk, d, torch.int8)
    # 5. D=32, Hk=2, legacy geometry (tests/test_numeric.py:82-103 shape)
    k = torch.randn(6, 2, 32, generator=g) * 1.5
    v = torch.randn(6, 2, 32, generator=g) * 1.5
    run("d32_hk2_bf16", k, v, list(range(6)), 3, 4, 2, 32, torch.bfloat16)
    # 6. exact .5 ties: min 0, max 3 -> scale 1, zero 0; x = j + 0.5 pins floor(+0.5)
    base = torch.tensor([0.0, 3.0, 0.5, 1.5, 2.5, 1.0, 2.0, 0.49999997, 2.5000002]).repeat(8)[:64]
    k = base[None, None, :].expand(3, 1, 64).contiguous().clone()
    k[1] *= 0.25
    k[2] = k[2] * 6.0 - 7.0
    v = k.flip(-1).contiguous()
    run("ties_d64", k, v, [4, 5, 6], 2, 8, 1, 64, torch.int8)
    # 7. duplicate slot inside one call (last writer wins on the CPU index_put_ path)
    n, hk, d = 5, 1, 64
    k = torch.randn(n, hk, d, generator=g)
    v = torch.randn(n, hk, d, generator=g)
    run("dup_slot_d64", k, v, [2, 9, 2, 5, 9], 4, 4, hk, d, torch.int8)
    return cases


def gen_clip(ref, torch):
    g = torch.Generator().manual_seed(99)
    x = outliers(torch.randn(16, 2, 256, generator=g)).bfloat16().float()
    rot = torch.linalg.qr(torch.randn(256, 256, generator=g)).Q.contiguous()
    impl = NS(_oscar_warned_quantile=True)
    out = dict(x=f32(x), rot=f32(rot))
    for ratio in (0.0, 0.5, 0.92, 0.96, 1.0):
        y = ref.backend.AscendOscarAttentionBackendImpl._rotate_clip(impl, x, rot, ratio)
        out[f"y_{int(round(ratio * 100))}"] = f32(y)
    return {"clip": out}


def _meta(torch, slots, ends, seqs, bt=None):
    return NS(
        num_actual_tokens=len(slots),
        slot_mapping=torch.tensor(slots),
        query_start_loc=torch.tensor([0] + ends),
        actual_seq_lengths_q=ends,
        seq_lens=torch.tensor(seqs),
        seq_lens_cpu=torch.tensor(seqs),
        seq_lens_list=seqs,
        block_tables=torch.tensor(bt or [[0, 1, 2, 3]], dtype=torch.int32),
    )


def _fixture_impl(ref, torch, hk=1, d=64, hq_per=2, sink=4, recent=4, staging=8, nb=8, bs=4, cache_dtype=None):
    Impl = ref.backend.AscendOscarAttentionBackendImpl
    impl = Impl.__new__(Impl)
    impl.head_size, impl.num_kv_heads, impl.num_heads = d, hk, hk * hq_per
    impl.scale = d**-0.5
    impl.key_cache = impl.value_cache = None
    impl._oscar_setup()
    impl._oscar.sink_tokens = sink
    impl._oscar.recent_tokens = recent
    impl._oscar.staging_tokens = staging
    layer = NS(layer_name="model.layers.0.self_attn.attn")
    cache = [torch.zeros(nb, bs, hk, d, dtype=cache_dtype or torch.bfloat16) for _ in range(2)]
    impl._set_caches(cache)
    return impl, layer, cache


def gen_staging(ref, torch):
    """A sequence of staging writes + invalidations on the reference fixture
    geometry (tests/test_backend.py:27-106)."""
    g = torch.Generator().manual_seed(5)
    impl, layer, cache = _fixture_impl(ref, torch)
    impl._ensure_staging(layer, cache)
    eye = torch.eye(64)
    rk = torch.linalg.qr(torch.randn(64, 64, generator=g)).Q
    rv = torch.linalg.qr(torch.randn(64, 64, generator=g)).Q
    layer._oscar_rots = (rk, rv)
    del eye
    rows = layer._oscar_stage_rows
    steps = [
        # (slots, ends, seqs) ; invalidate-only steps use ends=None
        ([0, 1, 2, 3], [4], [4]),
        ([4], [1], [5]),
        (list(range(12)), [12], [100]),
        ([0, rows * 4], [1, 2, 4], [1, 1, 1]),          # collision + padding request
        ([5, 6, 7, -1, 9, 10], [2, 6], [7, 4]),          # negative slot inside
        ([1, 2], None, None),                            # direct do_kv_cache_update invalidation
        ([16, 17, 18, 19, 20, 21, 22, 23, 24], [3, 9], [3, 40]),
    ]
    rec = dict(rows=np.int64(rows), bs=np.int64(4), sink_eff=np.int64(impl.sink_eff),
               recent=np.int64(impl._oscar.recent_tokens), rk=f32(rk), rv=f32(rv))
    for i, (slots, ends, seqs) in enumerate(steps):
        n = len(slots)
        k = torch.randn(n, 1, 64, generator=g)
        v = torch.randn(n, 1, 64, generator=g)
        if ends is None:
            impl.do_kv_cache_update(layer, k, v, cache, torch.tensor(slots))
            kind = 1
        else:
            impl._staging_write(layer, k, v, _meta(torch, slots, ends, seqs))
            kind = 0
        rec[f"s{i}_kind"] = np.int64(kind)
        rec[f"s{i}_slots"] = np.asarray(slots, np.int64)
        rec[f"s{i}_qsl"] = np.asarray([0] + (ends or []), np.int64)
        rec[f"s{i}_seqs"] = np.asarray(seqs or [], np.int64)
        rec[f"s{i}_k"] = f32(k)
        rec[f"s{i}_v"] = f32(v)
        rec[f"s{i}_owner"] = layer._oscar_slot_owner.numpy().copy()
        rec[f"s{i}_stage_k"] = f32(layer._oscar_stage_k)
        rec[f"s{i}_stage_v"] = f32(layer._oscar_stage_v)
    rec["nsteps"] = np.int64(len(steps))
    return {"staging": rec}


def _attn_case(ref, torch, *, seed, d, hk, g_heads, bs, prefixes, lengths, fresh, window,
               qdtype, cache_dtype, outlier=False, nb_extra=3):
    gen = torch.Generator().manual_seed(seed)
    hq = hk * g_heads
    seqs = [p + n if fresh else p for p, n in zip(prefixes, lengths)]
    width = max(1, math.ceil(max(max(seqs, default=0), 1) / bs))
    blocks = len(seqs) * width + nb_extra
    bt = torch.randperm(blocks, generator=gen)[: len(seqs) * width].reshape(len(seqs), width).int()
    kc = torch.zeros(blocks, bs, hk, d, dtype=cache_dtype)
    vc = torch.zeros_like(kc)
    qsl, slots = [0], []
    for req, (prefix, n) in enumerate(zip(prefixes, lengths)):
        pos = torch.arange(prefix)
        slots.append(bt[req, pos // bs].long() * bs + pos % bs)
        qsl.append(qsl[-1] + n)
    old = [torch.randn(sum(prefixes), hk, d, generator=gen) for _ in range(2)]
    if outlier:
        old = [outliers(o) for o in old]
    ref.store.oscar_store_ref(*old, kc, vc, torch.cat(slots) if slots else torch.zeros(0, dtype=torch.long))
    q = torch.randn(qsl[-1], hq, d, generator=gen).to(qdtype)
    k = v = None
    if fresh:
        k, v = [torch.randn(qsl[-1], hk, d, generator=gen).to(qdtype) for _ in range(2)]
    stage = None
    if window:
        rows = max(3, math.ceil(blocks / 6))
        sk = torch.zeros(rows, bs, hk, d)
        sv = torch.zeros(rows, bs, hk, d)
        owner = torch.full((rows, bs), -1, dtype=torch.int64)
        offset = 0
        for req, prefix in enumerate(prefixes):
            retained = list(range(min(bs, prefix))) + list(range(max(bs, prefix - 2 * bs), prefix))
            for pos in retained:
                block = int(bt[req, pos // bs])
                row, col = block % rows, pos % bs
                owner[row, col] = block
                sk[row, col], sv[row, col] = old[0][offset + pos], old[1][offset + pos]
            offset += prefix
        # a stale owner tag that must NOT hit (different block id on the same seat)
        owner[0, 0] = 10_000 + owner.shape[0] * 3
        stage = (sk, sv, owner)
    args = (q, k, v, kc, vc, bt, qsl, seqs, d**-0.5, stage)
    out, lse = ref.stream.streaming_attention_ref(*args)
    sout, slse = ref.slab.slab_attention(*args, chunk_tokens=37, workspace_bytes=64 * 2 * hk * d * 2)
    rec = dict(
        q=f32(q), k_new=f32(k) if k is not None else np.zeros(0, np.float32),
        v_new=f32(v) if v is not None else np.zeros(0, np.float32), has_new=np.int64(fresh),
        k8=u8(kc), v8=u8(vc), bt=bt.numpy(), qsl=np.asarray(qsl, np.int64), seqs=np.asarray(seqs, np.int64),
        scale=np.float32(d**-0.5), has_stage=np.int64(window), qdtype=np.array(str(qdtype).split(".")[-1]),
        cache_dtype=np.array(str(cache_dtype).split(".")[-1]),
        out=f32(out), lse=f32(lse),
    )
    # the reference's two CPU read paths agree (tests/test_slab_attention.py:21-35)
    torch.testing.assert_close(sout, out, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(slse, lse, atol=2e-5, rtol=2e-5)
    if window:
        rec.update(stage_k=f32(stage[0]), stage_v=f32(stage[1]), owner=stage[2].numpy())
    return rec


def gen_attention(ref, torch):
    bf16, f16, i8 = torch.bfloat16, torch.float16, torch.int8
    specs = {
        "mixed_d256": dict(seed=1, d=256, hk=1, g_heads=6, bs=16, prefixes=[0, 129, 300, 0], lengths=[1, 4, 3, 0],
                           fresh=True, window=True, qdtype=bf16, cache_dtype=i8, outlier=True),
        "mtp_hk2_d256": dict(seed=2, d=256, hk=2, g_heads=6, bs=16, prefixes=[257, 95], lengths=[4, 4],
                             fresh=True, window=True, qdtype=bf16, cache_dtype=i8),
        "nowin_d256": dict(seed=3, d=256, hk=1, g_heads=6, bs=32, prefixes=[400], lengths=[4],
                           fresh=True, window=False, qdtype=bf16, cache_dtype=i8, outlier=True),
        "cache_only_multi": dict(seed=4, d=256, hk=1, g_heads=6, bs=16, prefixes=[3, 263], lengths=[7, 9],
                                 fresh=False, window=True, qdtype=bf16, cache_dtype=i8),
        "cache_only_empty": dict(seed=5, d=256, hk=1, g_heads=6, bs=16, prefixes=[0, 257], lengths=[1, 1],
                                 fresh=False, window=False, qdtype=bf16, cache_dtype=i8),
        "cached_prefill": dict(seed=6, d=256, hk=1, g_heads=6, bs=16, prefixes=[129], lengths=[40],
                               fresh=True, window=True, qdtype=bf16, cache_dtype=i8),
        "legacy_hk2_d64_f16": dict(seed=7, d=64, hk=2, g_heads=6, bs=8, prefixes=[67, 1, 15], lengths=[4, 1, 0],
                                   fresh=True, window=True, qdtype=f16, cache_dtype=bf16),
        "hk4_d128_f16": dict(seed=8, d=128, hk=4, g_heads=2, bs=8, prefixes=[40, 9], lengths=[3, 2],
                             fresh=True, window=False, qdtype=f16, cache_dtype=i8),
        "f32_query_d64": dict(seed=9, d=64, hk=1, g_heads=2, bs=4, prefixes=[21], lengths=[3],
                              fresh=True, window=True, qdtype=torch.float32, cache_dtype=bf16),
    }
    return {f"attn_{name}": _attn_case(ref, torch, **spec) for name, spec in specs.items()}


def gen_merge(ref, torch):
    """tests/test_slab_attention.py:220-259 edge cases (-inf, +-1000, NaN)."""
    torch.manual_seed(91)
    out = torch.randn(5, 2, 64)
    lse = torch.tensor([[-torch.inf, 1000.0], [2.0, -torch.inf], [1.0, 3.0], [0.0, 0.0], [0.0, 0.0]])
    part = torch.randn(3, 2, 64).half()
    logs = torch.tensor([[-torch.inf, -1000.0], [float("nan"), 4.0], [3.0, -torch.inf]])
    out[0, 0] = part[0, 0] = torch.nan
    rec = dict(out=f32(out), lse=f32(lse), part=f32(part), part_lse=f32(logs))
    for name, ids, start in (("contig", None, 0), ("contig2", None, 2), ("indexed", torch.tensor([0, 3, 1], dtype=torch.int32), 0)):
        o, l = out.clone(), lse.clone()
        ref.slab.merge_slab(o, l, part, logs, start, ids)
        rec[f"{name}_out"] = f32(o)
        rec[f"{name}_lse"] = f32(l)
        rec[f"{name}_start"] = np.int64(start)
        rec[f"{name}_ids"] = ids.numpy() if ids is not None else np.zeros(0, np.int32)
    return {"merge": rec}


def gen_backend(ref, torch):
    """Two full layer steps through the reference backend (CPU path): a cached
    continuation that writes history, then a 4-token MTP step; rotations are
    QR-of-Gaussian, clip 0.96/0.92, sink/recent windows on."""
    g = torch.Generator().manual_seed(31)
    d, hk, gh, bs = 256, 2, 6, 16
    impl, layer, cache = _fixture_impl(ref, torch, hk=hk, d=d, hq_per=gh, sink=16, recent=32, staging=256,
                                       nb=40, bs=bs, cache_dtype=torch.int8)
    impl._oscar.k_clip_ratio, impl._oscar.v_clip_ratio = 0.96, 0.92
    impl._oscar.attention_mode = "streaming"
    rk = torch.linalg.qr(torch.randn(d, d, generator=g)).Q.contiguous()
    rv = torch.linalg.qr(torch.randn(d, d, generator=g)).Q.contiguous()
    layer._oscar_rots = (rk, rv)
    bt = torch.randperm(40, generator=g)[:36].reshape(2, 18).int()
    rec = dict(rk=f32(rk), rv=f32(rv), bt=bt.numpy(), d=np.int64(d), hk=np.int64(hk), hq=np.int64(hk * gh),
               bs=np.int64(bs), nb=np.int64(40), sink=np.int64(16), recent=np.int64(32), staging=np.int64(256),
               k_clip=np.float32(0.96), v_clip=np.float32(0.92))
    impl._ensure_staging(layer, cache)
    # step 0: fresh prefill of request 0 (150 tokens) and request 1 (90 tokens)
    # step 1: 4-token MTP step on both
    # step 2: cache-only decode of 1 token each (key=None)
    steps = [([0, 0], [100, 60]), ([100, 60], [4, 4])]
    for i, (prefixes, lengths) in enumerate(steps):
        n = sum(lengths)
        qsl = [0]
        slots = []
        for r, (p, L) in enumerate(zip(prefixes, lengths)):
            pos = torch.arange(p, p + L)
            slots.append(bt[r, pos // bs].long() * bs + pos % bs)
            qsl.append(qsl[-1] + L)
        seqs = [p + L for p, L in zip(prefixes, lengths)]
        q = outliers(torch.randn(n, hk * gh, d, generator=g)).bfloat16()
        k = outliers(torch.randn(n, hk, d, generator=g)).bfloat16()
        v = outliers(torch.randn(n, hk, d, generator=g)).bfloat16()
        md = NS(num_actual_tokens=n, slot_mapping=torch.cat(slots), actual_seq_lengths_q=qsl[1:],
                seq_lens_list=seqs, block_tables=bt)
        out = impl.forward(layer, q, k, v, cache, md,
                           output=torch.empty(n, hk * gh * d, dtype=torch.bfloat16))
        rec.update({f"s{i}_q": f32(q), f"s{i}_k": f32(k), f"s{i}_v": f32(v), f"s{i}_qsl": np.asarray(qsl),
                    f"s{i}_seqs": np.asarray(seqs), f"s{i}_slots": f32(torch.cat(slots)).astype(np.int64),
                    f"s{i}_out": f32(out)})
    rec.update(k8=u8(cache[0]), v8=u8(cache[1]), owner=layer._oscar_slot_owner.numpy().copy(),
               stage_k=f32(layer._oscar_stage_k), stage_v=f32(layer._oscar_stage_v))
    # step 2: cache-only decode
    n = 2
    q = outliers(torch.randn(n, hk * gh, d, generator=g)).bfloat16()
    md = NS(num_actual_tokens=n, slot_mapping=torch.tensor([-1, -1]), actual_seq_lengths_q=[1, 2],
            seq_lens_list=[104, 64], block_tables=bt)
    out = impl.forward(layer, q, None, None, cache, md, output=torch.empty(n, hk * gh * d, dtype=torch.bfloat16))
    rec.update(s2_q=f32(q), s2_qsl=np.asarray([0, 1, 2]), s2_seqs=np.asarray([104, 64]), s2_out=f32(out))
    rec["rows"] = np.int64(layer._oscar_stage_rows)
    return {"backend": rec}


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("OSCAR_REFERENCE")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_ROOT (or set OSCAR_REFERENCE)")
    ref = _import_reference(root)
    import torch

    torch.set_num_threads(4)
    out = {}
    out.update(gen_store(ref, torch))
    out.update(gen_clip(ref, torch))
    out.update(gen_staging(ref, torch))
    out.update(gen_attention(ref, torch))
    out.update(gen_merge(ref, torch))
    out.update(gen_backend(ref, torch))
    for name, rec in out.items():
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **rec)
        print(f"wrote {path.name} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
