"""Kernel-level API over the C ABI (torch tensors in, device work out).

Mirrors the reference's kernel entry points for the hot path:
  * ``oscar_store``       kernels/store_kernel.py:54-102 / :247-279 (+ clip of backend.py:140-146)
  * ``staging_invalidate`` backend.py:172-176
  * ``staging_write``     backend.py:513-555
  * ``slab_attention``    kernels/slab_attention.py:376-476 (semantics of
                          kernels/streaming_attention.py:134-196)
  * ``slab_attention_shard`` one history shard of slab_attention.py:458-475
                          (split-KV across GPUs)
  * ``merge_slab``        kernels/slab_attention.py:341-373

Layout problems raise ValueError with the reference's messages; every call
is asynchronous on the current CUDA stream and never synchronises the host.
There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native
from ._native import check
from .format import check_d

# bound on the attention workspace (split partials, then the continuation pre-pass tiles:
# ceil(seq / 64) x Hk x 64 KiB per request); the allocation is what a call needs, up to this
DEFAULT_WORKSPACE_BYTES = 512 * 1024 * 1024

_DTYPES = {torch.float32: _native.DTYPE_F32, torch.bfloat16: _native.DTYPE_BF16, torch.float16: _native.DTYPE_F16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("OSCAR B200 kernels require CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _byte_view(cache: torch.Tensor) -> torch.Tensor:
    c8 = cache.view(torch.uint8)
    if c8.ndim != 4 or not c8.is_contiguous():
        raise ValueError("OSCAR requires contiguous [blocks, tokens, heads, bytes] caches")
    return c8


def _clip_ok(r: float) -> float:
    r = float(r)
    if not 0.0 <= r <= 1.0:
        raise ValueError("OSCAR clip ratios must be finite and in [0, 1]")
    return r


# ---------------------------------------------------------------------------
def oscar_store(k_rot: torch.Tensor, v_rot: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                slot_mapping: torch.Tensor, k_clip_ratio: float = 0.0, v_clip_ratio: float = 0.0) -> None:
    """Clip, INT2-quantize, pack and scatter rotated K/V [N, Hk, D] into the
    paged caches in place; slot < 0 is skipped.  Bit-exact with
    oscar_store_ref for identical rotated fp32 input (clip ratios 0)."""
    dev = _require_cuda(k_rot, v_rot, k_cache, v_cache, slot_mapping)
    if k_rot.shape != v_rot.shape or k_rot.ndim != 3:
        raise ValueError("k_rot/v_rot must be [N, H, D] with equal shapes")
    n, h, d = k_rot.shape
    check_d(d)
    k8, v8 = _byte_view(k_cache), _byte_view(v_cache)
    if k8.shape[:3] != v8.shape[:3] or k8.shape[2] != h:
        raise ValueError("cache geometry does not match [N, H, D] input")
    k_rot = k_rot.to(torch.float32).contiguous()
    v_rot = v_rot.to(torch.float32).contiguous()
    slots = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    if slots.numel() < n:
        raise ValueError("slot_mapping shorter than the token count")
    check(_native.lib().oscar_store_int2(
        k_rot.data_ptr(), v_rot.data_ptr(), n, h, d, _clip_ok(k_clip_ratio), _clip_ok(v_clip_ratio),
        k8.data_ptr(), v8.data_ptr(), k8.shape[0], k8.shape[1], *k8.stride()[:3], *v8.stride()[:3],
        slots.data_ptr(), _stream(dev)))


def oscar_store_ref(k_rot, v_rot, k_cache, v_cache, slot_mapping) -> None:
    """Name-compatible alias of kernels/store_kernel.py:54 (runs on the GPU)."""
    oscar_store(k_rot, v_rot, k_cache, v_cache, slot_mapping)


# ---------------------------------------------------------------------------
def staging_invalidate(slot_mapping: torch.Tensor, owner: torch.Tensor, block_size: int) -> None:
    """owner[seat(slot)] = -1 for every slot >= 0 (backend.py:172-176)."""
    dev = _require_cuda(slot_mapping, owner)
    if owner.dtype != torch.int64 or owner.ndim != 2 or not owner.is_contiguous():
        raise ValueError("owner must be a contiguous int64 [rows, block_size] tensor")
    slots = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    check(_native.lib().oscar_staging_invalidate(slots.data_ptr(), slots.numel(), owner.data_ptr(),
                                                 owner.shape[0], int(block_size), _stream(dev)))


def staging_write(k_rot: torch.Tensor, v_rot: torch.Tensor, slot_mapping: torch.Tensor, qsl: torch.Tensor,
                  seqs: torch.Tensor, sink_eff: int, recent_tokens: int, stage_k: torch.Tensor,
                  stage_v: torch.Tensor, owner: torch.Tensor, seat_winner: torch.Tensor, epoch: int) -> None:
    """Sink/recent staging write of rotated, unclipped fp32 K/V [N, Hk, D]
    (backend.py:513-555).  qsl/seqs are device int32 tensors [B+1], [B]."""
    dev = _require_cuda(k_rot, v_rot, slot_mapping, qsl, seqs, stage_k, stage_v, owner, seat_winner)
    n, h, d = k_rot.shape
    rows, bs = owner.shape
    if stage_k.shape != (rows, bs, h, d) or stage_v.shape != stage_k.shape:
        raise ValueError("Invalid streaming staging geometry")
    if seat_winner.numel() != rows * bs or seat_winner.dtype != torch.int64:
        raise ValueError("seat_winner must be int64 [rows * block_size]")
    for t in (stage_k, stage_v, owner, seat_winner):
        if not t.is_contiguous():
            raise ValueError("Streaming staging tensors must be contiguous")
    k_rot = k_rot.to(torch.float32).contiguous()
    v_rot = v_rot.to(torch.float32).contiguous()
    slots = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    qsl = qsl.to(device=dev, dtype=torch.int32).contiguous()
    seqs = seqs.to(device=dev, dtype=torch.int32).contiguous()
    check(_native.lib().oscar_staging_write(
        k_rot.data_ptr(), v_rot.data_ptr(), n, h, d, slots.data_ptr(), qsl.data_ptr(), seqs.data_ptr(),
        seqs.numel(), int(sink_eff), int(recent_tokens), stage_k.data_ptr(), stage_v.data_ptr(), owner.data_ptr(),
        rows, bs, seat_winner.data_ptr(), int(epoch) & 0xFFFFFFFF, _stream(dev)))


WRITE_STEP_MAX_TOKENS = 256
WRITE_STEP_MAX_REQUESTS = 256


def write_step(k_rot: torch.Tensor, v_rot: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               slot_mapping: torch.Tensor, k_clip_ratio: float, v_clip_ratio: float, qsl: torch.Tensor,
               seqs: torch.Tensor, sink_eff: int, recent_tokens: int, stage_k: torch.Tensor, stage_v: torch.Tensor,
               owner: torch.Tensor) -> None:
    """oscar_store + staging_write of the same tokens in one launch (at most
    WRITE_STEP_MAX_TOKENS tokens and WRITE_STEP_MAX_REQUESTS requests): the
    write side of a decode step with the staging window on.  Needs no seat
    scratch and no epoch, so it can be captured in a CUDA graph."""
    dev = _require_cuda(k_rot, v_rot, k_cache, v_cache, slot_mapping, qsl, seqs, stage_k, stage_v, owner)
    if k_rot.shape != v_rot.shape or k_rot.ndim != 3:
        raise ValueError("k_rot/v_rot must be [N, H, D] with equal shapes")
    n, h, d = k_rot.shape
    check_d(d)
    k8, v8 = _byte_view(k_cache), _byte_view(v_cache)
    if k8.shape[:3] != v8.shape[:3] or k8.shape[2] != h:
        raise ValueError("cache geometry does not match [N, H, D] input")
    rows, bs = owner.shape
    if stage_k.shape != (rows, bs, h, d) or stage_v.shape != stage_k.shape or bs != k8.shape[1]:
        raise ValueError("Invalid streaming staging geometry")
    for t in (stage_k, stage_v, owner):
        if not t.is_contiguous():
            raise ValueError("Streaming staging tensors must be contiguous")
    k_rot = k_rot.to(torch.float32).contiguous()
    v_rot = v_rot.to(torch.float32).contiguous()
    slots = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    qsl = qsl.to(device=dev, dtype=torch.int32).contiguous()
    seqs = seqs.to(device=dev, dtype=torch.int32).contiguous()
    if slots.numel() < n:
        raise ValueError("slot_mapping shorter than the token count")
    check(_native.lib().oscar_write_step(
        k_rot.data_ptr(), v_rot.data_ptr(), n, h, d, _clip_ok(k_clip_ratio), _clip_ok(v_clip_ratio),
        k8.data_ptr(), v8.data_ptr(), k8.shape[0], k8.shape[1], *k8.stride()[:3], *v8.stride()[:3],
        slots.data_ptr(), qsl.data_ptr(), seqs.data_ptr(), seqs.numel(), int(sink_eff), int(recent_tokens),
        stage_k.data_ptr(), stage_v.data_ptr(), owner.data_ptr(), rows, _stream(dev)))


def staging_write_noalloc(k_rot: torch.Tensor, v_rot: torch.Tensor, slot_mapping: torch.Tensor, qsl: torch.Tensor,
                          seqs: torch.Tensor, sink_eff: int, recent_tokens: int, stage_k: torch.Tensor,
                          stage_v: torch.Tensor, owner: torch.Tensor) -> None:
    """staging_write with the library's built-in seat scratch, cleared on every
    call instead of tagged by a host epoch: no caller scratch and no host state,
    so it can be captured in a CUDA graph and replayed with new slots."""
    dev = _require_cuda(k_rot, v_rot, slot_mapping, qsl, seqs, stage_k, stage_v, owner)
    n, h, d = k_rot.shape
    rows, bs = owner.shape
    if stage_k.shape != (rows, bs, h, d) or stage_v.shape != stage_k.shape:
        raise ValueError("Invalid streaming staging geometry")
    for t in (stage_k, stage_v, owner):
        if not t.is_contiguous():
            raise ValueError("Streaming staging tensors must be contiguous")
    for t in (k_rot, v_rot, slot_mapping, qsl, seqs):
        if not t.is_contiguous():
            raise ValueError("staging_write_noalloc: inputs must be contiguous")
    if k_rot.dtype != torch.float32 or v_rot.dtype != torch.float32 or slot_mapping.dtype != torch.int64 \
            or qsl.dtype != torch.int32 or seqs.dtype != torch.int32:
        raise ValueError("staging_write_noalloc: fp32 rows, int64 slots and int32 qsl / seqs expected")
    check(_native.lib().oscar_staging_write_noalloc(
        k_rot.data_ptr(), v_rot.data_ptr(), n, h, d, slot_mapping.data_ptr(), qsl.data_ptr(), seqs.data_ptr(),
        seqs.numel(), int(sink_eff), int(recent_tokens), stage_k.data_ptr(), stage_v.data_ptr(), owner.data_ptr(),
        rows, bs, _stream(dev)))


# ---------------------------------------------------------------------------
def _validate_tensors(q, k, v, kc, vc, bt, qsl, seqs, stage):
    """streaming_attention._validate_tensors (streaming_attention.py:32-65)."""
    if q.ndim != 3 or kc.ndim != 4 or kc.shape != vc.shape or kc.shape[3] != q.shape[2]:
        raise ValueError("Streaming attention requires [tokens,heads,D] queries and native 4-D caches")
    if not kc.is_contiguous() or not vc.is_contiguous():
        raise ValueError("Streaming caches must be contiguous")
    if (k is None) != (v is None):
        raise ValueError("Both new K and V must be supplied together")
    if k is not None and (k.shape != v.shape or k.shape != (q.shape[0], kc.shape[2], q.shape[2])
                          or k.dtype != q.dtype or v.dtype != q.dtype):
        raise ValueError("Current K/V must match query tokens, dtype and KV geometry")
    if bt.ndim != 2 or bt.shape[0] < len(seqs):
        raise ValueError("Missing request block-table rows")
    for a, b, seq in zip(qsl, qsl[1:], seqs):
        prefix = seq - (b - a) if k is not None else seq
        if b > a and -(-prefix // kc.shape[1]) > bt.shape[1]:
            raise ValueError("Block table cannot cover the history")
    if stage is not None:
        sk, sv, owner = stage
        shape = (owner.shape[0], kc.shape[1], kc.shape[2], q.shape[2])
        if owner.shape != shape[:2] or sk.shape != shape or sv.shape != shape or shape[0] < 1:
            raise ValueError("Invalid streaming staging geometry")
        if not all(t.is_contiguous() for t in stage):
            raise ValueError("Streaming staging tensors must be contiguous")


def slab_attention(q, k_new, v_new, kc, vc, table, qsl, seqs, scale, stage=None, *,
                   workspace_bytes: int = DEFAULT_WORKSPACE_BYTES, chunk_tokens: int | None = None):
    """Exact attention of rotated queries over paged INT2 history (+ staged
    fp32 overrides) and the causal current chunk.  Returns (out [n, Hq, D]
    fp32, lse [n, Hq] fp32 natural log).  ``qsl``/``seqs`` are host lists.

    ``workspace_bytes`` bounds the workspace: split-KV partials, then (head dim
    256, q-blocks of 128 rows) the keys' tiles written once by a pre-pass.  Any
    value is valid; a smaller one only lowers parallelism or makes each
    attention CTA dequantise its own tiles.  ``chunk_tokens`` is accepted for
    signature compatibility: the fused kernel never materialises a slab."""
    del chunk_tokens
    qsl = [int(x) for x in qsl]
    seqs = [int(x) for x in seqs]
    if (q.ndim != 3 or kc.ndim != 4 or q.shape[1] < 1 or kc.shape[2] < 1 or len(qsl) != len(seqs) + 1
            or not qsl or qsl[0] != 0 or qsl[-1] != q.shape[0] or q.shape[1] % kc.shape[2]):
        raise ValueError("Invalid slab query layout")
    if any(a > b or seq < 0 or (k_new is not None and seq < b - a) for a, b, seq in zip(qsl, qsl[1:], seqs)):
        raise ValueError("Sequence length must cover its query chunk")
    _validate_tensors(q, k_new, v_new, kc, vc, table, qsl, seqs, stage)
    dev = _require_cuda(q, k_new, v_new, kc, vc, table, *(stage or ()))
    out_dtype = q.dtype
    if q.dtype == torch.float32:
        # fp32 queries: fp16 tensor-core operands (history is fp16-exact on this path)
        q = q.half()
        k_new = None if k_new is None else k_new.half()
        v_new = None if v_new is None else v_new.half()
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported query dtype {out_dtype}")
    n, hq, d = q.shape
    hk = kc.shape[2]
    q = q.contiguous()
    k_new = None if k_new is None else k_new.contiguous()
    v_new = None if v_new is None else v_new.contiguous()
    table = table.to(device=dev, dtype=torch.int32).contiguous()
    k8, v8 = _byte_view(kc), _byte_view(vc)
    sk = sv = owner = None
    rows = 0
    if stage is not None:
        sk, sv, owner = stage
        if sk.dtype != torch.float32 or sv.dtype != torch.float32 or owner.dtype != torch.int64:
            raise ValueError("staging arena must be fp32 K/V and int64 owner tags")
        rows = owner.shape[0]
    out = torch.empty(n, hq, d, dtype=torch.float32, device=dev)
    lse = torch.empty(n, hq, dtype=torch.float32, device=dev)
    if n == 0:
        return out, lse
    lib = _native.lib()
    qsl_a = np.ascontiguousarray(qsl, dtype=np.int32)
    seqs_a = np.ascontiguousarray(seqs, dtype=np.int32)
    qsl_p, seqs_p = qsl_a.ctypes.data, seqs_a.ctypes.data
    need = lib.oscar_slab_attention_workspace(qsl_p, seqs_p, len(seqs), int(k_new is not None), hq, hk, d)
    ws_bytes = max(0, min(int(need), int(workspace_bytes)))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    dtype = _DTYPES[q.dtype]
    check(lib.oscar_slab_attention(
        q.data_ptr(), _ptr(k_new), _ptr(v_new), dtype, n, hq, hk, d,
        k8.data_ptr(), v8.data_ptr(), k8.shape[0], k8.shape[1], *k8.stride()[:3], *v8.stride()[:3],
        table.data_ptr(), table.shape[0], table.stride(0), qsl_p, seqs_p, len(seqs), float(scale),
        _ptr(sk), _ptr(sv), _ptr(owner), rows, out.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws_bytes,
        _stream(dev)))
    return out, lse


def slab_attention_shard(q, kc, vc, table, qsl, history_lens, scale, stage=None, *,
                         workspace_bytes: int = DEFAULT_WORKSPACE_BYTES):
    """Partial attention of rotated queries over one shard of the paged
    history: request r's keys [0, history_lens[r]) through table row r, all of
    them visible to all of its queries, no current chunk.  Returns (out, lse)
    like ``slab_attention``; shards of one history are combined with
    ``merge_slab`` (the split-KV merge of slab_attention.py:458-475 across
    GPUs).  Decode-sized steps at head dim 256 only (the tensor-core decode
    kernel or the CUDA-core decode kernel); other layouts raise ValueError."""
    qsl = [int(x) for x in qsl]
    hist = [int(x) for x in history_lens]
    if (q.ndim != 3 or kc.ndim != 4 or q.shape[1] < 1 or kc.shape[2] < 1 or len(qsl) != len(hist) + 1
            or not qsl or qsl[0] != 0 or qsl[-1] != q.shape[0] or q.shape[1] % kc.shape[2]):
        raise ValueError("Invalid slab query layout")
    if any(a > b or h < 0 for a, b, h in zip(qsl, qsl[1:], hist)):
        raise ValueError("Sequence length must cover its query chunk")
    _validate_tensors(q, None, None, kc, vc, table, qsl, hist, stage)
    dev = _require_cuda(q, kc, vc, table, *(stage or ()))
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported query dtype {q.dtype}")
    n, hq, d = q.shape
    hk = kc.shape[2]
    q = q.contiguous()
    table = table.to(device=dev, dtype=torch.int32).contiguous()
    k8, v8 = _byte_view(kc), _byte_view(vc)
    sk = sv = owner = None
    rows = 0
    if stage is not None:
        sk, sv, owner = stage
        if sk.dtype != torch.float32 or sv.dtype != torch.float32 or owner.dtype != torch.int64:
            raise ValueError("staging arena must be fp32 K/V and int64 owner tags")
        rows = owner.shape[0]
    out = torch.empty(n, hq, d, dtype=torch.float32, device=dev)
    lse = torch.empty(n, hq, dtype=torch.float32, device=dev)
    if n == 0:
        return out, lse
    lib = _native.lib()
    qsl_a = np.ascontiguousarray(qsl, dtype=np.int32)
    hist_a = np.ascontiguousarray(hist, dtype=np.int32)
    # the shard's plan is the one of a step with the history as prefix and the
    # queries as its chunk
    seqs_a = np.ascontiguousarray([h + b - a for h, a, b in zip(hist, qsl, qsl[1:])], dtype=np.int32)
    need = lib.oscar_slab_attention_workspace(qsl_a.ctypes.data, seqs_a.ctypes.data, len(hist), 1, hq, hk, d)
    ws_bytes = max(0, min(int(need), int(workspace_bytes)))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    check(lib.oscar_slab_attention_shard(
        q.data_ptr(), _DTYPES[q.dtype], n, hq, hk, d,
        k8.data_ptr(), v8.data_ptr(), k8.shape[0], k8.shape[1], *k8.stride()[:3], *v8.stride()[:3],
        table.data_ptr(), table.shape[0], table.stride(0), qsl_a.ctypes.data, hist_a.ctypes.data, len(hist),
        float(scale), _ptr(sk), _ptr(sv), _ptr(owner), rows, out.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws_bytes,
        _stream(dev)))
    return out, lse


def decode_step_scratch_bytes(n: int, hq: int, hk: int, d: int, workspace_bytes: int) -> int:
    """Scratch of decode_layer_step for up to n tokens: the rotated rows and
    the attention output, then `workspace_bytes` of attention workspace."""
    fixed = int(_native.lib().oscar_decode_layer_step_scratch(n, hq, hk, d, _native.DTYPE_BF16))
    if fixed < 0:
        raise ValueError("decode_layer_step: invalid geometry")
    return fixed + max(0, int(workspace_bytes))


def decode_layer_step(q, k, v, token_strides, n, hq, hk, d, rot_k, rot_v, rot_vt, k_clip_ratio, v_clip_ratio,
                      k_cache, v_cache, slot_mapping, qsl_dev, seqs_dev, table, qsl, seqs, sink_eff, recent_tokens,
                      scale, stage_k, stage_v, owner, out, scratch) -> None:
    """One decode-sized layer step in one native call (oscar_decode_layer_step):
    rotations, clip + INT2 store + staging write, rotated attention, output
    rotation into ``out``.  The backend's fast path: the caller has checked
    the layouts (heads contiguous per token, ``token_strides`` = the token
    row strides of q, k, v, out in elements; int64 slots, int32 device qsl /
    seqs and block table, host lists ``qsl`` / ``seqs``); the C side checks
    sizes and alignment and raises through ``check``."""
    lib = _native.lib()
    k8, v8 = k_cache.view(torch.uint8), v_cache.view(torch.uint8)
    qsl_a = np.asarray(qsl, dtype=np.int32)
    seqs_a = np.asarray(seqs, dtype=np.int32)
    kst, vst = k8.stride(), v8.stride()
    check(lib.oscar_decode_layer_step(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _DTYPES[q.dtype], token_strides[0], token_strides[1],
        token_strides[2], n, hq, hk, d, rot_k.data_ptr(), rot_v.data_ptr(), rot_vt.data_ptr(), _clip_ok(k_clip_ratio),
        _clip_ok(v_clip_ratio), k8.data_ptr(), v8.data_ptr(), k8.shape[0], k8.shape[1], kst[0], kst[1], kst[2],
        vst[0], vst[1], vst[2], slot_mapping.data_ptr(), qsl_dev.data_ptr(), seqs_dev.data_ptr(), table.data_ptr(),
        table.shape[0], table.stride(0), qsl_a.ctypes.data, seqs_a.ctypes.data, len(seqs), int(sink_eff),
        int(recent_tokens), float(scale), stage_k.data_ptr(), stage_v.data_ptr(), owner.data_ptr(), owner.shape[0],
        out.data_ptr(), token_strides[3], scratch.data_ptr(), scratch.numel(), _stream(q.device)))


def merge_slab(output, lse, part, part_lse, start, ids) -> None:
    """In-place LSE merge of part into output[start:start+n] (or output[ids])."""
    dev = _require_cuda(output, lse, part, part_lse, ids)
    n, hq, d = part.shape
    if output.dtype != torch.float32 or lse.dtype != torch.float32 or not output.is_contiguous() or not lse.is_contiguous():
        raise ValueError("output/lse must be contiguous fp32")
    if part.dtype not in _DTYPES:
        raise ValueError(f"unsupported partial dtype {part.dtype}")
    part = part.contiguous()
    part_lse = part_lse.to(torch.float32).contiguous()
    ids_t = None if ids is None else ids.to(device=dev, dtype=torch.int32).contiguous()
    if output.shape[1:] != part.shape[1:] or lse.shape != output.shape[:2] or part_lse.shape != part.shape[:2]:
        raise ValueError("merge: output/lse/part geometry mismatch")
    check(_native.lib().oscar_merge_slab(output.data_ptr(), lse.data_ptr(), output.shape[0], part.data_ptr(),
                                         _DTYPES[part.dtype],
                                         part_lse.data_ptr(), n, hq, d, int(start), _ptr(ids_t), _stream(dev)))


_PATHS = {"auto": 0, "tile": 1, "decode": 2, "tensor": 3}


def rotate_rows(x: torch.Tensor, rot: torch.Tensor, *, transpose: bool = False, out: torch.Tensor | None = None,
                out_f32: torch.Tensor | None = None, out_dtype: torch.dtype | None = None):
    """y = x @ R (or x @ R^T) over the last dim of x in fp32 (the per-layer
    rotations of backend.py:238-246).  x: [..., D] (fp32/bf16/fp16, rows with a
    uniform stride); writes `out` (given, or new of `out_dtype`) and/or
    `out_f32`, both [..., D] views with uniform row strides.  Returns (out, out_f32)."""
    d = x.shape[-1]
    if rot.shape != (d, d) or rot.dtype != torch.float32:
        raise ValueError(f"rotation must be fp32 [{d}, {d}], got {tuple(rot.shape)} {rot.dtype}")
    rot = rot.contiguous()
    x2 = x.reshape(-1, d)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) % 8) or x2.data_ptr() % 16:
        x2 = x2.clone(memory_format=torch.contiguous_format)
    rows = x2.shape[0]
    if out is None and out_f32 is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    o2 = None if out is None else out.view(-1, d)
    f2 = None if out_f32 is None else out_f32.view(-1, d)
    for t in (x2, o2, f2):
        if t is not None and rows > 1 and t.stride(-1) != 1:
            raise ValueError("rotate_rows: rows must be contiguous in the last dim")
    dev = _require_cuda(x, rot)
    check(_native.lib().oscar_rotate_rows(
        _ptr(x2), _DTYPES[x2.dtype], rows, x2.stride(0), d, _ptr(rot), 1 if transpose else 0,
        _ptr(o2), _DTYPES[o2.dtype] if o2 is not None else 0, o2.stride(0) if o2 is not None else 0,
        _ptr(f2), f2.stride(0) if f2 is not None else 0, _stream(dev)))
    return out, out_f32


def rotate_rows_many(jobs) -> None:
    """Several rotate_rows calls in one launch.  ``jobs``: up to four
    ``(x, rot, out, out_f32)`` tuples (x @ R, no transpose) whose x share one
    dtype and D and whose ``out`` tensors share one dtype; each output is
    preallocated ([..., D] rows with uniform strides) or None."""
    if not jobs:
        return
    if len(jobs) > 4:
        raise ValueError("rotate_rows_many: at most 4 jobs per launch")
    dev = _require_cuda(*[t for job in jobs for t in job])
    d = jobs[0][0].shape[-1]
    x_dt = jobs[0][0].dtype
    out_dt = next((o.dtype for _, _, o, _ in jobs if o is not None), torch.float32)
    segs = (_native.RotateSeg * len(jobs))()
    keep = []
    for i, (x, rot, out, out_f32) in enumerate(jobs):
        if x.shape[-1] != d or x.dtype != x_dt or (out is not None and out.dtype != out_dt):
            raise ValueError("rotate_rows_many: jobs must share x dtype, D and out dtype")
        if rot.shape != (d, d) or rot.dtype != torch.float32:
            raise ValueError(f"rotation must be fp32 [{d}, {d}], got {tuple(rot.shape)} {rot.dtype}")
        rot = rot.contiguous()
        keep.append(rot)
        x2 = x.reshape(-1, d)
        if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) % 8) or x2.data_ptr() % 16:
            x2 = x2.clone(memory_format=torch.contiguous_format)
        o2 = None if out is None else out.view(-1, d)
        f2 = None if out_f32 is None else out_f32.view(-1, d)
        for t in (o2, f2):
            if t is not None and t.shape[0] > 1 and t.stride(-1) != 1:
                raise ValueError("rotate_rows_many: rows must be contiguous in the last dim")
        keep.append(x2)
        segs[i] = _native.RotateSeg(_ptr(x2), x2.shape[0], x2.stride(0), _ptr(rot), 0,
                                    _ptr(o2), o2.stride(0) if o2 is not None else 0,
                                    _ptr(f2), f2.stride(0) if f2 is not None else 0)
    check(_native.lib().oscar_rotate_rows_batch(segs, len(jobs), _DTYPES[x_dt], d, _DTYPES[out_dt], _stream(dev)))


def set_attention_path(path: str) -> None:
    """Kernel family for slab_attention: "auto" (tensor-core decode kernel,
    else the mma.sync decode kernel, else the tile kernel, whichever is
    eligible first), "tensor" or "decode" (that decode kernel where eligible,
    else the tile kernel) or "tile" (tile kernel only).  All compute the same
    function."""
    check(_native.lib().oscar_set_attention_path(_PATHS[path]))


_ROT_PATHS = {"auto": 0, "fma": 1, "tensor": 2, "fma_big": 3}


def set_rotation_path(path: str) -> None:
    """Rotation kernel for rotate_rows / rotate_rows_many and the layer step:
    "auto" (per tensor, by its own size: tcgen05 kind::tf32 with split
    precision for fp32 tensors of at least 2560 rows -- the output rotation --,
    register-tiled fp32 FMAs for 16-bit ones of at least 6144 rows -- the
    k / v / q rotations of long chunks; 64-row tiles below 16384 rows, 128-row
    tiles from there --, 16-row FMA tiles for the rest), "fma" (16-row FMA
    tiles), "tensor" or "fma_big" (register-tiled FMAs, D 128 or 256).  All
    compute x @ R to within a few fp32 ulps."""
    check(_native.lib().oscar_set_rotation_path(_ROT_PATHS[path]))


def device_error(device=None) -> int:
    """Synchronise and return/clear the kernels' bounds-violation flag (debug)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return int(_native.lib().oscar_device_error(_stream(dev)))
