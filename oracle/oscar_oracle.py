"""CPU oracle for the OSCAR INT2 rotated KV-cache hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and there only as the checker or the timed CPU baseline.  The product
path (``oscar_b200``) never imports it and has no CPU fallback.

This is a numpy restatement of the reference's own torch CPU path
(oscar-ascend 0.2.0, ``OSCAR_ASCEND_USE_TRITON=0``).  Every function cites the
reference function it restates.  Parity is PINNED: ``tests/test_oracle_golden.py``
checks each function against golden vectors produced by running the reference
itself (``tests/golden/make_golden.py``).

Numeric conventions (same as the reference):
  * all arithmetic is float32, one IEEE rounding per elementwise op;
  * bf16 / fp16 tensors are carried as float32 arrays holding exactly
    representable values; ``round_to(dtype, x)`` performs the cast;
  * caches are uint8 arrays ``[num_blocks, block_size, num_kv_heads, slot_bytes]``
    (the byte view of the reference's int8 "packed x2" or bf16 legacy caches).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# oscar_ascend/format.py:19-38
LEVELS = 4
VALUES_PER_BYTE = 4
META_BYTES = 8
PAD_BYTES = 24
K_IDX_OFF = 32
K_SLOT_BYTES = 96
SCALE_FLOOR = F32(2.0**-14)


def check_d(d: int) -> None:
    """format.py:41-45."""
    if d % VALUES_PER_BYTE != 0:
        raise ValueError(f"D={d} must be a multiple of {VALUES_PER_BYTE}")
    if d // VALUES_PER_BYTE > K_SLOT_BYTES - META_BYTES - PAD_BYTES:
        raise ValueError(f"D={d} exceeds the slot capacity")


# ---------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------
def round_bf16(x) -> np.ndarray:
    """float32 -> bfloat16 -> float32, round-to-nearest-even (torch's cast)."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = r.view(F32).copy()
    nan = np.isnan(x)
    out[nan] = x[nan]
    return out


def round_f16(x) -> np.ndarray:
    """float32 -> float16 -> float32 (round-to-nearest-even)."""
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def round_to(dtype: str, x) -> np.ndarray:
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return round_f16(x)
    if dtype == "f32":
        return np.asarray(x, dtype=F32)
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# INT2 format: format.py:51-119
# ---------------------------------------------------------------------------
def vector_scales(x):
    """format.vector_scales (format.py:51-64): fp16-rounded scale/zero per vector."""
    x = np.asarray(x, dtype=F32)
    vmin = x.min(axis=-1, keepdims=True)
    vmax = x.max(axis=-1, keepdims=True)
    scale = (vmax - vmin) / F32(LEVELS - 1)
    scale = np.where(scale > SCALE_FLOOR, scale, SCALE_FLOOR).astype(F32)
    return round_f16(scale), round_f16(vmin)


def quantize(x):
    """format.quantize (format.py:67-88) -> (packed uint8 [..,D/4], scale, zero)."""
    x = np.asarray(x, dtype=F32)
    scale, zero = vector_scales(x)
    q = np.floor((x - zero) / scale + F32(0.5))
    q = np.clip(q, 0, LEVELS - 1).astype(np.int32)
    q4 = q.reshape(*q.shape[:-1], q.shape[-1] // VALUES_PER_BYTE, VALUES_PER_BYTE)
    packed = q4[..., 0] | (q4[..., 1] << 2) | (q4[..., 2] << 4) | (q4[..., 3] << 6)
    return packed.astype(np.uint8), scale, zero


def unpack(packed, d: int) -> np.ndarray:
    """format._unpack (format.py:99-110): low index in the low two bits."""
    p = np.asarray(packed).astype(np.int32)
    q = np.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], axis=-1)
    return q.reshape(*p.shape[:-1], d)


def dequant(packed, scale, zero, d: int) -> np.ndarray:
    """format.dequant (format.py:91-96): q * scale + zero, two fp32 roundings."""
    q = unpack(packed, d).astype(F32)
    return (q * scale).astype(F32) + zero


def f16_bytes(x) -> np.ndarray:
    """format.f16_le (format.py:113-119): [...,1] -> [...,2] little-endian bytes."""
    h = np.ascontiguousarray(np.asarray(x, dtype=F32).astype(np.float16))
    return h.view(np.uint8).reshape(*h.shape[:-1], 2)


def f16_from_bytes(b) -> np.ndarray:
    """format.f16_be_from_le (format.py:122-125): [...,2] LE bytes -> [...,1] fp32."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    return b.view(np.float16).astype(F32)


def make_slot_bytes(k_rot, v_rot) -> np.ndarray:
    """format.make_slot_bytes (format.py:131-154): logical 160-byte slot."""
    n, h, d = k_rot.shape
    check_d(d)
    db = d // VALUES_PER_BYTE
    kp, ks, kz = quantize(k_rot)
    vp, vs, vz = quantize(v_rot)
    slot = np.zeros((n, h, 160), np.uint8)
    slot[..., 0:2] = f16_bytes(ks)
    slot[..., 2:4] = f16_bytes(kz)
    slot[..., 4:6] = f16_bytes(vs)
    slot[..., 6:8] = f16_bytes(vz)
    slot[..., 32 : 32 + db] = kp
    slot[..., 96 : 96 + db] = vp
    return slot


# ---------------------------------------------------------------------------
# write path
# ---------------------------------------------------------------------------
def rotate_clip(x, rot, clip_ratio: float) -> np.ndarray:
    """backend._rotate_clip (backend.py:130-148): x @ R, then per-vector clamp at
    the idx-th smallest |x|, idx = min(int(ratio * D), D - 1)."""
    y = np.asarray(x, dtype=F32) @ np.asarray(rot, dtype=F32)
    y = y.astype(F32)
    if clip_ratio > 0.0:
        d = y.shape[-1]
        idx = min(int(clip_ratio * d), d - 1)
        thr = np.sort(np.abs(y), axis=-1)[..., idx : idx + 1]
        y = np.minimum(np.maximum(y, -thr), thr)
    return y


def clip_only(y, clip_ratio: float) -> np.ndarray:
    """The clamp half of backend._rotate_clip (backend.py:140-146) on a rotated input."""
    y = np.asarray(y, dtype=F32)
    if clip_ratio > 0.0:
        d = y.shape[-1]
        idx = min(int(clip_ratio * d), d - 1)
        thr = np.sort(np.abs(y), axis=-1)[..., idx : idx + 1]
        y = np.minimum(np.maximum(y, -thr), thr)
    return y


def store(k_rot, v_rot, k8, v8, slot_mapping) -> None:
    """kernels/store_kernel.oscar_store_ref (store_kernel.py:54-102), in place.

    k8/v8: uint8 [num_blocks, bs, hk, slot_bytes].  Negative slots are skipped.
    K slot: [0:2] K scale, [2:4] K zero, [4:6] V scale, [6:8] V zero,
    [32:32+D/4] K codes.  V slot: [0:D/4] V codes (store_kernel.py:4-9)."""
    k_rot = np.asarray(k_rot, dtype=F32)
    v_rot = np.asarray(v_rot, dtype=F32)
    n, h, d = k_rot.shape
    check_d(d)
    db = d // VALUES_PER_BYTE
    bs = k8.shape[1]
    slots = np.asarray(slot_mapping, dtype=np.int64).reshape(-1)
    valid = slots >= 0
    slots, k_rot, v_rot = slots[valid], k_rot[valid], v_rot[valid]
    if slots.size == 0:
        return
    blk, off = slots // bs, slots % bs
    kp, ks, kz = quantize(k_rot)
    vp, vs, vz = quantize(v_rot)
    meta = np.concatenate([f16_bytes(ks), f16_bytes(kz), f16_bytes(vs), f16_bytes(vz)], -1)
    if np.unique(slots).size == slots.size:
        k8[blk, off, :, 0:META_BYTES] = meta
        k8[blk, off, :, K_IDX_OFF : K_IDX_OFF + db] = kp
        v8[blk, off, :, 0:db] = vp
        return
    # index_put_ with duplicate slots: the last occurrence wins on the CPU path.
    for i in range(slots.size):
        k8[blk[i], off[i], :, 0:META_BYTES] = meta[i]
        k8[blk[i], off[i], :, K_IDX_OFF : K_IDX_OFF + db] = kp[i]
        v8[blk[i], off[i], :, 0:db] = vp[i]


def dequant_split(k8, v8, blocks, pos, hk: int, d: int):
    """kernels/store_kernel.dequant_split_ref (store_kernel.py:105-133) -> fp32 [T,H,D]."""
    db = d // VALUES_PER_BYTE
    ks = k8[blocks, pos][..., :, 0:META_BYTES]  # [T, H, 8]
    k_scale = f16_from_bytes(ks[..., 0:2])
    k_zero = f16_from_bytes(ks[..., 2:4])
    v_scale = f16_from_bytes(ks[..., 4:6])
    v_zero = f16_from_bytes(ks[..., 6:8])
    kp = k8[blocks, pos][..., K_IDX_OFF : K_IDX_OFF + db]
    vp = v8[blocks, pos][..., 0:db]
    return dequant(kp, k_scale, k_zero, d), dequant(vp, v_scale, v_zero, d)


# ---------------------------------------------------------------------------
# staging window (backend.py:492-555, :172-176)
# ---------------------------------------------------------------------------
class Staging:
    """backend._ensure_staging (backend.py:492-511)."""

    def __init__(self, bs, hk, d, sink_tokens, recent_tokens, staging_tokens):
        self.bs = bs
        self.recent = recent_tokens
        self.sink_eff = (sink_tokens // bs) * bs
        sink_pages = self.sink_eff // bs
        tail_pages = (recent_tokens + bs - 1) // bs + 1
        self.rows = max((staging_tokens + bs - 1) // bs, sink_pages + tail_pages + 2)
        self.stage_k = np.zeros((self.rows, bs, hk, d), F32)
        self.stage_v = np.zeros_like(self.stage_k)
        self.owner = np.full((self.rows, bs), -1, np.int64)

    def invalidate(self, slot_mapping):
        """do_kv_cache_update owner invalidation (backend.py:172-176)."""
        s = np.asarray(slot_mapping, np.int64)
        s = s[s >= 0]
        self.owner[(s // self.bs) % self.rows, s % self.bs] = -1

    def write(self, key, value, rk, rv, slot_mapping, qsl, seqs, n):
        """backend._staging_write (backend.py:513-555)."""
        if n == 0:
            return
        slot = np.asarray(slot_mapping, np.int64)[:n]
        lengths = [max(0, min(e, n) - min(s, n)) for s, e in zip(qsl, qsl[1:])]
        req = np.repeat(np.arange(len(lengths)), lengths)
        seq = np.asarray(seqs[: len(lengths)], np.int64)
        ends = np.asarray(qsl[1:], np.int64)
        pos = seq[req] - ends[req] + np.arange(n)
        keep = (pos >= seq[req] - self.recent) | (pos < self.sink_eff)
        bs = self.bs
        valid = np.nonzero(slot >= 0)[0]
        seats = ((slot[valid] // bs) % self.rows) * bs + slot[valid] % bs
        order = np.argsort(seats, kind="stable")
        sorted_seats = seats[order]
        last = np.concatenate([sorted_seats[1:] != sorted_seats[:-1], np.ones(min(1, sorted_seats.size), bool)])
        selected = valid[order[last]]
        seats = sorted_seats[last]
        rows, offs = seats // bs, seats % bs
        self.owner[rows, offs] = np.where(keep[selected], slot[selected] // bs, -1)
        ret = keep[selected]
        selected, rows, offs = selected[ret], rows[ret], offs[ret]
        if selected.size == 0:
            return
        hk, d = self.stage_k.shape[2:]
        kk = np.asarray(key, F32)[:n].reshape(n, hk, d)[selected]
        vv = np.asarray(value, F32)[:n].reshape(n, hk, d)[selected]
        self.stage_k[rows, offs] = (kk @ np.asarray(rk, F32)).astype(F32)
        self.stage_v[rows, offs] = (vv @ np.asarray(rv, F32)).astype(F32)

    def tuple(self):
        return self.stage_k, self.stage_v, self.owner


# ---------------------------------------------------------------------------
# read path
# ---------------------------------------------------------------------------
def read_tile(k8, v8, bt_row, start, end, prefix, k_new, v_new, stage, dtype, d):
    """kernels/streaming_attention._read_tile (streaming_attention.py:103-131).

    History is dequantized (owner-tag hits read the fp32 staging arena), then
    rounded to fp16 and then to the query dtype; current tokens are raw."""
    hk = k8.shape[2]
    k = np.empty((end - start, hk, d), F32)
    v = np.empty_like(k)
    old_end = min(end, prefix)
    if start < old_end:
        pos = np.arange(start, old_end)
        bs = k8.shape[1]
        blocks = np.asarray(bt_row, np.int64)[pos // bs]
        oldk, oldv = dequant_split(k8, v8, blocks, pos % bs, hk, d)
        if stage is not None:
            sk, sv, owner = stage
            row, off = blocks % owner.shape[0], pos % bs
            hit = (owner[row, off] == blocks)[:, None, None]
            oldk = np.where(hit, sk[row, off], oldk)
            oldv = np.where(hit, sv[row, off], oldv)
        c = old_end - start
        k[:c] = round_to(dtype, round_f16(oldk))
        v[:c] = round_to(dtype, round_f16(oldv))
    fresh = max(start, prefix)
    if fresh < end:
        if k_new is None or v_new is None:
            raise ValueError("Missing current KV")
        k[fresh - start :] = k_new[fresh - prefix : end - prefix]
        v[fresh - start :] = v_new[fresh - prefix : end - prefix]
    return k, v


def validate_layout(q, k_new, kc_shape, bt, qsl, seqs, stage):
    """streaming_attention._validate_tensors (:32-65) + slab_attention checks (:394-410)."""
    n, hq, d = q.shape
    nb, bs, hk, _ = kc_shape
    if hq < 1 or hk < 1 or hq % hk or len(qsl) != len(seqs) + 1 or not len(qsl) or qsl[0] != 0 or qsl[-1] != n:
        raise ValueError("Invalid slab query layout")
    for a, b, seq in zip(qsl, qsl[1:], seqs):
        if a > b or seq < 0 or (k_new is not None and seq < b - a):
            raise ValueError("Sequence length must cover its query chunk")
    if bt.ndim != 2 or bt.shape[0] < len(seqs):
        raise ValueError("Missing request block-table rows")
    for a, b, seq in zip(qsl, qsl[1:], seqs):
        prefix = seq - (b - a) if k_new is not None else seq
        if b > a and -(-prefix // bs) > bt.shape[1]:
            raise ValueError("Block table cannot cover the history")
    if stage is not None:
        sk, sv, owner = stage
        shape = (owner.shape[0], bs, hk, d)
        if owner.shape != shape[:2] or sk.shape != shape or sv.shape != shape or shape[0] < 1:
            raise ValueError("Invalid streaming staging geometry")


def streaming_attention(q, k_new, v_new, k8, v8, bt, qsl, seqs, scale, stage=None, *,
                        dtype="bf16", kv_tile=128, query_tile=32, rows=None):
    """kernels/streaming_attention.streaming_attention_ref (streaming_attention.py:134-196).

    Exact fp32 online softmax over [paged INT2 history with staged overrides]
    followed by the causal current chunk.  Returns rotated-space output
    [n, Hq, D] fp32 and natural-log LSE [n, Hq] (scale included).  Queries that
    see no key produce 0 and -inf.  ``rows`` (economy for large test cases): a
    list of [start, end) query-row ranges; only query tiles meeting one are
    computed, the other rows stay 0 / -inf."""
    q = np.asarray(q, F32)
    n, hq, d = q.shape
    hk = k8.shape[2]
    bt = np.asarray(bt)
    validate_layout(q, k_new, (k8.shape[0], k8.shape[1], hk, d), bt, qsl, seqs, stage)
    g = hq // hk
    scale = F32(scale)
    output = np.zeros((n, hq, d), F32)
    lse = np.full((n, hq), -np.inf, F32)
    for req, (a, b, seq) in enumerate(zip(qsl, qsl[1:], seqs)):
        prefix = seq - (b - a) if k_new is not None else seq
        newk = None if k_new is None else np.asarray(k_new, F32)[a:b]
        newv = None if v_new is None else np.asarray(v_new, F32)[a:b]
        for qa in range(a, b, query_tile):
            qb = min(qa + query_tile, b)
            if rows is not None and not any(r0 < qb and qa < r1 for r0, r1 in rows):
                continue
            qpart = q[qa:qb].transpose(1, 0, 2)  # [hq, nq, d]
            ends = seq - (b - a) + np.arange(qa - a, qb - a) + 1
            maximum = np.full((hq, qb - qa), -np.inf, F32)
            denom = np.zeros_like(maximum)
            acc = np.zeros((hq, qb - qa, d), F32)
            visible_end = seq - (b - a) + qb - a
            for start in range(0, visible_end, kv_tile):
                end = min(start + kv_tile, visible_end)
                k, v = read_tile(k8, v8, bt[req], start, end, prefix, newk, newv, stage, dtype, d)
                kh = np.repeat(k.transpose(1, 0, 2), g, axis=0)
                vh = np.repeat(v.transpose(1, 0, 2), g, axis=0)
                scores = (qpart @ kh.transpose(0, 2, 1)).astype(F32) * scale
                valid = np.arange(start, end)[None, :] < ends[:, None]
                scores = np.where(valid[None], scores, F32(-np.inf))
                with np.errstate(invalid="ignore"):
                    new_max = np.maximum(maximum, scores.max(-1))
                    safe_max = np.where(np.isfinite(new_max), new_max, F32(0))
                    old_w = np.exp(maximum - safe_max)
                    probs = np.exp(scores - safe_max[..., None])
                acc = acc * old_w[..., None] + (probs @ vh).astype(F32)
                denom = denom * old_w + probs.sum(-1, dtype=F32)
                maximum = new_max
            safe = np.where(denom > 0, denom, F32(1))
            output[qa:qb] = (acc / safe[..., None]).transpose(1, 0, 2)
            lse[qa:qb] = (maximum + np.log(safe)).T
    return output, lse


def merge_slab(output, lse, part, part_lse, start, ids=None) -> None:
    """kernels/slab_attention.merge_slab CPU branch (slab_attention.py:341-355),
    in place: empty (-inf) partials contribute nothing, NaN propagates."""
    target = slice(start, start + part.shape[0]) if ids is None else np.asarray(ids, np.int64)
    old_lse = lse[target]
    part_lse = np.asarray(part_lse, F32)
    with np.errstate(invalid="ignore", over="ignore"):
        maximum = np.maximum(old_lse, part_lse)
        safe = np.where(maximum == -np.inf, F32(0), maximum)
        alpha = np.exp(old_lse - safe)
        beta = np.exp(part_lse - safe)
        denom = alpha + beta
        denom = np.where(denom == 0.0, F32(1), denom)
        old = np.where((old_lse == -np.inf)[..., None], F32(0), output[target])
        new = np.where((part_lse == -np.inf)[..., None], F32(0), np.asarray(part, F32))
        output[target] = (old * alpha[..., None] + new * beta[..., None]) / denom[..., None]
        lse[target] = maximum + np.log(denom)
