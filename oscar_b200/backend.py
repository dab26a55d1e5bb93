"""OSCAR INT2 FULL-attention implementation for vLLM on B200.

Drop-in for oscar_ascend/backend.py:96-572 (AscendOscarAttentionBackendImpl):
the plugin swaps ``layer.impl.__class__`` to a subclass of the impl's own
class with :class:`OscarAttentionImplMixin` in front (see plugin.py), so only
``forward`` / ``do_kv_cache_update`` and the OSCAR store / staging / read
paths change.  Everything on the device runs in the CUDA kernels of
``csrc/`` through :mod:`oscar_b200.kernels`, the per-layer rotations
included (``csrc/rotate.cuh``).  There is no dense-history path and no CPU
fallback.
"""
from __future__ import annotations

import abc
from itertools import pairwise

import numpy as np
import torch

from . import kernels
from .config import OscarConfig
from .format import K_IDX_OFF, VALUES_PER_BYTE, check_d
from .rotation import get_layer_rotation


def metadata_batch_lists(attn_metadata) -> tuple[list, list]:
    """Host (query_start_loc, seq_lens) lists (backend.py:26-56).

    Host-side fields are preferred so the hot path never reads device
    metadata; a device tensor is only converted when nothing else exists."""

    def _as_list(x, name: str) -> list:
        if x is None:
            raise RuntimeError(f"attn_metadata.{name} is missing")
        if hasattr(x, "tolist"):
            return x.tolist()
        return list(x)

    q_sl_cpu = getattr(attn_metadata, "query_start_loc_cpu", None)
    ends = getattr(attn_metadata, "actual_seq_lengths_q", None)
    if q_sl_cpu is not None:
        qsl = _as_list(q_sl_cpu, "query_start_loc_cpu")
    elif ends is not None:
        qsl = [0] + _as_list(ends, "actual_seq_lengths_q")
    else:
        qsl = _as_list(attn_metadata.query_start_loc, "query_start_loc")
    seq_cpu = getattr(attn_metadata, "seq_lens_cpu", None)
    if seq_cpu is None:
        seq_cpu = getattr(attn_metadata, "_seq_lens_cpu", None)
    seq_list = getattr(attn_metadata, "seq_lens_list", None)
    seqs = _as_list(seq_list if seq_list is not None else (seq_cpu if seq_cpu is not None else attn_metadata.seq_lens),
                    "seq_lens")
    return qsl, seqs


def block_table_of(attn_metadata) -> torch.Tensor:
    """vLLM-Ascend names it ``block_tables``, vLLM-CUDA ``block_table``."""
    bt = getattr(attn_metadata, "block_tables", None)
    if bt is None:
        bt = getattr(attn_metadata, "block_table", None)
    if bt is None:
        raise RuntimeError("attn_metadata has no block table")
    return bt


_STEP_DTYPES = (torch.bfloat16, torch.float16)


def _token_stride(t: torch.Tensor, heads: int, d: int):
    """Elements between token rows of a [n, heads * D] or [n, heads, D] tensor
    whose heads are contiguous within a token; None for any other layout."""
    if t.dim() == 2 and t.shape[1] == heads * d and t.stride(1) == 1:
        ts = t.stride(0)
    elif t.dim() == 3 and t.shape[1] == heads and t.shape[2] == d and t.stride(2) == 1 and t.stride(1) == d:
        ts = t.stride(0)
    else:
        return None
    if (t.shape[0] > 1 and ts % 8) or t.data_ptr() % 16:
        return None
    return ts


def _device_ints(values, device) -> torch.Tensor:
    t = torch.from_numpy(np.asarray(values, dtype=np.int32))
    if device.type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


def _device_batch(attn_metadata, qsl: list, seqs: list, device) -> tuple:
    """Device int32 (query_start_loc [B+1], seq_lens [B]) for the staging write:
    the metadata's own device tensors when it carries them (as vLLM's does:
    no host-to-device copy, and the call stays capturable in a CUDA graph),
    else copies of the host lists."""
    b = len(qsl) - 1
    dq = getattr(attn_metadata, "query_start_loc", None)
    ds = getattr(attn_metadata, "seq_lens", None)
    if isinstance(dq, torch.Tensor) and isinstance(ds, torch.Tensor) and dq.device == device and \
            ds.device == device and dq.dtype == torch.int32 and ds.dtype == torch.int32 and \
            dq.numel() >= b + 1 and ds.numel() >= b:
        return dq[: b + 1].contiguous(), ds[:b].contiguous()
    return _device_ints(qsl, device), _device_ints(seqs[:b], device)


class OscarAttentionImplMixin(metaclass=abc.ABCMeta):
    """The OSCAR read/write/window paths.  The plugin builds a subclass of the
    running vLLM attention impl with these methods in front of its own
    (plugin.oscar_impl_class, oscar_b200.surgery)."""

    # decode-sized steps run as one native call (_native_step); False keeps them
    # on the per-kernel path (the two are bit-identical)
    _oscar_native_step = True

    # ------------------------------------------------------------------ setup
    def _oscar_setup(self) -> None:
        """backend.py:100-123."""
        if getattr(self, "_oscar_cfg", None) is not None:
            return
        cfg = OscarConfig.from_env(head_dim=self.head_size)
        check_d(cfg.head_dim)
        if self.num_heads % self.num_kv_heads:
            raise ValueError("OSCAR requires Hq divisible by Hk")
        self._oscar_cfg = cfg
        self._oscar_stage_ready = False
        self._oscar_stats = {"writes": 0, "kv_bytes_written": 0, "reads": 0}
        if cfg.verbose:
            print(f"[oscar-b200] OSCAR active: D={self.head_size} Hq={self.num_heads} Hk={self.num_kv_heads} "
                  f"slot=160B (K 96B + V 64B) K-rot={'loaded' if cfg.k_rotation_path else 'identity'} "
                  f"V-rot={'loaded' if cfg.v_rotation_path else 'identity'} "
                  f"window(sink={cfg.sink_tokens}, recent={cfg.recent_tokens}) clip={cfg.k_clip_ratio}/{cfg.v_clip_ratio}")

    @property
    def _oscar(self) -> OscarConfig:
        return self._oscar_cfg

    # ------------------------------------------------------------------ caches / rotations
    def _set_caches(self, kv_cache) -> None:
        """backend.py:200-236: bind (K, V) caches and check the slot geometry once."""
        if isinstance(kv_cache, (tuple, list)) and len(kv_cache) >= 2:
            self.key_cache, self.value_cache = kv_cache[0], kv_cache[1]
        elif isinstance(kv_cache, torch.Tensor) and kv_cache.dim() > 0:
            self.key_cache, self.value_cache = kv_cache[0], kv_cache[1]
        if getattr(self, "key_cache", None) is None or getattr(self, "value_cache", None) is None:
            raise ValueError("OSCAR: KV cache is not bound")
        if not getattr(self, "_oscar_geo_ok", False):
            k8 = self.key_cache.view(torch.uint8)
            v8 = self.value_cache.view(torch.uint8)
            if k8.ndim != 4 or v8.ndim != 4 or not k8.is_contiguous() or not v8.is_contiguous():
                raise ValueError("OSCAR requires contiguous [blocks, tokens, heads, bytes] caches")
            slot_k, slot_v = int(k8.stride(2)), int(v8.stride(2))
            need_k = K_IDX_OFF + self.head_size // VALUES_PER_BYTE
            need_v = self.head_size // VALUES_PER_BYTE
            if slot_k not in (self.head_size, 2 * self.head_size):
                raise ValueError(f"OSCAR geometry: K slot of {slot_k} B (expected {self.head_size} packed or "
                                 f"{2 * self.head_size} legacy)")
            if need_k > slot_k or need_v > slot_v:
                raise ValueError(f"OSCAR geometry: K needs {need_k} B / V {need_v} B, slots are {slot_k}/{slot_v} B")
            self._oscar_geo_ok = True

    def _layer_rots(self, layer, device):
        """backend.py:238-246: per-layer (R_k, R_v), loaded once, strict."""
        rots = getattr(layer, "_oscar_rots", None)
        if not rots:
            cfg = self._oscar
            rk = get_layer_rotation(cfg.k_rotation_path, layer.layer_name, self.head_size, device, mode="k", strict=True)
            rv = get_layer_rotation(cfg.v_rotation_path, layer.layer_name, self.head_size, device, mode="v", strict=True)
            layer._oscar_rots = (rk, rv)
            rots = layer._oscar_rots
        rk, rv = rots
        if rk.device != device:
            rk, rv = rk.to(device), rv.to(device)
            layer._oscar_rots = (rk, rv)
            layer._oscar_rvt = None
        return rk, rv

    def _layer_rvt(self, layer, device):
        """R_v^T (contiguous), cached per layer: o @ R_v^T reads it row-major."""
        rvt = getattr(layer, "_oscar_rvt", None)
        _, rv = self._layer_rots(layer, device)
        if rvt is None or rvt.device != device:
            rvt = rv.t().contiguous()
            layer._oscar_rvt = rvt
        return rvt

    def _rotate(self, x: torch.Tensor, rot: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
        """x @ R in fp32, [N, H, D] -> [N, H, D] of out_dtype (rotate_rows)."""
        return kernels.rotate_rows(x, rot, out_dtype=out_dtype)[0]

    # ------------------------------------------------------------------ write path
    def _store(self, layer, key, value, slot_mapping, *, invalidate: bool, query_rows=None):
        """Rotate, clip/INT2-store; returns (k_rot, v_rot, k_lo, v_lo, q_lo):
        fp32 rows for the store / staging window, the model-dtype rows the
        attention reads (x @ R then .to(dtype), backend.py:360-366) and, when
        ``query_rows`` is given, the rotated queries (q @ R_k, query dtype),
        all from one rotation launch."""
        n = slot_mapping.shape[0]
        if invalidate and getattr(layer, "_oscar_stage_ready", False):
            kernels.staging_invalidate(slot_mapping, layer._oscar_slot_owner, self.stage_block)
        rotated = self._rotate_step(layer, key, value, n, query_rows)
        kernels.oscar_store(rotated[0], rotated[1], self.key_cache, self.value_cache, slot_mapping,
                            self._oscar.k_clip_ratio, self._oscar.v_clip_ratio)
        self._oscar_stats["writes"] += 1
        self._oscar_stats["kv_bytes_written"] += n * self.num_kv_heads * 160
        return rotated

    def _rotate_step(self, layer, key, value, n, query_rows=None):
        """(k_rot, v_rot, k_lo, v_lo, q_lo) of the step's n tokens, from one
        rotation launch (q_lo is None when query_rows is not given)."""
        hk, d = self.num_kv_heads, self.head_size
        k = key[:n].reshape(n, hk, d)
        v = value[:n].reshape(n, hk, d)
        rk, rv = self._layer_rots(layer, k.device)
        k_rot, v_rot = (torch.empty(n, hk, d, dtype=torch.float32, device=k.device) for _ in range(2))
        k_lo = torch.empty((n, hk, d), dtype=k.dtype, device=k.device)
        v_lo = torch.empty((n, hk, d), dtype=v.dtype, device=v.device)
        jobs = [(k, rk, k_lo, k_rot), (v, rv, v_lo, v_rot)]
        q_lo = None
        if query_rows is not None and query_rows.dtype == k.dtype == v.dtype:
            q_lo = torch.empty(query_rows.shape, dtype=query_rows.dtype, device=k.device)
            jobs.append((query_rows, rk, q_lo, None))
        if k.dtype == v.dtype:
            kernels.rotate_rows_many(jobs)
        else:
            kernels.rotate_rows(k, rk, out=k_lo, out_f32=k_rot)
            kernels.rotate_rows(v, rv, out=v_lo, out_f32=v_rot)
        return k_rot, v_rot, k_lo, v_lo, q_lo

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping) -> None:
        """backend.py:151-198: owner invalidation -> rotate -> clip/INT2 store."""
        if key is None or value is None:
            return
        slot_mapping = slot_mapping.to(device=key.device, dtype=torch.int64)
        if slot_mapping.shape[0] <= 0:
            return
        self._set_caches(kv_cache)
        self._store(layer, key, value, slot_mapping, invalidate=True)

    # ------------------------------------------------------------------ staging window
    def _ensure_staging(self, layer, kv_cache) -> None:
        """backend.py:492-511."""
        if getattr(layer, "_oscar_stage_ready", False):
            return
        bs = self.key_cache.shape[1]
        cfg = self._oscar
        self.stage_block = bs
        self.sink_eff = (cfg.sink_tokens // bs) * bs
        self.sink_pages = self.sink_eff // bs
        self.tail_pages = (cfg.recent_tokens + bs - 1) // bs + 1
        rows = max((cfg.staging_tokens + bs - 1) // bs, self.sink_pages + self.tail_pages + 2)
        dev = self.key_cache.device
        layer._oscar_stage_k = torch.zeros(rows, bs, self.num_kv_heads, self.head_size, dtype=torch.float32, device=dev)
        layer._oscar_stage_v = torch.zeros_like(layer._oscar_stage_k)
        layer._oscar_slot_owner = torch.full((rows, bs), -1, dtype=torch.int64, device=dev)
        layer._oscar_seat_winner = torch.zeros(rows * bs, dtype=torch.int64, device=dev)
        layer._oscar_stage_epoch = 0
        layer._oscar_stage_rows = rows
        layer._oscar_stage_ready = True
        self._oscar_stage_ready = True

    def _staging_write(self, layer, key, value, attn_metadata, rotated=None) -> None:
        """backend.py:513-555: last writer per seat; kept rows store rotated
        unclipped fp32.  ``rotated`` reuses the store path's x @ R."""
        n = attn_metadata.num_actual_tokens
        if n == 0:
            return
        dev = key.device
        slot = attn_metadata.slot_mapping[:n].to(device=dev, dtype=torch.int64)
        qsl, seqs = metadata_batch_lists(attn_metadata)
        if rotated is None:
            rk, rv = self._layer_rots(layer, dev)
            hk, d = self.num_kv_heads, self.head_size
            rotated = (self._rotate(key[:n].reshape(n, hk, d), rk), self._rotate(value[:n].reshape(n, hk, d), rv))
        k_rot, v_rot = rotated
        qsl_d, seqs_d = _device_batch(attn_metadata, qsl, seqs, dev)
        if torch.cuda.is_current_stream_capturing():
            # a replayed graph cannot advance a host epoch: the built-in scratch is cleared per call
            kernels.staging_write_noalloc(k_rot, v_rot, slot.contiguous(), qsl_d, seqs_d, self.sink_eff,
                                          self._oscar.recent_tokens, layer._oscar_stage_k, layer._oscar_stage_v,
                                          layer._oscar_slot_owner)
            return
        layer._oscar_stage_epoch += 1
        kernels.staging_write(k_rot, v_rot, slot, qsl_d, seqs_d, self.sink_eff, self._oscar.recent_tokens,
                              layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner,
                              layer._oscar_seat_winner, layer._oscar_stage_epoch)

    def _stage(self, layer):
        if self._oscar.window_enabled and getattr(self, "_oscar_stage_ready", False) and \
                getattr(layer, "_oscar_stage_ready", False):
            return layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner
        return None

    # ------------------------------------------------------------------ main entry
    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        """backend.py:249-282 (streaming mode)."""
        if output is None:
            raise ValueError("Output tensor must be provided.")
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("OSCAR fused output quantization is unsupported")
        if attn_metadata is None:
            return output.fill_(0)
        self._set_caches(kv_cache)
        if key is not None and value is not None and self._oscar_native_step and \
                self._native_step(layer, query, key, value, attn_metadata, output):
            return output
        if key is not None and value is not None:
            n = attn_metadata.num_actual_tokens
            slots = attn_metadata.slot_mapping[:n].to(device=key.device, dtype=torch.int64)
            rotated = None
            qsl, seqs = metadata_batch_lists(attn_metadata)
            fused = self._oscar.window_enabled and 0 < n <= kernels.WRITE_STEP_MAX_TOKENS and \
                len(qsl) - 1 <= kernels.WRITE_STEP_MAX_REQUESTS and slots.shape[0] == n
            if slots.shape[0] > 0:
                q_rows = self._whole_batch_rotated_queries(query, key, attn_metadata)
                if fused:
                    # store + staging write of a decode-sized step in one launch
                    self._ensure_staging(layer, kv_cache)
                    rotated = self._rotate_step(layer, key, value, n, q_rows)
                    qsl_d, seqs_d = _device_batch(attn_metadata, qsl, seqs, key.device)
                    kernels.write_step(rotated[0], rotated[1], self.key_cache, self.value_cache, slots,
                                       self._oscar.k_clip_ratio, self._oscar.v_clip_ratio, qsl_d, seqs_d,
                                       self.sink_eff, self._oscar.recent_tokens, layer._oscar_stage_k,
                                       layer._oscar_stage_v, layer._oscar_slot_owner)
                    self._oscar_stats["writes"] += 1
                    self._oscar_stats["kv_bytes_written"] += n * self.num_kv_heads * 160
                else:
                    rotated = self._store(layer, key, value, slots, invalidate=not self._oscar.window_enabled,
                                          query_rows=q_rows)
            if self._oscar.window_enabled and not (fused and slots.shape[0] > 0):
                self._ensure_staging(layer, kv_cache)
                self._staging_write(layer, key, value, attn_metadata, rotated=None if rotated is None else rotated[:2])
            return self._streaming_attention(layer, query, key, value, kv_cache, attn_metadata, output,
                                             rotated_lo=None if rotated is None else rotated[2:])
        return self._streaming_attention(layer, query, key, value, kv_cache, attn_metadata, output)

    def _native_step(self, layer, query, key, value, md, output) -> bool:
        """A decode-sized step (window on, <= 256 tokens and requests, every
        request with cached history, 16-bit activations whose heads are
        contiguous per token) as one native call: rotations, write step,
        attention and output rotation (kernels.decode_layer_step).  Returns
        False, having done nothing, for any other step."""
        cfg = self._oscar
        n = md.num_actual_tokens
        dt = query.dtype
        if (not cfg.window_enabled or n <= 0 or n > kernels.WRITE_STEP_MAX_TOKENS or dt not in _STEP_DTYPES
                or key.dtype != dt or value.dtype != dt or output.dtype != dt):
            return False
        qsl, seqs = metadata_batch_lists(md)
        b = len(qsl) - 1
        if b < 1 or b > kernels.WRITE_STEP_MAX_REQUESTS or qsl[-1] != n or len(seqs) < b:
            return False
        if any(bq - aq >= s_ for aq, bq, s_ in zip(qsl, qsl[1:], seqs) if bq > aq):
            return False  # a prefix-free request attends in the model's domain
        hq, hk, d = self.num_heads, self.num_kv_heads, self.head_size
        rows = []
        for t, heads in ((query, hq), (key, hk), (value, hk), (output, hq)):
            ts = _token_stride(t, heads, d)
            if ts is None:
                return False
            rows.append(ts)
        slots = md.slot_mapping
        if slots.dtype != torch.int64 or slots.device != query.device or slots.shape[0] < n or \
                (slots.dim() == 1 and slots.stride(0) != 1):
            return False
        self._ensure_staging(layer, None)
        qsl_d, seqs_d = _device_batch(md, qsl, seqs, query.device)
        table = block_table_of(md)
        if table.dtype != torch.int32 or not table.is_contiguous():
            table = table.to(torch.int32).contiguous()
        rk, rv = self._layer_rots(layer, query.device)
        rvt = self._layer_rvt(layer, query.device)
        if output.shape[0] > n:
            output[n:].zero_()
        kernels.decode_layer_step(query, key, value, rows, n, hq, hk, d, rk, rv, rvt, cfg.k_clip_ratio,
                                  cfg.v_clip_ratio, self.key_cache, self.value_cache, slots, qsl_d, seqs_d, table,
                                  qsl, seqs[:b], self.sink_eff, cfg.recent_tokens, self.scale, layer._oscar_stage_k,
                                  layer._oscar_stage_v, layer._oscar_slot_owner, output,
                                  self._step_scratch(query.device))
        self._oscar_stats["writes"] += 1
        self._oscar_stats["kv_bytes_written"] += n * hk * 160
        return True

    def _step_scratch(self, device) -> torch.Tensor:
        """The impl's scratch for native steps (rotated rows, attention output
        and the attention workspace up to the configured bound), grown on
        demand and shared by the impl's layers (their steps run in stream order)."""
        buf = getattr(self, "_oscar_scratch", None)
        if buf is None or buf.device != device:
            # sized once for the largest native step plus the configured workspace bound
            need = kernels.decode_step_scratch_bytes(kernels.WRITE_STEP_MAX_TOKENS, self.num_heads, self.num_kv_heads,
                                                     self.head_size, self._oscar.stream_workspace_bytes)
            buf = torch.empty(need, dtype=torch.uint8, device=device)
            self._oscar_scratch = buf
        return buf

    def _whole_batch_rotated_queries(self, query, key, metadata):
        """The query rows [covered, Hq, D] when every active request takes the
        rotated (cached-history) path of _streaming_attention, else None."""
        actual = min(query.shape[0], metadata.num_actual_tokens)
        if actual == 0:
            return None
        starts, seqs = metadata_batch_lists(metadata)
        starts = [min(x, actual) for x in starts]
        active = [i for i, (a, b) in enumerate(pairwise(starts)) if b > a]
        if not active or any(seqs[i] == starts[i + 1] - starts[i] for i in active):
            return None
        return query[:starts[-1]].view(starts[-1], self.num_heads, self.head_size)

    def _streaming_attention(self, layer, query, key, value, kv_cache, metadata, output, rotated_lo=None):
        """backend.py:334-393: prefix-free requests attend their own chunk in
        the model's domain; cached requests go through the rotated INT2 path.
        ``rotated_lo`` holds the store path's (x @ R).to(dtype) rows of key and
        value (and of the queries, or None), reused instead of rotating them
        again."""
        if (key is None) != (value is None):
            raise ValueError("Both new K and V must be supplied together")
        actual = min(query.shape[0], metadata.num_actual_tokens)
        out_rows = output.view(output.shape[0], -1)
        if actual == 0:
            return output.zero_()
        starts, seqs = metadata_batch_lists(metadata)
        starts = [min(x, actual) for x in starts]
        covered = starts[-1]
        if covered < out_rows.shape[0]:
            out_rows[covered:].zero_()
        active = [i for i, (a, b) in enumerate(pairwise(starts)) if b > a]
        fresh_only = [i for i in active if key is not None and seqs[i] == starts[i + 1] - starts[i]]
        fresh_set = set(fresh_only)
        cached = [i for i in active if i not in fresh_set]
        table = block_table_of(metadata)
        hq, hk, d = self.num_heads, self.num_kv_heads, self.head_size
        q_all = query[:actual].view(actual, hq, d)
        k_all = None if key is None else key[:actual].view(actual, hk, d)
        v_all = None if value is None else value[:actual].view(actual, hk, d)
        for group, rotate in ((fresh_only, False), (cached, True)):
            if not group:
                continue
            if len(group) == len(active):
                # the whole batch takes this path: no gather, inactive requests are skipped by the kernel
                ids, sub_starts, sub_seqs, sub_table = None, starts, seqs[: len(starts) - 1], table
                q_in = q_all[:covered]
                k_in = None if k_all is None else k_all[:covered]
                v_in = None if v_all is None else v_all[:covered]
            else:
                tok = [t for i in group for t in range(starts[i], starts[i + 1])]
                ids = torch.as_tensor(tok, device=query.device)
                lengths = [starts[i + 1] - starts[i] for i in group]
                sub_starts = [0]
                for length in lengths:
                    sub_starts.append(sub_starts[-1] + length)
                sub_seqs = [seqs[i] for i in group]
                sub_table = table[torch.as_tensor(group, device=table.device)]
                q_in = q_all[ids]
                k_in = None if k_all is None else k_all[ids]
                v_in = None if v_all is None else v_all[ids]
            if rotate:
                rk, rv = self._layer_rots(layer, query.device)
                q_lo = None if rotated_lo is None else rotated_lo[2]
                if ids is None and q_lo is not None and q_lo.shape[0] == covered:
                    q_in = q_lo
                else:
                    q_in = self._rotate(q_in, rk, query.dtype)
                if k_in is not None and rotated_lo is not None and rotated_lo[0].shape[0] >= covered:
                    k_lo, v_lo = rotated_lo[:2]
                    k_in = k_lo[:covered] if ids is None else k_lo[ids]
                    v_in = v_lo[:covered] if ids is None else v_lo[ids]
                else:
                    k_in = None if k_in is None else self._rotate(k_in, rk, query.dtype)
                    v_in = None if v_in is None else self._rotate(v_in, rv, query.dtype)
                stage = self._stage(layer)
            else:
                stage = None
            out, _ = kernels.slab_attention(q_in, k_in, v_in, self.key_cache, self.value_cache, sub_table, sub_starts,
                                            sub_seqs, self.scale, stage,
                                            workspace_bytes=self._oscar.stream_workspace_bytes)
            if rotate:
                m = out.shape[0]
                rvt = self._layer_rvt(layer, query.device)
                if ids is None and out_rows.is_contiguous():
                    # o @ R_v^T straight into the output rows, in the output dtype
                    kernels.rotate_rows(out, rvt, out=out_rows[:m].view(m, hq, d))
                    continue
                out = kernels.rotate_rows(out, rvt, out_dtype=output.dtype)[0]
            result = out.to(output.dtype).view(out.shape[0], hq * d)
            if ids is None:
                out_rows[: result.shape[0]].copy_(result)
            else:
                out_rows[ids] = result
        return output


class OscarAttentionBackendImpl(OscarAttentionImplMixin):
    """Stand-alone impl (no vLLM base class) used by tests, probes and the bench:
    construct with ``OscarAttentionBackendImpl.create(num_heads, num_kv_heads, head_size, scale)``."""

    @classmethod
    def create(cls, num_heads: int, num_kv_heads: int, head_size: int, scale: float | None = None):
        impl = cls.__new__(cls)
        impl.num_heads, impl.num_kv_heads, impl.head_size = num_heads, num_kv_heads, head_size
        impl.scale = head_size**-0.5 if scale is None else scale
        impl.key_cache = impl.value_cache = None
        impl._oscar_setup()
        return impl


# the reference's class name, for code that imports it by name
AscendOscarAttentionBackendImpl = OscarAttentionBackendImpl
