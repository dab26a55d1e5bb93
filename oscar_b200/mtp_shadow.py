"""MTP draft-layer bf16 shadow pool (oscar_ascend/mtp_shadow.py:29-61).

With a packed int8 KV pool, the MTP draft layer must keep bf16 KV: its
``kv_cache`` argument is swapped for a plugin-owned bf16 pool of the same
logical shape (block ids map one to one), and everything else runs the
framework's own attention.  vLLM-CUDA writes the cache through
``do_kv_cache_update`` before ``forward``; both hooks swap the pool.
A shadow-pool failure raises (never silently writes bf16 into an int8 pool).
"""
from __future__ import annotations

import abc

import torch

from .surgery import compose

_CLASSES: dict = {}


class MTPShadowMixin(metaclass=abc.ABCMeta):
    def _shadow_kv(self, kv_cache):
        sh = getattr(self, "_oscar_shadow_kv", None)
        if sh is not None:
            return sh
        k_native, v_native = kv_cache[0], kv_cache[1]
        if k_native.dtype == torch.bfloat16 and v_native.dtype == torch.bfloat16:
            return kv_cache
        if isinstance(kv_cache, torch.Tensor):
            self._oscar_shadow_kv = torch.zeros(kv_cache.shape, dtype=torch.bfloat16, device=kv_cache.device)
        else:
            self._oscar_shadow_kv = (torch.zeros(k_native.shape, dtype=torch.bfloat16, device=k_native.device),
                                     torch.zeros(v_native.shape, dtype=torch.bfloat16, device=v_native.device))
        return self._oscar_shadow_kv

    @staticmethod
    def _needs_shadow(kv_cache) -> bool:
        return (isinstance(kv_cache, (tuple, list, torch.Tensor)) and len(kv_cache) >= 2 and kv_cache[0] is not None
                and kv_cache[0].dtype != torch.bfloat16)

    def do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping):
        if self._needs_shadow(kv_cache):
            kv_cache = self._shadow_kv(kv_cache)
        return self._oscar_base.do_kv_cache_update(self, layer, key, value, kv_cache, slot_mapping)

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs):
        if self._needs_shadow(kv_cache):
            kv_cache = self._shadow_kv(kv_cache)
        return self._oscar_base.forward(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs)


def shadow_impl_class(base: type) -> type:
    if issubclass(base, MTPShadowMixin):
        return base
    cls = _CLASSES.get(base)
    if cls is None:
        cls = compose(MTPShadowMixin, base, f"MTPShadow{base.__name__}", __name__)
        _CLASSES[base] = cls
    return cls
