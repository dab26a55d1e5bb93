"""vLLM ``general_plugins`` entry point: class surgery onto FULL-attention impls.

Drop-in for oscar_ascend/plugin.py:60-267.  ``load_plugin()`` (no arguments,
idempotent) wraps ``Attention.__init__`` with an after-hook.  For decoder
FULL-attention layers of hybrid models the hook swaps ``layer.impl.__class__``
to ``OscarImpl[<original impl class>]`` (a subclass of the original class
with the methods of OscarAttentionImplMixin in front, oscar_b200.surgery),
runs ``_oscar_setup()`` and rolls the instance back if setup fails.  MTP draft layers keep bf16 KV (optionally in a shadow pool,
OSCAR_ASCEND_PACKED=1); sliding-window, sink and non-decoder layers are
skipped.  The Ascend platform bootstrap (plugin.py:27-57) has no CUDA
counterpart and is not part of this package.

Register with:  [project.entry-points."vllm.general_plugins"]
                oscar_b200 = "oscar_b200.plugin:load_plugin"
"""
from __future__ import annotations

import os

_HEARTBEAT: dict = {"loaded": 0, "layers": [], "errors": []}
_PATCHED = False
_SKIP_REASONS_LOGGED: set = set()
_IMPL_CLASSES: dict = {}


def oscar_impl_class(base: type) -> type:
    """Subclass of the running impl class with the OSCAR paths in front (cached)."""
    from .backend import OscarAttentionImplMixin
    from .surgery import compose

    if issubclass(base, OscarAttentionImplMixin):
        return base
    cls = _IMPL_CLASSES.get(base)
    if cls is None:
        cls = compose(OscarAttentionImplMixin, base, f"Oscar{base.__name__}", __name__)
        _IMPL_CLASSES[base] = cls
    return cls


def install_impl(impl, target_class) -> None:
    """Commit class surgery only if setup succeeds; preserve original state (plugin.py:60-70)."""
    old_class, old_state = impl.__class__, impl.__dict__.copy()
    try:
        impl.__class__ = target_class
        impl._oscar_setup()
    except Exception:
        impl.__class__ = old_class
        impl.__dict__.clear()
        impl.__dict__.update(old_state)
        raise


def _is_hybrid_config(model_config) -> bool:
    """plugin.py:184-196: registry flag, else any non-attention layer type."""
    if getattr(model_config, "is_hybrid", False):
        return True
    hf = getattr(model_config, "hf_text_config", None) or getattr(model_config, "hf_config", None)
    layer_types = getattr(hf, "layer_types", None) or []
    return any(lt != "attention" for lt in layer_types)


def _is_mtp_layer(layer_name: str) -> bool:
    return ".mtp." in layer_name or layer_name.startswith("mtp.")


def _has_sliding_window(impl) -> bool:
    """vLLM-CUDA impls encode "no window" as (-1, -1) (the Ascend impl as None)."""
    window = getattr(impl, "sliding_window", None)
    if window is None:
        return False
    if isinstance(window, (tuple, list)):
        return any(w is not None and w >= 0 for w in window)
    return True


def _skip_reasons(impl, model_config) -> list[str]:
    reasons = []
    if not _is_hybrid_config(model_config):
        reasons.append("not-hybrid")
    at = getattr(impl, "attn_type", "decoder")
    at_value = getattr(at, "value", at)
    if str(at_value) != "decoder":
        reasons.append(f"attn_type={at!r}")
    if _has_sliding_window(impl):
        reasons.append("sliding-window")
    if getattr(impl, "sinks", None) is not None:
        reasons.append("sinks")
    return reasons


def _should_oscar(layer, impl, model_config=None) -> bool:
    """plugin.py:202-253: decoder FULL layers of hybrid models; MTP drafts rejected first."""
    layer_name = getattr(layer, "layer_name", "") or ""
    if _is_mtp_layer(layer_name):
        return False
    try:
        if model_config is None:
            from vllm.config import get_current_vllm_config

            model_config = get_current_vllm_config().model_config
        reasons = _skip_reasons(impl, model_config)
    except Exception as exc:  # pragma: no cover - depends on a live vLLM config
        print(f"[oscar-b200][SKIP] _should_oscar failed: {exc}")
        return False
    if reasons:
        key = ",".join(reasons)
        if key not in _SKIP_REASONS_LOGGED:
            _SKIP_REASONS_LOGGED.add(key)
            print(f"[oscar-b200][SKIP] {layer_name} -> not replaced: {key}")
        return False
    return True


def _install_worker_hooks() -> None:
    """The worker seams (oscar_b200.integration) once an OSCAR layer exists
    (plugin.py:150-151 of the reference); an engine without vLLM-CUDA's worker
    classes runs without them."""
    try:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner
        from vllm.v1.worker.gpu_worker import Worker
    except ImportError as exc:  # pragma: no cover - depends on the engine build
        if "worker-hooks" not in _SKIP_REASONS_LOGGED:
            _SKIP_REASONS_LOGGED.add("worker-hooks")
            _HEARTBEAT["errors"].append(f"worker hooks: {exc}")
            print(f"[oscar-b200] vLLM-CUDA worker classes unavailable, memory seams not installed: {exc}")
        return
    from .integration import install_runner_hooks

    install_runner_hooks(Worker, GPUModelRunner)


def attach(attention_layer) -> bool:
    """The after-hook body for one constructed ``Attention`` layer."""
    impl = getattr(attention_layer, "impl", None)
    if impl is None:
        return False
    layer_name = getattr(attention_layer, "layer_name", "") or ""
    if os.environ.get("OSCAR_ASCEND_PACKED", "0") == "1" and _is_mtp_layer(layer_name):
        from .mtp_shadow import shadow_impl_class

        impl.__class__ = shadow_impl_class(impl.__class__)
        return True
    if not _should_oscar(attention_layer, impl):
        return False
    install_impl(impl, oscar_impl_class(impl.__class__))
    _install_worker_hooks()
    _HEARTBEAT["loaded"] += 1
    _HEARTBEAT["layers"].append(f"{layer_name}:heads={impl.num_heads}/kv={impl.num_kv_heads}/d={impl.head_size}")
    return True


def load_plugin() -> None:
    """vllm.load_general_plugins() entry (plugin.py:73-181)."""
    global _PATCHED
    if _PATCHED:
        return
    if os.environ.get("OSCAR_ASCEND_ENABLE", "auto") == "0":
        print("[oscar-b200] OSCAR_ASCEND_ENABLE=0: not injecting")
        _PATCHED = True
        return
    try:
        from vllm.model_executor.layers.attention.attention import Attention
    except Exception as exc:  # pragma: no cover - vLLM absent
        _HEARTBEAT["errors"].append(f"attention import: {exc}")
        print(f"[oscar-b200] cannot locate Attention (not injecting): {exc}")
        _PATCHED = True
        return
    orig_init = Attention.__init__

    def _patched_init(self, *args, **kwargs):
        orig_init(self, *args, **kwargs)
        try:
            attach(self)
        except Exception as exc:
            _HEARTBEAT["errors"].append(str(exc))
            raise RuntimeError(f"[oscar-b200] injection failed: {getattr(self, 'layer_name', '?')}: {exc}") from exc

    Attention.__init__ = _patched_init
    _PATCHED = True
    print("[oscar-b200] plugin injected: Attention.__init__ after-hook")


def heartbeat() -> dict:
    return dict(_HEARTBEAT)
