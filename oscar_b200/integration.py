"""Worker seams for vLLM-CUDA: the KV budget that leaves room for OSCAR's
persistent buffers, their allocation at cache set-up, and the READY manifest.

Counterpart of oscar_ascend/integration.py:17-245 for vLLM 0.22's CUDA worker
(``vllm.v1.worker.gpu_worker.Worker`` and
``vllm.v1.worker.gpu_model_runner.GPUModelRunner``); no vLLM file is edited.

* ``Worker.determine_available_memory`` is wrapped: from the memory vLLM
  profiled for the KV cache it deducts what OSCAR keeps per layer (the
  rotations and the fp32 staging arena of every OSCAR layer), the bf16 shadow
  pool of MTP draft layers (per cache block) and the transient bytes of one
  forward of ``max_num_batched_tokens`` tokens (the attention workspace bound
  plus the rotated rows and fp32 partial outputs), and returns the budget
  left for cache blocks (``memory_budget``).
* ``GPUModelRunner.initialize_kv_cache_tensors`` is wrapped: after vLLM has
  allocated the caches, every OSCAR layer binds its packed int8 cache (whose
  slots the engine allocates with ``--kv-cache-dtype int8_per_token_head``:
  D bytes per K and per V slot), loads its rotations and allocates its
  staging arena; every MTP draft layer allocates its bf16 shadow pool.  The
  hook then checks that the allocation stays inside the profiled budget and
  that every FULL-attention layer of the model is an OSCAR layer, and prints
  the READY manifest (one JSON line).

The arithmetic of the budget is the reference's; what is counted per layer is
this implementation's (two fp32 rotations and the cached R_v^T, no
transposed copies of R_k; the attention workspace bound instead of slab
buffers).
"""
from __future__ import annotations

import hashlib
import json
from copy import deepcopy
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent


def memory_budget(available: int, native_per_block: int, shadow_per_block: int, fixed_bytes: int) -> int:
    """Bytes of native cache blocks that fit once ``fixed_bytes`` are set aside
    and every block also carries ``shadow_per_block`` bytes of shadow pool
    (integration.py:17-23)."""
    if native_per_block <= 0 or available <= fixed_bytes:
        raise ValueError("Insufficient memory for OSCAR persistent buffers")
    blocks = (available - fixed_bytes) // (native_per_block + shadow_per_block)
    if blocks < 1:
        raise ValueError("OSCAR memory budget cannot hold one cache block")
    return blocks * native_per_block


def is_oscar_impl(impl) -> bool:
    return hasattr(impl, "_oscar_cfg")


def is_shadow_impl(impl) -> bool:
    from .mtp_shadow import MTPShadowMixin

    return isinstance(impl, MTPShadowMixin)


def rotation_bytes(impl) -> int:
    """R_k, R_v and the cached R_v^T of one layer, fp32."""
    return 3 * impl.head_size * impl.head_size * 4


def staging_rows(cfg, block_size: int) -> int:
    """Arena rows of one layer (the rule of backend._ensure_staging)."""
    sink_pages = (cfg.sink_tokens // block_size)
    tail_pages = (cfg.recent_tokens + block_size - 1) // block_size + 1
    return max((cfg.staging_tokens + block_size - 1) // block_size, sink_pages + tail_pages + 2)


def staging_bytes(impl, block_size: int) -> int:
    """fp32 K/V rows, owner tags and seat scratch of one layer's arena."""
    if not impl._oscar.window_enabled:
        return 0
    seats = staging_rows(impl._oscar, block_size) * block_size
    return seats * (2 * impl.num_kv_heads * impl.head_size * 4 + 8 + 8)


def transient_bytes(impls, max_tokens: int, act_bytes: int = 2) -> int:
    """The largest transient footprint of one forward over ``max_tokens``
    tokens: the attention workspace bound, the rotated K/V rows (fp32 and
    model dtype), the rotated queries and the fp32 attention output and LSE."""
    active = [i for i in impls if i._oscar.attention_mode == "streaming"]
    if not active:
        return 0
    if max_tokens <= 0:
        raise ValueError("Streaming reserve requires max_num_batched_tokens")
    return max(i._oscar.stream_workspace_bytes
               + max_tokens * (i.num_kv_heads * i.head_size * 2 * (4 + act_bytes)
                               + i.num_heads * i.head_size * (act_bytes + 4) + i.num_heads * 4)
               for i in active)


def shadow_block_bytes(spec) -> int:
    """bf16 K and V of one cache block of an MTP draft layer."""
    head_v = getattr(spec, "head_size_v", None) or spec.head_size
    return spec.block_size * spec.num_kv_heads * (spec.head_size + head_v) * 2


def verify_layers(layer_types, actual_ids) -> None:
    """Every FULL-attention layer of the model carries OSCAR (integration.py:65-74)."""
    expected = {i for i, kind in enumerate(layer_types) if kind in ("full_attention", "attention")}
    if not expected or set(actual_ids) != expected or len(actual_ids) != len(expected):
        raise RuntimeError(f"Incomplete OSCAR layers: expected={sorted(expected)}, actual={sorted(actual_ids)}")


def source_fingerprint() -> str:
    """sha256 over the package's Python sources and its native library."""
    from . import _native

    digest = hashlib.sha256()
    files = sorted(PACKAGE.rglob("*.py")) + [Path(_native.LIB_PATH)]
    for path in files:
        if path.exists():
            digest.update(str(path.relative_to(PACKAGE)).encode())
            digest.update(path.read_bytes())
    return digest.hexdigest()


def plan_memory(available: int, ctx: dict, specs: dict, native_per_block: int, max_tokens: int) -> dict:
    """The memory plan of one worker: ``ctx`` maps layer names to attention
    modules, ``specs`` layer names to their KV cache specs, and
    ``native_per_block`` is the bytes one cache block takes over all layers."""
    shadow = fixed = 0
    oscar_impls = []
    for name, module in ctx.items():
        impl = getattr(module, "impl", None)
        if impl is None:
            continue
        if is_shadow_impl(impl):
            shadow += shadow_block_bytes(specs[name])
        elif is_oscar_impl(impl):
            oscar_impls.append(impl)
            # the engine's page size bounds the arena of the kernel block size
            fixed += rotation_bytes(impl) + staging_bytes(impl, specs[name].block_size)
    transient = transient_bytes(oscar_impls, max_tokens)
    fixed += transient
    budget = memory_budget(available, native_per_block, shadow, fixed)
    return {"available": available, "native": native_per_block, "shadow": shadow, "fixed": fixed,
            "budget": budget, "streaming_transient_bytes": transient}


def _native_per_block(vllm_config, specs: dict, available: int) -> int:
    from vllm.v1.core.kv_cache_utils import get_kv_cache_config_from_groups, get_kv_cache_groups

    groups = get_kv_cache_groups(vllm_config, deepcopy(specs))
    provisional = get_kv_cache_config_from_groups(vllm_config, groups, available)
    if provisional.num_blocks < 1:
        raise ValueError("No native cache blocks fit")
    return sum(t.size for t in provisional.kv_cache_tensors) // provisional.num_blocks


def _check_engine(cfg) -> None:
    if getattr(cfg.cache_config, "num_gpu_blocks_override", None) is not None:
        raise ValueError("num_gpu_blocks_override bypasses OSCAR memory budgeting")
    if getattr(cfg.parallel_config, "data_parallel_size", 1) != 1:
        raise ValueError("OSCAR manifest validation currently supports DP=1")
    if getattr(cfg.parallel_config, "pipeline_parallel_size", 1) != 1:
        raise ValueError("OSCAR memory accounting currently supports PP=1")


def bind_layers(ctx: dict, caches: dict) -> dict:
    """Cache set-up of every OSCAR and shadow layer; returns what was bound
    and the persistent bytes allocated."""
    import torch

    from .rotation import layer_index_from_name

    names, ids, shadows = [], [], []
    persistent = 0
    for name, module in ctx.items():
        impl = getattr(module, "impl", None)
        if impl is None:
            continue
        if is_shadow_impl(impl):
            pool = impl._shadow_kv(caches[name])
            persistent += sum(t.numel() * t.element_size() for t in pool)
            shadows.append(name)
        elif is_oscar_impl(impl):
            cache = caches[name]
            impl._set_caches(cache)
            if impl.key_cache.dtype != torch.int8:
                raise RuntimeError(f"OSCAR layer {name}: the engine allocated a {impl.key_cache.dtype} cache; start it "
                                   "with --kv-cache-dtype int8_per_token_head (packed INT2 slots of D bytes)")
            impl._layer_rvt(module, impl.key_cache.device)  # loads R_k / R_v and caches R_v^T
            persistent += rotation_bytes(impl)
            if impl._oscar.window_enabled:
                impl._ensure_staging(module, cache)
                persistent += sum(t.numel() * t.element_size() for t in (
                    module._oscar_stage_k, module._oscar_stage_v, module._oscar_slot_owner,
                    module._oscar_seat_winner))
            names.append(name)
            ids.append(layer_index_from_name(name))
    return {"layers": names, "layer_ids": ids, "shadow_layers": shadows, "persistent_bytes": persistent}


def ready_manifest(bound: dict, plan: dict, native_bytes: int, rank: int, world: int) -> dict:
    return {"rank": rank, "world_size": world, "layers": sorted(bound["layers"]),
            "layer_ids": sorted(bound["layer_ids"]), "shadow_layers": bound["shadow_layers"],
            "native_bytes": native_bytes, "persistent_bytes": bound["persistent_bytes"],
            "streaming_transient_bytes": plan["streaming_transient_bytes"], "source": str(PACKAGE),
            "sha256": source_fingerprint(), "verified": True}


def install_runner_hooks(worker_cls=None, runner_cls=None) -> None:
    """Wrap the worker's memory profile and the runner's cache set-up (once
    per class).  The classes default to vLLM-CUDA's Worker and GPUModelRunner."""
    if worker_cls is None:
        from vllm.v1.worker.gpu_worker import Worker as worker_cls
    if runner_cls is None:
        from vllm.v1.worker.gpu_model_runner import GPUModelRunner as runner_cls
    if getattr(worker_cls, "_oscar_memory_hook", False):
        return
    original_memory = worker_cls.determine_available_memory
    original_caches = runner_cls.initialize_kv_cache_tensors

    def determine_available_memory(worker):
        available = original_memory(worker)
        runner = worker.model_runner
        ctx = runner.compilation_config.static_forward_context
        if not any(is_oscar_impl(getattr(m, "impl", None)) for m in ctx.values()):
            return available
        cfg = runner.vllm_config
        _check_engine(cfg)
        specs = runner.get_kv_cache_spec()
        max_tokens = getattr(getattr(cfg, "scheduler_config", None), "max_num_batched_tokens", 0)
        plan = plan_memory(available, ctx, specs, _native_per_block(cfg, specs, available), max_tokens)
        runner._oscar_memory_plan = plan
        worker.available_kv_cache_memory_bytes = plan["budget"]
        print("[oscar-b200] MEMORY " + json.dumps(plan, sort_keys=True), flush=True)
        return plan["budget"]

    def initialize_kv_cache_tensors(runner, kv_cache_config, *args, **kwargs):
        caches = original_caches(runner, kv_cache_config, *args, **kwargs)
        ctx = runner.compilation_config.static_forward_context
        bound = bind_layers(ctx, caches)
        if bound["layers"]:
            plan = getattr(runner, "_oscar_memory_plan", None)
            if plan is None:
                raise RuntimeError("OSCAR caches set up without the OSCAR memory plan (profile hook not run)")
            native = sum(t.size for t in kv_cache_config.kv_cache_tensors)
            if native + bound["persistent_bytes"] + plan["streaming_transient_bytes"] > plan["available"]:
                raise RuntimeError("Actual OSCAR persistent allocation exceeds profiled budget")
            hf = runner.model_config.hf_text_config
            verify_layers(getattr(hf, "layer_types", []) or [], bound["layer_ids"])
            try:
                import torch.distributed as dist

                rank = dist.get_rank() if dist.is_initialized() else 0
            except Exception:
                rank = 0
            world = runner.vllm_config.parallel_config.tensor_parallel_size
            manifest = ready_manifest(bound, plan, native, rank, world)
            runner._oscar_manifest = manifest
            print("[oscar-b200] READY " + json.dumps(manifest, sort_keys=True), flush=True)
        return caches

    worker_cls.determine_available_memory = determine_available_memory
    runner_cls.initialize_kv_cache_tensors = initialize_kv_cache_tensors
    worker_cls._oscar_memory_hook = True
