"""The plugin against the installed vLLM (0.22), on the CPU: real ``Attention``
layers built under ``load_plugin()`` with the engine's int8 KV dtype
(``int8_per_token_head``), then both worker seams of oscar_b200.integration
(memory budget, cache set-up + READY manifest) and the MTP draft layer's bf16
shadow pool on the int8 pool (oscar_ascend/integration.py:77-245,
mtp_shadow.py:29-61)."""
import json
from types import SimpleNamespace as NS

import pytest
import torch

vllm = pytest.importorskip("vllm")

FULL = "model.layers.3.self_attn.attn"
MTP = "model.mtp.layers.0.self_attn.attn"
LAYER_TYPES = ["linear_attention", "linear_attention", "linear_attention", "full_attention"]


@pytest.fixture
def engine(monkeypatch):
    """A CPU VllmConfig of a hybrid model with an int8 KV pool, the plugin
    loaded, and vLLM's classes restored afterwards."""
    from vllm.config import CacheConfig, DeviceConfig, VllmConfig
    from vllm.model_executor.layers.attention.attention import Attention
    from vllm.v1.worker.gpu_model_runner import GPUModelRunner
    from vllm.v1.worker.gpu_worker import Worker

    from oscar_b200 import plugin

    saved = (Attention.__init__, Worker.determine_available_memory, GPUModelRunner.initialize_kv_cache_tensors,
             plugin._PATCHED)
    monkeypatch.setenv("OSCAR_ASCEND_PACKED", "1")
    monkeypatch.setenv("OSCAR_ASCEND_SINK_TOKENS", "128")
    monkeypatch.setenv("OSCAR_ASCEND_STAGING_TOKENS", "1024")
    monkeypatch.setenv("OSCAR_ASCEND_VERBOSE", "0")
    cache = CacheConfig(cache_dtype="int8_per_token_head", block_size=128)
    cfg = VllmConfig(device_config=DeviceConfig(device="cpu"), cache_config=cache)
    model = NS(is_hybrid=True, is_mm_prefix_lm=False, hf_text_config=NS(layer_types=LAYER_TYPES),
               dtype=torch.bfloat16, use_mla=False)
    object.__setattr__(cfg, "model_config", model)
    plugin._PATCHED = False
    plugin.load_plugin()
    yield NS(cfg=cfg, cache=cache, model=model, Attention=Attention, Worker=Worker, Runner=GPUModelRunner)
    Attention.__init__, Worker.determine_available_memory, GPUModelRunner.initialize_kv_cache_tensors = saved[:3]
    plugin._PATCHED = saved[3]
    if "_oscar_memory_hook" in Worker.__dict__:
        delattr(Worker, "_oscar_memory_hook")


def build_layers(engine):
    from vllm.config import set_current_vllm_config
    from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend

    with set_current_vllm_config(engine.cfg):
        full = engine.Attention(num_heads=6, head_size=256, scale=1 / 16, num_kv_heads=1, prefix=FULL,
                                cache_config=engine.cache, attn_backend=TritonAttentionBackend)
        mtp = engine.Attention(num_heads=6, head_size=256, scale=1 / 16, num_kv_heads=1, prefix=MTP,
                               cache_config=engine.cache, attn_backend=TritonAttentionBackend)
    return {FULL: full, MTP: mtp}


def fake_worker_classes(engine, ctx, available):
    """Stand-ins for the profiling worker and the runner: profiling returns
    `available`; cache set-up allocates int8 pools as vLLM's does for the
    Triton backend ([2, blocks, block_size, Hk, D])."""

    class Runner:
        def __init__(self):
            self.compilation_config = NS(static_forward_context=ctx)
            self.vllm_config = engine.cfg
            self.model_config = engine.model

        def get_kv_cache_spec(self):
            return {name: m.get_kv_cache_spec(engine.cfg) for name, m in ctx.items()}

        def initialize_kv_cache_tensors(self, kv_cache_config, kernel_block_sizes):
            out = {}
            for t in kv_cache_config.kv_cache_tensors:
                for name in t.shared_by:
                    spec = self.get_kv_cache_spec()[name]
                    blocks = t.size // spec.page_size_bytes
                    out[name] = torch.zeros(2, blocks, spec.block_size, spec.num_kv_heads, spec.head_size,
                                            dtype=spec.dtype)
            return out

    class Worker:
        def __init__(self):
            self.model_runner = Runner()

        def determine_available_memory(self):
            return available

    return Worker, Runner


def test_plugin_swaps_real_attention_impls(engine):
    from oscar_b200.backend import OscarAttentionImplMixin
    from oscar_b200.mtp_shadow import MTPShadowMixin

    layers = build_layers(engine)
    assert isinstance(layers[FULL].impl, OscarAttentionImplMixin)
    assert layers[FULL].impl._oscar.sink_tokens == 128
    assert isinstance(layers[MTP].impl, MTPShadowMixin)
    assert not isinstance(layers[MTP].impl, OscarAttentionImplMixin)
    # the engine's own worker classes carry the seams once an OSCAR layer exists
    assert getattr(engine.Worker, "_oscar_memory_hook", False)
    spec = layers[FULL].get_kv_cache_spec(engine.cfg)
    assert spec.dtype == torch.int8 and spec.head_size == 256  # D bytes per packed K / V slot


def test_memory_seam_and_ready_manifest(engine, capsys):
    from vllm.v1.core.kv_cache_utils import get_kv_cache_config_from_groups, get_kv_cache_groups

    from oscar_b200 import integration

    layers = build_layers(engine)
    available = 1 << 30
    Worker, Runner = fake_worker_classes(engine, layers, available)
    integration.install_runner_hooks(Worker, Runner)
    worker = Worker()
    budget = worker.determine_available_memory()
    plan = worker.model_runner._oscar_memory_plan
    specs = worker.model_runner.get_kv_cache_spec()
    full_impl = layers[FULL].impl
    rows = integration.staging_rows(full_impl._oscar, 128)
    staging = rows * 128 * (2 * 1 * 256 * 4 + 16)
    rot = 3 * 256 * 256 * 4
    transient = full_impl._oscar.stream_workspace_bytes + 2048 * (1 * 256 * 2 * 6 + 6 * 256 * 6 + 6 * 4)
    assert plan["streaming_transient_bytes"] == transient
    assert plan["fixed"] == rot + staging + transient
    assert plan["shadow"] == 128 * 1 * 512 * 2  # the MTP layer's bf16 K and V per block
    assert budget == plan["budget"] and budget % plan["native"] == 0
    assert budget // plan["native"] == (available - plan["fixed"]) // (plan["native"] + plan["shadow"])
    assert worker.available_kv_cache_memory_bytes == budget
    assert "[oscar-b200] MEMORY" in capsys.readouterr().out

    groups = get_kv_cache_groups(engine.cfg, specs)
    kv_config = get_kv_cache_config_from_groups(engine.cfg, groups, budget)
    caches = worker.model_runner.initialize_kv_cache_tensors(kv_config, [128])
    impl = full_impl
    assert impl.key_cache.dtype == torch.int8 and impl.key_cache.shape[1:] == (128, 1, 256)
    assert impl.key_cache.data_ptr() == caches[FULL][0].data_ptr()
    assert layers[FULL]._oscar_stage_k.shape == (rows, 128, 1, 256)
    shadow = layers[MTP].impl._oscar_shadow_kv
    assert shadow.dtype == torch.bfloat16 and shadow.shape == caches[MTP].shape
    out = capsys.readouterr().out
    line = next(ln for ln in out.splitlines() if ln.startswith("[oscar-b200] READY "))
    manifest = json.loads(line[len("[oscar-b200] READY "):])
    assert manifest["layers"] == [FULL] and manifest["layer_ids"] == [3] and manifest["shadow_layers"] == [MTP]
    assert manifest["verified"] and len(manifest["sha256"]) == 64
    assert manifest["persistent_bytes"] == rot + staging + shadow.numel() * 2


def test_cache_seam_rejects_a_bf16_pool_and_missing_layers(engine):
    from oscar_b200 import integration

    layers = build_layers(engine)
    Worker, Runner = fake_worker_classes(engine, layers, 1 << 30)
    with pytest.raises(RuntimeError, match="int8_per_token_head"):
        integration.bind_layers({FULL: layers[FULL]}, {FULL: torch.zeros(2, 4, 128, 1, 256, dtype=torch.bfloat16)})
    with pytest.raises(RuntimeError, match="Incomplete OSCAR layers"):
        integration.verify_layers(LAYER_TYPES + ["full_attention"], [3])
    with pytest.raises(ValueError, match="Insufficient memory"):
        integration.memory_budget(100, 10, 0, 100)


def test_mtp_shadow_pool_on_the_int8_pool(engine, monkeypatch):
    """The draft layer's framework attention sees the bf16 shadow pool, never
    the int8 pool (mtp_shadow.py:29-61)."""
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl

    layers = build_layers(engine)
    seen = []
    monkeypatch.setattr(TritonAttentionImpl, "do_kv_cache_update",
                        lambda self, layer, key, value, kv_cache, slot_mapping: seen.append(("update", kv_cache)))
    monkeypatch.setattr(TritonAttentionImpl, "forward",
                        lambda self, layer, q, k, v, kv_cache, md, *a, **kw: seen.append(("forward", kv_cache)))
    impl = layers[MTP].impl
    pool = torch.zeros(2, 4, 128, 1, 256, dtype=torch.int8)
    q = torch.zeros(2, 6 * 256, dtype=torch.bfloat16)
    k = torch.zeros(2, 256, dtype=torch.bfloat16)
    impl.do_kv_cache_update(layers[MTP], k, k, pool, torch.tensor([0, 1]))
    impl.forward(layers[MTP], q, k, k, pool, None, output=q)
    assert [s[0] for s in seen] == ["update", "forward"]
    for _, kv in seen:
        assert kv.dtype == torch.bfloat16 and kv.shape == pool.shape
    assert seen[0][1] is seen[1][1]  # one pool, allocated once
