"""Host-side logic (no GPU): configuration, rotation checkpoints, plugin class
surgery and selection, metadata handling -- the reference's own unit tests
for these pieces (tests/test_backend.py, tests/test_numeric.py) restated."""
import os
from types import SimpleNamespace as NS

import pytest
import torch

from oscar_b200 import config, format as fmt, plugin
from oscar_b200.backend import OscarAttentionBackendImpl, OscarAttentionImplMixin, block_table_of, metadata_batch_lists
from oscar_b200.mtp_shadow import MTPShadowMixin, shadow_impl_class
from oscar_b200.rotation import get_layer_rotation, layer_index_from_name
from oscar_b200.synthetic import BASELINE_CONFIGS, make_case


def test_config_defaults_and_validation(monkeypatch):
    for k in list(os.environ):
        if k.startswith("OSCAR_ASCEND_"):
            monkeypatch.delenv(k)
    cfg = config.OscarConfig.from_env()
    assert (cfg.sink_tokens, cfg.recent_tokens, cfg.staging_tokens) == (64, 256, 8192)
    assert cfg.attention_mode == "streaming" and cfg.window_enabled
    # 128 MiB (the reference's 32 would push long continuations off the pre-pass path)
    assert cfg.stream_workspace_bytes == 128 * 1024 * 1024
    assert config.OscarConfig.from_env(environ={"OSCAR_ASCEND_STREAM_WORKSPACE_MIB": "32"}).stream_workspace_bytes \
        == 32 * 1024 * 1024
    # blank / unparsable numbers keep the default, negative counts clamp to 0
    odd = config.OscarConfig.from_env(environ={"OSCAR_ASCEND_SINK_TOKENS": " ", "OSCAR_ASCEND_RECENT_TOKENS": "x",
                                               "OSCAR_ASCEND_STAGING_TOKENS": "-5"})
    assert (odd.sink_tokens, odd.recent_tokens, odd.staging_tokens, odd.window_enabled) == (64, 256, 0, False)
    with pytest.raises(ValueError, match="native"):
        config.OscarConfig.from_env(environ={"OSCAR_ASCEND_ATTENTION_MODE": "native"})
    with pytest.raises(ValueError, match="streaming or native"):
        config.OscarConfig.from_env(environ={"OSCAR_ASCEND_ATTENTION_MODE": "dense"})
    monkeypatch.setenv("OSCAR_ASCEND_K_CLIP_RATIO", "1.5")
    with pytest.raises(ValueError, match="clip ratios"):
        config.OscarConfig.from_env()
    monkeypatch.setenv("OSCAR_ASCEND_K_CLIP_RATIO", "0.96")
    monkeypatch.setenv("OSCAR_ASCEND_GROUP_SIZE", "32")
    with pytest.raises(ValueError, match="per-vector"):
        config.OscarConfig.from_env()
    monkeypatch.setenv("OSCAR_ASCEND_GROUP_SIZE", "0")
    monkeypatch.setenv("OSCAR_ASCEND_STAGING_TOKENS", "0")
    assert not config.OscarConfig.from_env().window_enabled


def test_check_d_matches_reference_limits():
    fmt.check_d(256)
    fmt.check_d(32)
    with pytest.raises(ValueError):
        fmt.check_d(258)
    with pytest.raises(ValueError):
        fmt.check_d(260)
    assert fmt.slot_bytes_needed(256) == (96, 64)


def test_rotation_loader_schema(tmp_path):
    """tests/test_numeric.py:160-182 known answers."""
    d = 32
    r1, r2 = torch.eye(d), torch.eye(d) * 2
    p = tmp_path / "rot.pt"
    torch.save({"layers": {"3": {"layer_id": 3, "rotation": r1, "rotation_v": r2}}}, p)
    rk = get_layer_rotation(str(p), "model.layers.3.self_attn", d, torch.device("cpu"))
    rv = get_layer_rotation(str(p), "model.layers.3.self_attn", d, torch.device("cpu"), mode="v")
    assert torch.equal(rk, r1) and torch.equal(rv, r2)
    assert torch.equal(get_layer_rotation(str(p), "model.layers.9.self_attn", d, torch.device("cpu")), torch.eye(d))
    assert torch.equal(get_layer_rotation("", "x", d, torch.device("cpu")), torch.eye(d))
    with pytest.raises(ValueError, match="missing layer"):
        get_layer_rotation(str(p), "model.layers.9.self_attn", d, torch.device("cpu"), strict=True)
    stacked = tmp_path / "stack.pt"
    torch.save(torch.stack([torch.eye(d), -torch.eye(d)]), stacked)
    assert torch.equal(get_layer_rotation(str(stacked), "model.layers.1.attn", d, torch.device("cpu")), -torch.eye(d))
    assert layer_index_from_name("language_model.model.layers.11.self_attn.attn") == 11


def test_failed_surgery_restores_class_and_state():
    """tests/test_backend.py:137-150."""

    class Original:
        pass

    class Broken(Original):
        def _oscar_setup(self):
            self.partial = True
            raise ValueError("unsupported")

    impl = Original()
    impl.keep = 123
    with pytest.raises(ValueError):
        plugin.install_impl(impl, Broken)
    assert type(impl) is Original and vars(impl) == {"keep": 123}


def test_surgery_puts_oscar_paths_in_front_of_the_native_impl():
    class NativeImpl:
        def __init__(self):
            self.num_heads, self.num_kv_heads, self.head_size, self.scale = 6, 1, 256, 0.0625

        def forward(self, *a, **k):
            return "native"

        def do_kv_cache_update(self, *a):
            return "native-update"

    impl = NativeImpl()
    cls = plugin.oscar_impl_class(NativeImpl)
    assert plugin.oscar_impl_class(NativeImpl) is cls and plugin.oscar_impl_class(cls) is cls
    plugin.install_impl(impl, cls)
    assert isinstance(impl, NativeImpl) and isinstance(impl, OscarAttentionImplMixin)
    assert type(impl).forward is OscarAttentionImplMixin.forward
    assert impl._oscar.head_dim == 256
    bad = NativeImpl()
    bad.num_kv_heads = 4
    with pytest.raises(ValueError, match="divisible"):
        plugin.install_impl(bad, cls)
    assert type(bad) is NativeImpl


def test_hybrid_detection():
    """tests/test_numeric.py:218-244."""
    mc = NS(is_hybrid=False, hf_text_config=NS(layer_types=["linear_attention", "attention"]))
    assert plugin._is_hybrid_config(mc) is True
    assert plugin._is_hybrid_config(NS(is_hybrid=False, hf_text_config=NS(layer_types=["attention"]))) is False
    assert plugin._is_hybrid_config(NS(is_hybrid=True, hf_text_config=None)) is True


def test_should_oscar_selection():
    hybrid = NS(is_hybrid=True)

    class AT(str):
        @property
        def value(self):
            return str(self)

    impl = NS(attn_type=AT("decoder"), sliding_window=None, sinks=None)
    assert plugin._should_oscar(NS(layer_name="model.layers.3.self_attn.attn"), impl, hybrid)
    assert not plugin._should_oscar(NS(layer_name="model.mtp.layers.0.attn"), impl, hybrid)
    assert not plugin._should_oscar(NS(layer_name="x"), NS(attn_type="decoder", sliding_window=128, sinks=None), hybrid)
    assert not plugin._should_oscar(NS(layer_name="x"), NS(attn_type="encoder", sliding_window=None, sinks=None), hybrid)
    assert not plugin._should_oscar(NS(layer_name="x"), impl, NS(is_hybrid=False, hf_text_config=None))


def test_host_metadata_does_not_read_device_query_starts():
    """tests/test_backend.py:109-116."""

    class NoRead:
        def tolist(self):
            raise AssertionError("unexpected device sync")

    md = NS(query_start_loc=NoRead(), actual_seq_lengths_q=[1, 2], seq_lens_list=[9, 12], seq_lens=NoRead())
    assert metadata_batch_lists(md) == ([0, 1, 2], [9, 12])
    md = NS(query_start_loc_cpu=torch.tensor([0, 3]), seq_lens_cpu=torch.tensor([7]))
    assert metadata_batch_lists(md) == ([0, 3], [7])
    assert block_table_of(NS(block_table=torch.zeros(1, 2))).shape == (1, 2)
    assert block_table_of(NS(block_tables=torch.ones(1, 3), block_table=None)).shape == (1, 3)


def test_impl_geometry_check_accepts_packed_and_legacy_and_rejects_others():
    impl = OscarAttentionBackendImpl.create(6, 1, 256)
    impl._set_caches(torch.zeros(2, 4, 16, 1, 256, dtype=torch.int8))
    impl2 = OscarAttentionBackendImpl.create(6, 1, 256)
    impl2._set_caches([torch.zeros(4, 16, 1, 256, dtype=torch.bfloat16)] * 2)
    impl3 = OscarAttentionBackendImpl.create(6, 1, 256)
    with pytest.raises(ValueError, match="geometry"):
        impl3._set_caches([torch.zeros(4, 16, 1, 256, dtype=torch.float32)] * 2)


def test_forward_contract_without_gpu():
    impl = OscarAttentionBackendImpl.create(6, 1, 64)
    out = torch.ones(2, 6 * 64)
    assert torch.count_nonzero(impl.forward(None, torch.zeros(2, 6, 64), None, None, None, None, output=out)) == 0
    with pytest.raises(ValueError, match="Output tensor"):
        impl.forward(None, torch.zeros(2, 6, 64), None, None, None, NS())
    with pytest.raises(NotImplementedError):
        impl.forward(None, torch.zeros(2, 6, 64), None, None, None, NS(), output=out, output_scale=torch.ones(1))


def test_kernels_refuse_cpu_tensors():
    from oscar_b200 import kernels

    case = make_case([5], [2], d=64, bs=4, window=False)
    with pytest.raises(ValueError, match="CUDA"):
        kernels.slab_attention(*case.args())
    with pytest.raises(ValueError, match="CUDA"):
        kernels.oscar_store(case.old_k, case.old_v, case.kc, case.vc, case.slots)


def test_shadow_pool_class_surgery():
    class Native:
        def forward(self, layer, q, k, v, kv_cache, md, *a, **kw):
            return kv_cache

        def do_kv_cache_update(self, layer, k, v, kv_cache, slots):
            return kv_cache

    cls = shadow_impl_class(Native)
    assert issubclass(cls, MTPShadowMixin) and shadow_impl_class(cls) is cls
    impl = cls()
    int8_pool = torch.zeros(2, 3, 4, 1, 8, dtype=torch.int8)
    shadow = impl.forward(None, None, None, None, int8_pool, None)
    assert shadow.dtype == torch.bfloat16 and shadow.shape == int8_pool.shape
    assert impl.do_kv_cache_update(None, None, None, int8_pool, None) is shadow
    bf16_pool = torch.zeros(2, 3, 4, 1, 8, dtype=torch.bfloat16)
    assert cls().forward(None, None, None, None, bf16_pool, None) is bf16_pool


def test_synthetic_case_shapes_follow_probe_make_case():
    case = make_case([300, 0], [4, 3], hk=2, d=64, bs=16)
    assert case.q.shape == (7, 12, 64) and case.k_new.shape == (7, 2, 64)
    assert case.qsl == [0, 4, 7] and case.seqs == [304, 3]
    sk, sv, owner = case.stage
    hits = int((owner >= 0).sum())
    assert hits > 0 and sk.shape[1:] == (16, 2, 64)
    assert set(BASELINE_CONFIGS) == {"cfg1_mtp_8k", "cfg2_mtp_24k", "cfg3_mtp_8x24k", "cfg4_continuation", "cfg5_mixed_64"}
    lengths = BASELINE_CONFIGS["cfg5_mixed_64"]["prefixes"]
    assert len(lengths) == 64 and min(lengths) >= 1024 and max(lengths) <= 32768


def test_graph_wrappers_reject_host_tensors_and_empty_sequences():
    """CUDA-graph wrappers need device tensors; a sequence needs a forward."""
    import torch

    from oscar_b200.graphs import GraphedForward, GraphedSequence

    q = torch.zeros(1, 6, 256)
    with pytest.raises(ValueError):
        GraphedSequence([])
    with pytest.raises(ValueError):
        GraphedSequence([(None, None, q, q, q, None, None, q)])
    with pytest.raises(ValueError):
        GraphedForward(None, None, q, q, q, None, None, q)
