"""Plugin configuration from ``OSCAR_ASCEND_*`` environment variables.

Same keys, defaults and validation as oscar_ascend/config.py:35-103, so a
deployment switching to this package keeps its environment.  Keys that only
select Ascend code paths (USE_TRITON, USE_PAGED, FUSED_PREP) are parsed and
ignored: the B200 build has one device path.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

from .format import D_DEFAULT, LEVELS


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    if v is None or v.strip() == "":
        return default
    try:
        return int(v)
    except ValueError:
        return default


def _env_float(name: str, default: float) -> float:
    v = os.environ.get(name)
    if v is None or v.strip() == "":
        return default
    try:
        return float(v)
    except ValueError:
        return default


@dataclass
class OscarConfig:
    head_dim: int = D_DEFAULT
    key_quant_bits: int = 2
    value_quant_bits: int = 2
    k_clip_ratio: float = 0.0
    v_clip_ratio: float = 0.0
    k_rotation_path: str = ""
    v_rotation_path: str = ""
    sink_tokens: int = 64
    recent_tokens: int = 256
    staging_tokens: int = 8192
    group_size: int = 0
    window_enabled: bool = True
    attention_mode: str = "streaming"
    stream_workspace_bytes: int = 32 * 1024 * 1024
    verbose: bool = True
    extra: dict = field(default_factory=dict)

    @property
    def levels(self) -> int:
        return LEVELS

    @property
    def data_bytes(self) -> int:
        return (self.head_dim * self.key_quant_bits + 7) // 8

    @property
    def slot_bytes(self) -> int:
        return 160

    @property
    def num_groups(self) -> int:
        return 1 if self.group_size == 0 else -(-self.head_dim // self.group_size)

    @classmethod
    def from_env(cls, head_dim: int | None = None) -> OscarConfig:
        d = head_dim if head_dim is not None else _env_int("OSCAR_ASCEND_HEAD_DIM", D_DEFAULT)
        cfg = cls(
            head_dim=d,
            k_clip_ratio=_env_float("OSCAR_ASCEND_K_CLIP_RATIO", 0.0),
            v_clip_ratio=_env_float("OSCAR_ASCEND_V_CLIP_RATIO", 0.0),
            k_rotation_path=os.environ.get("OSCAR_ASCEND_K_ROTATION_PATH", ""),
            v_rotation_path=os.environ.get("OSCAR_ASCEND_V_ROTATION_PATH", ""),
            sink_tokens=max(0, _env_int("OSCAR_ASCEND_SINK_TOKENS", 64)),
            recent_tokens=max(0, _env_int("OSCAR_ASCEND_RECENT_TOKENS", 256)),
            staging_tokens=max(0, _env_int("OSCAR_ASCEND_STAGING_TOKENS", 8192)),
            group_size=_env_int("OSCAR_ASCEND_GROUP_SIZE", 0),
            verbose=os.environ.get("OSCAR_ASCEND_VERBOSE", "1") != "0",
        )
        cfg.window_enabled = cfg.staging_tokens > 0 and (cfg.sink_tokens > 0 or cfg.recent_tokens > 0)
        cfg.attention_mode = os.environ.get("OSCAR_ASCEND_ATTENTION_MODE", "streaming")
        cfg.stream_workspace_bytes = max(0, _env_int("OSCAR_ASCEND_STREAM_WORKSPACE_MIB", 32)) * 1024 * 1024
        if cfg.attention_mode not in ("streaming", "native"):
            raise ValueError("OSCAR_ASCEND_ATTENTION_MODE must be streaming or native")
        if not all(0 <= r <= 1 for r in (cfg.k_clip_ratio, cfg.v_clip_ratio)):
            raise ValueError("OSCAR clip ratios must be finite and in [0, 1]")
        if cfg.group_size != 0:
            raise ValueError("Only per-vector OSCAR quantization (GROUP_SIZE=0) is supported")
        cfg.extra["enable"] = os.environ.get("OSCAR_ASCEND_ENABLE", "auto")
        return cfg


# the reference's class name, for code that imports it by name
OscarAscendConfig = OscarConfig
