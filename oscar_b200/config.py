"""Plugin configuration read from ``OSCAR_ASCEND_*`` environment variables.

The keys, their defaults and the validation messages are the reference
plugin's configuration interface (oscar_ascend/config.py:35-103), kept so that
a deployment switching to this package keeps its environment.  The parsing is
driven by one table, ``SETTINGS``: each row names the attribute, the
environment key (without the ``OSCAR_ASCEND_`` prefix), how the raw string is
read and the default.  Keys that only pick Ascend code paths
(``USE_TRITON``, ``USE_PAGED``, ``FUSED_PREP``) have no row: this build has
one device path.

Two deliberate differences from the reference:
  * ``ATTENTION_MODE=native`` (the reference's legacy dense / paged read path,
    oscar_ascend/backend.py:281) is rejected with a message instead of being
    accepted, because this build only has the streaming path;
  * ``STREAM_WORKSPACE_MIB`` defaults to 128 instead of 32: the attention
    workspace also holds the continuation pre-pass tiles (about 101 MB for a
    15360-token chunk on 9256 tokens of history at 4 KV heads), and below that
    bound long continuations fall back to per-CTA dequantisation.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Callable, Mapping

from .format import D_DEFAULT, LEVELS

PREFIX = "OSCAR_ASCEND_"
MIB = 1024 * 1024


def _number(kind: type) -> Callable[[str | None, object], object]:
    """A reader for int / float keys: unset, blank or unparsable -> default."""

    def read(raw: str | None, default):
        if raw is None or not raw.strip():
            return default
        try:
            return kind(raw)
        except ValueError:
            return default

    return read


def _text(raw: str | None, default):
    return default if raw is None else raw


def _on_unless_zero(raw: str | None, default):
    return default if raw is None else raw != "0"


_int, _float = _number(int), _number(float)


def _at_least_zero(x):
    return max(0, x)


# attribute, key suffix, reader, default, post-processing of the read value
SETTINGS: tuple[tuple[str, str, Callable, object, Callable | None], ...] = (
    ("k_clip_ratio", "K_CLIP_RATIO", _float, 0.0, None),
    ("v_clip_ratio", "V_CLIP_RATIO", _float, 0.0, None),
    ("k_rotation_path", "K_ROTATION_PATH", _text, "", None),
    ("v_rotation_path", "V_ROTATION_PATH", _text, "", None),
    ("sink_tokens", "SINK_TOKENS", _int, 64, _at_least_zero),
    ("recent_tokens", "RECENT_TOKENS", _int, 256, _at_least_zero),
    ("staging_tokens", "STAGING_TOKENS", _int, 8192, _at_least_zero),
    ("group_size", "GROUP_SIZE", _int, 0, None),
    ("verbose", "VERBOSE", _on_unless_zero, True, None),
    ("attention_mode", "ATTENTION_MODE", _text, "streaming", None),
    ("stream_workspace_bytes", "STREAM_WORKSPACE_MIB", _int, 128, lambda mib: max(0, mib) * MIB),
)


@dataclass
class OscarConfig:
    """The settings of one OSCAR attention impl (attributes as the reference's)."""

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
    stream_workspace_bytes: int = 128 * MIB
    verbose: bool = True
    extra: dict = field(default_factory=dict)

    # -- derived geometry
    @property
    def levels(self) -> int:
        return LEVELS

    @property
    def data_bytes(self) -> int:
        """Packed code bytes of one vector."""
        return (self.head_dim * self.key_quant_bits + 7) // 8

    @property
    def slot_bytes(self) -> int:
        """Logical slot: K slot bytes [0, 96) + V slot bytes [0, 64)."""
        return 160

    @property
    def num_groups(self) -> int:
        return 1 if self.group_size == 0 else -(-self.head_dim // self.group_size)

    def window_on(self) -> bool:
        """The fp32 staging window is used when it has seats and something to keep."""
        return self.staging_tokens > 0 and (self.sink_tokens > 0 or self.recent_tokens > 0)

    def validate(self) -> None:
        if self.attention_mode == "native":
            raise ValueError("OSCAR_ASCEND_ATTENTION_MODE=native (the legacy dense/paged read path) is not provided "
                             "on B200: only streaming is")
        if self.attention_mode != "streaming":
            raise ValueError("OSCAR_ASCEND_ATTENTION_MODE must be streaming or native")
        if not all(0 <= r <= 1 for r in (self.k_clip_ratio, self.v_clip_ratio)):
            raise ValueError("OSCAR clip ratios must be finite and in [0, 1]")
        if self.group_size != 0:
            raise ValueError("Only per-vector OSCAR quantization (GROUP_SIZE=0) is supported")

    @classmethod
    def from_env(cls, head_dim: int | None = None, environ: Mapping[str, str] | None = None) -> OscarConfig:
        env = os.environ if environ is None else environ
        values = {}
        for attr, key, read, default, post in SETTINGS:
            value = read(env.get(PREFIX + key), default)
            values[attr] = post(value) if post is not None else value
        if head_dim is None:
            head_dim = _int(env.get(PREFIX + "HEAD_DIM"), D_DEFAULT)
        cfg = cls(head_dim=head_dim, **values)
        cfg.window_enabled = cfg.window_on()
        cfg.extra["enable"] = env.get(PREFIX + "ENABLE", "auto")
        cfg.validate()
        return cfg


# the reference's class name, for code that imports it by name
OscarAscendConfig = OscarConfig
