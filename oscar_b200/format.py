"""INT2 slot-format constants and geometry checks (oscar_ascend/format.py:19-45).

The numeric contract itself (per-vector asymmetric INT2, fp16-rounded
scale/zero, floor(x + 0.5), low index in low bits, little-endian fp16 meta)
is implemented on the device by ``csrc/store.cuh`` and checked bit-exactly
against the reference in the tests; the host only needs the layout.
"""
from __future__ import annotations

BITS = 2
LEVELS = 4
VALUES_PER_BYTE = 4
D_DEFAULT = 256
DATA_BYTES = D_DEFAULT // VALUES_PER_BYTE

SLOT_SIZE = 160            # logical slot = K slot [0:96] + V slot [0:64]
K_META_OFF = 0             # [0:2] K scale | [2:4] K zero | [4:6] V scale | [6:8] V zero
META_BYTES = 8
PAD_BYTES = 24             # [8:32], never written
K_IDX_OFF = 32             # [32:32+D/4] K codes
V_IDX_OFF = 96             # logical offset of the V codes (= V slot offset 0)
K_SLOT_BYTES = V_IDX_OFF
V_SLOT_BYTES = SLOT_SIZE - V_IDX_OFF

SCALE_FLOOR = 2.0**-14


def check_d(d: int) -> None:
    """format.check_d (format.py:41-45)."""
    if d % VALUES_PER_BYTE != 0:
        raise ValueError(f"D={d} must be divisible by {VALUES_PER_BYTE} (INT2 packing)")
    if d // VALUES_PER_BYTE > K_SLOT_BYTES - META_BYTES - PAD_BYTES:
        raise ValueError(f"D={d} exceeds the slot capacity")


def slot_bytes_needed(d: int) -> tuple[int, int]:
    """Bytes of the K and V slots the packed layout occupies for head dim d."""
    check_d(d)
    return K_IDX_OFF + d // VALUES_PER_BYTE, d // VALUES_PER_BYTE


__all__ = [
    "BITS", "LEVELS", "VALUES_PER_BYTE", "D_DEFAULT", "DATA_BYTES", "SLOT_SIZE", "K_META_OFF",
    "META_BYTES", "PAD_BYTES", "K_IDX_OFF", "V_IDX_OFF", "K_SLOT_BYTES", "V_SLOT_BYTES",
    "SCALE_FLOOR", "check_d", "slot_bytes_needed",
]
