"""Per-layer orthogonal rotations from a checkpoint.

The checkpoint schema is the reference's file format (oscar_ascend/rotation.py:1-129)
and is kept as is, so existing calibration outputs load unchanged:

  * ``{"layers": {key: {"rotation": R, "rotation_v": Rv, ...}}}`` or
    ``{"layers": {key: R}}``;
  * ``{key: R}`` or ``{key: {"rotation": R, ...}}`` (other top-level entries,
    such as ``format_version`` / ``objective``, are metadata);
  * a stacked ``[num_layers, D, D]`` tensor.

A key is an int, a digit string or a vLLM layer name.  Loading turns any of
these forms into one normal form, ``{layer index: {name: fp32 tensor}}``
(``RotationTable``), cached per path; ``get_layer_rotation`` is a single
lookup in it.  An empty path or a missing layer gives the identity unless
``strict`` asks for an error.
"""
from __future__ import annotations

import re
from functools import lru_cache

import torch

_LAYERS_SEGMENT = re.compile(r"\.layers\.(\d+)\.")
_DIGITS = re.compile(r"\d+")


def layer_index_from_name(layer_name: str) -> int | None:
    """Decoder layer index of a vLLM layer name: the ``.layers.N.`` segment,
    else the last integer in the name, else None."""
    seg = _LAYERS_SEGMENT.search(layer_name)
    if seg is not None:
        return int(seg.group(1))
    found = _DIGITS.findall(layer_name)
    return int(found[-1]) if found else None


def _key_index(key) -> int | None:
    if isinstance(key, int):
        return key
    if isinstance(key, str):
        return int(key) if key.isdigit() else layer_index_from_name(key)
    return None


def _entry(value) -> dict[str, torch.Tensor] | None:
    """One layer's tensors: a bare matrix is its ``rotation``."""
    if isinstance(value, torch.Tensor):
        return {"rotation": value.float().contiguous()}
    if isinstance(value, dict) and "rotation" in value:
        return {name: t.float().contiguous() for name, t in value.items() if isinstance(t, torch.Tensor)}
    return None


class RotationTable:
    """A checkpoint in normal form: ``layers[index] = {"rotation": R, ...}``."""

    def __init__(self, obj, origin: str = "<memory>"):
        self.origin = origin
        self.layers: dict[int, dict[str, torch.Tensor]] = {}
        if isinstance(obj, torch.Tensor):
            if obj.dim() != 3:
                raise ValueError(f"Unrecognized OSCAR rotation checkpoint structure at {origin!r}: {type(obj)}")
            self.layers = {i: {"rotation": obj[i].float().contiguous()} for i in range(obj.shape[0])}
            return
        if not isinstance(obj, dict):
            raise ValueError(f"Unrecognized OSCAR rotation checkpoint structure at {origin!r}: {type(obj)}")
        body = obj["layers"] if "layers" in obj else obj
        for key, value in body.items():
            idx, tensors = _key_index(key), _entry(value)
            if idx is not None and tensors is not None:
                self.layers[idx] = tensors

    @staticmethod
    def is_v2_recipe(obj) -> bool:
        """Calibrations that compose U @ H @ P_br record it (format_version >= 2)."""
        return isinstance(obj, dict) and obj.get("format_version", 0) >= 2 and "r_h_pbr" in str(obj.get("objective", ""))

    def lookup(self, layer_name: str, mode: str) -> tuple[int | None, torch.Tensor | None, bool]:
        """(layer index, matrix or None, layer present).  Mode "v" prefers
        ``rotation_v`` and falls back to ``rotation``."""
        idx = layer_index_from_name(layer_name)
        entry = self.layers.get(idx) if idx is not None else None
        if entry is None:
            return idx, None, False
        names = ("rotation_v", "rotation") if mode == "v" else ("rotation",)
        return idx, next((entry[n] for n in names if entry.get(n) is not None), None), True


@lru_cache(maxsize=8)
def load_table(path: str) -> RotationTable:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    if not RotationTable.is_v2_recipe(obj):
        print(f"[oscar-b200] rotation checkpoint {path!r} does not record the v2 (U@H@P_br) calibration recipe; "
              "per-vector INT2 accuracy will be much worse -- re-run the calibration")
    return RotationTable(obj, path)


def get_layer_rotation(path: str, layer_name: str, head_dim: int, device, dtype=torch.float32, mode: str = "k",
                       strict: bool = False) -> torch.Tensor:
    """The ``[D, D]`` rotation of one layer (contiguous, on ``device``)."""
    eye = torch.eye(head_dim, device=device, dtype=dtype)
    if not path:
        return eye
    idx, rot, present = load_table(path).lookup(layer_name, mode)
    if not present and strict:
        raise ValueError(f"Rotation checkpoint {path!r} is missing layer {layer_name}")
    if rot is None:
        return eye
    if tuple(rot.shape) != (head_dim, head_dim):
        raise ValueError(f"OSCAR rotation for layer {idx} has shape {tuple(rot.shape)}, expected ({head_dim}, {head_dim}).")
    if strict:
        orthogonal = torch.allclose(rot @ rot.t(), torch.eye(head_dim), atol=1e-3, rtol=1e-3)
        if not (torch.isfinite(rot).all() and orthogonal):
            raise ValueError(f"Rotation checkpoint {path!r} layer {idx} is not finite/orthogonal")
    return rot.to(device=device, dtype=dtype).contiguous()
