"""Per-layer orthogonal rotations (checkpoint schema of oscar_ascend/rotation.py:1-129).

Accepted checkpoint forms: ``{"layers": {id: {"rotation": R, "rotation_v": Rv, ...}}}``,
``{id: R}`` / ``{id: {"rotation": R}}``, or a stacked ``[num_layers, D, D]``
tensor.  Keys may be ints, digit strings or vLLM layer names.  An empty path
or a missing layer gives the identity (unless ``strict``).
"""
from __future__ import annotations

import re
from functools import lru_cache

import torch

_LAYER_IDX_RE = re.compile(r"\.layers\.(\d+)\.")


def layer_index_from_name(layer_name: str) -> int | None:
    m = _LAYER_IDX_RE.search(layer_name)
    if m is not None:
        return int(m.group(1))
    ints = re.findall(r"\d+", layer_name)
    return int(ints[-1]) if ints else None


def _resolve_lid(key) -> int | None:
    if isinstance(key, int):
        return key
    if isinstance(key, str):
        try:
            return int(key)
        except ValueError:
            return layer_index_from_name(key)
    return None


def _tensors(entry: dict) -> dict:
    return {k: v.float().contiguous() for k, v in entry.items() if isinstance(v, torch.Tensor)}


@lru_cache(maxsize=8)
def _load_checkpoint(path: str) -> dict[int, dict[str, torch.Tensor]]:
    obj = torch.load(path, map_location="cpu", weights_only=False)
    if not (isinstance(obj, dict) and obj.get("format_version", 0) >= 2 and "r_h_pbr" in str(obj.get("objective", ""))):
        print(f"[oscar-b200] rotation checkpoint {path!r} is not a v2 (U@H@P_br) recipe; "
              "per-vector INT2 accuracy will suffer")
    out: dict[int, dict[str, torch.Tensor]] = {}
    if isinstance(obj, dict) and "layers" in obj:
        for k, entry in obj["layers"].items():
            lid = _resolve_lid(k)
            if lid is None:
                continue
            out[lid] = _tensors(entry) if isinstance(entry, dict) and "rotation" in entry else {
                "rotation": entry.float().contiguous()}
    elif isinstance(obj, dict):
        for k, rot in obj.items():
            lid = _resolve_lid(k)
            if lid is None or not (isinstance(rot, torch.Tensor) or isinstance(rot, dict)):
                continue
            out[lid] = _tensors(rot) if isinstance(rot, dict) and "rotation" in rot else {
                "rotation": rot.float().contiguous()}
    elif torch.is_tensor(obj) and obj.dim() == 3:
        for lid in range(obj.shape[0]):
            out[lid] = {"rotation": obj[lid].float().contiguous()}
    else:
        raise ValueError(f"Unrecognized OSCAR rotation checkpoint structure at {path!r}: {type(obj)}")
    return out


def get_layer_rotation(path: str, layer_name: str, head_dim: int, device, dtype=torch.float32,
                       mode: str = "k", strict: bool = False) -> torch.Tensor:
    """[D, D] rotation of one layer (rotation.py:93-129): mode "v" prefers
    ``rotation_v`` and falls back to ``rotation``."""
    if not path:
        return torch.eye(head_dim, device=device, dtype=dtype)
    table = _load_checkpoint(path)
    lid = layer_index_from_name(layer_name)
    entry = table.get(lid) if lid is not None else None
    if entry is None:
        if strict:
            raise ValueError(f"Rotation checkpoint {path!r} is missing layer {layer_name}")
        return torch.eye(head_dim, device=device, dtype=dtype)
    rot = entry.get("rotation_v") if mode == "v" else entry.get("rotation")
    if rot is None:
        rot = entry.get("rotation")
    if rot is None:
        return torch.eye(head_dim, device=device, dtype=dtype)
    if tuple(rot.shape) != (head_dim, head_dim):
        raise ValueError(f"OSCAR rotation for layer {lid} has shape {tuple(rot.shape)}, expected ({head_dim}, {head_dim}).")
    if strict and (not torch.isfinite(rot).all() or not torch.allclose(rot @ rot.t(), torch.eye(head_dim), atol=1e-3, rtol=1e-3)):
        raise ValueError(f"Rotation checkpoint {path!r} layer {lid} is not finite/orthogonal")
    return rot.to(device=device, dtype=dtype).contiguous()
