"""Startup loading of OSCAR's calibrated K/V rotation files.

Same file format and checks as the reference (``oscar_ascend/rotations.py:7-53``):
a ``.pt`` holding ``{"layers": {idx: {"rotation": [256,256]}}}``, ``{idx: tensor}`` or a
``[L, 256, 256]`` tensor; a missing layer, wrong dimension, non-finite or non-orthogonal
matrix (fp32 check, atol/rtol 0.015) is an error, never a silent identity.
"""

from __future__ import annotations

import re
from functools import lru_cache


def layer_index(name: str) -> int:
    """Global decoder layer index from a module name like ``model.layers.3.self_attn.attn``."""
    match = re.search(r"(?:^|\.)layers\.(\d+)(?:\.|$)", name)
    if match is None:
        raise ValueError(f"Cannot resolve global decoder layer index: {name}")
    return int(match.group(1))


@lru_cache(maxsize=4)
def load_checkpoint(path: str):
    import torch

    if not path:
        raise ValueError("calibrated D256 K/V rotation paths are required")
    source = torch.load(path, map_location="cpu", weights_only=True)
    if torch.is_tensor(source) and source.ndim == 3:
        items = enumerate(source)
    elif isinstance(source, dict):
        items = source.get("layers", source).items()
    else:
        raise ValueError(f"Unsupported rotation checkpoint format: {path}")
    table = {}
    for key, entry in items:
        matrix = entry["rotation"] if isinstance(entry, dict) else entry
        if not torch.is_tensor(matrix):
            raise ValueError(f"Invalid matrix for layer {key} in {path}")
        table[int(key)] = matrix.float().contiguous()
    return table


def get_rotation(path: str, name: str, device, dim: int = 256):
    """bf16 ``[dim, dim]`` rotation of layer ``name`` on ``device`` (validated in fp32 on CPU)."""
    import torch

    index = layer_index(name)
    table = load_checkpoint(path)
    if index not in table:
        raise ValueError(f"Missing rotation for {name} (layer {index}) in {path}")
    matrix = table[index]
    if matrix.shape != (dim, dim):
        raise ValueError(f"Expected D{dim} rotation for {name}; got {tuple(matrix.shape)}")
    if not torch.isfinite(matrix).all():
        raise ValueError(f"Nonfinite rotation for {name}")
    identity = torch.eye(dim, dtype=matrix.dtype, device=matrix.device)
    if not torch.allclose(matrix.T @ matrix, identity, atol=0.015, rtol=0.015):
        raise ValueError(f"Rotation for {name} is not orthogonal")
    return matrix.to(device=device, dtype=torch.bfloat16).contiguous()
