"""Start-up loading of OSCAR's calibrated K/V rotation files.

File format (the reference's artifact, ``oscar_ascend/rotations.py:7-53``; the
calibration worker writes it): a ``torch.save``'d object in one of three shapes,

* a tensor ``[L, d, d]``: matrix ``i`` belongs to decoder layer ``i``;
* ``{"layers": {layer: entry}}``;
* ``{layer: entry}``;

where an entry is a matrix or ``{"rotation": matrix}``.  A layer whose matrix is
missing, of another dimension, non-finite or not orthogonal (``RᵀR`` within 0.015
absolute + 0.015 relative of the identity, checked in fp32 on the CPU whatever the
default dtype) is an error, never a silent identity.

Here a file is parsed once into a :class:`RotationFile`, and every matrix of it is
checked at load time in one batched pass (finiteness and ``RᵀR`` of all layers of a
dimension at once); asking for a layer then only reports what the load found.
"""

from __future__ import annotations

from collections.abc import Mapping
from functools import lru_cache

import torch

ORTHO_TOL = 0.015  # absolute and relative tolerance of RᵀR against I


def layer_index(name: str) -> int:
    """Global decoder layer of a module name: the integer after the first ``layers``
    component (``model.language_model.layers.63.self_attn.attn`` -> 63)."""
    parts = name.split(".")
    for here, after in zip(parts, parts[1:]):
        if here == "layers" and after.isdecimal():
            return int(after)
    raise ValueError(f"no decoder layer index in module name {name!r}")


def _entries(source, path):
    """(layer, matrix) pairs of a loaded rotation file, in file order."""
    if torch.is_tensor(source):
        if source.ndim != 3:
            raise ValueError(f"{path}: a stacked rotation file holds [L, d, d], not {tuple(source.shape)}")
        return list(enumerate(source))
    if not isinstance(source, dict):
        raise ValueError(f"{path}: not a rotation file (a [L, d, d] tensor or a dict of layers)")
    layers = source["layers"] if "layers" in source else source
    pairs = []
    for key, entry in layers.items():
        matrix = entry.get("rotation") if isinstance(entry, dict) else entry
        if not torch.is_tensor(matrix):
            raise ValueError(f"{path}: layer {key} holds no rotation matrix")
        pairs.append((int(key), matrix))
    return pairs


def _audit(matrices: dict) -> dict:
    """Problem per layer (absent: valid), all square matrices of one size checked in one
    batch: non-finite entries, then RᵀR against the identity."""
    problems = {}
    by_dim = {}
    for layer, m in matrices.items():
        if m.ndim != 2 or m.shape[0] != m.shape[1]:
            problems[layer] = f"shape {tuple(m.shape)} is not square"
        else:
            by_dim.setdefault(m.shape[0], []).append(layer)
    for dim, layers in by_dim.items():
        stack = torch.stack([matrices[i] for i in layers])
        finite = torch.isfinite(stack).flatten(1).all(dim=1)
        gram = torch.bmm(stack.transpose(1, 2), stack)
        eye = torch.eye(dim, dtype=torch.float32)
        excess = ((gram - eye).abs() - (ORTHO_TOL + ORTHO_TOL * eye)).flatten(1).amax(dim=1)
        for layer, fin, ex in zip(layers, finite.tolist(), excess.tolist()):
            if not fin:
                problems[layer] = "non-finite entries"
            elif not ex <= 0.0:
                problems[layer] = "matrix is not orthogonal (RᵀR differs from I)"
    return problems


class RotationFile(Mapping):
    """The checked contents of one rotation file: layer -> fp32 CPU matrix."""

    def __init__(self, path: str, matrices: dict, problems: dict):
        self.path, self._matrices, self.problems = path, matrices, problems

    def __getitem__(self, layer):
        return self._matrices[layer]

    def __iter__(self):
        return iter(self._matrices)

    def __len__(self):
        return len(self._matrices)

    def rotation(self, layer: int, dim: int, name: str) -> torch.Tensor:
        if layer not in self._matrices:
            raise ValueError(f"Missing rotation: {self.path} has no layer {layer} (module {name})")
        m = self._matrices[layer]
        if tuple(m.shape) != (dim, dim):
            raise ValueError(f"module {name} needs a D{dim} rotation; {self.path} layer {layer} is "
                             f"{tuple(m.shape)}")
        if layer in self.problems:
            raise ValueError(f"{self.path} layer {layer} (module {name}): {self.problems[layer]}")
        return m


@lru_cache(maxsize=4)
def load_checkpoint(path: str) -> RotationFile:
    """Parse and check a rotation file once per path."""
    if not path:
        raise ValueError("calibrated D256 K and V rotation files are required (no identity default)")
    source = torch.load(path, map_location="cpu", weights_only=True)
    matrices = {}
    for layer, m in _entries(source, path):
        matrices[layer] = m.detach().to(torch.float32).contiguous()
    return RotationFile(path, matrices, _audit(matrices))


def get_rotation(path: str, name: str, device, dim: int = 256) -> torch.Tensor:
    """bf16 ``[dim, dim]`` rotation of module ``name`` on ``device``."""
    m = load_checkpoint(path).rotation(layer_index(name), dim, name)
    return m.to(device=device, dtype=torch.bfloat16).contiguous()
