"""Reversible replacement of every gated MLP with OracleSparseMLP.

Same interface as reference end_to_end/model_patcher.py:12-33:
``OracleMLPPatcher(model, telemetry=None, norm_chunk_columns=256)`` with
``dense()``, ``apply_schedule(per-layer retentions)``, ``restore()`` and
``norm_computation_count``.  MLP discovery: the longest ``nn.ModuleList`` whose
entries contain a module with ``gate_proj``/``up_proj``/``down_proj`` (the
shallowest such module per layer), the rule of reference
extract/extract_ffn.py:34-55.
"""
from __future__ import annotations

from torch import nn

from .oracle_sparse_mlp import OracleSparseMLP

_PROJECTIONS = ("gate_proj", "up_proj", "down_proj")


def _is_gated_mlp(module: nn.Module) -> bool:
    return all(isinstance(getattr(module, name, None), nn.Module) for name in _PROJECTIONS)


def find_gated_mlps(model: nn.Module) -> list[str]:
    """Dotted paths of the per-layer gated MLPs, in layer order."""
    best: tuple[int, str] | None = None
    for path, layers in model.named_modules():
        if isinstance(layers, nn.ModuleList) and len(layers) and any(
                _is_gated_mlp(m) for m in layers[0].modules()):
            if best is None or len(layers) > best[0]:
                best = (len(layers), path)
    if best is None:
        raise RuntimeError("could not locate a ModuleList of layers with gate_proj, up_proj and down_proj")
    layers_path = best[1]
    layers = model.get_submodule(layers_path)
    paths = []
    for index, layer in enumerate(layers):
        found = sorted(((rel.count("."), len(rel), rel) for rel, m in layer.named_modules()
                        if rel and _is_gated_mlp(m)))
        if not found:
            raise RuntimeError(f"layer {index} of {layers_path} has no gated MLP")
        paths.append(".".join(p for p in (layers_path, str(index), found[0][2]) if p))
    return paths


class OracleMLPPatcher:
    def __init__(self, model: nn.Module, telemetry=None, norm_chunk_columns: int = 256):
        self.model = model
        self.wrappers: dict[int, OracleSparseMLP] = {}
        self.originals: dict[int, tuple[nn.Module, str, nn.Module]] = {}
        for index, path in enumerate(find_gated_mlps(model)):
            parent_path, name = path.rsplit(".", 1)
            parent = model.get_submodule(parent_path)
            original = getattr(parent, name)
            wrapper = OracleSparseMLP(original, index, 1.0, telemetry, norm_chunk_columns)
            setattr(parent, name, wrapper)
            self.wrappers[index] = wrapper
            self.originals[index] = (parent, name, original)

    @property
    def norm_computation_count(self) -> int:
        return sum(w.norm_computation_count for w in self.wrappers.values())

    def dense(self) -> None:
        for wrapper in self.wrappers.values():
            wrapper.set_mode(False)

    def apply_schedule(self, schedule: list[float]) -> None:
        if len(schedule) != len(self.wrappers):
            raise ValueError(f"schedule has {len(schedule)} layers; model has {len(self.wrappers)}")
        for index, wrapper in self.wrappers.items():
            wrapper.set_mode(True, schedule[index])

    def restore(self) -> None:
        for index, wrapper in self.wrappers.items():
            wrapper.close()
            parent, name, original = self.originals[index]
            setattr(parent, name, original)
