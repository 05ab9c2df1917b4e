"""Ant residency planning for the CUDA backend's VRAM tier.

`plan_residency` restates the reference planner `Ant::plan_residency`
(`src/ant.rs:655-710`) so a host that drives the library without the Rust
engine (tests, the benchmark) produces the same unit -> tier map the engine
passes to the loader (`BackendLoader`, `registry.rs:138-146`), which
`cheetah_cuda_model_open_ex` takes:

1. pinned units (`resident_units`) go to "vram" unconditionally and do not
   count against the pool;
2. the others are visited in numeric `layer_id` order, then by unit id, so
   the VRAM boundary falls inside one deterministic layer;
3. each takes the first tier where it still fits: the VRAM pool, then the RAM
   budget, then "disk"; a unit larger than the whole VRAM pool goes straight
   to "disk".

A disabled Ant (`enabled=False`) plans nothing (an empty map: every unit
HBM-resident, as `ant.rs:667-669`).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, List, Sequence

# `AntSettings::default` (`ant.rs:70-85`).
DEFAULT_VRAM_POOL = 8 * 1024 ** 3
DEFAULT_RAM_BUDGET = 16 * 1024 ** 3


@dataclass(frozen=True)
class AntUnit:
    """The planner's view of one `cheetah_units.json` entry (`ant.rs:87-123`)."""
    unit_id: str
    bytes: int
    layer_id: int


def units_of(prepared) -> List[AntUnit]:
    """Planner units of a `prepared.PreparedModel` (its units manifest)."""
    return [AntUnit(u.unit_id, int(u.nbytes), int(u.layer_id)) for u in prepared.units.values()]


def plan_residency(units: Iterable[AntUnit], vram_pool_bytes: int = DEFAULT_VRAM_POOL,
                   ram_budget_bytes: int = DEFAULT_RAM_BUDGET, resident_units: Sequence[str] = (),
                   enabled: bool = True) -> Dict[str, str]:
    """unit id -> "vram" | "ram" | "disk" (`Ant::plan_residency`, `ant.rs:655-710`)."""
    if not enabled:
        return {}
    pinned = set(resident_units)
    ordered = sorted(units, key=lambda u: (u.unit_id not in pinned, u.layer_id, u.unit_id))
    vram_used = ram_used = 0
    plan: Dict[str, str] = {}
    for unit in ordered:
        size = unit.bytes
        if unit.unit_id in pinned:
            tier = "vram"
        elif size > vram_pool_bytes:
            tier = "disk"
        elif vram_used + size <= vram_pool_bytes:
            vram_used += size
            tier = "vram"
        elif ram_used + size <= ram_budget_bytes:
            ram_used += size
            tier = "ram"
        else:
            tier = "disk"
        plan[unit.unit_id] = tier
    return plan


@dataclass
class LayerResidency:
    """Per-layer units and bytes in each tier (`AntLayerResidency`, `ant.rs:125-154`)."""
    layer_id: int
    vram_units: int = 0
    vram_bytes: int = 0
    ram_units: int = 0
    ram_bytes: int = 0
    disk_units: int = 0
    disk_bytes: int = 0

    def state(self) -> str:
        """"full_vram" / "full_ram" / "full_disk", or "partial" when the layer spans tiers."""
        key = (self.vram_units > 0, self.ram_units > 0, self.disk_units > 0)
        return {(True, False, False): "full_vram", (False, True, False): "full_ram",
                (False, False, True): "full_disk"}.get(key, "partial")


def layer_residency_summary(units: Iterable[AntUnit], plan: Dict[str, str]) -> List[LayerResidency]:
    """`Ant::layer_residency_summary` (`ant.rs:619-652`): units not in the plan count as "vram"."""
    layers: Dict[int, LayerResidency] = {}
    for u in units:
        tier = plan.get(u.unit_id, "vram")
        entry = layers.setdefault(u.layer_id, LayerResidency(u.layer_id))
        if tier == "vram":
            entry.vram_units += 1
            entry.vram_bytes += u.bytes
        elif tier == "ram":
            entry.ram_units += 1
            entry.ram_bytes += u.bytes
        else:
            entry.disk_units += 1
            entry.disk_bytes += u.bytes
    return [layers[k] for k in sorted(layers)]
