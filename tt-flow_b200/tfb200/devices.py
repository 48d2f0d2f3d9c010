"""The device table of the B200 backend, with the lookup API of the reference's
``tensixflow.devices`` (python/tensixflow/devices.py: ``DEVICES``, ``ALIASES``,
``DEFAULT_DEVICE``, ``lookup``, ``valid_device_names``, ``all_devices``).

The values come from ``spec/devices.json`` (the B200 entry, in the layout of
the reference's device table), the same figures the C++ planner uses. Fields
that only describe Tensix hardware (NoC, matrix-unit tiles) have no B200
counterpart; the B200's own figures (TMEM, L2, the pool's measured peaks) are
added.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

_SPEC_PATH = Path(__file__).resolve().parents[1] / "spec" / "devices.json"


@dataclass(frozen=True)
class DeviceSpec:
    """One device entry, a static planning input."""

    name: str
    arch: str
    compute_grid_x: int          # SMs per die
    compute_grid_y: int          # dies
    chips: int
    l1_usable_bytes: int         # shared memory one CTA may request
    l1_nominal_bytes: int        # shared memory per SM
    tmem_columns: int
    l2_bytes: int
    clock_hz: int
    flops_per_cycle_per_core: int
    dram_bytes: int
    dram_bandwidth_bytes_per_second: int
    measured_hbm_bytes_per_second: float
    measured_bf16_flops_per_second: float
    power_watts: int

    @property
    def total_cores(self) -> int:
        """SMs across the board's dies."""
        return self.chips * self.compute_grid_x * self.compute_grid_y

    def cb_budget(self, reserve_bytes: int = 0) -> int:
        """Shared-memory bytes a CTA has for its stage rings after a reserve."""
        return max(0, self.l1_usable_bytes - reserve_bytes)


def _load():
    spec = json.loads(_SPEC_PATH.read_text())
    devices, aliases = {}, {}
    for name, e in spec["devices"].items():
        devices[name] = DeviceSpec(
            name=name, arch=e["arch"], compute_grid_x=e["compute"]["grid_x"], compute_grid_y=e["compute"]["grid_y"],
            chips=e["chips"], l1_usable_bytes=e["l1"]["usable_bytes"], l1_nominal_bytes=e["l1"]["nominal_bytes"],
            tmem_columns=e["tmem"]["columns"], l2_bytes=e["l2_bytes"], clock_hz=e["clock_hz"],
            flops_per_cycle_per_core=e["matrix_unit"]["flops_per_cycle_per_core"], dram_bytes=e["dram"]["bytes"],
            dram_bandwidth_bytes_per_second=e["dram"]["bandwidth_bytes_per_second"],
            measured_hbm_bytes_per_second=e["measured"]["hbm_bytes_per_second"],
            measured_bf16_flops_per_second=e["measured"]["bf16_flops_per_second"], power_watts=e["power_watts"])
        for a in e.get("aliases", []):
            aliases[a] = name
    return spec["default_device"], devices, aliases


DEFAULT_DEVICE, DEVICES, ALIASES = _load()


def valid_device_names() -> str:
    """Comma-separated device names for error messages."""
    return ", ".join(DEVICES)


def lookup(name: str) -> DeviceSpec:
    """Return the spec for a name or alias; raise KeyError if unknown."""
    if name in DEVICES:
        return DEVICES[name]
    resolved = ALIASES.get(name)
    if resolved is None:
        raise KeyError(f"unknown device {name!r}; valid devices: {valid_device_names()}")
    return DEVICES[resolved]


def all_devices() -> tuple[DeviceSpec, ...]:
    """Every device entry in source order."""
    return tuple(DEVICES.values())
