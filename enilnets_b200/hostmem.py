"""Host memory placement for the copies on either side of the attention path.

Every call through the public API with host buffers (NumPy in, NumPy out)
copies its inputs up and its result down through pinned host memory, one
process per GPU. On a multi-socket host, a rank whose pinned buffers were
first touched from the far socket sends every copy across the socket link.
With eight ranks copying at once, that traffic, not PCIe, sets the
end-to-end rate.

`local_to(device)` runs a block on the CPUs NVML reports as closest to the
GPU, then restores the caller's CPU set. Pinned buffers allocated and filled
inside the block are placed on the GPU's NUMA node (Linux places a page on
the node of the CPU that first touches it). Only this process's CPU affinity
changes; nothing on the GPU is changed, and NVML is only read. When NVML or
the device cannot answer (no GPU, no driver, an unknown bus id), the block
runs unbound.
"""
from __future__ import annotations

import contextlib
import os
from typing import Iterator, List, Optional


def _bus_id(device: int) -> str:
    import torch
    props = torch.cuda.get_device_properties(device)
    return f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"


def gpu_local_cpus(device: int) -> Optional[List[int]]:
    """CPUs closest to CUDA device `device` that this process may run on, or
    None when that cannot be determined."""
    try:
        import pynvml
        bus = _bus_id(device)
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = ((os.cpu_count() or 1) + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        return None
    cpus = [64 * i + b for i, word in enumerate(mask) for b in range(64) if (word >> b) & 1]
    allowed = os.sched_getaffinity(0)
    cpus = [c for c in cpus if c in allowed]
    return cpus or None


def numa_nodes() -> List[List[int]]:
    """CPUs of each NUMA node of the host (from sysfs), restricted to the
    CPUs this process may run on; [] when sysfs does not say."""
    base = "/sys/devices/system/node"
    nodes = []
    try:
        names = sorted((n for n in os.listdir(base) if n.startswith("node") and n[4:].isdigit()),
                       key=lambda n: int(n[4:]))
    except OSError:
        return []
    allowed = os.sched_getaffinity(0)
    for name in names:
        try:
            with open(os.path.join(base, name, "cpulist")) as f:
                text = f.read().strip()
        except OSError:
            continue
        cpus = []
        for part in filter(None, text.split(",")):
            lo, _, hi = part.partition("-")
            cpus.extend(range(int(lo), int(hi or lo) + 1))
        cpus = [c for c in cpus if c in allowed]
        if cpus:
            nodes.append(cpus)
    return nodes


def spread_cpus(rank: int) -> Optional[List[int]]:
    """CPUs of NUMA node rank % (number of nodes): spreads the ranks' pinned
    buffers over every node's memory, for hosts where every GPU reports the
    same local node; None on a single-node host."""
    nodes = numa_nodes()
    if len(nodes) < 2:
        return None
    return nodes[rank % len(nodes)]


@contextlib.contextmanager
def local_to(device: int, cpus: Optional[List[int]] = None) -> Iterator[Optional[List[int]]]:
    """Run the block on the GPU's local CPUs (or on `cpus` when given); yield
    the CPUs used (None: unbound)."""
    if cpus is None:
        cpus = gpu_local_cpus(device)
    before = os.sched_getaffinity(0)
    if cpus:
        os.sched_setaffinity(0, cpus)
    try:
        yield cpus
    finally:
        if cpus:
            os.sched_setaffinity(0, before)
