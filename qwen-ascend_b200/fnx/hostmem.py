"""Host-side placement for the pinned buffers that feed a GPU (``HostPipeline`` batches).

A pinned host buffer crosses the GPU's PCIe link, and, when its pages sit on the other CPU
socket, the inter-socket link as well.  ``bind_to_device`` restricts the calling process to
the CPUs the kernel lists as local to the GPU's PCI device (sysfs ``local_cpulist``), so
that pinned buffers allocated afterwards land on the GPU's NUMA node (pages are placed on
the node of the thread that first touches them, which for ``cudaHostAlloc`` is the caller).
Nothing here changes a GPU setting.
"""
from __future__ import annotations

import os

import torch


def _parse_cpulist(text):
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def device_locality(device):
    """``{"pci": bus id, "numa_node": n or None, "cpus": set}`` of a CUDA device, from sysfs
    (empty ``cpus`` when the platform does not say)."""
    idx = torch.device(device).index
    p = torch.cuda.get_device_properties(idx if idx is not None else torch.cuda.current_device())
    bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    base = f"/sys/bus/pci/devices/{bus}"
    node, cpus = None, set()
    try:
        with open(f"{base}/numa_node") as f:
            node = int(f.read().strip())
        with open(f"{base}/local_cpulist") as f:
            cpus = _parse_cpulist(f.read())
    except (OSError, ValueError):
        pass
    return {"pci": bus, "numa_node": node if node is not None and node >= 0 else None, "cpus": cpus}


def bind_to_device(device):
    """Restrict this process to the CPUs local to ``device`` (those it may run on anyway).
    Returns a summary: the device's NUMA node, how many CPUs it is bound to, and whether the
    binding changed anything (False when every allowed CPU is already local, or the platform
    gives no locality)."""
    loc = device_locality(device)
    allowed = os.sched_getaffinity(0)
    local = loc["cpus"] & allowed
    changed = bool(local) and local != allowed
    if changed:
        os.sched_setaffinity(0, local)
    return {"pci": loc["pci"], "numa_node": loc["numa_node"],
            "cpus": len(local) if local else len(allowed), "bound": changed}
