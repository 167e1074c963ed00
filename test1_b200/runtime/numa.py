"""CPU / NUMA placement of the local ranks.

Each local rank gets a contiguous block of the CPUs of its GPU's NUMA node:
``control`` cores for the Python/launch thread and the rest for the host
worker pool that runs LayerAdam and the CPU reduction.  Unlike the reference
launcher (numa_launch.sh:199-237), which gives the spare cores to rank 0
alone because only rank 0 runs the optimizer, every rank here gets an equal
share: the optimizer is sharded across ranks.

Topology comes from sysfs (``/sys/devices/system/cpu``,
``/sys/devices/system/node``, ``/sys/bus/pci/devices/<bus>/numa_node``);
``root`` lets tests point it at a fake tree.
"""
from __future__ import annotations

import argparse
import glob
import os
import re
import subprocess
from typing import Dict, List, Optional


def parse_cpulist(s: str) -> List[int]:
    out: List[int] = []
    for part in s.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            out.extend(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return out


def format_cpulist(cpus: List[int]) -> str:
    return ",".join(str(c) for c in cpus)


def numa_nodes(root: str = "/") -> Dict[int, List[int]]:
    nodes: Dict[int, List[int]] = {}
    for d in glob.glob(os.path.join(root, "sys/devices/system/node/node[0-9]*")):
        n = int(re.findall(r"node(\d+)$", d)[0])
        try:
            with open(os.path.join(d, "cpulist")) as f:
                nodes[n] = parse_cpulist(f.read())
        except OSError:
            continue
    return nodes


def physical_cores(cpus: List[int], root: str = "/") -> List[int]:
    """One logical CPU per physical core (the lowest sibling), order kept."""
    seen, out = set(), []
    for c in cpus:
        path = os.path.join(root, f"sys/devices/system/cpu/cpu{c}/topology/thread_siblings_list")
        try:
            with open(path) as f:
                sib = tuple(parse_cpulist(f.read()))
        except OSError:
            sib = (c,)
        key = min(sib)
        if key not in seen:
            seen.add(key)
            out.append(c)
    return out


def gpu_numa_node(gpu: int, root: str = "/", bus_ids: Optional[List[str]] = None) -> int:
    if bus_ids is None:
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=pci.bus_id", "--format=csv,noheader"],
                                 capture_output=True, text=True, timeout=30).stdout
            bus_ids = [l.strip() for l in out.splitlines() if l.strip()]
        except Exception:
            bus_ids = []
    if gpu >= len(bus_ids):
        return 0
    bus = bus_ids[gpu].lower()
    if bus.count(":") == 2 and len(bus.split(":")[0]) == 8:
        bus = bus[4:]  # 00000000:53:00.0 -> 0000:53:00.0
    try:
        with open(os.path.join(root, f"sys/bus/pci/devices/{bus}/numa_node")) as f:
            n = int(f.read().strip())
        return max(n, 0)
    except OSError:
        return 0


def plan(local_rank: int, local_world: int, gpu: int, allowed: List[int], control: int = 1,
         root: str = "/", bus_ids: Optional[List[str]] = None) -> Dict[str, str]:
    nodes = numa_nodes(root)
    node = gpu_numa_node(gpu, root, bus_ids) if nodes else 0
    node_cpus = [c for c in nodes.get(node, allowed) if c in set(allowed)] or list(allowed)
    cores = physical_cores(node_cpus, root) or node_cpus
    # ranks sharing this node split its cores evenly
    if nodes:
        same_node = [r for r in range(local_world)
                     if gpu_numa_node(r, root, bus_ids) == node] if bus_ids is not None else list(range(local_world))
    else:
        same_node = list(range(local_world))
    k = same_node.index(local_rank) if local_rank in same_node else 0
    per = max(1, len(cores) // max(1, len(same_node)))
    mine = cores[k * per:(k + 1) * per] or cores[-per:]
    ctl = mine[:control] if len(mine) > control else mine[:1]
    pool = mine[control:] if len(mine) > control else mine
    return {
        "NUMA_NODE": str(node),
        "NUMA_CONTROL_CORES": format_cpulist(ctl),
        "NUMA_CPU_ADAM_CORES": format_cpulist(pool),
        "T1_HOST_THREADS": str(len(pool)),
        "OMP_NUM_THREADS": "1",
        "MKL_NUM_THREADS": "1",
    }


def main() -> None:
    ap = argparse.ArgumentParser(description="print per-rank CPU placement as shell exports")
    ap.add_argument("--local-rank", type=int, default=int(os.environ.get("LOCAL_RANK", "0")))
    ap.add_argument("--local-world", type=int, default=int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
    ap.add_argument("--control", type=int, default=int(os.environ.get("CONTROLLER_CORES", "1")))
    ap.add_argument("--root", default="/")
    args = ap.parse_args()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu = int(vis.split(",")[args.local_rank]) if vis else args.local_rank
    env = plan(args.local_rank, args.local_world, gpu, sorted(os.sched_getaffinity(0)),
               args.control, args.root)
    for k, v in env.items():
        print(f"export {k}={v}")


if __name__ == "__main__":
    main()
