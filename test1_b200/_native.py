"""Loaders for the in-tree native extensions.

``host()`` returns the C++ host runtime (``test1_b200._host``) and ``cuda()``
the sm_100a kernel library (``test1_b200._cuda``).  Both are built in-tree by
``python setup.py build_ext --inplace`` (``__graft_entry__.build()`` does the
same).  There is no silent fallback: if an extension is missing, the call
raises with the build command, so a GPU run can never quietly execute a
PyTorch substitute for a native kernel.
"""
from __future__ import annotations

import importlib
import os
import threading

_lock = threading.Lock()
_mods: dict = {}

_BUILD_HINT = "build it with `python setup.py build_ext --inplace` from the repository root"


def _load(name: str):
    with _lock:
        if name in _mods:
            return _mods[name]
        try:
            mod = importlib.import_module(f"test1_b200.{name}")
        except ImportError as exc:  # pragma: no cover - exercised only when unbuilt
            raise ImportError(f"native extension test1_b200.{name} is not built: {exc}; {_BUILD_HINT}") from exc
        _mods[name] = mod
        return mod


def host():
    """The host runtime extension (always required, CPU-only machines included)."""
    mod = _load("_host")
    if not getattr(host, "_configured", False):
        n = int(os.environ.get("T1_HOST_THREADS", "0") or 0)
        cpus = _cpu_list_from_env() or _rank_cpu_slice()
        if n <= 0:
            n = len(cpus) if cpus else len(os.sched_getaffinity(0))
        mod.configure_threads(n, cpus)
        host._configured = True
    return mod


def _rank_cpu_slice() -> list[int]:
    """Without an explicit CPU list, local ranks split the process affinity
    mask evenly (contiguous blocks), so N ranks on one host do not run N
    full-size worker pools on the same cores."""
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1") or 1)
    if local_world <= 1:
        return []
    local_rank = int(os.environ.get("LOCAL_RANK", "0") or 0)
    cpus = sorted(os.sched_getaffinity(0))
    per = max(1, len(cpus) // local_world)
    part = cpus[local_rank * per:(local_rank + 1) * per]
    return part or cpus[-per:]


def cuda():
    """The sm_100a kernel library.  Importing it loads libcuda; it is only
    needed on a machine with a B200.  With ``T1_BOUNDS_CHECK=1`` the
    bounds-checked build (``_cuda_checked``, built with
    ``T1_BUILD_CHECKED=1``) is loaded instead; ``bounds_errors()`` then
    reports the first out-of-range index each kernel file met."""
    if os.environ.get("T1_BOUNDS_CHECK", "0") == "1":
        return _load("_cuda_checked")
    return _load("_cuda")


def cuda_available() -> bool:
    try:
        cuda()
        return True
    except ImportError:
        return False


def _cpu_list_from_env() -> list[int]:
    """CPU list for the host worker pool: ``NUMA_CPU_ADAM_CORES`` (set by
    numa_launch.sh) wins, else the process affinity mask."""
    spec = os.environ.get("NUMA_CPU_ADAM_CORES", "").strip()
    if not spec:
        return []
    out: list[int] = []
    for part in spec.split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            out.extend(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return out
