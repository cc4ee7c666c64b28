"""GPU / host detection without touching CUDA (flodl-hw/src/lib.rs:1-103).

``detect_gpus()`` parses ``nvidia-smi`` (no CUDA context is created, so it is
safe before forking rank processes). ``FLODL_TESTING_GPU_JSON`` replaces the
detection with a JSON list for tests (flodl-hw/src/testing.rs).
"""
from __future__ import annotations

import json
import os
import shutil
import subprocess
from dataclasses import asdict, dataclass
from typing import List


@dataclass
class GpuInfo:
    index: int
    name: str
    vendor: str
    memory_mb: int
    compute_capability: str = ""


def detect_gpus() -> List[GpuInfo]:
    spoof = os.environ.get("FLODL_TESTING_GPU_JSON")
    if spoof:
        return [GpuInfo(**g) for g in json.loads(spoof)]
    exe = shutil.which("nvidia-smi")
    if exe is None:
        return []
    try:
        out = subprocess.run([exe, "--query-gpu=index,name,memory.total,compute_cap",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True,
                             timeout=20).stdout
    except Exception:
        return []
    gpus = []
    for line in out.strip().splitlines():
        parts = [p.strip() for p in line.split(",")]
        if len(parts) < 3:
            continue
        try:
            gpus.append(GpuInfo(int(parts[0]), parts[1], "nvidia", int(float(parts[2])),
                                parts[3] if len(parts) > 3 else ""))
        except ValueError:
            continue
    return gpus


def host_memory_mb() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    return int(line.split()[1]) // 1024
    except OSError:
        pass
    return 0


def survey() -> dict:
    return {"gpus": [asdict(g) for g in detect_gpus()], "host_memory_mb": host_memory_mb(),
            "cpus": os.cpu_count()}
