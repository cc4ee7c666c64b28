"""Hardware survey without a CUDA context, spoofable for tests.

Reference roles: flodl-hw/src/{gpu,nvidia,vendor,report,mem,metrics,testing}.rs.

* :func:`survey` - every GPU on the machine, ignoring visibility masks (the
  provisioning view), plus findings (:class:`SurveyNote`). NVIDIA devices come
  from NVML (``nvidia_ml_py``) when it loads, else from ``nvidia-smi``; both
  are read-only queries and create no CUDA context, so the survey is safe
  before forking rank processes. A machine that exposes an AMD compute node
  (``/dev/kfd``) gets a ``vendor_mismatch`` note: this framework's kernels are
  sm_100a only.
* :func:`survey_visible` - the same with ``CUDA_VISIBLE_DEVICES`` applied
  (indices; a UUID mask that cannot be resolved leaves a ``mask_applied``
  note). :func:`detect_gpus` returns its devices.
* ``FLODL_TESTING_GPU_JSON`` replaces the sweep (plain JSON, typed by a
  developer): a bare device array or ``{"gpus": [...], "notes": [...]}``.
  Device keys: ``arch`` (required; ``sm`` is an alias), ``vendor`` (default
  ``nvidia``), ``index`` (default: position), ``name`` (default: generated),
  ``vram_mb`` (default 0). Unknown keys and malformed values raise - a test
  that silently fell back to real hardware would report on the wrong machine.
* :func:`gpu_metrics` - utilisation, memory, temperature and power through
  NVML (read-only); :func:`mem_info` - host RAM from ``/proc/meminfo``.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import subprocess
from dataclasses import asdict, dataclass, field
from typing import List, Optional

ENV_TESTING_GPU_JSON = "FLODL_TESTING_GPU_JSON"
NOTE_KINDS = ("hardware_unusable", "tool_failed", "unparsable", "mask_applied", "vendor_mismatch")
VENDORS = ("nvidia", "amd")


# ----------------------------------------------------------------- arch
@dataclass(frozen=True)
class GpuArch:
    vendor: str
    major: int = 0
    minor: int = 0
    gfx: str = ""

    @staticmethod
    def parse(vendor: str, token: str) -> Optional["GpuArch"]:
        t = token.strip().lower()
        if vendor == "nvidia":
            m = re.fullmatch(r"(\d+)\.(\d+)", t)
            if m:
                return GpuArch("nvidia", int(m.group(1)), int(m.group(2)))
            m = re.fullmatch(r"sm_?(\d+)([a-z]?)", t)
            if m and len(m.group(1)) >= 2:
                d = m.group(1)
                return GpuArch("nvidia", int(d[:-1]), int(d[-1]))
            return None
        if vendor == "amd":
            m = re.fullmatch(r"(gfx[0-9a-f]+)(:.*)?", t)
            return GpuArch("amd", gfx=m.group(1)) if m else None
        return None

    def __str__(self) -> str:
        return f"sm_{self.major}{self.minor}" if self.vendor == "nvidia" else self.gfx

    def archs_token(self) -> str:
        return f"{self.major}.{self.minor}" if self.vendor == "nvidia" else self.gfx

    def covered_by(self, archs: str) -> bool:
        """Whether a build for ``archs`` ("9.0;10.0", "gfx1030") runs here:
        NVIDIA matches any minor of the same major (PTX forward compatibility
        within a major), AMD needs the exact target. Tokens are parsed, never
        substring-matched (the "5" inside "7.5" is not sm_50)."""
        for tok in re.split(r"[;, ]+", archs):
            a = GpuArch.parse(self.vendor, tok) if tok else None
            if a is None:
                continue
            if self.vendor == "nvidia" and a.major == self.major:
                return True
            if self.vendor == "amd" and a.gfx == self.gfx:
                return True
        return False


# ----------------------------------------------------------------- devices and findings
@dataclass
class GpuInfo:
    index: int
    vendor: str
    name: str
    arch: GpuArch
    total_memory_mb: int = 0
    uuid: str = ""

    def sm_version(self) -> Optional[str]:
        return f"sm_{self.arch.major}{self.arch.minor}" if self.vendor == "nvidia" else None

    def vram_bytes(self) -> int:
        return self.total_memory_mb * (1 << 20)

    def short_name(self) -> str:
        n = self.name
        for p in ("NVIDIA ", "GeForce ", "AMD ", "Advanced Micro Devices, Inc. "):
            n = n.replace(p, "")
        return n

    def covered_by(self, archs: str) -> bool:
        return self.arch.covered_by(archs)

    def to_json(self) -> dict:
        return {"index": self.index, "vendor": self.vendor, "name": self.name,
                "arch": str(self.arch), "vram_mb": self.total_memory_mb}


@dataclass
class SurveyNote:
    vendor: str
    kind: str
    message: str

    def __post_init__(self):
        if self.kind not in NOTE_KINDS:
            raise ValueError(f"note kind {self.kind!r} is not one of {', '.join(NOTE_KINDS)}")


@dataclass
class GpuSurvey:
    devices: List[GpuInfo] = field(default_factory=list)
    notes: List[SurveyNote] = field(default_factory=list)

    def require_devices(self) -> List[GpuInfo]:
        if self.devices:
            return self.devices
        why = "; ".join(n.message for n in self.notes) or "no GPU detected"
        raise RuntimeError(f"no usable GPU: {why}")

    def has_vendor(self, vendor: str) -> bool:
        return any(d.vendor == vendor for d in self.devices)

    def vendors(self) -> List[str]:
        return sorted({d.vendor for d in self.devices})

    def to_json(self) -> dict:
        return {"gpus": [d.to_json() for d in self.devices], "notes": [asdict(n) for n in self.notes]}


# ----------------------------------------------------------------- spoofing
_DEVICE_KEYS = {"arch", "sm", "vendor", "index", "name", "vram_mb"}


def parse_survey(raw: str) -> GpuSurvey:
    v = json.loads(raw)
    notes = []
    if isinstance(v, dict):
        extra = set(v) - {"gpus", "notes"}
        if extra:
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: unknown keys {sorted(extra)}")
        devs = v.get("gpus", [])
        for n in v.get("notes", []):
            if set(n) - {"vendor", "kind", "message"}:
                raise ValueError(f"{ENV_TESTING_GPU_JSON}: unknown note keys in {n}")
            notes.append(SurveyNote(n.get("vendor", "nvidia"), n["kind"], n.get("message", "")))
    elif isinstance(v, list):
        devs = v
    else:
        raise ValueError(f"{ENV_TESTING_GPU_JSON}: expected an array or an object")
    out = []
    for i, d in enumerate(devs):
        if not isinstance(d, dict):
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: device {i} is not an object")
        extra = set(d) - _DEVICE_KEYS
        if extra:
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: device {i}: unknown keys {sorted(extra)}")
        vendor = d.get("vendor", "nvidia")
        if vendor not in VENDORS:
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: device {i}: unknown vendor {vendor!r}")
        tok = d.get("arch", d.get("sm"))
        if tok is None:
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: device {i}: 'arch' is required")
        arch = GpuArch.parse(vendor, str(tok))
        if arch is None:
            raise ValueError(f"{ENV_TESTING_GPU_JSON}: device {i}: arch {tok!r} does not fit {vendor}")
        out.append(GpuInfo(int(d.get("index", i)), vendor,
                           d.get("name", f"spoofed {vendor} {arch}"), arch, int(d.get("vram_mb", 0))))
    return GpuSurvey(out, notes)


# ----------------------------------------------------------------- detection
def _nvml():
    try:
        import pynvml
        pynvml.nvmlInit()
        return pynvml
    except Exception:
        return None


def _nvidia_nvml(nv) -> List[GpuInfo]:
    out = []
    for i in range(nv.nvmlDeviceGetCount()):
        h = nv.nvmlDeviceGetHandleByIndex(i)
        name = nv.nvmlDeviceGetName(h)
        name = name.decode() if isinstance(name, bytes) else name
        major, minor = nv.nvmlDeviceGetCudaComputeCapability(h)
        mem = nv.nvmlDeviceGetMemoryInfo(h).total // (1 << 20)
        uuid = nv.nvmlDeviceGetUUID(h)
        uuid = uuid.decode() if isinstance(uuid, bytes) else uuid
        out.append(GpuInfo(i, "nvidia", name, GpuArch("nvidia", major, minor), int(mem), uuid))
    return out


def _nvidia_smi(notes: List[SurveyNote]) -> List[GpuInfo]:
    exe = shutil.which("nvidia-smi")
    if exe is None:
        if os.path.exists("/dev/nvidiactl"):
            notes.append(SurveyNote("nvidia", "hardware_unusable",
                                    "NVIDIA driver nodes exist but neither NVML nor nvidia-smi loads"))
        return []
    try:
        r = subprocess.run([exe, "--query-gpu=index,name,memory.total,compute_cap,uuid",
                            "--format=csv,noheader,nounits"], capture_output=True, text=True,
                           timeout=20)
    except Exception as e:
        notes.append(SurveyNote("nvidia", "tool_failed", f"nvidia-smi: {e}"))
        return []
    if r.returncode != 0:
        notes.append(SurveyNote("nvidia", "tool_failed", f"nvidia-smi exited {r.returncode}"))
        return []
    out = []
    for line in r.stdout.strip().splitlines():
        p = [x.strip() for x in line.split(",")]
        arch = GpuArch.parse("nvidia", p[3]) if len(p) > 3 else None
        try:
            out.append(GpuInfo(int(p[0]), "nvidia", p[1], arch, int(float(p[2])),
                               p[4] if len(p) > 4 else ""))
            if arch is None:
                raise ValueError
        except (ValueError, IndexError):
            if out and out[-1].arch is None:
                out.pop()
            notes.append(SurveyNote("nvidia", "unparsable", f"nvidia-smi row {line!r}"))
    return out


def survey(nvml=None) -> GpuSurvey:
    """All GPUs on the machine (masks ignored). ``nvml`` injects a fake NVML."""
    raw = os.environ.get(ENV_TESTING_GPU_JSON, "")
    if raw.strip():
        return parse_survey(raw)
    notes: List[SurveyNote] = []
    nv = nvml if nvml is not None else _nvml()
    devices = []
    if nv is not None:
        try:
            devices = _nvidia_nvml(nv)
        except Exception as e:
            notes.append(SurveyNote("nvidia", "tool_failed", f"NVML: {e}"))
    if not devices and nvml is None:
        devices = _nvidia_smi(notes)
    if os.path.exists("/dev/kfd"):
        notes.append(SurveyNote("amd", "vendor_mismatch",
                                "AMD compute devices present; this build's kernels target sm_100a only"))
    return GpuSurvey(devices, notes)


def _apply_mask(s: GpuSurvey, mask: Optional[str]) -> GpuSurvey:
    if mask is None:
        return s
    nv = [d for d in s.devices if d.vendor == "nvidia"]
    other = [d for d in s.devices if d.vendor != "nvidia"]
    notes = list(s.notes)
    picked = []
    for tok in filter(None, (t.strip() for t in mask.split(","))):
        if tok.isdigit():
            hit = [d for d in nv if d.index == int(tok)]
        else:
            hit = [d for d in nv if d.uuid and d.uuid.startswith(tok)]
        if not hit:  # CUDA stops enumerating at the first invalid entry
            notes.append(SurveyNote("nvidia", "mask_applied",
                                    f"CUDA_VISIBLE_DEVICES entry {tok!r} matches no device"))
            break
        picked.append(hit[0])
    if len(picked) != len(nv):
        notes.append(SurveyNote("nvidia", "mask_applied",
                                f"CUDA_VISIBLE_DEVICES={mask!r} exposes {len(picked)} of {len(nv)}"))
    return GpuSurvey(picked + other, notes)


def survey_visible(nvml=None) -> GpuSurvey:
    return _apply_mask(survey(nvml), os.environ.get("CUDA_VISIBLE_DEVICES"))


def detect_gpus(nvml=None) -> List[GpuInfo]:
    """Usable devices: visible and addressable by this build (NVIDIA)."""
    return [d for d in survey_visible(nvml).devices if d.vendor == "nvidia"]


def detect_gpus_physical(nvml=None) -> List[GpuInfo]:
    return survey(nvml).devices


def nvidia_driver_version(nvml=None) -> Optional[str]:
    nv = nvml if nvml is not None else _nvml()
    if nv is None:
        return None
    try:
        v = nv.nvmlSystemGetDriverVersion()
        return v.decode() if isinstance(v, bytes) else v
    except Exception:
        return None


# ----------------------------------------------------------------- metrics (read-only)
@dataclass
class GpuMetrics:
    util_percent: Optional[int] = None
    mem_used_mb: Optional[int] = None
    mem_total_mb: Optional[int] = None
    temp_c: Optional[float] = None
    power_w: Optional[float] = None
    sm_clock_mhz: Optional[int] = None

    def is_empty(self) -> bool:
        return all(v is None for v in asdict(self).values())


def gpu_metrics(index: int, nvml=None) -> GpuMetrics:
    """Live counters of one device through NVML; empty when NVML is absent."""
    nv = nvml if nvml is not None else _nvml()
    m = GpuMetrics()
    if nv is None:
        return m
    try:
        h = nv.nvmlDeviceGetHandleByIndex(index)
    except Exception:
        return m
    for attr, fn in (("util_percent", lambda: nv.nvmlDeviceGetUtilizationRates(h).gpu),
                     ("mem_used_mb", lambda: nv.nvmlDeviceGetMemoryInfo(h).used >> 20),
                     ("mem_total_mb", lambda: nv.nvmlDeviceGetMemoryInfo(h).total >> 20),
                     ("temp_c", lambda: float(nv.nvmlDeviceGetTemperature(h, 0))),
                     ("power_w", lambda: nv.nvmlDeviceGetPowerUsage(h) / 1000.0),
                     ("sm_clock_mhz", lambda: nv.nvmlDeviceGetClockInfo(h, 1))):
        try:
            setattr(m, attr, fn())
        except Exception:
            pass
    return m


# ----------------------------------------------------------------- host memory
@dataclass
class MemInfo:
    total_kb: int
    available_kb: int

    def total_gb(self) -> int:
        return round(self.total_kb / (1 << 20))


def mem_info(path: str = "/proc/meminfo") -> Optional[MemInfo]:
    vals = {}
    try:
        with open(path) as f:
            for line in f:
                k, _, rest = line.partition(":")
                vals[k] = int(rest.split()[0])
    except (OSError, ValueError, IndexError):
        return None
    if "MemTotal" not in vals:
        return None
    return MemInfo(vals["MemTotal"], vals.get("MemAvailable", vals.get("MemFree", 0)))


def host_memory_mb() -> int:
    m = mem_info()
    return m.total_kb // 1024 if m else 0


def cpu_package_count(path: str = "/proc/cpuinfo") -> Optional[int]:
    try:
        with open(path) as f:
            ids = {line.split(":")[1].strip() for line in f if line.startswith("physical id")}
    except OSError:
        return None
    return len(ids) or None


def report() -> dict:
    """The ``probe`` report: visible GPUs, findings, host memory and CPUs."""
    s = survey_visible()
    m = mem_info()
    return {**s.to_json(), "driver": nvidia_driver_version(),
            "host_memory_mb": m.total_kb // 1024 if m else 0,
            "host_available_mb": m.available_kb // 1024 if m else 0,
            "cpus": os.cpu_count(), "cpu_packages": cpu_package_count()}
