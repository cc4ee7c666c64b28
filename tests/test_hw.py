"""Hardware survey: spoofing, arch parsing and coverage, visibility masks,
NVML read-only metrics through a fake (reference: flodl-hw/src/testing.rs,
vendor.rs, gpu.rs tests)."""
import json
from types import SimpleNamespace

import pytest

from flodl_b200.utils import hw


def test_arch_parse_and_coverage():
    a = hw.GpuArch.parse("nvidia", "10.0")
    assert str(a) == "sm_100" and a == hw.GpuArch.parse("nvidia", "sm_100a")
    assert hw.GpuArch.parse("nvidia", "sm_90").major == 9
    assert a.covered_by("9.0;10.0") and a.covered_by("10.3") and not a.covered_by("9.0 12.0")
    sm50 = hw.GpuArch.parse("nvidia", "5.0")
    assert not sm50.covered_by("7.0 7.5 8.0 8.6 8.9 9.0 12.0")  # the "5" in "7.5" is not sm_50
    g = hw.GpuArch.parse("amd", "gfx906:sramecc-:xnack-")
    assert str(g) == "gfx906" and g.covered_by("gfx906;gfx1030") and not g.covered_by("gfx90a")
    assert hw.GpuArch.parse("nvidia", "gfx906") is None


def test_spoofed_survey_array_and_envelope(monkeypatch):
    monkeypatch.setenv(hw.ENV_TESTING_GPU_JSON, json.dumps(
        [{"arch": "10.0", "vram_mb": 183359, "name": "NVIDIA B200"}, {"sm": "sm_100"}]))
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    s = hw.survey()
    assert [d.index for d in s.devices] == [0, 1] and s.devices[0].short_name() == "B200"
    assert s.devices[0].vram_bytes() == 183359 << 20 and s.devices[1].sm_version() == "sm_100"
    assert len(hw.detect_gpus()) == 2
    monkeypatch.setenv(hw.ENV_TESTING_GPU_JSON, json.dumps(
        {"gpus": [], "notes": [{"vendor": "amd", "kind": "hardware_unusable", "message": "no ROCm"}]}))
    s = hw.survey()
    assert not s.devices and s.notes[0].kind == "hardware_unusable"
    with pytest.raises(RuntimeError, match="no ROCm"):
        s.require_devices()


@pytest.mark.parametrize("bad", ['[{"vram_mb": 1}]', '[{"arch": "10.0", "vrm_mb": 1}]',
                                 '[{"arch": "10.0", "vendor": "intel"}]', '{"gpu": []}',
                                 '[{"arch": "gfx906"}]', 'not json'])
def test_spoof_errors_are_loud(monkeypatch, bad):
    monkeypatch.setenv(hw.ENV_TESTING_GPU_JSON, bad)
    with pytest.raises(ValueError):
        hw.survey()


def test_visibility_mask_applies_on_top_of_spoof(monkeypatch):
    monkeypatch.setenv(hw.ENV_TESTING_GPU_JSON, json.dumps([{"arch": "10.0"}] * 4))
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "2,0")
    s = hw.survey_visible()
    assert [d.index for d in s.devices] == [2, 0]
    assert any(n.kind == "mask_applied" for n in s.notes)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "1,9,3")  # enumeration stops at the bad entry
    assert [d.index for d in hw.detect_gpus()] == [1]


class _FakeNvml:
    """Read-only NVML surface; any setter would be an AttributeError."""

    def nvmlDeviceGetCount(self):
        return 2

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetCudaComputeCapability(self, h):
        return (10, 0)

    def nvmlDeviceGetMemoryInfo(self, h):
        return SimpleNamespace(total=183359 << 20, used=(1000 + h) << 20)

    def nvmlDeviceGetUUID(self, h):
        return f"GPU-{h:04d}"

    def nvmlDeviceGetUtilizationRates(self, h):
        return SimpleNamespace(gpu=87)

    def nvmlDeviceGetTemperature(self, h, sensor):
        return 55

    def nvmlDeviceGetPowerUsage(self, h):
        return 712000

    def nvmlDeviceGetClockInfo(self, h, kind):
        return 1965

    def nvmlSystemGetDriverVersion(self):
        return "580.159"


def test_nvml_survey_and_metrics_through_a_fake(monkeypatch):
    monkeypatch.delenv(hw.ENV_TESTING_GPU_JSON, raising=False)
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-0001")
    nv = _FakeNvml()
    s = hw.survey(nvml=nv)
    assert len(s.devices) == 2 and s.devices[0].arch == hw.GpuArch("nvidia", 10, 0)
    assert [d.uuid for d in hw.detect_gpus(nvml=nv)] == ["GPU-0001"]
    m = hw.gpu_metrics(1, nvml=nv)
    assert (m.util_percent, m.mem_used_mb, m.temp_c, m.power_w, m.sm_clock_mhz) == (87, 1001, 55.0, 712.0, 1965)
    assert hw.nvidia_driver_version(nvml=nv) == "580.159"
    assert hw.GpuMetrics().is_empty()


def test_host_memory(tmp_path):
    p = tmp_path / "meminfo"
    p.write_text("MemTotal:       263840764 kB\nMemFree:  1000 kB\nMemAvailable:   200000000 kB\n")
    m = hw.mem_info(str(p))
    assert m.total_gb() == 252 and m.available_kb == 200000000
    assert hw.mem_info(str(tmp_path / "missing")) is None
