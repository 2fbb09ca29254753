"""Launcher GPU checks and the opt-in power / clock settings against a
stand-in NVML (CPU; no real GPU setting is read or changed)."""
import pytest

from k8v4_xpu_b200.tools import gpu_setup


class FakeNVML:
    """Devices as dicts; records every setter call."""
    NVML_CLOCK_SM = 1

    def __init__(self, devices):
        self.devs = devices
        self.calls = []

    def nvmlDeviceGetCount(self):
        return len(self.devs)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetRemappedRows(self, h):
        d = self.devs[h]
        if "remap" not in d:
            raise RuntimeError("not supported")
        return d["remap"]

    def nvmlDeviceGetTotalEccErrors(self, h, kind, counter):
        assert (kind, counter) == (1, 0)  # uncorrected, volatile
        return self.devs[h].get("ecc", 0)

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.devs[h].get("reasons", 0)

    def nvmlDeviceGetMaxClockInfo(self, h, clock):
        return 1965

    def nvmlDeviceGetApplicationsClock(self, h, clock):
        return self.devs[h].get("app_clock", 1965)

    def nvmlDeviceGetPowerManagementLimitConstraints(self, h):
        return (200000, 1000000)

    def nvmlDeviceGetPowerManagementLimit(self, h):
        return self.devs[h].get("power", 1000000)

    def nvmlDeviceSetPowerManagementLimit(self, h, mw):
        if self.devs[h].get("denied"):
            raise PermissionError("insufficient permissions")
        self.calls.append(("power", h, mw))
        self.devs[h]["power"] = mw

    def nvmlDeviceSetGpuLockedClocks(self, h, lo, hi):
        self.calls.append(("lock", h, lo, hi))

    def nvmlDeviceResetGpuLockedClocks(self, h):
        self.calls.append(("unlock", h))


def test_preflight_reports_what_is_wrong_and_only_reads():
    nv = FakeNVML([{"remap": (0, 0, 0, 0)},
                   {"remap": (0, 2, 1, 0), "ecc": 3},
                   {"reasons": 0x8 | 0x4, "app_clock": 1000},
                   {}])
    w = gpu_setup.preflight(nv)
    assert not [x for x in w if x.startswith("GPU 0") or x.startswith("GPU 3")]
    assert any("GPU 1" in x and "pending" in x for x in w)
    assert any("GPU 1" in x and "2 rows" in x for x in w)
    assert any("GPU 1" in x and "3 uncorrected ECC" in x for x in w)
    assert any("GPU 2" in x and "hardware slowdown" in x for x in w)
    assert not any("power" in x for x in w)  # the power cap alone is normal under load
    assert any("GPU 2" in x and "1000 MHz" in x for x in w)
    assert nv.calls == []


def test_settings_are_off_unless_asked_and_restore_what_they_changed():
    nv = FakeNVML([{}, {"denied": True}])
    assert gpu_setup.apply_settings(nv, [0, 1]) == {} and nv.calls == []
    done = gpu_setup.apply_settings(nv, [0, 1], power_limit_w=120.0, clock_range=(400, 1800))
    assert done[0]["power_mw"] == (1000000, 200000)  # clamped to the card's minimum
    assert done[0]["clocks"] == (400, 1800)
    assert "power_error" in done[1] and done[1]["clocks"] == (400, 1800)
    gpu_setup.restore(nv, done)
    assert ("power", 0, 1000000) in nv.calls and ("unlock", 0) in nv.calls and ("unlock", 1) in nv.calls
    assert nv.devs[0]["power"] == 1000000


def test_clock_range_parsing():
    assert gpu_setup.parse_clock_range(None) is None
    assert gpu_setup.parse_clock_range("400, 1800") == (400, 1800)
    for bad in ("1800", "a,b", "1800,400", "0,100"):
        with pytest.raises(ValueError):
            gpu_setup.parse_clock_range(bad)


def test_serve_start_up_checks(capsys):
    from k8v4_xpu_b200 import cli, config
    nv = FakeNVML([{"remap": (0, 0, 1, 0)}, {}])
    cfg = config.resolve(["--model", "tiny"], env={})
    assert cfg.gpu_power_limit is None and cfg.gpu_clock_range is None
    assert cli.gpu_checks(cfg, 0, nvml=nv) is None and nv.calls == []
    assert "GPU 0: a row remap is pending" in capsys.readouterr().err
    assert cli.gpu_checks(cfg, 1, nvml=nv) is None
    assert capsys.readouterr().err == ""  # only local rank 0 prints the warnings
    cfg = config.resolve(["--model", "tiny", "--gpu-power-limit", "700", "--gpu-clock-range", "500,1900"], env={})
    got = cli.gpu_checks(cfg, 1, nvml=nv)
    assert got is not None and got[1][1]["power_mw"] == (1000000, 700000)
    assert ("lock", 1, 500, 1900) in nv.calls and not [c for c in nv.calls if c[1] == 0]
    with pytest.raises(ValueError):
        config.resolve(["--gpu-clock-range", "9,1"], env={})
    with pytest.raises(ValueError):
        config.resolve(["--gpu-power-limit", "-5"], env={})
