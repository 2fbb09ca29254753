"""Launcher GPU checks (read-only) and the opt-in power / clock settings.

The reference launcher looks for an earlier GPU fault in the kernel log
before it starts a server (``k8v4_v030/launch.sh:201-203``: a "CAT error"
warning) and sets each card's power limit and frequency range with
``xpu-smi`` (``launch.sh:204-213``). Here:

* :func:`preflight` reads, through NVML, what says a B200 is not in a clean
  state: pending row remaps or remap failures, uncorrected ECC errors since
  the driver loaded, throttling by hardware slowdown or heat, and SM clocks
  held below their maximum by a clock lock. It only reads; the launcher
  prints its warnings and starts anyway, as the reference does with old
  faults;
* :func:`apply_settings` sets a power limit and/or a locked SM clock range.
  It is OFF by default: it runs only when ``serve`` is given
  ``--gpu-power-limit`` or ``--gpu-clock-range``, and a setting outlasts the
  process, so whoever uses it owns putting it back (``restore`` below gives
  the values it replaced). The tests drive it with a stand-in NVML only.

``nvml`` is the ``pynvml`` module (nvidia-ml-py) or an object with the same
functions.
"""
from __future__ import annotations

# clocks event reason bits (NVML's values; the module's names differ by version)
_HW_SLOWDOWN = 0x8
_SW_THERMAL = 0x20
_HW_THERMAL = 0x40
_HW_POWER_BRAKE = 0x80
_SW_POWER_CAP = 0x4
_UNCORRECTED, _VOLATILE = 1, 0


def load_nvml():
    """The NVML module, initialised, or None when NVML is not there."""
    try:
        import pynvml
        pynvml.nvmlInit()
        return pynvml
    except Exception:
        return None


def _reasons(nvml, h) -> int:
    fn = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
        getattr(nvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
    return int(fn(h))


def preflight(nvml) -> list[str]:
    """Warnings (one line each) about every GPU NVML sees; empty when clean."""
    warnings = []
    for i in range(int(nvml.nvmlDeviceGetCount())):
        h = nvml.nvmlDeviceGetHandleByIndex(i)
        try:
            corr, unc, pending, failure = nvml.nvmlDeviceGetRemappedRows(h)
            if pending:
                warnings.append("GPU %d: a row remap is pending (the GPU needs a reset to apply it)" % i)
            if failure:
                warnings.append("GPU %d: a row remap failed (its memory may be unreliable)" % i)
            if unc:
                warnings.append("GPU %d: %d rows remapped after uncorrectable errors" % (i, unc))
        except Exception:
            pass  # not supported on this part
        try:
            ecc = int(nvml.nvmlDeviceGetTotalEccErrors(h, _UNCORRECTED, _VOLATILE))
            if ecc:
                warnings.append("GPU %d: %d uncorrected ECC errors since the driver loaded" % (i, ecc))
        except Exception:
            pass
        try:
            r = _reasons(nvml, h)
            for bit, what in ((_HW_SLOWDOWN, "hardware slowdown"), (_HW_THERMAL, "hardware thermal slowdown"),
                              (_SW_THERMAL, "software thermal slowdown"), (_HW_POWER_BRAKE, "power brake")):
                if r & bit:
                    warnings.append("GPU %d: clocks held down by %s" % (i, what))
        except Exception:
            pass
        try:
            sm = getattr(nvml, "NVML_CLOCK_SM", 1)
            mx = int(nvml.nvmlDeviceGetMaxClockInfo(h, sm))
            app = int(nvml.nvmlDeviceGetApplicationsClock(h, sm))
            if mx and app and app < 0.8 * mx:
                warnings.append("GPU %d: application SM clock %d MHz of %d MHz (a clock setting is in place)"
                                % (i, app, mx))
        except Exception:
            pass
    return warnings


def parse_clock_range(text: str | None) -> tuple[int, int] | None:
    """``"MIN,MAX"`` in MHz, or None."""
    if not text:
        return None
    parts = [p.strip() for p in str(text).split(",")]
    if len(parts) != 2 or not all(p.isdigit() for p in parts):
        raise ValueError("--gpu-clock-range takes MIN,MAX in MHz, got %r" % text)
    lo, hi = int(parts[0]), int(parts[1])
    if not 0 < lo <= hi:
        raise ValueError("--gpu-clock-range needs 0 < MIN <= MAX, got %r" % text)
    return lo, hi


def apply_settings(nvml, devices: list[int], power_limit_w: float | None = None,
                   clock_range: tuple[int, int] | None = None) -> dict:
    """Set the power limit (watts, clamped to the card's allowed range) and/or
    lock the SM clocks to ``clock_range`` on ``devices``. Does nothing when
    both are None. Returns ``{device: {"power_mw": (old, new), "clocks":
    (lo, hi)}}`` for what it changed; failures (no permission, not supported)
    are reported per device and do not raise."""
    done: dict = {}
    if power_limit_w is None and clock_range is None:
        return done
    for i in devices:
        h = nvml.nvmlDeviceGetHandleByIndex(i)
        rec: dict = {}
        if power_limit_w is not None:
            try:
                lo, hi = nvml.nvmlDeviceGetPowerManagementLimitConstraints(h)
                want = int(min(max(power_limit_w * 1000.0, lo), hi))
                old = int(nvml.nvmlDeviceGetPowerManagementLimit(h))
                nvml.nvmlDeviceSetPowerManagementLimit(h, want)
                rec["power_mw"] = (old, want)
            except Exception as e:
                rec["power_error"] = str(e)
        if clock_range is not None:
            try:
                nvml.nvmlDeviceSetGpuLockedClocks(h, int(clock_range[0]), int(clock_range[1]))
                rec["clocks"] = tuple(clock_range)
            except Exception as e:
                rec["clocks_error"] = str(e)
        done[i] = rec
    return done


def restore(nvml, done: dict) -> None:
    """Put back what :func:`apply_settings` changed: the old power limits, and
    the SM clocks unlocked."""
    for i, rec in done.items():
        h = nvml.nvmlDeviceGetHandleByIndex(i)
        if "power_mw" in rec:
            try:
                nvml.nvmlDeviceSetPowerManagementLimit(h, int(rec["power_mw"][0]))
            except Exception:
                pass
        if "clocks" in rec:
            try:
                nvml.nvmlDeviceResetGpuLockedClocks(h)
            except Exception:
                pass
