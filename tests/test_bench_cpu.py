"""Host-side pieces of bench.py that need no GPU: the clock sampler's windowing and reason decoding
(against a fake NVML), and the JSON contract keys of the reference arm's line."""

import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


class FakeNVML:
    NVML_CLOCK_SM = 1

    def __init__(self, reasons_after=None):
        self.t0 = None
        self.reasons_after = reasons_after
        self.closed = False

    def nvmlInit(self):
        self.t0 = time.perf_counter()

    def nvmlShutdown(self):
        self.closed = True

    def nvmlDeviceGetHandleByUUID(self, u):
        assert u.startswith("GPU-")
        return "h"

    def nvmlDeviceGetHandleByIndex(self, i):
        return "h"

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, kind):
        return 1965 if self.reasons_after is None else 1800

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4 | 0x40 if self.reasons_after is not None else 0


def test_clock_sampler_window_and_reasons():
    import bench

    nv = FakeNVML()
    with bench.ClockSampler(0, "0123", nvml=nv) as clk:
        time.sleep(0.02)  # idle samples before the region are not counted
        with clk.window():
            time.sleep(0.05)
        time.sleep(0.02)
    s = clk.summary()
    assert nv.closed
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965 and s["reasons"] == []
    assert 3 <= s["samples"] < len(clk.samples)
    assert all(clk.win[0] <= t <= clk.win[1] for t, _, _ in clk.samples[:0])

    nv = FakeNVML(reasons_after=0)
    with bench.ClockSampler(0, None, nvml=nv) as clk:
        with clk.window():
            time.sleep(0.03)
    s = clk.summary()
    assert s["sm_mhz"] == 1800 and s["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_clock_sampler_without_nvml_or_smi(monkeypatch):
    """No NVML and no nvidia-smi: the summary says so instead of raising."""
    import subprocess

    import bench

    class Broken(FakeNVML):
        def nvmlInit(self):
            raise RuntimeError("no driver")

    def no_smi(*a, **k):
        raise FileNotFoundError("nvidia-smi")

    monkeypatch.setattr(subprocess, "Popen", no_smi)
    with bench.ClockSampler(0, None, nvml=Broken()) as clk:
        with clk.window():
            pass
    s = clk.summary()
    assert s["samples"] == 0 and s["sm_mhz"] is None


def test_compositing_rooflines_arithmetic():
    """Forward: 3 SFU ops per pixel-pair against 148 x 16 MUFU per clock; backward: 40 FP32 ops against
    148 x 128 lanes; frac = roofline time / measured time."""
    import bench

    r = bench.compositing_rooflines({"fields_fwd": {"ms_per_replay": 0.05}, "fields_bwd": {"ms_per_replay": 0.1}},
                                    pairs=1000, f_mhz=1000.0)
    pp = 64000
    assert r["pixel_pairs"] == pp
    f, b = r["fields_fwd"], r["fields_bwd"]
    assert f["bound"] == "sfu" and abs(f["roofline_ms"] - pp * 3 / (148 * 16 * 1e9) * 1e3) < 1e-15
    assert abs(f["frac"] - f["roofline_ms"] / 0.05) < 1e-12
    assert b["bound"] == "fp32" and abs(b["roofline_ms"] - pp * 40 / (148 * 128 * 1e9) * 1e3) < 1e-15
    assert "fields_fwd" not in bench.compositing_rooflines({}, pairs=10, f_mhz=1965.0)


def test_binning_roofline_arithmetic():
    """Octave tile counts (768^2 -> 12,289 tiles; 384^2 -> 3,074, the grids of the two renders) and the
    algorithmic bytes N*36 + N*4 + pairs*8 + (tiles+1)*4 over the binning stage time."""
    import bench

    assert bench.octave_tiles(768, 768) == 12289 and bench.octave_tiles(384, 384) == 3074
    r = bench.binning_roofline({"binning": {"ms_per_replay": 0.1}}, pairs=1000, N=100, H=768, W=768, hbm_gbs=1000.0)
    nbytes = 100 * 40 + 1000 * 8 + 12290 * 4
    assert r["algorithmic_bytes"] == nbytes
    assert abs(r["achieved_gbs"] - nbytes / 1e-4 / 1e9) < 1e-9 and abs(r["frac"] - r["achieved_gbs"] / 1000.0) < 1e-12
    assert bench.binning_roofline({}, 1000, 100, 768, 768, 1000.0) is None


def test_reference_arm_line():
    """`bench.py --impl reference` (host CPU, no GPU): one JSON line with the contract's keys, the same
    metric/unit/scaling as our arm's line for the workload, and an e2e entry with no host-device bytes."""
    import json
    import subprocess

    import bench

    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "render",
                        "--steps", "1", "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference" and line["value"] > 0 and line["warmup"] >= 3
    assert (line["metric"], line["unit"], line["scaling"]) == (bench.RenderWorkload.metric, "images/s", "weak")
    assert line["config"]["splats"] == 92160 and line["config"]["H"] == 768
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and "render fwd+bwd" in cb["sample"]
