"""Measurement helpers shared by bench.py and the layer-pipeline bench: SM clock and
throttle sampling during a timed region, the measured roofline denominators, and the
algorithmic bytes of a decode step."""

from __future__ import annotations

import json
import statistics
import subprocess
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch
        self.sel = None
        try:
            self.sel = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            pass
        self.proc = None

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.sel:
            cmd += ["-i", self.sel]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(dict(sm=float(f[1]), smax=float(f[2]), power=float(f[3]),
                                 hw=f[5], hwt=f[6], swt=f[7], swp=f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows), "sm_max_mhz": rows[0]["smax"],
                "power_w_max": max(r["power"] for r in rows), "reasons": sorted(reasons),
                "samples": len(rows)}


# --------------------------------------------------------------------------- peaks
def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]),
                "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}



def alg_bytes(stack, idx_layers, T) -> tuple[int, list[int]]:
    """Algorithmic bytes of one step and of each gate/up launch: distinct routed experts'
    int4 sections (gate+up for gate/up; all three for the step) + router + activations."""
    import numpy as np
    s = stack.shape
    mat = (s.inter * s.hidden) // 2 + 2 * 2 * (s.inter * s.hidden) // s.group_size
    total, gu = 0, []
    for li in idx_layers:
        d = len(np.unique(li[li >= 0]))
        total += d * 3 * mat + s.n_experts * s.hidden * 2 + T * s.hidden * (2 + 4)
        gu.append(d * 2 * mat + T * s.hidden * 2)
    return total, gu


