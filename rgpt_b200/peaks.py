"""Roofline denominators: the measured B200 peaks (MEASURED_PEAKS.json at the repo root,
written per GPU pool), else the pool's earlier measurement as a fallback."""
import json
import os

_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "of measured (MEASURED_PEAKS.json)"}
    except (OSError, KeyError, ValueError):
        return dict(_FALLBACK, source="of fallback (no MEASURED_PEAKS.json)")
