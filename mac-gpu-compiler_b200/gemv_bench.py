"""Benchmark config 3: the isolated bf16 GEMV microbenchmark.

y = W x with W bf16 ~ N(0, 0.02) [rows x cols], x f32 ~ N(0, 1), at the decode step's shapes:
q [2048x1024], k+v [1024x1024]... o [1024x2048], fused gate+up [6144x1024], down [1024x3072] and
lm_head [151936x1024]. Runs qw_gemv_bf16 — the decode kernel's own weight-streaming GEMV — over
enough distinct copies of W (>= 2x the 126 MB L2) that every launch reads from HBM, and reports
GB/s of the algorithmic bytes R*C*2 + C*4 + R*4 against the measured copy bandwidth, plus the
max-abs error against float64 accumulation (one JSON line per shape).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

import cuda_inference as ci  # noqa: E402

SHAPES = {"q": (2048, 1024), "kv": (1024, 1024), "o": (1024, 2048), "gate_up": (6144, 1024),
          "down": (1024, 3072), "lm_head": (151936, 1024)}
L2_BYTES = 126 << 20


def peak_gbs() -> float:
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return 6650.0


def run(name: str, rows: int, cols: int, iters: int) -> dict:
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    wbytes = rows * cols * 2
    copies = max(2, -(-2 * L2_BYTES // wbytes))
    ws = [(torch.randn(rows, cols, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for _ in range(copies)]
    x = torch.randn(cols, device="cuda", generator=g)
    y = torch.empty(rows, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for i in range(3):
        ci.gemv_bf16(0, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, stream)
    torch.cuda.synchronize()
    ref = ws[2 % copies].double() @ x.double()
    err = float((y.double() - ref).abs().max())
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(iters):
        ci.gemv_bf16(0, ws[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), rows, cols, stream)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    algo = rows * cols * 2 + cols * 4 + rows * 4
    gbs = algo / (ms * 1e-3) / 1e9
    return {"shape": name, "rows": rows, "cols": cols, "us_per_launch": ms * 1e3, "GB_s": gbs,
            "frac_of_measured_copy": gbs / peak_gbs(), "frac_of_8TBs_spec": gbs / 8000.0,
            "max_abs_err_vs_f64": err, "weight_copies": copies}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--shapes", default=",".join(SHAPES))
    a = ap.parse_args()
    for name in a.shapes.split(","):
        print(json.dumps(run(name, *SHAPES[name], a.iters)), flush=True)


if __name__ == "__main__":
    main()
