"""Fine-grid effective-L2-capacity (C_eff) measurement on one B200.

Port of profiling/portable/cliff_finegrain.py:30-89: the coarse 14-point grid of
measure_params.c_eff (0.4..1.5 x nominal L2) can only place the residency cliff
in one of a fixed set of cells, so this sweep re-reads the warm re-read
bandwidth (measure_params.read_bw, graph-timed) at 0.5 MB steps between 0.55 and
1.0 x nominal L2, three repeats. Same detection rule as the reference: the first
size more than 5 % below the running maximum is the break; C_eff is the midpoint
of the argmax and the break.

    python cache-barrier_b200/harness/cliff_finegrain.py --out cliff_finegrain_b200.json
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

from common import ClockSampler, gpu_info, save_json  # noqa: E402
from measure_params import read_bw  # noqa: E402

STEP_MB = 0.5
REPEATS = 3


def detect(points):
    """(C_eff, argmax, break): the first point > 5 % below the running maximum."""
    run_max, m_max = 0.0, None
    for m, b in points:
        if b > run_max:
            run_max, m_max = b, m
        elif b < 0.95 * run_max:
            return (m_max + m) / 2, m_max, m
    return None, m_max, None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--step-mb", type=float, default=STEP_MB)
    ap.add_argument("--repeats", type=int, default=REPEATS)
    args = ap.parse_args()
    torch.manual_seed(0)
    props = torch.cuda.get_device_properties(0)
    l2_mb = props.L2_cache_size / 2**20
    lo, hi = 0.55 * l2_mb, 1.0 * l2_mb
    print(f"{props.name}: nominal L2 {l2_mb:.1f} MB, sweep {lo:.1f}-{hi:.1f} MB at {args.step_mb} MB, "
          f"{args.repeats} repeats", flush=True)
    runs = []
    with ClockSampler(0) as clk:
        for rep in range(args.repeats):
            pts = []
            mb = lo
            while mb <= hi + 1e-9:
                bw = read_bw(mb)
                bw = bw[0] if isinstance(bw, tuple) else bw
                pts.append((round(mb, 2), round(float(bw), 3)))
                mb += args.step_mb
            c, m_arg, m_brk = detect(pts)
            runs.append({"c_eff_mb": round(c, 2) if c else None, "argmax_mb": m_arg, "break_mb": m_brk,
                         "ratio": round(c / l2_mb, 4) if c else None, "points": pts})
            print(f"rep {rep}: C_eff {runs[-1]['c_eff_mb']} MB (argmax {m_arg}, break {m_brk})", flush=True)
    vals = sorted(r["c_eff_mb"] for r in runs if r["c_eff_mb"] is not None)
    med = vals[len(vals) // 2] if vals else None
    out = {"experiment": "cliff_finegrain", "gpu": gpu_info(), "nominal_l2_mb": round(l2_mb, 1),
           "step_mb": args.step_mb,
           "detection": "first point > 5 % below the running max; C_eff = midpoint of argmax and break",
           "runs": runs, "c_eff_mb_median": med, "ratio_median": round(med / l2_mb, 4) if med else None,
           "clocks": clk.info}
    print(f"median C_eff {med} MB", flush=True)
    if args.out:
        save_json(args.out, out)


if __name__ == "__main__":
    main()
