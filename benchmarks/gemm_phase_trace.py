"""Per-k-tile phase trace of the tcgen05 GEMM (clock64 stamps of CTAs 0 and 1).

    python benchmarks/gemm_phase_trace.py [gemm3|wgrad3]

Runs the 3xTF32 product of ``profile_kernels.py`` (32768x768 @ 768x2048, or
the weight-gradient (32768x768)^T @ 32768x2048) with ``ext().gemm_trace`` on
and prints, per CTA, the stamps of a few k-tiles and the steady-state medians:
k-tile period of the producer / converter / MMA issuer, TMA latency (issue to
converter), converter time, converter done to MMA start, MMA issue time, and
the epilogue's chunk drain. Clocks are per SM: compare stamps within a CTA.
"""
from __future__ import annotations

import os
import statistics
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from abacus_b200.ops import gemm, precision  # noqa: E402
from abacus_b200.ops._ext import check_status, ext  # noqa: E402

SLOTS = ("tma", "conv_in", "conv_out", "mma_in", "mma_out")


def main() -> None:
    case = sys.argv[1] if len(sys.argv) > 1 else "gemm3"
    precision.set_precision("fp32")
    x = torch.randn(32768, 768, device="cuda")
    other = torch.randn(768, 2048, device="cuda") if case == "gemm3" else torch.randn(32768, 2048, device="cuda")

    def run():
        if case == "gemm3":
            gemm.matmul(x, other)
        else:
            gemm.matmul(x, other, trans_a=True)

    for _ in range(3):
        run()
    buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
    ext().gemm_trace(buf)
    run()
    torch.cuda.synchronize()
    ext().gemm_trace(None)
    check_status()
    t = buf.view(2, 16, 128).cpu()

    def med(values):
        values = [v for v in values if v is not None]
        return statistics.median(values) if values else -1

    for cta in range(2):
        def stamp(slot, i):
            v = t[cta, slot, i].item()
            return v if v else None

        base = t[cta, 0, 0].item()
        print(f"== CTA {cta} ({case}, CTA pairs in the last launch: {ext().gemm_pair_clusters()})")
        print(" kt " + " ".join(f"{s:>8s}" for s in SLOTS))
        for i in list(range(0, 8)) + list(range(40, 48)):
            row = [stamp(s, i) for s in range(5)]
            if row[0] is None:
                continue
            print(f"{i:3d} " + " ".join(f"{(v - base) if v else -1:8d}" for v in row))

        def period(slot):
            v = [stamp(slot, i) for i in range(20, 100)]
            v = [x for x in v if x]
            return med([v[i + 1] - v[i] for i in range(len(v) - 1)])

        def lat(a, b):
            return med([(stamp(b, i) - stamp(a, i)) if stamp(a, i) and stamp(b, i) else None for i in range(20, 100)])

        print(f"period: producer {period(0)} converter {period(2)} mma {period(4)} clk | TMA {lat(0, 1)} "
              f"converter {lat(1, 2)} converted->MMA {lat(2, 3)} MMA issue {lat(3, 4)} clk")
        print(f"converter: A split + TMEM store issue {lat(1, 8)}, B lo {lat(8, 9)}, TMEM store wait {lat(9, 10)}, "
              f"fences {lat(10, 2)} clk; chunk drain {lat(5, 6)} clk")


if __name__ == "__main__":
    main()
