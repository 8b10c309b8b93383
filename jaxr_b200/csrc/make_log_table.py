"""Writes log_table.h: the 128-entry table of the samplers' table-driven logarithm.

The float64 normal sampler needs w = -log(t), t = 1 - x*x in (0, 1], to an absolute
accuracy well below 1e-15 (it is held to 1e-12 relative), and the float32 and 16-bit
samplers need logarithms accurate enough to round to the same float as the exact value
(within ~1e-16 relative; their inputs sit at least 1.2e-14 from a float rounding
boundary).  The logarithm (log_tab_core, samplers.cuh) takes the table-driven method of
P. T. P. Tang, "Table-driven implementation of the logarithm function in IEEE
floating-point arithmetic", ACM TOMS 16(4), 1990: t = 2^k z with z in [0.75, 1.5); the
top 7 bits of z above 0.75 pick an interval of width 2^-8 (z < 1) or 2^-7 (z >= 1) with
midpoint c (c = 1 for the two intervals next to 1); for inv = 1/c rounded to double,
    log t = k log 2 + log(1 / inv) + log1p(z inv - 1),   |z inv - 1| < 2^-7,
where z inv - 1 is one fused multiply-add and log1p is a degree-7 Taylor polynomial
(truncation below 2e-18, and below 5e-20 away from the two intervals next to 1).  Each
entry holds (inv, -log(inv)), the logarithm evaluated in 60-digit arithmetic (mpmath) and
rounded once, so the identity holds for the stored inv.

    python jaxr_b200/csrc/make_log_table.py      # rewrites log_table.h beside this file
"""

from __future__ import annotations

import os

import mpmath

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "log_table.h")
N = 128


def entries():
    mpmath.mp.dps = 60
    rows = []
    for i in range(N):
        if i < 64:  # z in [0.75, 1): intervals of 2^-8
            lo, width = mpmath.mpf(3) / 4 + i * mpmath.mpf(2) ** -8, mpmath.mpf(2) ** -8
        else:  # z in [1, 1.5): intervals of 2^-7
            lo, width = 1 + (i - 64) * mpmath.mpf(2) ** -7, mpmath.mpf(2) ** -7
        # the two intervals next to 1 take c = 1 exactly (inv = 1, log = 0): there
        # z inv - 1 = z - 1 is exact, so log t keeps its full relative accuracy as t -> 1
        # and log 1 is exactly 0; |z - 1| < 2^-7 still bounds the polynomial's argument
        c = mpmath.mpf(1) if i in (63, 64) else lo + width / 2
        inv = float(1 / c)  # rounded to double
        neg_log_inv = float(-mpmath.log(mpmath.mpf(inv)))
        rows.append((inv, neg_log_inv))
    return rows


def main():
    lines = [
        "/* (1 / c, -log(1 / c)) for the 128 intervals of z in [0.75, 1.5) that the samplers'",
        " * table-driven logarithm (log_tab_core, samplers.cuh) reads: 64 of width 2^-8",
        " * below 1, 64 of width 2^-7 above; c is the interval's midpoint (1 for the two next",
        " * to 1, where log 1 must be exactly 0), 1 / c is rounded to",
        " * double and -log(1 / c) is computed in 60-digit arithmetic and rounded once.",
        " * Written by make_log_table.py; do not edit. */",
        "#pragma once",
        "",
        "#define JXR_LOG_TABLE_N 128",
        "#define JXR_LOG_TABLE \\",
    ]
    rows = entries()
    for i, (inv, nl) in enumerate(rows):
        sep = ", \\" if i + 1 < len(rows) else ""
        lines.append(f"  {{{inv.hex()}, {nl.hex()}}}{sep}")
    with open(OUT, "w") as f:
        f.write("\n".join(lines) + "\n")
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
