"""Writes erfinv_tables.h: the coefficients of the accurate erf_inv (the lowering of erf_inv
when jax_accurate_erf_inv is set, R/lax_special.R:1022-1082).

The coefficients are Sollya fits that JAX ships in jax/_src/lax/erf.py; the reference holds
them as exact hexadecimal literals in `sp_erf_tables` (R/lax_special.R:641-): ERFINV32_P1,
ERFINV32_P2 (float32, w < 3.5 and w >= 3.5) and ERFINV64_P1 .. ERFINV64_P3 (float64,
w < 4.5, 4.5 <= w < 16, w >= 16), lowest degree first.  The accurate erf_inv of the
samplers has no far-tail pieces, so the others are not used.  Results match the
reference's only with these exact values, so they are read from its source as text, as
tests/golden/make_golden.py reads the recorded samples; the header is committed.

    python jaxr_b200/csrc/make_erfinv_tables.py JAXR_SOURCE_DIR   # or $JAXR_REFERENCE_DIR
"""

from __future__ import annotations

import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "erfinv_tables.h")
sys.path.insert(0, os.path.join(HERE, "..", "..", "tests", "golden"))

from make_golden import _balanced, read_r  # noqa: E402

TABLES = ["ERFINV32_P1", "ERFINV32_P2", "ERFINV64_P1", "ERFINV64_P2", "ERFINV64_P3"]


def read_tables(ref):
    path = os.path.join(ref, "R", "lax_special.R")
    text = open(path).read()
    out = {}
    for name in TABLES:
        m = re.search(rf"\b{name} = c\(", text)
        start = m.end() - 2
        vals = read_r(text[start:_balanced(text, start + 1)])
        out[name] = (vals, text.count("\n", 0, m.start()) + 1)
    return out


def literal(v, single):
    h = float(v).hex()
    if single:
        assert float(v) == float(__import__("numpy").float32(v)), v
        return h + "f"
    return h


def main(argv):
    ref = argv[1] if len(argv) > 1 else os.environ.get("JAXR_REFERENCE_DIR")
    if not ref:
        sys.exit(f"usage: {argv[0]} JAXR_SOURCE_DIR (or set $JAXR_REFERENCE_DIR): the root "
                 "of the jaxR source tree to read")
    tables = read_tables(ref)
    lines = [
        "/* Coefficients of the accurate erf_inv (jax_accurate_erf_inv), lowest degree first:",
        " * JAX's Sollya fits (jax/_src/lax/erf.py) as the reference holds them in",
        " * R/lax_special.R sp_erf_tables.  Written by make_erfinv_tables.py; do not edit. */",
        "#pragma once",
        "",
    ]
    for name in TABLES:
        vals, line = tables[name]
        single = name.startswith("ERFINV32")
        body = ", ".join(literal(v, single) for v in vals)
        lines.append(f"/* {name}: {len(vals)} coefficients, R/lax_special.R:{line} */")
        lines.append(f"#define JXR_{name} {body}")
        lines.append(f"#define JXR_{name}_N {len(vals)}")
        lines.append("")
    with open(OUT, "w") as f:
        f.write("\n".join(lines))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main(sys.argv)
