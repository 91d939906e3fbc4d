"""Writes dc_exp2_table.cuh: 2^(j/64), j = 0..63, as double-double pairs (hi =
the double nearest, lo = the double nearest the remainder), and ln2/64 split
so that k * hi is exact for |k| < 2^17, for the table-driven exp in
dc_math.cuh.  The values come from Python's decimal module at 60 digits (every
step correctly rounded at that precision), converted to the nearest doubles.

    python daisychain-infer_b200/csrc/gen_exp2_table.py
"""
import os
from decimal import Decimal, getcontext

getcontext().prec = 60
HERE = os.path.dirname(os.path.abspath(__file__))


def hexd(v: float) -> str:
    import struct
    return "0x%016XULL" % struct.unpack("<Q", struct.pack("<d", v))[0]


def main() -> None:
    ln2 = Decimal(2).ln()
    rows = []
    for j in range(64):
        t = Decimal(2) ** (Decimal(j) / Decimal(64))
        hi = float(t)
        lo = float(t - Decimal(hi))
        rows.append((hi, lo))
    l64 = ln2 / 64
    # hi: l64 rounded down to a multiple of 2^-42 (at most 36 significant bits)
    hi_l = float(Decimal(int(l64 * (Decimal(2) ** 42))) / (Decimal(2) ** 42))
    lo_l = float(l64 - Decimal(hi_l))
    inv = float(Decimal(64) / ln2)
    out = ["// dc_exp2_table.cuh -- written by gen_exp2_table.py (do not edit).",
           "// 2^(j/64) as double-double (hi, lo) bit patterns, and ln2/64 = hi + lo",
           "// with k * hi exact for |k| < 2^17; 64/ln2 rounded to nearest.  The table",
           "// sits in global memory: kernels copy it to shared memory once.",
           "#pragma once",
           "#include <stdint.h>",
           "namespace dcm {",
           "static __device__ const uint64_t kExp2Tab[64][2] = {"]
    for hi, lo in rows:
        out.append("    {%s, %s}," % (hexd(hi), hexd(lo)))
    out += ["};",
            "constexpr uint64_t kLn2Over64Hi = %s;" % hexd(hi_l),
            "constexpr uint64_t kLn2Over64Lo = %s;" % hexd(lo_l),
            "constexpr uint64_t kInvLn2Times64 = %s;" % hexd(inv),
            "}  // namespace dcm", ""]
    with open(os.path.join(HERE, "dc_exp2_table.cuh"), "w") as f:
        f.write("\n".join(out))


if __name__ == "__main__":
    main()
