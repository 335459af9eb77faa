"""Generates the double constants of splat_atan2f / splat_tanf (aaa.cuh) and
of their CPU restatement (oracle/aaa_oracle.cpp): atan(i/8) for i = 0..8,
1/(2k+1) for the arctangent series and 1/n! for the sine and cosine series,
each the double nearest to its exact value (50-digit decimal arithmetic,
then one correctly rounded conversion).  Run it to print the tables; the
CPU tests check that both sources hold exactly these values."""

from __future__ import annotations

from decimal import Decimal, getcontext
from fractions import Fraction
from math import factorial

getcontext().prec = 60


def _atan(x: Decimal) -> Decimal:
    # two half-angle steps, then the alternating series to 1e-55
    for _ in range(2):
        x = x / (1 + (1 + x * x).sqrt())
    total, term, k, x2 = Decimal(0), x, 0, x * x
    while abs(term) > Decimal(10) ** -58:
        total += term / (2 * k + 1) * (1 if k % 2 == 0 else -1)
        term *= x2
        k += 1
    return 4 * total


def _nearest(value) -> float:
    return float(value)  # Decimal / Fraction -> float rounds to nearest


ATAN_TABLE = [_nearest(_atan(Decimal(i) / 8)) for i in range(9)]
TWO_OVER_PI = _nearest(Decimal(2) / (4 * _atan(Decimal(1))))  # the tangent's reduction
ATAN_SERIES = [_nearest(Fraction(1, 2 * k + 1)) for k in range(8)]   # u^(2k+1) / (2k+1)
SIN_SERIES = [_nearest(Fraction(1, factorial(2 * j + 1))) for j in range(11)]  # r^(2j+1)/(2j+1)!
COS_SERIES = [_nearest(Fraction(1, factorial(2 * j))) for j in range(12)]      # r^(2j)/(2j)!


def tables() -> dict[str, list[float]]:
    return {"kTwoOverPi": [TWO_OVER_PI], "kAtanTable": ATAN_TABLE, "kAtanSeries": ATAN_SERIES, "kSinSeries": SIN_SERIES,
            "kCosSeries": COS_SERIES}


if __name__ == "__main__":
    for name, values in tables().items():
        body = ", ".join(repr(v) for v in values)
        print(f"constexpr double {name}[{len(values)}] = {{{body}}};")
