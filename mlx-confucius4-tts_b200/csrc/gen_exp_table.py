"""Prints the constants of c4s_exp.cuh: 2^(j/64) for j = 0..63, 64/ln 2 and
ln 2/64 split into a leading double and the rounded remainder, each the
nearest double to the value computed with 80-digit decimal arithmetic."""
from decimal import Decimal, getcontext
from fractions import Fraction

getcontext().prec = 80
ln2 = Decimal(2).ln()


def nearest(x):
    return float(Fraction(x))      # Fraction -> float rounds to nearest


if __name__ == "__main__":
    hi = nearest(ln2 / 64)
    print("INV_LN2_64", nearest(64 / ln2).hex())
    print("LN2_64_HI", hi.hex())
    print("LN2_64_LO", float(Fraction(ln2 / 64) - Fraction(hi)).hex())
    tab = [nearest(Decimal(2) ** (Decimal(j) / 64)) for j in range(64)]
    for j in range(0, 64, 4):
        print("  " + ", ".join(t.hex() for t in tab[j:j + 4]) + ",")
