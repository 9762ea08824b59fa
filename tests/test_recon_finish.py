"""The arithmetic of the reconstruction's finish on the CPU: a step-by-step restatement of recon_pair_kernel
and crt_finish_biased / round_scaled (oztt_b200/csrc/recon.cu), checked against exact rational arithmetic.

The CRT digits are made from a chosen C' as the GEMM epilogue makes them, k_s = C' (M/m_s)^-1 mod m_s (so that
sum_s k_s M/m_s = C' mod M), and every magnitude of C' is reached: the
largest the window margin allows, values whose top words are zero, single units, zero and negatives. The
kernel's result must be C' * 2^e rounded to nearest even in binary64, with results below 2^-1022 flushed
to +-0 (the reference's pack_f64, ozaki2 recon_elem.h) and above the range +-inf. Reference counterpart of
the reconstruction: src/backend/ozaki2/kernels/recon_crt.cpp:219-338.
"""
import math
import random
from fractions import Fraction

import pytest

# the moduli of the 16384^3 metric plan (S = 17, b = 56), a shorter even-S set, and a longer one whose
# product (about 2^150) takes five words, so that C' has halves under the top two
MODULI_17 = [255, 254, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199, 197, 29, 37]
MODULI_8 = [255, 254, 253, 251, 247, 241, 239, 233]
MODULI_20 = MODULI_17 + [193, 191, 181]

TWO52 = 2.0 ** 52
MAGIC = 1.5 * 2.0 ** 52


def fma(a: float, b: float, c: float) -> float:
    """fma(a, b, c) rounded once to nearest even (int / int true division is correctly rounded)."""
    r = Fraction(a) * Fraction(b) + Fraction(c)
    return r.numerator / r.denominator if r else 0.0


def consts(moduli):
    """The constants recon_const derives: M, its words, the pairs' multipliers and limbs, 2^(32 l)/M."""
    M = math.prod(moduli)
    L = max(1, (M.bit_length() + 31) // 32)
    pairs = []
    for p in range((len(moduli) + 1) // 2):
        s0, s1 = 2 * p, 2 * p + 1
        if s1 < len(moduli):
            ms, mt = moduli[s0], moduli[s1]
            pairs.append((ms, mt, ms * mt, M // (ms * mt)))
        else:
            pairs.append((0, 1, moduli[s0], M // moduli[s0]))
    nl = max(1, (max(q for *_, q in pairs).bit_length() + 31) // 32)
    rl = [float(Fraction(2 ** (32 * l), M)) for l in range(max(nl, L))]
    return M, L, nl, pairs, rl


def finish(kvals, moduli, g, two_b):
    """recon_pair_kernel for one element: the pair sums on top of 2^52, then crt_finish_biased."""
    M, L, NL, pairs, rl = consts(moduli)
    kv = list(kvals) + [0]
    lim = [TWO52] * NL
    for p, (ms, mt, mm, qp) in enumerate(pairs):
        u2 = kv[2 * p] * mt + kv[2 * p + 1] * ms
        u = min(u2, (u2 - mm) % 2 ** 32)  # the 32-bit wrap of u2 - mm when u2 < mm
        assert u < mm
        for l in range(NL):
            limb = (qp >> (32 * l)) & 0xFFFFFFFF
            nxt = lim[l] + u * limb  # the fused multiply-add, exact while below 2^53
            assert nxt < 2.0 ** 53 and nxt == int(lim[l]) + u * limb
            lim[l] = float(nxt)
    # q from the limbs l >= L - 3, unbiased exactly
    xm = 0.0
    for l in range(NL - 1, max(L - 3, 0) - 1, -1):
        xm = fma(lim[l] - TWO52, rl[l], xm)
    q = int(xm + MAGIC) & 0xFFFFFFFF  # the low word of the pattern of xm + 1.5 2^52 (an exact integer)
    # C' = X' - q M in L words (two's complement)
    y, cr = [], 0
    for l in range(L):
        v = cr - q * ((M >> (32 * l)) & 0xFFFFFFFF)
        if l < NL:
            v += int(lim[l]) - 2 ** 52
        y.append(v & 0xFFFFFFFF)
        cr = v >> 32
    return round_scaled(y, g, two_b)


def round_scaled(y, g, two_b):
    """round_scaled: sign, the top 64-bit half and the one below it with a sticky bit, one conversion, the
    scale."""
    nw = len(y)
    neg = (y[-1] >> 31) != 0
    if neg:
        c = 1
        for w in range(nw):
            t = ((~y[w]) & 0xFFFFFFFF) + c
            y[w], c = t & 0xFFFFFFFF, t >> 32
    halves = [((y[2 * i + 1] if 2 * i + 1 < nw else 0) << 32) | y[2 * i] for i in range((nw + 1) // 2)]
    hh, t0, t1, a, sticky, below = -1, 0, 0, 0, False, False
    for i, h in enumerate(halves):
        if h:
            hh, t0, t1, sticky = i, h, a, below
        below = below or a != 0
        a = h
    if hh < 0:
        return 0.0
    lz = 64 - t0.bit_length()
    top64 = ((t0 << lz) | (t1 >> (64 - lz))) & (2 ** 64 - 1) if lz else t0
    sticky = sticky or ((t1 << lz) & (2 ** 64 - 1)) != 0
    v = float(top64 | (1 if sticky else 0))  # int -> float rounds to nearest even
    p = 64 * hh + 63 - lz
    lead = p + g - two_b + (1 if v == 2.0 ** 64 else 0)
    if lead < -1022:
        r = 0.0
    elif lead > 1023:
        r = math.inf
    else:
        r = math.ldexp(v, p - 63 + g - two_b)
    return -r if neg else r


def expected(c, g, two_b):
    """C' 2^(g - 2b) rounded once to nearest even; below 2^-1022 -> +-0, above the range -> +-inf."""
    if c == 0:
        return 0.0
    v = float(c)  # C' < 2^127 rounds without overflow
    e = g - two_b
    lead = math.frexp(abs(v))[1] - 1 + e
    if lead < -1022:
        r = 0.0
    elif lead > 1023:
        r = math.inf
    else:
        r = math.ldexp(abs(v), e)
    return -r if v < 0 else r


def digits(c, moduli):
    """The CRT digits of C': k_s = C' (M/m_s)^-1 mod m_s."""
    M = math.prod(moduli)
    return [c * pow(M // m, -1, m) % m for m in moduli]


def cases(M, rng, count):
    """C' values over every magnitude the window allows (|C'| <= M/2 - M 2^-31.4), both signs, and zero."""
    hi = int(Fraction(M, 2) - Fraction(M) * Fraction(2) ** -31) - 1
    out = [0, 1, -1, 2 ** 31, -(2 ** 32), 2 ** 32 - 1, 2 ** 64 + 1, -(2 ** 64) - 1, hi, -hi, 2 ** 52 + 1,
           (2 ** 53 + 1) * 2 ** 40, -((2 ** 53 + 1) * 2 ** 70), (2 ** 53 + 3) * 2 ** 60,  # ties of the rounding
           2 ** 54 - 1, -(2 ** 54 - 1)]  # rounds up to 2^54: at e = -1076 onto 2^-1022, kept
    # exact ties of the rounding to 53 bits, (2^53 + odd) 2^k, and the same one unit above or below in some
    # lower bit j: the bit decides the direction through the sticky bit of the halves under the top two or of
    # the bits shifted out of the second
    for k in (1, 11, 31, 40, 60, 70, 90, 96):
        for j in (0, 5, k - 1):
            if j < 0 or j >= k:
                continue
            for odd in (1, 3, 2 ** 52 - 1):
                base = (2 ** 53 + odd) * 2 ** (k - 1)  # the half-unit bit of the 53-bit rounding set
                out += [base, base + 2 ** j, base - 2 ** j, -(base + 2 ** j), -(base - 2 ** j)]
    for _ in range(count):
        bits = rng.randint(1, hi.bit_length())
        v = rng.getrandbits(bits)
        v = min(v, hi)
        out.append(v if rng.random() < 0.5 else -v)
    return [c for c in out if abs(c) <= hi]


@pytest.mark.parametrize("moduli", [MODULI_17, MODULI_8, MODULI_20], ids=["S17", "S8", "S20"])
def test_finish_matches_exact_rounding(moduli):
    rng = random.Random(20261202)
    M = math.prod(moduli)
    two_b = 112
    for c in cases(M, rng, 400):
        kvals = digits(c, moduli)
        for g in (two_b, two_b - 60, two_b + 40, -900, two_b - 1076, two_b - 1100):
            got = finish(kvals, moduli, g, two_b)
            want = expected(c, g, two_b)
            assert got == want and math.copysign(1.0, got) == math.copysign(1.0, want), (c, g, got, want)


def test_limb_sums_stay_exact_for_the_largest_digits():
    """Every digit at its largest (k_s = m_s - 1) keeps each biased limb sum below 2^53 (asserted inside)."""
    for moduli in (MODULI_17, MODULI_8, [255, 254] * 12):
        kvals = [m - 1 for m in moduli]
        finish(kvals, moduli, 0, 0)
