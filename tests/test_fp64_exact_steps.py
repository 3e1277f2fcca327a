"""Exact model of the fp64 steps the integer kernels use, checked against the oracle. CPU only.

The kernels get floored fixed-point products from one fp64 FMA rounded toward minus infinity:
with a, b exact doubles, fma_rd(a, b, 1.5 * 2^52) = 1.5 * 2^52 + floor(a b) whenever
|floor(a b)| < 2^51, because every double in [2^52, 2^53) is an integer and IEEE 754 rounds the exact
a b + 1.5 * 2^52 once. Here that step is modelled as floor(Fraction(a) * Fraction(b)) with the
window checked, plain double arithmetic is Python's (IEEE round to nearest), and the algorithms of
k_pv (k_attn.cu), exp_taylor30_fp / ln2_reduce / silu_gate30 / muldiv_trunc (slx_device.cuh) and
the softmax's p_div are restated on top, then compared with the reference's Int128 arithmetic
(the oracle's FixedExp, FixedSiLU, and exact integer division).
"""
import math
import random
from fractions import Fraction

import numpy as np

WINDOW = 1 << 51
LN2 = 744261117  # (long)(0.6931471805599453 * 2^30)


def rd_floor(a: float, b: float, base: int = 0) -> int:
    """fma_rd(a, b, 1.5 * 2^52 + base) - 1.5 * 2^52, for base an integer."""
    v = base + math.floor(Fraction(a) * Fraction(b))
    assert -WINDOW < v < WINDOW, "outside the exact window"
    return v


def fma_rn_exact(a: float, b: float, c: float) -> float:
    """fma_rn when the exact result is representable (the kernels use it only so)."""
    exact = Fraction(a) * Fraction(b) + Fraction(c)
    out = float(exact)
    assert Fraction(out) == exact
    return out


def umulhi(a: int, b: int) -> int:
    return (a * b) >> 32


def exp_taylor30(r: int) -> int:
    """The all-integer form: term_n = floor(floor(t r / 2^30) / n) by multiply-high constants."""
    r4 = r << 2
    t, s = r, (1 << 30) + r
    t = umulhi(t, r4) >> 1; s += t
    t = umulhi(umulhi(t, r4), 1431655766); s += t
    t = umulhi(t, r4) >> 2; s += t
    t = umulhi(umulhi(t, r4), 858993460); s += t
    t = umulhi(umulhi(t, r4), 715827883); s += t
    t = umulhi(umulhi(t, r4), 613566757); s += t
    t = umulhi(t, r4) >> 3; s += t
    t = umulhi(umulhi(t, r4), 477218589); s += t
    t = umulhi(umulhi(t, r4), 429496730); s += t
    return s & 0xFFFFFFFF


def exp_taylor30_fp(r: int) -> int:
    """exp_taylor30_fp: floor(t r / 2^30) (and the terms n = 2, 4, 8) as rounded-down FMAs."""
    rd = float(r)
    r4 = r << 2
    r30 = rd * 2.0 ** -30
    s = (1 << 30) + r
    y = rd_floor(rd, rd * 2.0 ** -31); t = y; s += t                       # n = 2
    t = umulhi(umulhi(t, r4), 1431655766); s += t                           # n = 3
    y = rd_floor(float(t), rd * 2.0 ** -32); t = y; s += t                  # n = 4
    y = rd_floor(float(y), r30); t = umulhi(y, 858993460); s += t           # n = 5
    y = rd_floor(float(t), r30); t = umulhi(y, 715827883); s += t           # n = 6
    t = umulhi(umulhi(t, r4), 613566757); s += t                            # n = 7
    y = rd_floor(float(t), rd * 2.0 ** -33); t = y; s += t                  # n = 8
    y = rd_floor(float(y), r30); t = umulhi(y, 477218589); s += t           # n = 9
    y = rd_floor(float(t), r30); t = umulhi(y, 429496730); s += t           # n = 10
    return s & 0xFFFFFFFF


def ln2_reduce(y: int):
    """k = floor(y / ln2) and r = y - k ln2 from an fp64 estimate fixed by the exact remainder."""
    yd = float(y)
    assert Fraction(yd) == y
    k1 = rd_floor(yd, 1.0 / float(LN2))
    r = fma_rn_exact(-float(k1), float(LN2), yd)
    k = k1
    if r < 0.0:
        k -= 1; r += float(LN2)
    elif r >= float(LN2):
        k += 1; r -= float(LN2)
    return k, int(r)


def exp_nonpos30(x: int) -> int:
    if x < -30 * LN2:
        return 0
    k, r = ln2_reduce(x)
    return exp_taylor30_fp(r) >> -k


def p_div(e: int, total: int) -> int:
    """k_attn.cu p_div: the floor of the fp64 product, checked by the exact remainder only when the
    product lies within 2^-22 of an integer."""
    inv30 = 1073741824.0 / float(total)
    q = rd_floor(float(e), inv30)
    frac = float(Fraction(e) * Fraction(inv30) - q)  # fma_rn(e, inv30, -q)
    if frac < 2.0 ** -22 or frac > 1.0 - 2.0 ** -22:
        rem = (e << 30) - q * total
        if rem < 0:
            q -= 1
        elif rem >= total:
            q += 1
    return q


def muldiv_trunc(a: int, w: int, d: int) -> int:
    """slx_device.cuh muldiv_trunc: the floor of the fp64 quotient, checked by the exact remainder
    only when the quotient lies within (q + 1) 2^-50 of an integer."""
    lim = 1 << 51
    if -lim < a < lim and -lim < w < lim and d < (1 << 60):
        rd = 1.0 / float(d)
        P = abs(float(a) * float(w))
        q = rd_floor(P, rd) if P * rd < 2.0 ** 50 else None
        if q is not None and q < (1 << 49):
            frac = float(Fraction(P) * Fraction(rd) - q)  # fma_rn(P, rd, -q)
            tol = (q + 1) * 2.0 ** -50
            if frac < tol or frac > 1.0 - tol:
                rem = abs(a) * abs(w) - q * d  # the kernel's wrapping 64-bit value, exact since |rem| < 2 d
                assert abs(rem) < 2 * d
                while rem < 0:
                    q -= 1; rem += d
                while rem >= d:
                    q += 1; rem -= d
            return -q if (a < 0) != (w < 0) else q
    p = a * w
    return -(abs(p) // d) if p < 0 else p // d


def silu_gate30(g: int, u: int) -> int:
    one, thr = 1 << 30, 20 << 30
    if g > thr:
        s = g
    elif g < -thr:
        s = 0
    else:
        k, r = ln2_reduce(-g)
        total = exp_taylor30_fp(r)
        e = total << k if k >= 0 else total >> -k
        den = one + e
        den_d = fma_rn_exact(float(total), 2.0 ** k, 1073741824.0) if k >= 0 else float(den)
        assert Fraction(den_d) == den
        rcp = 1.0 / den_d
        q = rd_floor(2.0 ** 60, rcp)
        frac = float(Fraction(2 ** 60) * Fraction(rcp) - q)  # fma_rn(2^60, rcp, -q)
        if frac < 2.0 ** -22 or frac > 1.0 - 2.0 ** -22:
            rem = (1 << 60) - q * den
            while rem < 0:
                q -= 1; rem += den
            while rem >= den:
                q += 1; rem -= den
        s = rd_floor(float(g), float(q) * 2.0 ** -30)
    lim = 1 << 51
    if -lim < s < lim and -lim < u < lim and abs(float(s) * float(u)) < 2.0 ** 80:
        return rd_floor(float(s), float(u) * 2.0 ** -30)
    return (s * u) >> 30


def test_split_taylor_equals_integer_recurrence():
    rng = random.Random(1)
    rs = list(range(0, 4096)) + [LN2 - 1 - i for i in range(4096)] + [rng.randrange(LN2) for _ in range(20000)]
    for r in rs:
        assert exp_taylor30_fp(r) == exp_taylor30(r), r


def test_softmax_exp_matches_fixed_exp(oracle):
    rng = random.Random(2)
    xs = [0, -1, -LN2, -LN2 + 1, -LN2 - 1, -30 * LN2, -30 * LN2 - 1]
    xs += [-c * LN2 + d for c in range(31) for d in (-2, -1, 0, 1, 2) if -c * LN2 + d <= 0]
    xs += [-rng.randrange(30 * LN2 + 100) for _ in range(6000)]
    for x in xs:
        assert exp_nonpos30(x) == oracle.fixed_exp(x), x


def test_softmax_division(oracle):
    rng = random.Random(3)
    for _ in range(3000):
        n = rng.randrange(1, 600)
        es = [oracle.fixed_exp(-rng.randrange(12 * LN2)) for _ in range(n)]
        total = sum(es)
        if total == 0:
            continue
        for e in es[:20]:
            assert p_div(e, total) == (e << 30) // total
    # extremes: one key takes everything, a sum of one, sums near the 2^41 bound
    for e, total in [(1 << 30, 1 << 30), (1, 1), (0, 1), ((1 << 30) - 1, (1 << 41) - 1), (1 << 30, (1 << 41) - 1),
                     (12345, 12346), ((1 << 30), (1 << 30) + 1)]:
        assert p_div(e, total) == (e << 30) // total, (e, total)
    # quotients within 2^-22 of an integer k (total = e 2^30 / k rounded, +-1), where the fp64 product
    # alone can round across k: every one takes the remainder check, and some need its correction
    wrong = 0
    for _ in range(6000):
        m = rng.randrange(1 << 6, 1 << 11)
        k = rng.randrange(1, m << 6)
        e = k * m + rng.randrange(0, k)
        base = (e << 30) // k
        for total in (base - 1, base, base + 1):
            if e > (1 << 30) or total < e or total >= (1 << 41):
                continue
            inv30 = 1073741824.0 / float(total)
            wrong += rd_floor(float(e), inv30) != (e << 30) // total
            assert p_div(e, total) == (e << 30) // total, (e, total)
    assert wrong > 0  # the fast product alone is not enough there


def test_norm_division_matches_int128():
    rng = random.Random(4)
    cases = [(0, 5, 3), (-7, 3, 2), (7, -3, 2), ((1 << 51) - 1, (1 << 51) - 1, (1 << 60) - 1), (1 << 51, 3, 5),
             (-(1 << 40), 1 << 30, (1 << 30) + 1), (123456789, -987654321, 1)]
    for _ in range(40000):
        cases.append((rng.getrandbits(64) - (1 << 63) >> rng.randrange(63), rng.getrandbits(64) - (1 << 63) >> rng.randrange(63),
                      1 + (rng.getrandbits(63) >> rng.randrange(63))))
        isq = 1 + rng.randrange(1 << 36)
        cases.append((rng.randrange(-(1 << 40), 1 << 40), rng.randrange(-(1 << 31), 1 << 31), isq))
    for a, w, d in cases:
        p = a * w
        want = -(abs(p) // d) if p < 0 else p // d
        assert muldiv_trunc(a, w, d) == want, (a, w, d)


def test_norm_division_near_integers():
    """Quotients a w / d just around an integer k (d = floor(a w / k) + {-1, 0, 1}), from k = 1 to
    2^48: every one takes the remainder check, and at the large ones the fp64 quotient alone rounds
    across k."""
    rng = random.Random(14)
    wrong = checked = 0
    for _ in range(12000):
        a = rng.randrange(1, 1 << rng.randrange(1, 51))
        w = rng.randrange(1, 1 << rng.randrange(1, 51))
        k = rng.randrange(1, 1 << rng.randrange(1, 49))
        p = a * w
        for d in (p // k - 1, p // k, p // k + 1):
            if not 1 <= d < (1 << 60) or p // d >= (1 << 49):
                continue
            for sa, sw in ((1, 1), (-1, 1), (1, -1)):
                pp = sa * a * sw * w
                want = -(abs(pp) // d) if pp < 0 else pp // d
                assert muldiv_trunc(sa * a, sw * w, d) == want, (sa * a, sw * w, d)
            checked += 1
            wrong += rd_floor(abs(float(a) * float(w)), 1.0 / float(d)) != p // d
    assert checked > 10000
    assert wrong > 0  # the fast quotient alone is not enough there


def test_silu_gate_matches_fixed_silu(oracle):
    rng = random.Random(5)
    thr = 20 << 30
    gs = [0, 1, -1, thr, thr + 1, -thr, -thr - 1, thr - 1, -thr + 1, 1 << 51, -(1 << 51), LN2, -LN2, 5 << 30,
          (1 << 62), -(1 << 62)]
    us = [0, 1, -1, 1 << 30, -(1 << 30), (1 << 51) - 1, -(1 << 51) + 1, 1 << 51, (1 << 62), -(1 << 62), 123456789012]
    pairs = [(g, u) for g in gs for u in us]
    pairs += [(rng.randrange(-thr - 1000, thr + 1000), rng.getrandbits(64) - (1 << 63) >> rng.randrange(64))
              for _ in range(4000)]
    for g, u in pairs:
        want = (oracle.fixed_silu(g) * u) >> 30
        want = (want + (1 << 63)) % (1 << 64) - (1 << 63)  # the reference's (long) of the Int128
        got = silu_gate30(g, u)
        got = (got + (1 << 63)) % (1 << 64) - (1 << 63)
        assert got == want, (g, u)


def test_pv_window_holds_for_softmax_weights():
    """The P.V accumulator stays inside [2^52, 2^53): sum_s p_s <= 2^30 and |v| < 2^50 bound every
    partial sum of floor(p v / 2^30) by |v|max + T < 2^51; the chained floors equal the reference's
    per-term (long)((Int128)p v >> 30) sums."""
    rng = np.random.default_rng(6)
    for T in (1, 7, 512, 2000):
        e = rng.integers(0, 1 << 30, T)
        p = (e.astype(object) << 30) // int(e.sum()) if e.sum() else np.full(T, (1 << 30) // T, dtype=object)
        assert sum(p) <= 1 << 30
        v = [int(x) for x in rng.integers(-(1 << 50), 1 << 50, T)]
        v[0] = (1 << 50) - 1
        acc = 0
        for ps, vs in zip(p, v):
            acc = rd_floor(float(ps), float(vs) * 2.0 ** -30, acc)
        assert acc == sum((int(ps) * vs) >> 30 for ps, vs in zip(p, v))
