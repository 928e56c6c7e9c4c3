"""The operand splits the tensor-core kernels rely on, checked on the CPU with
an exact bf16 restatement (round to nearest even on the fp32 bits):

* the list scan's two-way split x = x_hi + x_lo + e, x_hi = bf16(x),
  x_lo = bf16(x - x_hi): |x - x_hi| is at most half a bf16 ulp of x, and the
  rounding of x_lo at most half a bf16 ulp of that, so |e| <= 2^-17 |x|;
  the four products of (x_hi + x_lo)(q_hi + q_lo) are then within 2^-16 (plus
  2^-34) of x q;
* every bf16 x bf16 product is exact in fp32 (8 + 8 significant bits).
"""
import numpy as np


def bf16_rn(x):
    """x (float32) rounded to the nearest bf16 value, ties to even, as float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return r.astype(np.uint32).view(np.float32)


def split(x):
    hi = bf16_rn(x)
    lo = bf16_rn((x - hi).astype(np.float32))
    return hi, lo


def sample(rng, n):
    # magnitudes over many binades, both signs, plus values near bf16 rounding ties
    m = rng.standard_normal(n) * np.exp2(rng.integers(-30, 30, n))
    x = m.astype(np.float32)
    ties = (bf16_rn(x[: n // 8]).view(np.uint32) + np.uint32(0x8000)).view(np.float32)
    x[: n // 8] = ties
    return x


def test_two_way_split_error():
    rng = np.random.default_rng(0)
    x = sample(rng, 1 << 20)
    hi, lo = split(x)
    e = np.abs(x.astype(np.float64) - hi.astype(np.float64) - lo.astype(np.float64))
    assert np.all(e <= 2.0 ** -17 * np.abs(x.astype(np.float64)))
    assert np.all(bf16_rn(hi) == hi) and np.all(bf16_rn(lo) == lo)


def test_products_of_split_operands():
    rng = np.random.default_rng(1)
    x, q = sample(rng, 1 << 18), sample(rng, 1 << 18)
    xh, xl = split(x)
    qh, ql = split(q)
    exact = x.astype(np.float64) * q.astype(np.float64)
    four = sum(a.astype(np.float64) * b.astype(np.float64)
               for a in (xh, xl) for b in (qh, ql))
    assert np.all(np.abs(four - exact) <= (2.0 ** -16 + 2.0 ** -34) * np.abs(exact))
    # each bf16 x bf16 product is representable in fp32
    for a in (xh, xl):
        for b in (qh, ql):
            p64 = a.astype(np.float64) * b.astype(np.float64)
            assert np.all(p64.astype(np.float32).astype(np.float64) == p64)


def test_coarse_gemm_three_products():
    """The coarse GEMM's operands [hi | hi | lo] . [hi | lo | hi] leave out lo lo
    (|lo| <= 2^-8 |x|): hi hi + hi lo + lo hi is within 2^-16 + 2 * 2^-17 (+2^-34)
    of x q, inside the 3.02 * 2^-16 its error bound allows for representation."""
    rng = np.random.default_rng(2)
    x, q = sample(rng, 1 << 20), sample(rng, 1 << 20)
    xh, xl = split(x)
    qh, ql = split(q)
    f = lambda a: a.astype(np.float64)  # noqa: E731
    exact = f(x) * f(q)
    three = f(xh) * f(qh) + f(xh) * f(ql) + f(xl) * f(qh)
    bound = (2.0 ** -16 + 2 * 2.0 ** -17 + 2.0 ** -34) * np.abs(exact)
    assert np.all(np.abs(three - exact) <= bound)
    assert 2.0 ** -16 + 2 * 2.0 ** -17 + 2.0 ** -34 <= 3.02 * 2.0 ** -16
