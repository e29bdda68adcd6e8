"""The division-free code computation of the one-pass quantize+repack kernel
(csrc/prep.cu, codes8), restated in numpy float32 arithmetic and checked on
the CPU against quantize_cpu's per-element rule (src/reference.cu:6-26:
q = clamp(int(rint(x / s)), -8, 7)), for every FP16 x a group with a finite
normal scale s can hold, over a set of scales that includes exact ties. The
GPU test test_quantize_repack_one_pass_matches_three_step compares the kernel
itself with the oracle byte for byte (zero, subnormal and infinite scales,
which the kernel sends to the exact division, included)."""
import numpy as np

import oracle

F = np.float32


def exact_codes(x: np.ndarray, s: np.float32) -> np.ndarray:
    """quantize_cpu's code of each x for scale s (as int, before masking);
    x86's int() of NaN / out-of-range values gives INT_MIN."""
    with np.errstate(all="ignore"):
        q = np.rint(x / s)
        ok = (q >= F(-2147483648.0)) & (q < F(2147483648.0))
        qi = np.where(ok, q, 0).astype(np.int64)
    qi = np.where(ok, qi, -2147483648)
    return np.clip(qi, -8, 7)


def method_codes(x: np.ndarray, s: np.float32):
    """codes8's arithmetic for a finite normal s: (codes, mask of elements
    it decides; the rest take the exact division)."""
    with np.errstate(all="ignore"):
        r = F(1) / s                                        # __frcp_rn
        y = (x * r).astype(F)                               # __fmul2_rn
        t = (y + F(12582912.0)).astype(F)                   # + 1.5 * 2^23
        n = (t - F(12582912.0)).astype(F)
        d = (y - n).astype(F)                               # exact
        decided = np.abs(d) < F(0.5) - F(2.0 ** -18)
    code = (t.view(np.uint32) & 15).astype(np.int64)
    return np.where(code >= 8, code - 16, code), decided


def all_halves() -> np.ndarray:
    return oracle.h2f(np.arange(65536, dtype=np.uint16))


def normal_scales():
    fixed = [1.0, 0.75, 0.5, 1.0 / 7.0, 2.0 ** -14, 6.2e-5, 0.002856, 0.0029, 65504.0, 3.0,
             1.0e-3, 9357.0]
    rng = np.random.default_rng(11)
    rand = rng.uniform(1e-4, 0.02, 40).tolist()
    return [oracle.h2f(oracle.f2h(np.array([v], F)))[0] for v in fixed + rand]


def test_method_equals_quantize_cpu_on_every_half():
    """For a finite normal s = half(vmax / 7), a group holds |x| <= vmax <=
    7 s (1 + 2^-11) or NaN: every such FP16 x is checked."""
    x = all_halves()
    slow = checked = 0
    for s in normal_scales():
        m = np.isnan(x) | (np.abs(x) <= F(7.004) * s)
        want = exact_codes(x[m], s)
        got, decided = method_codes(x[m], s)
        assert np.array_equal(got[decided], want[decided]), float(s)
        nan = np.isnan(x[m])
        assert not decided[nan].any()   # NaN always takes the division
        slow += int((~decided[~nan]).sum())
        checked += int((~nan).sum())
    # apart from NaN (2046 of the FP16 codes), the exact division is rare
    assert checked > 100000 and slow < 0.001 * checked, (slow, checked)


def test_method_matches_the_oracle_quantizer():
    """End to end on a weight matrix with planted ties and a zero group:
    codes from the method where the scale is finite normal and it decides,
    the exact rule elsewhere, equal oracle.quantize's."""
    K, N, g = 256, 64, 32
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((K, N)) * 0.02).astype(F)
    pattern = [5.25] + [(-1) ** k * (k + 0.5) * 0.75 for k in range(7)]
    w[:, 7] = [pattern[i % len(pattern)] for i in range(K)]   # s = 0.75, exact ties
    w[:, 8] = [((i % 29) - 14) * 0.5 for i in range(K)]        # s = 1, exact ties
    w[0:32, 9] = 0.0                                            # zero scale
    w[32:64, 10] = 2.0 ** -20                                   # subnormal scale
    w16 = oracle.f2h(w)
    packed, scales = oracle.quantize(w16, K, N, g)
    xs = oracle.h2f(w16).reshape(K, N)
    sc = oracle.h2f(scales).reshape(K // g, N)
    codes = np.empty((K, N), np.int64)
    slow = 0
    for gi in range(K // g):
        for n in range(N):
            x, s = xs[gi * g:(gi + 1) * g, n], sc[gi, n]
            if 2.0 ** -14 <= s <= 65504.0:
                c, dec = method_codes(x, s)
                c[~dec] = exact_codes(x[~dec], s)
                slow += int((~dec).sum())
            else:
                c = exact_codes(x, s)
            codes[gi * g:(gi + 1) * g, n] = c
    nib = (codes & 15).astype(np.uint8).reshape(K, N // 2, 2)
    mine = nib[:, :, 0] | (nib[:, :, 1] << 4)
    np.testing.assert_array_equal(mine.reshape(-1), packed)
    assert slow > 0  # the planted ties reach the exact division
