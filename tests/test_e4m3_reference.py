"""Pins the reference the FP8 tests use: torch's float32 -> float8_e4m3fn
conversion, against an independent restatement of e4m3 (OCP FP8 E4M3: 1 sign,
4 exponent bits with bias 7, 3 mantissa bits, no infinities, 448 the largest
finite value) with round-to-nearest-even.  CPU only."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")


def e4m3_table():
    """(code, value) of the 127 non-negative finite e4m3 codes, ascending."""
    out = []
    for code in range(0x7F):  # 0x7F is NaN
        e, m = code >> 3, code & 7
        v = (m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
        out.append((code, v))
    return out


def rne_e4m3(x: float) -> int:
    """Code of the nearest e4m3 value, ties to the even code (even mantissa)."""
    tab = e4m3_table()
    s = 0x80 if np.signbit(x) else 0
    a = abs(x)
    if a >= 448.0:
        return s | 0x7E if a < 464.0 else None  # beyond the midpoint to 480: not finite
    vals = np.array([v for _, v in tab])
    i = int(np.searchsorted(vals, a))
    if i < len(vals) and vals[i] == a:
        return s | tab[i][0]
    lo, hi = tab[i - 1], tab[i]
    dl, dh = a - lo[1], hi[1] - a
    if dl < dh or (dl == dh and lo[0] % 2 == 0):
        return s | lo[0]
    return s | hi[0]


def test_table_values():
    tab = e4m3_table()
    assert tab[1][1] == 2.0 ** -9 and tab[0x7E][1] == 448.0 and tab[0x08][1] == 2.0 ** -6
    got = torch.tensor([v for _, v in tab], dtype=torch.float32).to(torch.float8_e4m3fn)
    assert got.view(torch.uint8).tolist() == [c for c, _ in tab]


def test_torch_conversion_is_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.exp(rng.uniform(-9, 6, 4000)).astype(np.float32),
        # exact midpoints between neighbouring codes (ties), both signs
        np.array([(a + b) / 2 for (_, a), (_, b) in zip(e4m3_table()[:-1], e4m3_table()[1:])],
                 np.float32),
        -np.array([(a + b) / 2 for (_, a), (_, b) in zip(e4m3_table()[:-1], e4m3_table()[1:])],
                  np.float32),
    ])
    x = x[np.abs(x) <= 448.0]
    got = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    want = np.array([rne_e4m3(float(v)) for v in x], np.uint8)
    assert np.array_equal(got, want)
