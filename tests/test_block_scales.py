"""Host-side checks of the adversarial block-scale builders the GPU byte tests use, and of the
checker's exact-range test (xref_q4b_check) at the bound's edge. No GPU."""
import numpy as np
import pytest

import spmodel


def test_f16_k_round_trip_every_finite_pattern():
    for h in range(1 << 16):
        if ((h >> 10) & 31) == 31:
            continue
        k = spmodel.f16_k(h)
        back = spmodel.k_to_f16(k)
        # -0 and +0 are the same integer; every other pattern comes back unchanged
        assert back == h or (k == 0 and (back & 0x7FFF) == 0), hex(h)
        v = np.array([h], np.uint16).view(np.float16).astype(np.float64)[0]
        assert v * 2.0 ** 24 == k


def _spread(h):
    e = (h >> 10) & 31
    m = np.where(e > 0, (h & 1023) | 1024, h & 1023)
    s = np.where(e > 0, e.astype(np.int64) - 1, 0)
    out = 0
    for r in range(h.shape[0]):
        nz = s[r][m[r] != 0]
        if nz.size:
            out = max(out, int(nz.max() - nz.min()))
    return out


@pytest.mark.parametrize("kind,lo,hi", [("signs", 0, 10), ("large", 0, 1), ("spread1", 0, 1),
                                        ("spread9", 2, 9), ("spread17", 10, 17), ("full", 18, 29)])
def test_adversarial_kinds(xr, kind, lo, hi):
    h = spmodel.adversarial_bscale(5, 48, 15360, kind)
    sp = _spread(h)
    assert lo <= sp <= hi, sp
    e = (h >> 10) & 31
    assert e.max() <= 30
    if kind == "large":
        assert e.min() >= 22                      # every scale >= 128
    if kind in ("signs", "spread9", "full"):
        assert (h >> 15).any() and not (h >> 15).all()   # both signs
    codes = spmodel.gen_codes(5, 1, 48, 15360)
    assert xr.q4b_check(spmodel.Q4B(codes, h, 48, 15360)) == 0


def test_bound_edge_rows(xr):
    nblk = 480
    inside = spmodel.bound_edge_row(nblk, spmodel.BOUND_LIMIT - 1)
    at = spmodel.bound_edge_row(nblk, spmodel.BOUND_LIMIT)
    assert sum(spmodel.f16_k(int(x)) for x in inside) == spmodel.BOUND_LIMIT - 1
    assert sum(spmodel.f16_k(int(x)) for x in at) == spmodel.BOUND_LIMIT
    codes = np.zeros((2, nblk * 16), np.uint8)
    ok = spmodel.Q4B(codes, np.stack([inside, inside]), 2, nblk * 32)
    bad = spmodel.Q4B(codes, np.stack([inside, at]), 2, nblk * 32)
    assert xr.q4b_check(ok) == 0
    assert xr.q4b_check(bad) == -1
    inf = np.array(inside)
    inf[7] = 0x7C00
    assert xr.q4b_check(spmodel.Q4B(codes[:1], inf[None], 1, nblk * 32)) == -1
