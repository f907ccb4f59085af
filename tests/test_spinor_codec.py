"""The Spinor KV block codec of the checker (oracle/xref_spinor.c) pinned to the reference's
own codec (core/vht2/spinor_block.c, vht2.c, mobius_reorder.c): the committed golden blocks
(tests/golden/make_golden.py spinor), live comparisons on fresh rows where the compiled
reference is present, and the frozen properties the reference's T_VHT tests check."""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import GOLDEN, rng

G = np.load(os.path.join(GOLDEN, "spinor_vectors.npz"))
NG = len([k for k in G.files if k.endswith("_v")])


@pytest.mark.parametrize("i", range(NG))
def test_spinor_golden_blocks(xr, i):
    v = G[f"sp{i}_v"]
    blk = xr.spinor_encode(v)
    assert np.array_equal(blk, G[f"sp{i}_blocks"])
    dec, rc = xr.spinor_decode(G[f"sp{i}_blocks"], v.size)
    assert rc == 0
    assert np.array_equal(dec.view(np.uint32), G[f"sp{i}_dec"].view(np.uint32))


def test_spinor_frozen_split_and_sizes(xr):
    # T_VHT_7 (a): ceil(k / 55), at least one block; head_dim 128 -> 43/43/42
    for k, nb in [(1, 1), (55, 1), (56, 2), (110, 2), (111, 3), (128, 3), (256, 5)]:
        assert xr.spinor_blocks_for(k) == nb
    v = rng(5).standard_normal(128).astype(np.float32)
    blk = xr.spinor_encode(v)
    for b, (off, n) in enumerate([(0, 43), (43, 43), (86, 42)]):
        assert np.array_equal(blk[b * 63:(b + 1) * 63], xr.spinor_encode(v[off:off + n]))


def test_spinor_crc_detects_single_bit_errors(xr):
    # T_VHT_4: CRC-8 over header || body catches every single-bit flip
    v = rng(6).standard_normal(55).astype(np.float32)
    blk = xr.spinor_encode(v)
    for bit in range(62 * 8):
        bad = blk.copy()
        bad[bit // 8] ^= np.uint8(1 << (bit % 8))
        _, rc = xr.spinor_decode(bad, 55)
        assert rc == 1


def test_spinor_header_little_endian(xr):
    # T_VHT_5: 0.15625f = 0x3E200000 stored as 00 00 20 3E; exponent, basis, reserved 0
    v = np.zeros(10, np.float32)
    v[3] = -0.15625
    blk = xr.spinor_encode(v)
    assert list(blk[:7]) == [0x00, 0x00, 0x20, 0x3E, 0, 0, 0]


def test_spinor_kv_rows(xr):
    """The cache transform of the exact path: a K row on the 2^16 grid and a V row of floats
    round-trip through the codec to lrintf(decoded * 65536); V out of range is refused."""
    r = rng(7)
    kg = r.integers(-(1 << 24) + 1, 1 << 24, 256).astype(np.int32)
    blocks, grid, rc = xr.spinor_kv_row(256, kg=kg)
    assert rc == 0
    assert np.array_equal(blocks, xr.spinor_encode(kg.astype(np.float32) * np.float32(1 / 65536)))
    dec, _ = xr.spinor_decode(blocks, 256)
    assert np.array_equal(grid, np.rint(dec.astype(np.float64) * 65536).astype(np.int32))
    v = (r.standard_normal(128) * 40).astype(np.float32)
    blocks, grid, rc = xr.spinor_kv_row(128, vf=v)
    assert rc == 0 and np.array_equal(blocks, xr.spinor_encode(v))
    assert np.abs(grid.astype(np.int64) - np.rint(v.astype(np.float64) * 65536)).max() <= 65536 * np.abs(v).max() / 127
    v[5] = 16384.0
    assert xr.spinor_kv_row(128, vf=v)[2] == -50


def test_spinor_live_vs_reference(xr, reflib):
    L = reflib.lib
    L.sp_spinor_encode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.sp_spinor_decode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    L.sp_crc8.argtypes = [C.c_void_p, C.c_int]
    L.sp_crc8.restype = C.c_uint8
    r = rng(8)
    for it in range(300):
        k = int(r.integers(1, 300))
        v = (r.standard_normal(k) * 10.0 ** r.uniform(-4, 3)).astype(np.float32)
        if it % 7 == 0:
            v[r.integers(0, k, max(1, k // 3))] = 0.0
        if it % 11 == 0:
            v = np.round(v * 2) / 2
        want = np.zeros(xr.spinor_blocks_for(k) * 63, np.uint8)
        L.sp_spinor_encode_vec(v.ctypes.data, k, want.ctypes.data)
        got = xr.spinor_encode(v)
        assert np.array_equal(got, want), (it, k)
        d0 = np.zeros(k, np.float32)
        assert L.sp_spinor_decode_vec(want.ctypes.data, k, d0.ctypes.data) == 0
        d1, rc = xr.spinor_decode(want, k)
        assert rc == 0 and np.array_equal(d0.view(np.uint32), d1.view(np.uint32))
        buf = r.integers(0, 256, 62, dtype=np.uint8)
        assert L.sp_crc8(buf.ctypes.data, 62) == xr.lib.xref_crc8(buf.ctypes.data, 62)
