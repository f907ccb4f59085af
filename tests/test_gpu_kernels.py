"""Kernel-level parity on the GPU: every kernel through the C ABI against XREF, bit for bit."""
import ctypes as C

import numpy as np
import pytest

import spb200
import spmodel
from conftest import rng

pytestmark = pytest.mark.gpu


def t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(x):
    return C.c_void_p(x.data_ptr())


def sync():
    import torch
    torch.cuda.synchronize()


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("n,rows,scale", [(3840, 4, 1.0), (256, 8, 0.01), (64, 16, 3.0), (15360, 2, 0.5),
                                          (4096, 3, 50.0), (128, 5, 1e-3)])
def test_rmsnorm_rows(xr, spb, cuda_ok, n, rows, scale):
    r = rng(n + rows)
    x = (r.standard_normal((rows, n)) * scale).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(n)).astype(np.float32)
    dx, dw = t(x), t(w)
    import torch
    out = torch.empty_like(dx)
    spb200.check(spb.spb_rmsnorm_exact_dev(ptr(dx), ptr(dw), n, rows, ptr(out), None))
    sync()
    want = np.stack([xr.rmsnorm(x[i], w) for i in range(rows)])
    assert np.array_equal(u32(out.cpu().numpy()), u32(want))
    assert spb.spb_take_device_errors() == 0


def test_rmsnorm_range_error_flag(spb, cuda_ok):
    import torch
    x = t(np.full((1, 64), 40000.0, np.float32))
    w = t(np.ones(64, np.float32))
    out = torch.empty_like(x)
    spb200.check(spb.spb_rmsnorm_exact_dev(ptr(x), ptr(w), 64, 1, ptr(out), None))
    sync()
    assert spb.spb_take_device_errors() != 0
    assert spb.spb_take_device_errors() == 0


@pytest.mark.parametrize("op", ["gelu", "silu"])
def test_gelu_silu(xr, spb, cuda_ok, op):
    import torch
    r = rng(7)
    x = np.concatenate([r.standard_normal(100000) * 3, np.linspace(-40, 40, 20001),
                        [0.0, -0.0, 1e-6, -1e-6, 2047.0, -2047.0]]).astype(np.float32)
    dx = t(x)
    out = torch.empty_like(dx)
    f = spb.spb_gelu_exact_dev if op == "gelu" else spb.spb_silu_exact_dev
    spb200.check(f(ptr(dx), x.size, ptr(out), None))
    sync()
    want = xr.gelu(x) if op == "gelu" else xr.silu(x)
    assert np.array_equal(u32(out.cpu().numpy()), u32(want))


@pytest.mark.parametrize("d,base", [(64, 10000.0), (128, 1e6), (256, 1e6), (256, 10000.0)])
def test_rope_cordic(xr, spb, cuda_ok, d, base):
    import torch
    r = rng(d)
    rows = 64
    v = (r.standard_normal((rows, d)) * 2).astype(np.float32)
    pos = np.concatenate([[0, 1, 2, 4095, 8191, 65535, 1 << 20], r.integers(0, 10000, rows - 7)]).astype(np.int32)
    dv, dp = t(v), t(pos)
    out = torch.empty((rows, d), dtype=torch.int32, device="cuda")
    spb200.check(spb.spb_rope_cordic_dev(ptr(dv), d, rows, ptr(dp), base, ptr(out), None))
    W = xr.rope_table(base, d)
    want = np.stack([xr.rope(v[i], int(pos[i]), W)[0] for i in range(rows)])
    assert np.array_equal(out.cpu().numpy(), want)


GEMV_SHAPES = [(3840, 3840), (15360, 3840), (3840, 15360), (4096, 3840), (96, 256), (1000, 512)]


@pytest.mark.parametrize("rows,cols", GEMV_SHAPES)
@pytest.mark.parametrize("m", [1, 4, 16])
def test_gemv_vs_xref(xr, spb, cuda_ok, rows, cols, m):
    import torch
    w = spmodel.gen_matrix(rows + m, "blk.0.ffn_gate.weight", rows, cols)
    r = rng(rows * 7 + m)
    x = r.standard_normal((m, cols)).astype(np.float32)
    # config-2 activations: N(0,1) through the exact RMSNorm island
    g = np.ones(cols, np.float32)
    x = np.stack([xr.rmsnorm(x[i], g) for i in range(m)])
    dc, ds, dx = t(w.codes), t(w.bscale.view(np.int16)), t(x)
    y = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    spb200.check(spb.spb_gemv_q4b(ptr(dc), ptr(ds), rows, cols, ptr(dx), m, ptr(y), None))
    sync()
    assert np.array_equal(u32(y.cpu().numpy()), u32(xr.matvec(w, x)))


def test_gemv_lm_head_full_size(xr, spb, cuda_ok):
    """262144 x 3840 (the 12B LM head): a random row subset against XREF, and the
    scale-invariance property (x * 8 -> identical output, since the quantizer divides
    by max|x|) over every row."""
    import torch
    rows, cols, m = 262144, 3840, 4
    w = spmodel.gen_matrix(9, "token_embd.weight", rows, cols)
    x = rng(3).standard_normal((m, cols)).astype(np.float32)
    dc, ds, dx = t(w.codes), t(w.bscale.view(np.int16)), t(x)
    y = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    spb200.check(spb.spb_gemv_q4b(ptr(dc), ptr(ds), rows, cols, ptr(dx), m, ptr(y), None))
    y2 = torch.empty_like(y)
    dx8 = dx * 8   # referenced until the kernel has run
    spb200.check(spb.spb_gemv_q4b(ptr(dc), ptr(ds), rows, cols, ptr(dx8), m, ptr(y2), None))
    sync()
    yh = y.cpu().numpy()
    assert np.array_equal(u32(yh * np.float32(8)), u32(y2.cpu().numpy()))
    sel = np.sort(rng(4).choice(rows, 2048, replace=False))
    sub = spmodel.Q4B(w.codes[sel], w.bscale[sel], sel.size, cols)
    assert np.array_equal(u32(yh[:, sel]), u32(xr.matvec(sub, x)))


def test_gemv_rejects_bad_args(spb, cuda_ok):
    assert spb.spb_gemv_q4b(None, None, 4, 64, None, 1, None, None) == spb200.SPB_EBADARG
    import torch
    d = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    assert spb.spb_gemv_q4b(ptr(d), ptr(d), 4, 64, ptr(d), 3, ptr(d), None) == spb200.SPB_EBADARG
