"""The gated GEMV epilogue (exact GELU/SiLU(gate) * up) and the pre-quantized GEMV entry
points, against XREF, at every supported token-row count."""
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


def P(x):
    return C.c_void_p(x.data_ptr())


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("rows,cols", [(1536, 512), (4000, 3840), (512, 15360)])
def test_gated_gemv(xr, spb, cuda_ok, m, act, rows, cols):
    import torch
    wg = spmodel.gen_matrix(1, "blk.0.ffn_gate.weight", rows, cols)
    wu = spmodel.gen_matrix(2, "blk.0.ffn_up.weight", rows, cols)
    x = rng(rows + m + act).standard_normal((m, cols)).astype(np.float32)
    dx = t(x)
    q = torch.empty((m, cols), dtype=torch.int8, device="cuda")
    bs = torch.empty((m, cols // 32), dtype=torch.int32, device="cuda")
    sc = torch.empty(m, dtype=torch.float32, device="cuda")
    spb200.check(spb.spb_quantize_rows(P(dx), cols, m, P(q), P(bs), P(sc), None))
    y = torch.empty((m, rows), dtype=torch.float32, device="cuda")
    # keep every device buffer referenced until the kernel has run
    dev = [t(wg.codes), t(wg.bscale.view(np.int16)), t(wu.codes), t(wu.bscale.view(np.int16))]
    spb200.check(spb.spb_gemv_q4b_gated_q(P(dev[0]), P(dev[1]), P(dev[2]), P(dev[3]), rows, cols, P(q), P(bs),
                                          P(sc), m, act, P(y), None))
    torch.cuda.synchronize()
    g = xr.matvec(wg, x)
    u = xr.matvec(wu, x)
    f = xr.gelu if act == 0 else xr.silu
    want = (np.stack([f(g[i]) for i in range(m)]) * u).astype(np.float32)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))
    q2, s2 = xr.quant(x[0])
    assert float(sc[0].item()) == s2
