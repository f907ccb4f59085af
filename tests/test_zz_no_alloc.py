"""spb_gemv_q4b_noalloc: the dequant-GEMV for callers that must not allocate device memory
(for example when all device memory already belongs to another pool, or when a
latency-critical loop must not reach the allocator and its implicit device sync).

It must give the same bytes as spb_gemv_q4b, whose scratch comes from cudaMalloc, on two
calls in a row (the second reuses the fixed scratch the first one left behind), and reject
sizes beyond its fixed scratch. This file sorts last so a stopping run has already run every
other test; it also passes alone in a fresh process (its first call does the set-up).
"""
import ctypes as C

import numpy as np
import pytest

import spb200
import spmodel

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_gemv_matches_allocating_gemv_twice(spb, cuda_ok):
    import torch
    # the last case fills the fixed scratch exactly: 16 rows x 16384 columns = 262144 elements,
    # the widest row the GEMV takes, so the scratch's last activation and block-sum bytes are used
    cases = [(3840, 3840, 1, 11), (1000, 15360, 16, 12), (512, 16384, 16, 13)]
    for rows, cols, m, seed in cases:
        w = spmodel.gen_matrix(seed, "blk.0.ffn_down.weight", rows, cols)
        x = np.random.default_rng(seed).standard_normal((m, cols)).astype(np.float32)
        codes, scales, dx = _dev(w.codes), _dev(w.bscale.view(np.int16)), _dev(x)
        y_ref = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        y_na = torch.full((m, rows), float("nan"), dtype=torch.float32, device="cuda")
        spb200.check(spb.spb_gemv_q4b(_p(codes), _p(scales), rows, cols, _p(dx), m, _p(y_ref), None))
        spb200.check(spb.spb_gemv_q4b_noalloc(_p(codes), _p(scales), rows, cols, _p(dx), m, _p(y_na), None))
        torch.cuda.synchronize()
        assert np.array_equal(y_na.cpu().numpy().view(np.uint32), y_ref.cpu().numpy().view(np.uint32))


def test_noalloc_gemv_rejects_oversize(spb, cuda_ok):
    import torch
    d = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    rc = spb.spb_gemv_q4b_noalloc(_p(d), _p(d), 8, 16384, _p(d), 32, _p(d), None)
    assert rc == spb200.SPB_EBADARG                       # n_tok outside {1, 2, 4, 8, 16}
    rc = spb.spb_gemv_q4b_noalloc(_p(d), _p(d), 8, 32768, _p(d), 1, _p(d), None)
    assert rc == spb200.SPB_EBADARG                       # one row, but wider than the GEMV takes
    assert b"16384-column limit" in spb.spb_last_error()
    rc = spb.spb_gemv_q4b_noalloc(_p(d), _p(d), 8, 16416, _p(d), 16, _p(d), None)
    assert rc == spb200.SPB_EBADARG
    assert b"16384-column limit" in spb.spb_last_error()
