"""Block scales the seeded generator never makes, on the GPU, byte for byte against XREF.

Real OK_Q4B weights (build_packed_q4b, sp_model_bridge.c:114-148) carry a separate f16 scale
per 32-column block, with exponents that vary within a row; the dequant rule is
frobenius_lift.c:200-209. These tests drive the GEMV (1-8 token rows), the token-batch GEMM in
both its small-scale and general forms (16 and more rows) and the whole forward with
hand-built scales: negative, subnormal and zero scales, scales >= 128, rows whose blocks span
the whole f16 exponent range, and rows at the exact int64 bound's edge."""
import ctypes as C

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(x):
    return C.c_void_p(x.data_ptr())


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def expected_info(h):
    e = (h >> 10) & 31
    m = np.where(e > 0, (h & 1023) | 1024, h & 1023)
    s = np.where(e > 0, e.astype(np.int64) - 1, 0)
    spread = 0
    for r in range(h.shape[0]):
        nz = s[r][m[r] != 0]
        if nz.size:
            spread = max(spread, int(nz.max() - nz.min()))
    planes = 2 if spread <= 1 else 3 if spread <= 9 else 4 if spread <= 17 else 0
    return int(e.max() <= 21), planes


def run_matmul(w, x, n_tok):
    import torch
    dc, ds, dx = t(w.codes), t(w.bscale.view(np.int16)), t(x)
    pm = spb200.PreparedQ4B(ptr(dc), ptr(ds), w.rows, w.cols)
    y = torch.empty((n_tok, w.rows), dtype=torch.float32, device="cuda")
    pm.matmul(ptr(dx), n_tok, ptr(y))
    torch.cuda.synchronize()
    info = pm.info()
    pm.release()
    return y.cpu().numpy(), info


@pytest.mark.parametrize("kind", ["signs", "large", "spread1", "spread9", "spread17", "full"])
@pytest.mark.parametrize("rows,cols", [(1000, 3840), (520, 15360)])
def test_adversarial_scales_matmul(xr, spb, cuda_ok, kind, rows, cols):
    h = spmodel.adversarial_bscale(rows + cols, rows, cols, kind)
    w = spmodel.Q4B(spmodel.gen_codes(rows, 77, rows, cols), h, rows, cols)
    x = np.random.default_rng(rows).standard_normal((100, cols)).astype(np.float32)
    want = xr.matvec(w, x)
    for n_tok in (1, 4, 16, 64, 100):   # GEMV rows; the GEMM at 16, 64 and 64 + 36
        y, info = run_matmul(w, x[:n_tok], n_tok)
        assert np.array_equal(u32(y), u32(want[:n_tok])), f"{kind} n_tok={n_tok}"
    small, planes = expected_info(h)
    assert info["small"] == small and info["planes"] == planes, info
    assert spb.spb_take_device_errors() == 0


def test_isolated_gemv_entry_general_form(xr, spb, cuda_ok):
    """spb_gemv_q4b does not describe the scales, so its 16-row batch runs the GEMM's general
    (not small-scale) form: check it on scales >= 128 and on the full exponent range."""
    import torch
    for kind in ("large", "full"):
        rows, cols = 700, 4096
        w = spmodel.Q4B(spmodel.gen_codes(3, 9, rows, cols), spmodel.adversarial_bscale(4, rows, cols, kind),
                        rows, cols)
        x = np.random.default_rng(5).standard_normal((16, cols)).astype(np.float32)
        dc, ds, dx = t(w.codes), t(w.bscale.view(np.int16)), t(x)
        y = torch.empty((16, rows), dtype=torch.float32, device="cuda")
        spb200.check(spb.spb_gemv_q4b(ptr(dc), ptr(ds), rows, cols, ptr(dx), 16, ptr(y), None))
        torch.cuda.synchronize()
        assert np.array_equal(u32(y.cpu().numpy()), u32(xr.matvec(w, x))), kind


def test_bound_edge(xr, spb, cuda_ok):
    """A row whose scales sum to one below the exact bound is accepted and multiplied exactly
    (the int64 accumulator comes within a factor of the activations' size of 2^63); a row at
    the bound, or one with an infinite scale, is refused with SPB_ERANGE."""
    import torch
    rows, cols = 64, 15360
    nblk = cols // 32
    h = spmodel.adversarial_bscale(6, rows, cols, "spread9")
    h[5] = spmodel.bound_edge_row(nblk, spmodel.BOUND_LIMIT - 1)
    h[9] = spmodel.bound_edge_row(nblk, spmodel.BOUND_LIMIT - 1)[::-1]
    codes = spmodel.gen_codes(6, 3, rows, cols)
    codes[5] = 0x77          # every code +7: the largest same-sign block sums
    w = spmodel.Q4B(codes, h, rows, cols)
    assert xr.q4b_check(w) == 0
    x = np.random.default_rng(6).standard_normal((20, cols)).astype(np.float32)
    x[:, :] = np.abs(x)      # one sign: the accumulators run up to their bound
    want = xr.matvec(w, x)
    for n_tok in (1, 16, 20):
        y, _ = run_matmul(w, x[:n_tok], n_tok)
        assert np.array_equal(u32(y), u32(want[:n_tok])), n_tok
    for bad_row in (spmodel.bound_edge_row(nblk, spmodel.BOUND_LIMIT), None):
        hb = h.copy()
        if bad_row is None:
            hb[3, 17] = 0x7C00       # +inf
        else:
            hb[3] = bad_row
        dc, ds = t(codes), t(hb.view(np.int16))
        out = C.c_void_p()
        rc = spb.spb_q4b_prepare(ptr(dc), ptr(ds), rows, cols, None, C.byref(out))
        assert rc == spb200.SPB_ERANGE, rc
        assert b"bound" in spb.spb_last_error()


def _adversarial_model(cfg, seed):
    """Every matrix's scales from spmodel.model_bscale, with spreads 1, 6 and 12 in turn (2, 3
    and 4 digit planes), signs, zeros and subnormals."""
    T = spmodel.gen_model(cfg, seed=seed)
    mats = sorted(k for k, v in T.items() if isinstance(v, spmodel.Q4B))
    for i, name in enumerate(mats):
        w = T[name]
        T[name] = spmodel.Q4B(w.codes, spmodel.model_bscale(seed * 100 + i, w.rows, w.cols, (1, 6, 12)[i % 3]),
                              w.rows, w.cols)
    return T


@pytest.mark.parametrize("name", ["micro_gemma", "micro_qwen"])
def test_forward_with_adversarial_scales(xr, cuda_ok, name):
    """Whole prefill (16-64-row GEMM chunks) and decode (GEMV) through spb_model_upload with
    per-block scales of mixed signs, zeros, subnormals and within-row exponent spreads."""
    cfg = spmodel.CONFIGS[name]
    T = _adversarial_model(cfg, 8)
    m = spb200.Model.upload(cfg, T)
    s = m.session(cfg.max_context)
    xs = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    toks = spmodel.gen_tokens(40, 70, cfg.n_vocab)
    got, want = s.prefill(toks), xs.prefill(toks)
    assert np.array_equal(u32(got), u32(want))
    tok = int(want[-1].argmax())
    for i in range(6):
        a, am = s.step_argmax(tok)
        b = xs.step(tok)
        assert np.array_equal(u32(a), u32(b)), f"decode step {i}"
        tok = am
    s.close()
    m.free()


def test_upload_refuses_out_of_range_scales(cuda_ok):
    """An infinite block scale, or a row past the int64 bound (a 264-block FFN row is wide
    enough to reach it), makes spb_model_upload refuse the model with SPB_ERANGE."""
    import dataclasses
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_qwen"], n_ff=8448, n_layers=2)
    T = spmodel.gen_model(cfg, seed=9)
    for name, mutate in (("blk.0.attn_q.weight", "inf"), ("blk.1.ffn_down.weight", "bound")):
        T2 = dict(T)
        w = T[name]
        h = w.bscale.copy()
        if mutate == "inf":
            h[2, 3] = 0x7C00
        else:
            h[2] = spmodel.bound_edge_row(w.cols // 32, spmodel.BOUND_LIMIT)
        T2[name] = spmodel.Q4B(w.codes, h, w.rows, w.cols)
        with pytest.raises(spb200.SpbError) as ei:
            spb200.Model.upload(cfg, T2)
        assert ei.value.code == spb200.SPB_ERANGE, name
