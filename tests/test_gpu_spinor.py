"""Compressed K/V (SPB_KV_SPINOR, the reference's kv_mode 1: sp_session.c:233-244, 298-313) on
the GPU: every K and V head row kept as the reference's frozen 63-byte Spinor blocks, encoded by
the kernel that produces the row (k_rope_kv for prefill chunks, the attention's owning CTA for a
decode step) and decoded inside the attention from the blocks its bulk copies bring in.

Against XREF's Spinor session (oracle/xref_spinor.c, pinned to the reference's compiled codec by
tests/test_spinor_codec.py): every logit, the greedy tokens, and the cached blocks byte for
byte; clone and rewind; batches mixing Spinor and int32 sessions; and the refusals."""
import ctypes as C
import dataclasses

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def run(xr, cfg, seed, n_pre, n_dec, pmax, kv_positions):
    T = spmodel.gen_model(cfg, seed=seed)
    m = spb200.Model.upload(cfg, T)
    s = m.session(pmax, spinor=True)
    xs = xr.session(xref.build_desc(cfg, T), pmax, spinor=True)
    toks = spmodel.gen_tokens(seed + 1, n_pre, cfg.n_vocab)
    got, want = s.prefill(toks), xs.prefill(toks)
    assert np.array_equal(u32(got), u32(want)), "prefill logits"
    tok = int(want[-1].argmax())
    for i in range(n_dec):
        a, am = s.step_argmax(tok)
        b = xs.step(tok)
        assert np.array_equal(u32(a), u32(b)), f"decode step {i}"
        assert am == int(b.argmax())
        tok = am
    for L in range(cfg.n_layers):
        for p in kv_positions:
            for which in (0, 1):
                assert np.array_equal(s.kv_bytes(L, p, which), xs.kv_bytes(L, p, which)), (L, p, which)
    return m, s, xs, tok


@pytest.mark.parametrize("name", ["micro_gemma", "micro_qwen"])
def test_spinor_session_micro(xr, cuda_ok, name):
    """head_dim 64 (two 32-value blocks per row): prefill 40 + 20 decode steps."""
    cfg = spmodel.CONFIGS[name]
    m, s, xs, _ = run(xr, cfg, 51, 40, 20, cfg.max_context, (0, 17, 39, 59))
    s.close(); xs.close(); m.free()


@pytest.mark.parametrize("hd,nh,nkv,win", [(256, 4, 2, 40), (128, 8, 2, 300), (64, 8, 8, 24)])
def test_spinor_long_context(xr, cuda_ok, hd, nh, nkv, win):
    """Head widths 256 / 128 / 64 (5 / 3 / 2 blocks per row, ragged 52/51/51/51/51 and 43/43/42
    splits), 330 positions: several ring stages per CTA, clusters over long rows, sliding windows
    shorter than the context on the local layers."""
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_gemma"], n_layers=6, head_dim=hd, n_head=nh,
                              n_head_kv=nkv, sliding_window=win, max_context=384)
    m, s, xs, _ = run(xr, cfg, 52, 300, 30, cfg.max_context, (0, 127, 128, 299, 329))
    s.close(); xs.close(); m.free()


def test_spinor_clone_rewind(xr, cuda_ok):
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_qwen"], head_dim=128, n_head=4, n_head_kv=2)
    m, s, xs, tok = run(xr, cfg, 53, 30, 5, cfg.max_context, (0, 34))
    c, xc = s.clone(), xs.clone()
    for _ in range(3):
        a, b = c.step(tok), xc.step(tok)
        assert np.array_equal(u32(a), u32(b))
        tok = int(b.argmax())
    s.rewind(4); xs.rewind(4)
    for t in spmodel.gen_tokens(54, 6, cfg.n_vocab):
        assert np.array_equal(u32(s.step(int(t))), u32(xs.step(int(t))))
    for p in (26, 33):
        assert np.array_equal(s.kv_bytes(1, p, 0), xs.kv_bytes(1, p, 0))
    for o in (c, xc, s, xs):
        o.close()
    m.free()


def test_spinor_blocks_decode_with_reference_codec(xr, reflib, cuda_ok):
    """The device-written blocks decode with the reference's own sp_spinor_decode_vec (CRC
    verified) to exactly the grid rows the attention used (XREF's round-tripped K and V)."""
    cfg = spmodel.CONFIGS["micro_gemma"]
    T = spmodel.gen_model(cfg, seed=55)
    m = spb200.Model.upload(cfg, T)
    s = m.session(cfg.max_context, spinor=True)
    xs = xr.session(xref.build_desc(cfg, T), cfg.max_context, spinor=True)
    toks = spmodel.gen_tokens(56, 24, cfg.n_vocab)
    s.prefill(toks, logits=False)
    xs.prefill(toks, all_logits=False)
    s.step(int(toks[0]))
    xs.step(int(toks[0]))
    L = reflib.lib
    L.sp_spinor_decode_vec.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    hd, nkv = cfg.head_dim, cfg.n_head_kv
    rb = xr.spinor_blocks_for(hd) * 63
    for p in (0, 23, 24):
        for which in (0, 1):
            blk = s.kv_bytes(0, p, which)
            want = xs.kv(0, p, which)
            for g in range(nkv):
                dec = np.zeros(hd, np.float32)
                row = np.ascontiguousarray(blk[g * rb:(g + 1) * rb])
                assert L.sp_spinor_decode_vec(row.ctypes.data, hd, dec.ctypes.data) == 0
                grid = np.rint(dec.astype(np.float64) * 65536).astype(np.int32)
                assert np.array_equal(grid, want[g * hd:(g + 1) * hd]), (p, which, g)
    s.close()
    xs.close()
    m.free()


def test_spinor_refusals(cuda_ok):
    cfg = spmodel.CONFIGS["micro_gemma"]
    T = spmodel.gen_model(cfg, seed=57)
    m = spb200.Model.upload(cfg, T)
    L = spb200.load()
    h = C.c_void_p()
    assert L.spb_session_open_ex(m.h, 64, 2, C.byref(h)) == spb200.SPB_EBADARG
    s = m.session(64, spinor=True)
    o = np.zeros(cfg.n_head_kv * cfg.head_dim, np.int32)
    assert L.spb_session_kv_read(s.h, 0, 0, 0, o.ctypes.data) == spb200.SPB_EUNSUPPORTED
    plain = m.session(64)
    b = np.zeros(16, np.uint8)
    assert L.spb_session_kv_bytes(plain.h, 0, 0, 0, b.ctypes.data) == spb200.SPB_EBADARG
    s.close(); plain.close(); m.free()


def test_spinor_batch_rows(xr, cuda_ok):
    """spb_batch_decode_step over sessions at different positions, three keeping Spinor K/V and
    one int32 rows: every row's logits equal its own XREF session's (Spinor or not)."""
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_gemma"], head_dim=128, n_head=8, n_head_kv=2,
                              sliding_window=48, max_context=256)
    T = spmodel.gen_model(cfg, seed=58)
    m = spb200.Model.upload(cfg, T)
    d = xref.build_desc(cfg, T)
    kinds = [True, False, True, True]
    lens = [70, 33, 150, 9]
    ss, xs = [], []
    for i, (sp, n) in enumerate(zip(kinds, lens)):
        s = m.session(cfg.max_context, spinor=sp)
        x = xr.session(d, cfg.max_context, spinor=sp)
        toks = spmodel.gen_tokens(60 + i, n, cfg.n_vocab)
        s.prefill(toks, logits=False)
        x.prefill(toks, all_logits=False)
        ss.append(s)
        xs.append(x)
    L = spb200.load()
    arr = (C.c_void_p * len(ss))(*[s.h for s in ss])
    toks = np.array([3, 5, 7, 11], np.int32)
    for step in range(4):
        lg = np.empty((len(ss), cfg.n_vocab), np.float32)
        am = np.empty(len(ss), np.int32)
        spb200.check(L.spb_batch_decode_step(arr, len(ss), toks.ctypes.data, lg.ctypes.data, am.ctypes.data))
        for i, x in enumerate(xs):
            want = x.step(int(toks[i]))
            assert np.array_equal(u32(lg[i]), u32(want)), (step, i)
        toks = am.copy()
    for i, (s, x) in enumerate(zip(ss, xs)):
        p = lens[i] + 3
        if kinds[i]:
            assert np.array_equal(s.kv_bytes(1, p, 0), x.kv_bytes(1, p, 0))
            assert np.array_equal(s.kv_bytes(0, p, 1), x.kv_bytes(0, p, 1))
        s.close()
        x.close()
    m.free()
