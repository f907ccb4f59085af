"""The drop-in: the reference's own libshannonprime session (sp_prefill_chunk /
sp_decode_step / sp_session_clone / sp_session_rewind) with the B200 backend
registered through its section-6 and section-6b hooks, byte-identical to XREF."""
import ctypes as C

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module", params=["micro_gemma", "micro_qwen"])
def setup(request, reflib, xr, tmp_path_factory):
    cfg = spmodel.CONFIGS[request.param]
    T = spmodel.gen_model(cfg, seed=0)
    d = tmp_path_factory.mktemp("m")
    mp, tp = str(d / "m.sp-model"), str(d / "m.sp-tokenizer")
    spmodel.write_sp_model(mp, tp, cfg, T)
    model = reflib.load(mp, tp)
    l1 = spb200.load_l1()
    yield cfg, T, model, l1
    s = reflib.session(model, 16)   # the borrowed qwen3_model the hooks were handed
    qm = reflib.lib.sp_session_qwen3_model(s)
    reflib.lib.sp_session_destroy(s)
    l1.spb_l1_release_model(qm)
    reflib.lib.sp_model_unload(model)


def test_section6_prefill(reflib, xr, cuda_ok, setup):
    cfg, T, model, l1 = setup
    L = reflib.lib
    s = reflib.session(model, cfg.max_context)
    fn = C.cast(l1.spb_l1_forward, C.c_void_p)
    assert L.sp_session_register_forward_backend(s, l1.spb_l1_backend(), fn) == 0
    toks = spmodel.gen_tokens(31, 24, cfg.n_vocab)
    want = xr.session(xref.build_desc(cfg, T), cfg.max_context).prefill(toks)
    rc, lg = reflib.prefill(s, toks[:10], cfg.n_vocab)
    assert rc == 0, reflib.err()
    assert np.array_equal(u32(lg), u32(want[9]))
    rc, lg = reflib.prefill(s, toks[10:], cfg.n_vocab)      # re-runs the whole history
    assert rc == 0 and np.array_equal(u32(lg), u32(want[-1]))
    assert reflib.position(s) == 24
    L.sp_session_destroy(s)


def test_section6b_decode(reflib, xr, cuda_ok, setup):
    cfg, T, model, l1 = setup
    L = reflib.lib
    s = reflib.session(model, cfg.max_context)
    qm = L.sp_session_qwen3_model(s)
    dt = l1.spb_l1_kvdecode_table()
    OPEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p))
    PRE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int)
    REW = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int)
    POS = C.CFUNCTYPE(C.c_int, C.c_void_p)
    CLOSE = C.CFUNCTYPE(None, C.c_void_p)
    fns = (C.c_void_p * 6).from_address(dt)
    h = C.c_void_p()
    assert OPEN(fns[0])(qm, cfg.max_context, C.byref(h)) == 0
    toks = spmodel.gen_tokens(32, 16, cfg.n_vocab)
    xs = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    lx = xs.prefill(toks)[-1]
    # the caller drives prefill on both sides (sp_prefill_chunk does not feed section 6b)
    rc, _ = reflib.prefill(s, toks, cfg.n_vocab)
    assert rc == 0
    assert PRE(fns[1])(h, toks.ctypes.data, toks.size) == 0
    assert L.sp_session_register_kvdecode_backend(s, h, dt) == 0
    tok = int(lx.argmax())
    for i in range(10):
        lx = xs.step(tok)
        rc, lg = reflib.decode(s, tok, cfg.n_vocab)
        assert rc == 0, reflib.err()
        assert np.array_equal(u32(lg), u32(lx)), f"step {i}"
        tok = int(lg.argmax())
    assert POS(fns[4])(h) == 26 and reflib.position(s) == 26
    # rewind must be mirrored by the caller (sp_session_rewind does not call dt->rewind)
    assert L.sp_session_rewind(s, 2) == 0 and REW(fns[3])(h, 2) == 0
    assert xs.rewind(2) == 0
    lx = xs.step(7)
    rc, lg = reflib.decode(s, 7, cfg.n_vocab)
    assert rc == 0 and np.array_equal(u32(lg), u32(lx))
    # append-only clone row: fork the resident cache
    h2 = C.c_void_p()
    assert l1.spb_l1_kvdecode_clone(h, C.byref(h2)) == 0
    assert POS(fns[4])(h2) == POS(fns[4])(h)
    # bad token: the backend fails, the session reports SP_EBADSTATE with detail
    rc, _ = reflib.decode(s, cfg.n_vocab + 1, cfg.n_vocab)
    assert rc == -4
    CLOSE(fns[5])(h2)
    CLOSE(fns[5])(h)
    L.sp_session_register_kvdecode_backend(s, None, None)
    L.sp_session_destroy(s)


def test_section6b_spinor_kv(reflib, xr, cuda_ok, setup):
    """Caches opened through the section-6b table after spb_l1_set_kv_flags(SPB_KV_SPINOR) keep
    their K/V as Spinor blocks (the reference's SP_KV_SPINOR); the reference's own sp_decode_step
    then returns XREF's Spinor-session logits byte for byte."""
    cfg, T, model, l1 = setup
    L = reflib.lib
    assert l1.spb_l1_set_kv_flags(2) != 0   # unknown flag refused
    assert l1.spb_l1_set_kv_flags(spb200.SPB_KV_SPINOR) == 0
    try:
        s = reflib.session(model, cfg.max_context)
        qm = L.sp_session_qwen3_model(s)
        dt = l1.spb_l1_kvdecode_table()
        OPEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p))
        PRE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int)
        CLOSE = C.CFUNCTYPE(None, C.c_void_p)
        fns = (C.c_void_p * 6).from_address(dt)
        h = C.c_void_p()
        assert OPEN(fns[0])(qm, cfg.max_context, C.byref(h)) == 0
        toks = spmodel.gen_tokens(35, 16, cfg.n_vocab)
        xs = xr.session(xref.build_desc(cfg, T), cfg.max_context, spinor=True)
        lx = xs.prefill(toks)[-1]
        rc, _ = reflib.prefill(s, toks, cfg.n_vocab)
        assert rc == 0
        assert PRE(fns[1])(h, toks.ctypes.data, toks.size) == 0
        assert L.sp_session_register_kvdecode_backend(s, h, dt) == 0
        tok = int(lx.argmax())
        for i in range(8):
            lx = xs.step(tok)
            rc, lg = reflib.decode(s, tok, cfg.n_vocab)
            assert rc == 0, reflib.err()
            assert np.array_equal(u32(lg), u32(lx)), f"step {i}"
            tok = int(lg.argmax())
        L.sp_session_register_kvdecode_backend(s, None, None)
        CLOSE(fns[5])(h)
        L.sp_session_destroy(s)
    finally:
        assert l1.spb_l1_set_kv_flags(0) == 0


def test_non_q4b_model_rejected(reflib, cuda_ok, tmp_path):
    """A model whose weights are not OK_Q4B arena tensors is refused with a clear error."""
    l1 = spb200.load_l1()
    L = reflib.lib
    fn = C.cast(l1.spb_l1_forward, C.c_void_p)
    rc = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)(fn.value)(
        None, None, None, 1, None)
    assert rc != 0 and b"null model" in L.sp_last_error()


def test_section6b_extended_table_paged_clone(reflib, xr, cuda_ok, tmp_path):
    """The table with the appended clone row (its first six rows are the frozen table), on a
    model whose caches live in a page pool: the fork shares pages, both sides stay exact."""
    cfg = spmodel.CONFIGS["micro_qwen"]
    T = spmodel.gen_model(cfg, seed=4)
    mp, tp = str(tmp_path / "m.sp-model"), str(tmp_path / "m.sp-tokenizer")
    spmodel.write_sp_model(mp, tp, cfg, T)
    model = reflib.load(mp, tp)
    l1 = spb200.load_l1()
    assert l1.spb_l1_set_kv_pool(128, 16) == 0
    L = reflib.lib
    s = reflib.session(model, cfg.max_context)
    qm = L.sp_session_qwen3_model(s)
    ext = l1.spb_l1_kvdecode_table_ext()
    assert ext == l1.spb_l1_kvdecode_table()          # the frozen table is the extension's prefix
    fns = (C.c_void_p * 7).from_address(ext)
    OPEN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_void_p))
    PRE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int)
    DEC = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int32, C.c_void_p)
    POS = C.CFUNCTYPE(C.c_int, C.c_void_p)
    CLOSE = C.CFUNCTYPE(None, C.c_void_p)
    CLONE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_void_p))
    h = C.c_void_p()
    assert OPEN(fns[0])(qm, cfg.max_context, C.byref(h)) == 0
    toks = spmodel.gen_tokens(35, 40, cfg.n_vocab)
    assert PRE(fns[1])(h, toks.ctypes.data, toks.size) == 0
    xs = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    xs.prefill(toks, all_logits=False)
    h2 = C.c_void_p()
    assert CLONE(fns[6])(h, C.byref(h2)) == 0
    xc = xs.clone()
    lg = np.empty(cfg.n_vocab, np.float32)
    for tok_a, tok_b in ((3, 8), (4, 9), (5, 10)):
        assert DEC(fns[2])(h, tok_a, lg.ctypes.data) == 0
        assert np.array_equal(u32(lg), u32(xs.step(tok_a)))
        assert DEC(fns[2])(h2, tok_b, lg.ctypes.data) == 0
        assert np.array_equal(u32(lg), u32(xc.step(tok_b)))
    assert POS(fns[4])(h) == POS(fns[4])(h2) == 43
    CLOSE(fns[5])(h2)
    CLOSE(fns[5])(h)
    L.sp_session_destroy(s)
    l1.spb_l1_release_model(qm)
    assert l1.spb_l1_set_kv_pool(0, 0) == 0
    reflib.lib.sp_model_unload(model)
