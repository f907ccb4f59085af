"""Whole-forward parity on the GPU: resident sessions (section-6b semantics) and the
full forward (section-6) through the C ABI, byte-identical to XREF."""
import dataclasses

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module", params=["micro_gemma", "micro_qwen", "tiny"])
def pair(request, xr):
    cfg = spmodel.CONFIGS[request.param]
    T = spmodel.gen_model(cfg, seed=0)
    m = spb200.Model.upload(cfg, T)
    yield cfg, T, m, xref.build_desc(cfg, T)
    m.free()


def test_prefill_all_logits(xr, cuda_ok, pair):
    cfg, T, m, d = pair
    n = 40 if cfg.name != "tiny" else 64
    toks = spmodel.gen_tokens(21, n, cfg.n_vocab)
    want = xr.session(d, cfg.max_context).prefill(toks)
    s = m.session(cfg.max_context)
    got = s.prefill(toks)
    s.close()
    assert np.array_equal(u32(got), u32(want))


def test_decode_trajectory_and_kv(xr, cuda_ok, pair):
    cfg, T, m, d = pair
    n_pre, n_dec = (64, 64) if cfg.name == "tiny" else (20, 24)
    toks = spmodel.gen_tokens(22, n_pre, cfg.n_vocab)
    xs = xr.session(d, cfg.max_context)
    lx = xs.prefill(toks)[-1]
    s = m.session(cfg.max_context)
    s.prefill(toks, logits=False)
    tok = int(lx.argmax())
    for i in range(n_dec):
        lx = xs.step(tok)
        lg, am = s.step_argmax(tok)
        assert np.array_equal(u32(lg), u32(lx)), f"step {i}"
        assert am == int(lx.argmax())
        tok = am
    assert s.position() == xs.position() == n_pre + n_dec
    for L in (0, cfg.n_layers - 1):
        for p in (0, n_pre - 1, n_pre + n_dec - 1):
            for which in (0, 1):
                assert np.array_equal(s.kv(L, p, which), xs.kv(L, p, which))
    s.close()


def test_greedy_on_device(xr, cuda_ok, pair):
    cfg, T, m, d = pair
    toks = spmodel.gen_tokens(23, 16, cfg.n_vocab)
    xs = xr.session(d, cfg.max_context)
    tok = int(xs.prefill(toks)[-1].argmax())
    want = []
    t0 = tok
    for _ in range(12):
        t0 = int(xs.step(t0).argmax())
        want.append(t0)
    s = m.session(cfg.max_context)
    s.prefill(toks, logits=False)
    got = s.greedy(tok, 12)
    s.close()
    assert got.tolist() == want


def test_clone_rewind(xr, cuda_ok, pair):
    cfg, T, m, d = pair
    toks = spmodel.gen_tokens(24, 30, cfg.n_vocab)
    s = m.session(64)
    s.prefill(toks[:20], logits=False)
    c = s.clone()
    a = s.step(toks[20])
    b = c.step(toks[20])
    assert np.array_equal(u32(a), u32(b))
    s.step(toks[21]); s.step(toks[22])
    s.rewind(3)
    assert s.position() == 20
    assert np.array_equal(u32(s.step(toks[20])), u32(a))
    with pytest.raises(spb200.SpbError):
        s.rewind(1000)
    c.close(); s.close()


def test_full_forward_section6(xr, cuda_ok, pair):
    cfg, T, m, d = pair
    toks = spmodel.gen_tokens(25, 33, cfg.n_vocab)
    assert np.array_equal(u32(m.forward(toks)), u32(xr.session(d, 64).prefill(toks)))


def test_context_full_and_bad_token(cuda_ok, pair):
    cfg, T, m, d = pair
    s = m.session(4)
    s.prefill(np.array([1, 2, 3], np.int32), logits=False)
    s.step(5)
    with pytest.raises(spb200.SpbError) as e:
        s.step(6)
    assert e.value.code == spb200.SPB_ECONTEXT_FULL
    s.rewind(1)
    with pytest.raises(spb200.SpbError) as e:
        s.step(cfg.n_vocab + 5)
    assert e.value.code == spb200.SPB_ERANGE and "token" in str(e.value)
    assert s.position() == 3          # a failed step leaves the position unchanged
    s.step(5)                         # and the session usable
    s.close()


def test_synthetic_device_model_matches_host_generator(cuda_ok):
    cfg = spmodel.CONFIGS["micro_gemma"]
    T = spmodel.gen_model(cfg, seed=5)
    a = spb200.Model.upload(cfg, T)
    b = spb200.Model.synthetic(cfg, seed=5)
    toks = spmodel.gen_tokens(26, 12, cfg.n_vocab)
    assert np.array_equal(u32(a.forward(toks)), u32(b.forward(toks)))
    a.free(); b.free()


def test_sliding_window_long_context(xr, cuda_ok):
    """Local layers with a window of 16 over 100 positions, GQA group 4."""
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_gemma"], n_head=8, n_head_kv=2)
    T = spmodel.gen_model(cfg, seed=6)
    m = spb200.Model.upload(cfg, T)
    toks = spmodel.gen_tokens(27, 100, cfg.n_vocab)
    got = m.forward(toks)
    want = xr.session(xref.build_desc(cfg, T), 128).prefill(toks)
    m.free()
    assert np.array_equal(u32(got), u32(want))


@pytest.mark.parametrize("hd,nh,nkv", [(256, 8, 2), (128, 8, 8), (128, 16, 2), (256, 4, 2), (128, 8, 2),
                                       (128, 32, 8)])
def test_attention_head_shapes(xr, cuda_ok, hd, nh, nkv):
    """Head widths 128 / 256 and GQA groups 1-8: q held in registers (G * hd <= 512) or read
    from shared memory, one CTA per (row, KV head) when rows x KV heads fill the GPU (the
    64-row chunk with 8 KV heads) and clusters otherwise; a 70-token prefill spans several
    K/V stages."""
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_gemma"], n_layers=2, head_dim=hd, n_head=nh,
                              n_head_kv=nkv)
    T = spmodel.gen_model(cfg, seed=11)
    m = spb200.Model.upload(cfg, T)
    toks = spmodel.gen_tokens(31, 70, cfg.n_vocab)
    s = m.session(cfg.max_context)
    got = s.prefill(toks)
    want_s = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    want = want_s.prefill(toks)
    assert np.array_equal(u32(got), u32(want))
    for t in spmodel.gen_tokens(32, 3, cfg.n_vocab):
        assert np.array_equal(u32(s.step(int(t))), u32(want_s.step(int(t))))
    s.close()
    want_s.close()
    m.free()


@pytest.mark.parametrize("name", ["micro_qwen", "micro_gemma"])
def test_prefill_k_not_multiple_of_256(xr, cuda_ok, name):
    """Attention output projection with K = 128 and FFN down with K = 384 (what a
    tensor-parallel rank holds of a small model): no tensor-core GEMM for those matrices, so a
    40-row prefill chunk runs them as GEMV pieces of 32 + 8 rows; == XREF."""
    cfg = dataclasses.replace(spmodel.CONFIGS[name], n_layers=2, n_head=2, n_head_kv=1, n_ff=384)
    T = spmodel.gen_model(cfg, seed=12)
    m = spb200.Model.upload(cfg, T)
    toks = spmodel.gen_tokens(33, 40, cfg.n_vocab)
    got = m.forward(toks)
    want = xr.session(xref.build_desc(cfg, T), cfg.max_context).prefill(toks)
    m.free()
    assert np.array_equal(u32(got), u32(want))


@pytest.mark.parametrize("hd,nh,nkv,win", [(256, 4, 2, 40), (128, 8, 2, 300), (64, 8, 8, 24)])
def test_prefill_row_tiles_long_context(xr, cuda_ok, hd, nh, nkv, win):
    """Prefill chunks of 256 rows run attention in row tiles (16 query vectors of one KV head
    per CTA, each K/V slice staged once for all of them): 600 positions in chunks of 256 + 256
    + 88 rows, sliding windows shorter than a chunk (rows of one tile start their windows at
    different positions) on the local layers, the full context on the global one, then decode
    steps; every logit and K/V row == XREF."""
    cfg = dataclasses.replace(spmodel.CONFIGS["micro_gemma"], n_layers=6, head_dim=hd, n_head=nh,
                              n_head_kv=nkv, sliding_window=win, max_context=640)
    T = spmodel.gen_model(cfg, seed=13)
    m = spb200.Model.upload(cfg, T)
    toks = spmodel.gen_tokens(34, 600, cfg.n_vocab)
    s = m.session(cfg.max_context)
    want_s = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    s.prefill(toks, logits=False)
    want_s.prefill(toks, all_logits=False)
    for L in (0, 5):
        for p in (0, 255, 256, 511, 599):
            for w in (0, 1):
                assert np.array_equal(s.kv(L, p, w), want_s.kv(L, p, w)), (L, p, w)
    for t in spmodel.gen_tokens(35, 3, cfg.n_vocab):
        assert np.array_equal(u32(s.step(int(t))), u32(want_s.step(int(t))))
    s.close()
    want_s.close()
    m.free()
