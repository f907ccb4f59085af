"""The persistent decode-step kernel (one cooperative launch per token) against the
multi-kernel schedule and against XREF.

Both decode paths must give byte-identical logits, greedy tokens and KV rows. The
12B-width case runs the shapes the bench runs (16-row tiles, the 4-segment down matrix,
16/8 heads of 256) on two layers, with a context long enough that every KV head is
split over many CTAs and the sliding window cuts the local layers."""
import dataclasses

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture
def mode_restore(spb):
    prev = spb.spb_decode_mode(-1)
    yield spb
    spb.spb_decode_mode(prev)


def run_steps(m, cfg, toks, n_dec, pmax):
    s = m.session(pmax)
    s.prefill(toks, logits=False)
    tok = int(toks[-1])
    out = []
    for _ in range(n_dec):
        lg, am = s.step_argmax(tok)
        out.append((lg.copy(), am))
        tok = am
    kv = [s.kv(L, p, w) for L in (0, cfg.n_layers - 1) for p in (0, len(toks) + n_dec - 1) for w in (0, 1)]
    s.close()
    return out, kv


@pytest.mark.parametrize("name", ["micro_gemma", "micro_qwen", "tiny"])
def test_persistent_matches_xref(xr, cuda_ok, mode_restore, name):
    spb = mode_restore
    cfg = spmodel.CONFIGS[name]
    T = spmodel.gen_model(cfg, seed=3)
    m = spb200.Model.upload(cfg, T)
    toks = spmodel.gen_tokens(31, 37, cfg.n_vocab)
    xs = xr.session(xref.build_desc(cfg, T), cfg.max_context)
    xs.prefill(toks)
    spb.spb_decode_mode(1)
    got, _ = run_steps(m, cfg, toks, 10, cfg.max_context)
    tok = int(toks[-1])
    for i, (lg, am) in enumerate(got):
        lx = xs.step(tok)
        assert np.array_equal(u32(lg), u32(lx)), f"step {i}"
        assert am == int(lx.argmax())
        tok = am
    m.free()


@pytest.mark.parametrize("name,n_pre", [("micro_gemma", 150), ("micro_qwen", 200), ("tiny", 300)])
def test_persistent_matches_multikernel_long_context(cuda_ok, mode_restore, name, n_pre):
    spb = mode_restore
    cfg = spmodel.CONFIGS[name]
    m = spb200.Model.synthetic(cfg, seed=4)
    toks = spmodel.gen_tokens(32, n_pre, cfg.n_vocab)
    pmax = n_pre + 16
    spb.spb_decode_mode(0)
    a, kva = run_steps(m, cfg, toks, 8, pmax)
    spb.spb_decode_mode(1)
    b, kvb = run_steps(m, cfg, toks, 8, pmax)
    m.free()
    for i, ((la, ta), (lb, tb)) in enumerate(zip(a, b)):
        assert np.array_equal(u32(la), u32(lb)), f"step {i}"
        assert ta == tb
    for x, y in zip(kva, kvb):
        assert np.array_equal(x, y)


def test_persistent_12b_width(cuda_ok, mode_restore):
    spb = mode_restore
    cfg = dataclasses.replace(spmodel.CONFIGS["gemma12b"], n_layers=2, n_vocab=4096, swa_period=2,
                              sliding_window=256)
    m = spb200.Model.synthetic(cfg, seed=5)
    toks = spmodel.gen_tokens(33, 700, cfg.n_vocab)
    spb.spb_decode_mode(0)
    a, kva = run_steps(m, cfg, toks, 6, 720)
    spb.spb_decode_mode(1)
    b, kvb = run_steps(m, cfg, toks, 6, 720)
    m.free()
    for i, ((la, ta), (lb, tb)) in enumerate(zip(a, b)):
        assert np.array_equal(u32(la), u32(lb)), f"step {i}"
        assert ta == tb
    for x, y in zip(kva, kvb):
        assert np.array_equal(x, y)


def test_persistent_greedy_and_rewind(cuda_ok, mode_restore):
    spb = mode_restore
    cfg = spmodel.CONFIGS["micro_gemma"]
    m = spb200.Model.synthetic(cfg, seed=6)
    toks = spmodel.gen_tokens(34, 40, cfg.n_vocab)
    res = {}
    for mode in (0, 1):
        spb.spb_decode_mode(mode)
        s = m.session(128)
        s.prefill(toks, logits=False)
        g1 = s.greedy(int(toks[-1]), 20)
        s.rewind(20)
        g2 = s.greedy(int(toks[-1]), 20)
        res[mode] = (g1.tolist(), g2.tolist())
        s.close()
    m.free()
    assert res[0] == res[1]
    assert res[1][0] == res[1][1]
