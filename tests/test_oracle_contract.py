"""The builder-defined parts of the exact contract, checked on CPU:
exact int64 matvec (vs an independent numpy restatement), CORDIC-RoPE (vs float RoPE and
vs the product's own host tables), exact SiLU fidelity, XREF session semantics
(prefill == sequential decode, clone, rewind)."""
import numpy as np
import pytest

import spmodel
import xref
from conftest import rng


def numpy_matvec(t, X):
    """Independent restatement of the exact matvec: int64 numpy, one final rounding."""
    K = t.cols
    nib = t.codes.astype(np.int16)
    lo = nib & 0xF
    hi = nib >> 4
    c = np.empty((t.rows, K), np.int64)
    c[:, 0::2] = np.where(lo >= 8, lo - 16, lo)
    c[:, 1::2] = np.where(hi >= 8, hi - 16, hi)
    h = t.bscale.astype(np.int64)
    e = (h >> 10) & 31
    m = h & 1023
    k = np.where(e > 0, (m | 1024) << np.maximum(e - 1, 0), m)
    k = np.where(h & 0x8000, -k, k)
    out = []
    for x in np.atleast_2d(X):
        s = np.float32(np.abs(x).max())
        xs = (x / s).astype(np.float32) * np.float32(127)
        q = np.where(xs >= 0, np.floor(xs + np.float32(0.5)), np.ceil(xs - np.float32(0.5)))
        q = np.clip(q, -127, 127).astype(np.int64)
        isum = (c * q[None, :]).reshape(t.rows, -1, 32).sum(-1)
        acc = (isum * k).sum(-1)
        dsc = (np.float64(s) / 127.0) * 2.0 ** -24
        out.append((acc.astype(np.float64) * dsc).astype(np.float32))
    return np.array(out)


@pytest.mark.parametrize("rows,cols,m", [(64, 256, 1), (33, 512, 4), (128, 1024, 2)])
def test_matvec_exact_vs_numpy(xr, rows, cols, m):
    t = spmodel.gen_matrix(3, "blk.0.attn_q.weight", rows, cols)
    X = rng(rows).standard_normal((m, cols)).astype(np.float32)
    assert np.array_equal(xr.matvec(t, X), numpy_matvec(t, X))


def test_matvec_edge_cases(xr):
    t = spmodel.gen_matrix(4, "blk.1.ffn_up.weight", 16, 64)
    assert np.all(xr.matvec(t, np.zeros((1, 64), np.float32)) == 0)       # all-zero input
    x = np.zeros((1, 64), np.float32)
    x[0, 5] = -3.0                                                        # single spike
    assert np.array_equal(xr.matvec(t, x), numpy_matvec(t, x))
    # extreme codes: all -8 and all 7 nibbles
    for byte in (0x88, 0x77):
        t2 = spmodel.Q4B(np.full((4, 32), byte, np.uint8), t.bscale[:4, :2].copy(), 4, 64)
        X = rng(1).standard_normal((2, 64)).astype(np.float32)
        assert np.array_equal(xr.matvec(t2, X), numpy_matvec(t2, X))


def test_quantizer_scale_invariance(xr):
    """quant1(x * 2^k, s * 2^k) == quant1(x, s): the property the full-size GPU tests use."""
    x = rng(2).standard_normal(4096).astype(np.float32)
    q1, s1 = xr.quant(x)
    q2, s2 = xr.quant(x * np.float32(8.0))
    assert np.array_equal(q1, q2) and s2 == s1 * 8


@pytest.mark.parametrize("base,d", [(10000.0, 64), (1e6, 128), (1e6, 256), (500000.0, 128)])
def test_rope_table_and_fidelity(xr, base, d):
    W = xr.rope_table(base, d)
    ref = base ** (-2.0 * np.arange(d // 2) / d) / (2 * np.pi)
    assert np.max(np.abs(W.astype(np.float64) / 2.0 ** 64 - ref) / ref) < 1e-12
    r = rng(d)
    for p in (0, 1, 17, 1023, 8191, 40000):
        v = r.standard_normal(d).astype(np.float32)
        out, rc = xr.rope(v, p, W)
        assert rc == 0
        th = p * base ** (-2.0 * np.arange(d // 2) / d)
        a, b = v[: d // 2].astype(np.float64), v[d // 2:].astype(np.float64)
        want = np.concatenate([a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)])
        assert np.max(np.abs(out / 65536.0 - want)) < 2e-5


def test_rope_range_errors(xr):
    W = xr.rope_table(10000.0, 64)
    v = np.zeros(64, np.float32)
    v[3] = 300.0
    _, rc = xr.rope(v, 5, W)
    assert rc == xref.XREF_ERANGE


def test_product_host_tables_match_oracle(xr, spb):
    import spb200
    for base, d in [(10000.0, 64), (1e6, 256), (1e6, 128)]:
        assert np.array_equal(spb200.rope_table(base, d), xr.rope_table(base, d))
    T, g = spb200.cordic_tables()
    T2 = np.zeros(30, np.uint64)
    xr.lib.xref_cordic_atan_table(T2.ctypes.data)
    assert np.array_equal(T, T2) and g == xr.lib.xref_cordic_gain_q62()


def test_silu_fidelity(xr):
    x = np.linspace(-30, 30, 200001).astype(np.float32)
    y = xr.silu(x)
    ref = x.astype(np.float64) / (1 + np.exp(-x.astype(np.float64)))
    assert np.max(np.abs(y - ref)) < 3e-5


@pytest.fixture(scope="module")
def micro():
    cfg = spmodel.CONFIGS["micro_gemma"]
    T = spmodel.gen_model(cfg, seed=1)
    return cfg, T, xref.build_desc(cfg, T)


def test_prefill_equals_sequential_decode(xr, micro):
    cfg, T, d = micro
    toks = spmodel.gen_tokens(3, 24, cfg.n_vocab)
    a = xr.session(d, 64).prefill(toks)
    s = xr.session(d, 64)
    b = np.array([s.step(t) for t in toks])
    assert np.array_equal(a, b)


def test_clone_and_rewind(xr, micro):
    cfg, T, d = micro
    toks = spmodel.gen_tokens(4, 20, cfg.n_vocab)
    s = xr.session(d, 64)
    s.prefill(toks[:12], all_logits=False)
    c = s.clone()
    la = s.step(toks[12])
    lb = c.step(toks[12])
    assert np.array_equal(la, lb)
    s.step(toks[13]); s.step(toks[14])
    assert s.rewind(3) == 0 and s.position() == 12
    assert np.array_equal(s.step(toks[12]), la)
    assert s.rewind(100) != 0


def test_sliding_window_matters(xr, micro):
    """Local layers attend only to the last `sliding_window` positions (16 here)."""
    import dataclasses
    cfg, T, _ = micro
    toks = spmodel.gen_tokens(5, 40, cfg.n_vocab)
    a = xr.session(xref.build_desc(cfg, T), 64).prefill(toks)
    cfg2 = dataclasses.replace(cfg, sliding_window=0)
    b = xr.session(xref.build_desc(cfg2, T), 64).prefill(toks)
    assert np.array_equal(a[:16], b[:16])       # inside the window: identical
    assert not np.array_equal(a[-1], b[-1])     # beyond it: differs


def test_bad_token_rejected(xr, micro):
    cfg, T, d = micro
    s = xr.session(d, 8)
    with pytest.raises(RuntimeError):
        s.step(cfg.n_vocab)
