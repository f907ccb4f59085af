"""Paged, copy-on-write K/V on the GPU, byte for byte against XREF.

The reference forks a session by copying its whole cache (sp_session_clone, sp_session.c:773-816)
and rewinds in O(1) (:818-824). Paged sessions keep their K/V rows in pages of a pool shared by
the model's sessions: a clone takes the same pages and a page is copied only when one of the
sessions holding it writes into it. Every result must equal an unpaged session's and XREF's:
prefill across page boundaries, decode, clone and divergence, rewind into a shared page, the
speculative loop (clone, 4-token batched draft, rewind of 0-4 rejected tokens) over ragged
contexts, and a pool that runs out of pages."""
import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu

PG = 128


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module", params=["micro_gemma", "micro_qwen"])
def env(request):
    cfg = spmodel.CONFIGS[request.param]
    T = spmodel.gen_model(cfg, seed=5)
    m = spb200.Model.upload(cfg, T)
    pool = spb200.KvPool(m, PG, 64)
    yield cfg, T, m, pool
    pool.free()
    m.free()


def test_paged_matches_unpaged_and_xref(xr, cuda_ok, env):
    cfg, T, m, pool = env
    pmax = 520
    toks = spmodel.gen_tokens(61, 300, cfg.n_vocab)     # 300 positions: pages 0, 1, 2
    sp, su = pool.session(pmax), m.session(pmax)
    xs = xr.session(xref.build_desc(cfg, T), pmax)
    a, b, c = sp.prefill(toks), su.prefill(toks), xs.prefill(toks)
    assert np.array_equal(u32(a), u32(c)) and np.array_equal(u32(b), u32(c))
    tok = int(c[-1].argmax())
    for i in range(12):                                  # positions 300..311, then greedy on the device
        la, ta = sp.step_argmax(tok)
        lx = xs.step(tok)
        assert np.array_equal(u32(la), u32(lx)), i
        tok = ta
    g1 = sp.greedy(tok, 20)
    g2 = np.array([0] * 20)
    t2 = tok
    for i in range(20):
        t2 = int(xs.step(t2).argmax())
        g2[i] = t2
    assert g1.tolist() == g2.tolist()
    for L in (0, cfg.n_layers - 1):
        for p in (0, 127, 128, 255, 256, 331):
            for w in (0, 1):
                assert np.array_equal(sp.kv(L, p, w), xs.kv(L, p, w)), (L, p, w)
    sp.close()
    su.close()
    xs.close()
    assert pool.free_pages() == pool.n_pages


def test_clone_shares_pages_and_copies_on_write(xr, cuda_ok, env):
    cfg, T, m, pool = env
    pmax = 400
    toks = spmodel.gen_tokens(62, 150, cfg.n_vocab)     # pages 0 and 1 (positions 128..149)
    s = pool.session(pmax)
    s.prefill(toks, logits=False)
    xs = xr.session(xref.build_desc(cfg, T), pmax)
    xs.prefill(toks, all_logits=False)
    free0 = pool.free_pages()
    c = s.clone()
    assert pool.free_pages() == free0                    # the clone took no page
    xc = xs.clone()
    # the clone writes position 150 into the shared page 1: one page copied
    lc, tc = c.step_argmax(5)
    assert np.array_equal(u32(lc), u32(xc.step(5)))
    assert pool.free_pages() == free0 - 1
    # the original writes its own token at 150 into page 1, now its own: no further page
    ls, ts = s.step_argmax(9)
    assert np.array_equal(u32(ls), u32(xs.step(9)))
    assert pool.free_pages() == free0 - 1
    for i in range(8):                                   # both diverge, each exact
        lc, ntc = c.step_argmax(tc)
        ls, nts = s.step_argmax(ts)
        assert np.array_equal(u32(lc), u32(xc.step(tc))), ("clone", i)
        assert np.array_equal(u32(ls), u32(xs.step(ts))), ("orig", i)
        tc, ts = ntc, nts
    c.close()
    s.close()
    xs.close()
    xc.close()
    assert pool.free_pages() == pool.n_pages


def test_clone_trajectories_exact(xr, cuda_ok, env):
    cfg, T, m, pool = env
    pmax = 400
    toks = spmodel.gen_tokens(63, 140, cfg.n_vocab)
    s = pool.session(pmax)
    s.prefill(toks, logits=False)
    xs = xr.session(xref.build_desc(cfg, T), pmax)
    xs.prefill(toks, all_logits=False)
    c, xc = s.clone(), xs.clone()
    ts, tc = 11, 12
    for i in range(10):
        ls, ns = s.step_argmax(ts)
        lc, nc = c.step_argmax(tc)
        assert np.array_equal(u32(ls), u32(xs.step(ts))), ("orig", i)
        assert np.array_equal(u32(lc), u32(xc.step(tc))), ("clone", i)
        ts, tc = ns, nc
    # rewind the original back into the page the clone still shares, then write there again
    s.rewind(8)
    xs.rewind(8)
    ls, _ = s.step_argmax(3)
    assert np.array_equal(u32(ls), u32(xs.step(3)))
    lc, _ = c.step_argmax(tc)
    assert np.array_equal(u32(lc), u32(xc.step(tc)))
    for p in (139, 140, 142):
        assert np.array_equal(c.kv(0, p, 1), xc.kv(0, p, 1))
        assert np.array_equal(s.kv(0, p, 0), xs.kv(0, p, 0))
    for h in (s, c, xs, xc):
        h.close()


def test_speculative_loop_matches_sequential(xr, cuda_ok, env):
    """Six sessions of ragged contexts; each step: clone every session, draft 4 tokens on the
    clones in one batched decode per token, reject a seeded 0-4 of them (rewind), and keep the
    clone. XREF replays each session alone: the same 4 steps, the same rewind."""
    cfg, T, m, pool = env
    rng = np.random.default_rng(7)
    B, pmax = 6, 420
    ctx = rng.integers(20, 300, size=B)
    desc = xref.build_desc(cfg, T)
    sess, xss, nxt = [], [], []
    for i in range(B):
        t = spmodel.gen_tokens(100 + i, int(ctx[i]), cfg.n_vocab)
        s = pool.session(pmax)
        s.prefill(t, logits=False)
        x = xr.session(desc, pmax)
        lx = x.prefill(t)[-1]
        sess.append(s)
        xss.append(x)
        nxt.append(int(lx.argmax()))
    for step in range(5):
        clones = [s.clone() for s in sess]
        inputs = [list() for _ in range(B)]
        outs = [list() for _ in range(B)]
        toks = list(nxt)
        for k in range(4):
            lg, am = spb200.batch_decode(clones, toks)
            for i in range(B):
                lx = xss[i].step(toks[i])
                assert np.array_equal(u32(lg[i]), u32(lx)), (step, k, i)
                inputs[i].append(toks[i])
                outs[i].append(int(am[i]))
            toks = [int(a) for a in am]
        rej = rng.integers(0, 5, size=B)
        for i in range(B):
            r = int(rej[i])
            clones[i].rewind(r)
            assert xss[i].rewind(r) == 0
            nxt[i] = outs[i][3 - r] if r < 4 else nxt[i]
            sess[i].close()
            assert clones[i].position() == xss[i].position()
        sess = clones
    for s in sess:
        s.close()
    for x in xss:
        x.close()
    assert pool.free_pages() == pool.n_pages


def test_pool_exhaustion_is_reported(cuda_ok, env):
    cfg, T, m, _ = env
    small = spb200.KvPool(m, PG, 2)
    s = small.session(600)
    toks = spmodel.gen_tokens(64, 300, cfg.n_vocab)       # needs 3 pages
    with pytest.raises(spb200.SpbError) as ei:
        s.prefill(toks, logits=False)
    assert ei.value.code == spb200.SPB_EOOM
    s.prefill(toks[:200], logits=False)                    # 2 pages: fits, the session still works
    assert s.position() == 200 and small.free_pages() == 0
    s.close()
    assert small.free_pages() == 2
    small.free()


def test_batch_mixes_paged_and_unpaged(xr, cuda_ok, env):
    cfg, T, m, pool = env
    desc = xref.build_desc(cfg, T)
    sess, xss = [], []
    for i, paged in enumerate((True, False, True)):
        t = spmodel.gen_tokens(200 + i, 60 + 70 * i, cfg.n_vocab)
        s = pool.session(300) if paged else m.session(300)
        s.prefill(t, logits=False)
        x = xr.session(desc, 300)
        x.prefill(t, all_logits=False)
        sess.append(s)
        xss.append(x)
    toks = [3, 4, 5]
    for k in range(3):
        lg, am = spb200.batch_decode(sess, toks)
        for i in range(3):
            assert np.array_equal(u32(lg[i]), u32(xss[i].step(toks[i])))
        toks = [int(a) for a in am]
    for h in sess + xss:
        h.close()


def test_reopened_session_starts_clean(xr, cuda_ok, env):
    """A closed session's device buffer, stream and pinned staging go to the next open of the same
    shape (the clone-and-close loop then allocates nothing): the new session starts from an empty
    state, whatever the old one held, and its results equal XREF's, paged and unpaged."""
    cfg, T, m, pool = env
    d = xref.build_desc(cfg, T)
    for paged in (True, False):
        def open_():
            return pool.session(300) if paged else m.session(300)
        old = open_()
        old.prefill(spmodel.gen_tokens(70, 200, cfg.n_vocab), logits=False)
        old.greedy(5, 16)
        st = old.stream()
        old.close()
        s = open_()
        assert s.stream() == st, "closed session's stream not reused"
        xs = xr.session(d, 300)
        toks = spmodel.gen_tokens(71, 37, cfg.n_vocab)
        assert np.array_equal(u32(s.prefill(toks)), u32(xs.prefill(toks)))
        tok = int(toks[-1])
        for i in range(6):
            la, ta = s.step_argmax(tok)
            assert np.array_equal(u32(la), u32(xs.step(tok))), (paged, i)
            tok = ta
        for p in (0, 36, 42):
            assert np.array_equal(s.kv(1, p, 0), xs.kv(1, p, 0)), (paged, p)
        s.close()
        xs.close()
