"""Multi-session batched decode (spb_batch_decode_step) against each session decoding alone.

B sessions with ragged contexts step together: every row's logits, argmax and new KV rows
must be the bytes the same session produces with its own spb_session_decode_step (which the
other GPU tests tie to XREF). Row counts cover the dp4a GEMV (1, 2, 8), the tensor-core GEMM
with a partial 16-row tile (3, 20) and full tiles (16, 64)."""
import dataclasses

import numpy as np
import pytest

import spb200
import spmodel

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def sessions_with_history(m, cfg, B, seed, pmax):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(B):
        n = int(rng.integers(1, 60))
        toks = spmodel.gen_tokens(seed * 100 + i, n, cfg.n_vocab)
        s = m.session(pmax)
        s.prefill(toks, logits=False)
        out.append((s, int(toks[-1])))
    return out


@pytest.mark.parametrize("name,B", [("micro_gemma", 3), ("micro_gemma", 20), ("micro_qwen", 16),
                                    ("micro_qwen", 1), ("tiny", 8), ("tiny", 2), ("micro_gemma", 64),
                                    ("kv8", 64)])
def test_batch_matches_single_sessions(cuda_ok, name, B):
    if name == "kv8":   # 64 rows x 8 KV heads: one attention CTA per (row, KV head)
        cfg = dataclasses.replace(spmodel.CONFIGS["micro_qwen"], name="kv8", n_head=8, n_head_kv=8)
    else:
        cfg = spmodel.CONFIGS[name]
    m = spb200.Model.synthetic(cfg, seed=7)
    pmax = 96
    batch = sessions_with_history(m, cfg, B, 40 + B, pmax)
    alone = sessions_with_history(m, cfg, B, 40 + B, pmax)
    toks = [t for _, t in batch]
    for step in range(4):
        lg, am = spb200.batch_decode([s for s, _ in batch], toks)
        for i, (s, _) in enumerate(alone):
            l1, a1 = s.step_argmax(toks[i])
            assert np.array_equal(u32(lg[i]), u32(l1)), f"step {step} row {i}"
            assert am[i] == a1
        toks = [int(a) for a in am]
    for (sb, _), (sa, _) in zip(batch, alone):
        assert sb.position() == sa.position()
        p = sb.position() - 1
        for L in (0, cfg.n_layers - 1):
            for w in (0, 1):
                assert np.array_equal(sb.kv(L, p, w), sa.kv(L, p, w))
    for s, _ in batch + alone:
        s.close()
    m.free()


def test_batch_rejects_repeats_and_full_context(cuda_ok):
    cfg = spmodel.CONFIGS["micro_qwen"]
    m = spb200.Model.synthetic(cfg, seed=8)
    a, b = m.session(8), m.session(2)
    a.prefill(np.array([1, 2], np.int32), logits=False)
    b.prefill(np.array([3, 4], np.int32), logits=False)
    with pytest.raises(spb200.SpbError) as e:
        spb200.batch_decode([a, a], [5, 6])
    assert e.value.code == spb200.SPB_EBADARG
    with pytest.raises(spb200.SpbError) as e:
        spb200.batch_decode([a, b], [5, 6])
    assert e.value.code == spb200.SPB_ECONTEXT_FULL
    assert a.position() == 2 and b.position() == 2
    a.close(); b.close(); m.free()
