"""The benchmark geometries at full width on the GPU, two layers deep, byte for byte against XREF.

* Qwen3-8B: d_model 4096, 32 query / 8 KV heads of 128 (GQA group 4),
  SwiGLU FFN 12288 (the down projection's K = 12288 is 384 scale blocks, 12 code vectors per
  lane), untied LM head over the full 151936-token vocabulary (not a multiple of any tile).
  Reference path: qwen3_forward_ex2 (forward.c:87-291) / kv_step (sp_session.c:274-363).
* Gemma-3-12B widths: d_model 3840, 16/8 heads of 256, GeGLU FFN 15360,
  with a sliding window short enough that the prefill and the decode steps cross it.
  Reference path: gemma3_forward (gemma3.c:39-148) / kv_step_gemma3 (sp_session.c:380-464).

Prefill runs the token-batch GEMM in 64-row chunks plus a ragged last chunk; decode runs the
GEMV; every logit, the greedy tokens and cached K/V rows must equal XREF's."""
import dataclasses

import numpy as np
import pytest

import spb200
import spmodel
import xref

pytestmark = pytest.mark.gpu


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def run_case(xr, cfg, seed, n_pre, n_dec, pmax):
    T = spmodel.gen_model(cfg, seed=seed)
    m = spb200.Model.upload(cfg, T)
    s = m.session(pmax)
    xs = xr.session(xref.build_desc(cfg, T), pmax)
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
        for p in (0, n_pre - 1, n_pre + n_dec - 1):
            for which in (0, 1):
                assert np.array_equal(s.kv(L, p, which), xs.kv(L, p, which)), (L, p, which)
    s.close()
    xs.close()
    m.free()


def test_qwen8b_geometry(xr, cuda_ok):
    cfg = dataclasses.replace(spmodel.CONFIGS["qwen8b"], n_layers=2)
    run_case(xr, cfg, 41, 70, 4, 96)


def test_gemma12b_width_sliding_window(xr, cuda_ok):
    cfg = dataclasses.replace(spmodel.CONFIGS["gemma12b"], n_layers=2, n_vocab=4096, swa_period=2,
                              sliding_window=64)
    run_case(xr, cfg, 43, 150, 6, 192)
