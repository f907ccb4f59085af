"""CPU baselines for bench.py (benchmark infrastructure; never part of the product path).

Times the reference's OWN decode -- sp_decode_step of its float forward over OK_Q4B weights
(matmul_arena's Q4B branch, forward_dispatch.c:69-86, driven by kv_step_gemma3 / kv_step,
sp_session.c:274-464) -- from oracle/_ref/libspref.so, on the host cores, and the exact-integer
checker XREF (oracle/_ref/libxref.so) the same way.

Two measurements:

* `measure` -- the 12B shape, SCALED. A full 12B-shape decode token costs ~90 s per core, so
  each process times a bounded sample: a 1-layer model with the target's exact widths (E, FF,
  heads, head_dim) and a 2048-token vocabulary, written as a real .sp-model and driven through
  sp_session. The full model's per-token time is the sample step's time multiplied by the
  ratio of streamed weight parameters (every reference matvec is one pass over its weights at
  a fixed rate). What the scaling leaves out: attention over a long context (the sample runs
  at a context of a few tokens, the benchmark at ~2048) and the other 47 layers' cache
  traffic. P processes run concurrently, one per core, for the aggregate.
* `config1_e2e` -- BASELINE configs[0], UNSCALED: the tiny Gemma model end to end in one
  process, sp_prefill_chunk of 64 tokens then 64 greedy sp_decode_step calls (the reference's
  own session, sp_session.c:154,725), and XREF doing the same.
"""
from __future__ import annotations

import dataclasses
import multiprocessing as mp
import os
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (HERE, os.path.join(ROOT, "shannon-prime-system_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SAMPLE_VOCAB = 2048


def _params(cfg, n_layers, vocab):
    E, FF = cfg.n_embd, cfg.n_ff
    layer = (cfg.qd + 2 * cfg.kvd) * E + E * cfg.qd + 3 * FF * E
    return n_layers * layer + vocab * E


def sample_config(cfg):
    return dataclasses.replace(cfg, name=cfg.name + "_sample", n_layers=1, n_vocab=SAMPLE_VOCAB,
                               max_context=64)


def write_sample(cfg, directory):
    import spmodel
    sc = sample_config(cfg)
    T = spmodel.gen_model(sc, seed=0)
    mp_, tp = os.path.join(directory, "sample.sp-model"), os.path.join(directory, "sample.sp-tokenizer")
    spmodel.write_sp_model(mp_, tp, sc, T)
    return mp_, tp, sc


def _worker(args):
    model_path, tok_path, vocab, steps, warmup, barrier = args
    import xref
    R = xref.RefLib()
    m = R.load(model_path, tok_path)
    s = R.session(m, 64)
    rc, _ = R.prefill(s, [1], vocab)
    assert rc == 0, R.err()
    rc, _ = R.decode(s, 2, vocab)          # first decode backfills the prompt position
    assert rc == 0, R.err()
    for i in range(warmup):
        rc, _ = R.decode(s, 3 + i, vocab)
        assert rc == 0, R.err()
    times = []
    for i in range(steps):
        barrier.wait()                      # every process starts step i together
        t0 = time.perf_counter()
        rc, _ = R.decode(s, 3 + warmup + i, vocab)
        times.append(time.perf_counter() - t0)
        assert rc == 0, R.err()
    R.lib.sp_session_destroy(s)
    R.lib.sp_model_unload(m)
    return times


def measure(cfg, procs=None, steps=1, warmup=0):
    """The reference decode of `cfg`, sampled and scaled (see the module docstring). Each of the
    `steps` timed steps is one sample decode token in each of `procs` concurrent processes;
    step_wall_s is the slowest process's time for that step."""
    import xref
    if not os.path.exists(xref.SPREF_SO):
        return None
    procs = procs or os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as d:
        mp_, tp, sc = write_sample(cfg, d)
        ctx = mp.get_context("spawn")
        with ctx.Manager() as mgr:
            barrier = mgr.Barrier(procs)
            with ctx.Pool(procs) as pool:
                res = pool.map(_worker, [(mp_, tp, sc.n_vocab, steps, warmup, barrier)] * procs)
    walls = [max(r[i] for r in res) for i in range(steps)]
    per_step = sorted(t for r in res for t in r)
    med = per_step[len(per_step) // 2]
    scale = _params(cfg, cfg.n_layers, cfg.n_vocab) / _params(cfg, 1, SAMPLE_VOCAB)
    t_token = med * scale
    return {
        "value": procs / t_token,
        "per_core_tokens_per_s": 1.0 / t_token,
        "cores": procs,
        "steps_timed": steps,
        "step_wall_s": walls,
        "sample_step_s_median": med,
        "scale": scale,
        "scaled": True,
        "sample": (f"SCALED: reference sp_decode_step (float OK_Q4B forward, libspref from the reference "
                   f"sources) on a 1-layer {cfg.name}-width model (vocab {SAMPLE_VOCAB}), {steps} timed "
                   f"step(s) x {procs} concurrent processes; the median sample step x{scale:.1f} "
                   f"(streamed parameters of the full model / the sample) = one full-model token per "
                   f"process; leaves out attention at the benchmark's ~2048-token context"),
    }


def _config1_worker(args):
    which, n_pre, n_dec = args
    import numpy as np
    import spmodel
    import xref
    cfg = spmodel.CONFIGS["tiny"]
    T = spmodel.gen_model(cfg, seed=0)
    toks = spmodel.gen_tokens(1, n_pre, cfg.n_vocab)
    if which == "reference":
        R = xref.RefLib()
        with tempfile.TemporaryDirectory() as d:
            mp_, tp = os.path.join(d, "tiny.sp-model"), os.path.join(d, "tiny.sp-tokenizer")
            spmodel.write_sp_model(mp_, tp, cfg, T)
            m = R.load(mp_, tp)
        s = R.session(m, n_pre + n_dec + 8)
        t0 = time.perf_counter()
        rc, lg = R.prefill(s, toks, cfg.n_vocab)
        assert rc == 0, R.err()
        t1 = time.perf_counter()
        tok = int(np.argmax(lg))
        for _ in range(n_dec):
            rc, lg = R.decode(s, tok, cfg.n_vocab)
            assert rc == 0, R.err()
            tok = int(np.argmax(lg))
        t2 = time.perf_counter()
        R.lib.sp_session_destroy(s)
        R.lib.sp_model_unload(m)
    else:
        os.environ["XREF_THREADS"] = "1"
        xs = xref.Xref().session(xref.build_desc(cfg, T), n_pre + n_dec + 8)
        t0 = time.perf_counter()
        lg = xs.prefill(toks, all_logits=False)
        t1 = time.perf_counter()
        tok = int(np.argmax(lg))
        for _ in range(n_dec):
            tok = int(np.argmax(xs.step(tok)))
        t2 = time.perf_counter()
        xs.close()
    return {"prefill_s": t1 - t0, "decode_s": t2 - t1, "decode_tokens_per_s": n_dec / (t2 - t1),
            "e2e_tokens_per_s": (n_pre + n_dec) / (t2 - t0)}


def config1_e2e(which="reference", n_pre=64, n_dec=64):
    """BASELINE configs[0] end to end, unscaled, one process on one core: prefill n_pre tokens,
    then n_dec greedy decode steps. which = "reference" (the reference's float session) or
    "xref" (the exact-integer checker, single-threaded)."""
    import xref
    if which == "reference" and not os.path.exists(xref.SPREF_SO):
        return None
    ctx = mp.get_context("spawn")
    with ctx.Pool(1) as pool:
        r = pool.map(_config1_worker, [(which, n_pre, n_dec)])[0]
    r.update({"cores": 1, "kind": which, "scaled": False,
              "sample": f"tiny (BASELINE configs[0]): prefill {n_pre} + {n_dec} greedy decode steps, one process"})
    return r
