"""CPU baseline for bench.py (benchmark infrastructure; never part of the product path).

Times the reference's OWN decode -- sp_decode_step of its float forward over OK_Q4B
weights (matmul_arena's Q4B branch, forward_dispatch.c:69-86, driven by kv_step_gemma3 /
kv_step, sp_session.c:274-464) -- from oracle/_ref/libspref.so, on the host cores.

A full 12B-shape decode token costs ~90 s per core, so each process times a bounded
sample: a 1-layer model with the target's exact widths (E, FF, heads, head_dim) and a
small vocab, written as a real .sp-model and driven through sp_session. The per-token
time of the full model is that sample's time scaled by the ratio of streamed weight
parameters (every reference matvec is one pass over its weights at a fixed rate); the
attention term at the sample's short context is not scaled (it is a few percent of a
layer at context 2048). P processes run concurrently, one per core, and the aggregate
throughput is P tokens per scaled token-time.
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
    model_path, tok_path, vocab, steps = args
    import xref
    R = xref.RefLib()
    m = R.load(model_path, tok_path)
    s = R.session(m, 64)
    rc, _ = R.prefill(s, [1], vocab)
    assert rc == 0, R.err()
    rc, _ = R.decode(s, 2, vocab)          # first decode backfills the prompt position
    assert rc == 0, R.err()
    times = []
    for i in range(steps):
        t0 = time.perf_counter()
        rc, _ = R.decode(s, 3 + i, vocab)
        times.append(time.perf_counter() - t0)
        assert rc == 0, R.err()
    R.lib.sp_session_destroy(s)
    R.lib.sp_model_unload(m)
    return times


def measure(cfg, procs=None, steps=1):
    """Aggregate reference CPU decode tokens/s for `cfg`, scaled from the sample."""
    import xref
    if not os.path.exists(xref.SPREF_SO):
        return None
    procs = procs or os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as d:
        mp_, tp, sc = write_sample(cfg, d)
        ctx = mp.get_context("spawn")
        with ctx.Pool(procs) as pool:
            res = pool.map(_worker, [(mp_, tp, sc.n_vocab, steps)] * procs)
    per_step = sorted(t for r in res for t in r)
    med = per_step[len(per_step) // 2]
    scale = _params(cfg, cfg.n_layers, cfg.n_vocab) / _params(cfg, 1, SAMPLE_VOCAB)
    t_token = med * scale
    return {
        "value": procs / t_token,
        "per_core_tokens_per_s": 1.0 / t_token,
        "cores": procs,
        "sample_step_s": med,
        "scale": scale,
        "sample": (f"reference sp_decode_step (float OK_Q4B forward, libspref from the reference "
                   f"sources) on a 1-layer {cfg.name}-width model (vocab {SAMPLE_VOCAB}), "
                   f"{steps} timed step(s) x {procs} concurrent processes; per-token time scaled "
                   f"by streamed params x{scale:.1f}"),
    }
