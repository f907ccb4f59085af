#!/usr/bin/env python
"""bench.py -- byte-exact decode tokens/s at the Gemma-3-12B shape (B=1), plus the
dequant-GEMV's achieved HBM bandwidth against the measured peak.

Workload: Gemma-3-12B-shaped decoder (48 layers, d_model
3840, 16/8 heads, head_dim 256, FFN 15360 exact-GELU, vocab 262144, sliding window 1024
on 5 of every 6 layers), random-init OK_Q4B weights generated on the device from a
seed, batch 1: prefill --prefill random tokens (untimed), W warm-up decode steps, then
K timed greedy decode steps. A step is one decode token through the whole model.

  value    K tokens / device time of the K steps (CUDA events on the session stream;
           inputs resident: each step's token is the previous step's device argmax)
  e2e      the same K steps through the public C ABI call a user makes
           (spb_session_decode_step_argmax): the token copied host->device from pinned
           memory and the full-vocab logits copied device->host every step
  roofline the dequant-GEMV alone, per decode shape, CUDA-event timed over weights
           larger than L2, weighted by its share of a decode token's bytes
  prefill  the untimed --prefill ingestion timed with CUDA events: tokens/s and the
           tensor-core GEMM's int8 ops/s against an int8 dense peak (2 x measured bf16)
  b64      --batch sessions (default 64) decoding together (spb_batch_decode_step)
  tp       with --tp and N > 1: one session tensor-parallel over the N GPUs
Multi-GPU (torchrun): independent sessions spread one per GPU (weak scaling); the only
collectives are the barrier and the max-over-ranks of the timings.

--impl reference times the reference's own CPU decode (oracle/cpu_baseline.py) instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "shannon-prime-system_b200")
ORACLE = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

METRIC = "byte-exact decode tokens/s (12B shape, B=1/64); dequant-GEMV HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", default="spb", choices=["spb", "reference"])
    p.add_argument("--config", default="gemma12b")
    p.add_argument("--prefill", type=int, default=2048)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-roofline", action="store_true")
    # profiling-size overrides (smaller device footprint for ncu captures); a line printed
    # with either set is not the configs[2] measurement and says so in config.workload
    p.add_argument("--layers", type=int, default=0)
    p.add_argument("--vocab", type=int, default=0)
    p.add_argument("--batch", type=int, default=64,
                   help="sessions decoded together for the b64 figure (0: skip it)")
    p.add_argument("--batch-steps", type=int, default=16)
    p.add_argument("--no-sweep", action="store_true", help="skip the isolated matmul sweep (configs[1])")
    p.add_argument("--spec-sessions", type=int, default=8,
                   help="speculative-decode sessions per GPU (configs[4]: 64 over 8 GPUs); 0 skips it")
    p.add_argument("--spec-steps", type=int, default=8)
    p.add_argument("--q8-prefill", type=int, default=4096, help="configs[3] prefill tokens (0 skips configs[3])")
    p.add_argument("--q8-steps", type=int, default=512)
    p.add_argument("--spinor", type=int, default=1,
                   help="also time B=1 decode on a Spinor-block K/V session (SPB_KV_SPINOR); 0 skips it")
    p.add_argument("--spin-batch", type=int, default=16,
                   help="sessions of the long-context batch comparison (int32 against Spinor K/V); 0 skips it")
    p.add_argument("--spin-ctx", type=int, default=4096, help="their shared prefix length")
    p.add_argument("--spin-batch-steps", type=int, default=8)
    p.add_argument("--no-tp", action="store_true", help="N>1: skip the tensor-parallel objects")
    p.add_argument("--tp", action="store_true", help="(default with N>1) the tensor-parallel objects")
    p.add_argument("--probe-gemm", default="",
                   help="ROWS,COLS,M: time only spb_q4b_matmul of one prepared seeded matrix at M token "
                        "rows (a small case for ncu captures of the token-batch GEMM) and exit")
    p.add_argument("--probe-iters", type=int, default=5)
    return p.parse_args()


def bench_config(args):
    import dataclasses
    import spmodel
    cfg = spmodel.CONFIGS[args.config]
    over = {}
    if args.layers:
        over["n_layers"] = args.layers
    if args.vocab:
        over["n_vocab"] = args.vocab
    if over:
        cfg = dataclasses.replace(cfg, name=cfg.name + "_profile", **over)
    return cfg


def line_config(cfg, args, world):
    """The config object both arms print (the same workload, so the driver can pair them)."""
    return {"workload": f"{cfg.name} decode B=1 after a {args.prefill}-token prefill (BASELINE configs[2])",
            "model": "Gemma-3-12B shape: 48L d3840 16/8 heads hd256 FFN15360 vocab262144 SWA1024 (5 of 6)"
            if cfg.name == "gemma12b" else cfg.name,
            "global_batch": world, "seq_len": args.prefill + args.warmup + args.steps,
            "parallelism": f"sessions spread: {world} independent session(s), one per GPU",
            "l2": "weights 6.6 GB per step >> 126 MB L2: every step streams from HBM"}


def measure_config1_gpu(device):
    """BASELINE configs[0] (tiny Gemma) on the GPU through the public session API, the same
    steps as the CPU's unscaled config-1 run: spb_session_prefill of 64 tokens, then 64 greedy
    spb_session_decode_step_argmax calls with the full-vocab logits copied to host memory."""
    import torch
    import spb200
    import spmodel
    cfg = spmodel.CONFIGS["tiny"]
    m = spb200.Model.synthetic(cfg, seed=0, device=device)
    toks = spmodel.gen_tokens(1, 64, cfg.n_vocab)
    lg = np.empty(cfg.n_vocab, np.float32)
    for rep in range(2):   # the first pass builds the step graph; the second is timed
        s = m.session(64 + 64 + 8)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = s.prefill(toks)
        t1 = time.perf_counter()
        tok = int(out[-1].argmax())
        for _ in range(64):
            _, tok = s.step_argmax(tok, out=lg)
        t2 = time.perf_counter()
        s.close()
    m.free()
    return {"prefill_s": round(t1 - t0, 5), "decode_s": round(t2 - t1, 5),
            "decode_tokens_per_s": round(64 / (t2 - t1), 1), "e2e_tokens_per_s": round(128 / (t2 - t0), 1),
            "timing": "wall clock, host-buffer API (tokens in, every step's full-vocab logits out)"}


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait(timeout=10)
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


# ----------------------------------------------------------------------------- GEMV roofline
def gemv_shapes(cfg):
    """(name, rows, cols, gated, launches per decode token) of the decode step's GEMVs."""
    E, FF = cfg.n_embd, cfg.n_ff
    return [("qkv", cfg.qd + 2 * cfg.kvd, E, False, cfg.n_layers),
            ("o", E, cfg.qd, False, cfg.n_layers),
            ("gate_up", FF, E, True, cfg.n_layers),
            ("down", E, FF, False, cfg.n_layers),
            ("lm_head", cfg.n_vocab, E, False, 1)]


def gemv_bytes(rows, cols, gated, m=1):
    mats = 2 if gated else 1
    return mats * (rows * cols // 2 + rows * (cols // 32) * 2) + m * cols + m * (cols // 32) * 4 + m * rows * 4


def gemv_roofline(cfg, spb, device, stream, iters=60):
    import ctypes as C
    import torch
    L2 = 126 * 2 ** 20
    out = {}
    tot_b = tot_t = 0.0
    launches = 0
    for name, rows, cols, gated, per_tok in gemv_shapes(cfg):
        mats = 2 if gated else 1
        wbytes = mats * (rows * cols // 2 + rows * (cols // 32) * 2)
        copies = max(1, -(-3 * L2 // wbytes))          # rotate so the set exceeds L2 threefold
        codes = [torch.randint(0, 256, (mats, rows * cols // 2), dtype=torch.uint8, device=device)
                 for _ in range(copies)]
        scl = [(torch.randint(0, 1024, (mats, rows * (cols // 32)), dtype=torch.int16, device=device)
                | (5 << 10)) for _ in range(copies)]
        x = torch.randn(1, cols, device=device)
        q = torch.empty(cols, dtype=torch.int8, device=device)
        bs = torch.empty(cols // 32, dtype=torch.int32, device=device)
        sc = torch.empty(1, dtype=torch.float32, device=device)
        y = torch.empty(rows, dtype=torch.float32, device=device)
        P = lambda t: C.c_void_p(t.data_ptr())
        spb.spb_quantize_rows(P(x), cols, 1, P(q), P(bs), P(sc), stream.cuda_stream)

        def launch(i):
            c, s = codes[i % copies], scl[i % copies]
            if gated:
                rc = spb.spb_gemv_q4b_gated_q(P(c[0]), P(s[0]), P(c[1]), P(s[1]), rows, cols, P(q), P(bs),
                                             P(sc), 1, 0, P(y), stream.cuda_stream)
            else:
                rc = spb.spb_gemv_q4b_q(P(c[0]), P(s[0]), rows, cols, P(q), P(bs), P(sc), 1, P(y),
                                        stream.cuda_stream)
            assert rc == 0, spb.spb_last_error()
        for i in range(5):
            launch(i)
        torch.cuda.synchronize()
        n = iters if name != "lm_head" else max(10, iters // 3)
        # capture the n launches once (the library's own capture helpers) so host enqueue
        # cost cannot hide between kernels; replay and time on the launching stream
        assert spb.spb_graph_begin(stream.cuda_stream) == 0, spb.spb_last_error()
        for i in range(n):
            launch(i)
        gexec = C.c_void_p()
        assert spb.spb_graph_end(stream.cuda_stream, C.byref(gexec)) == 0, spb.spb_last_error()
        assert spb.spb_graph_launch(gexec, stream.cuda_stream) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        assert spb.spb_graph_launch(gexec, stream.cuda_stream) == 0
        e1.record(stream)
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / n
        spb.spb_graph_free(gexec)
        if gemv_bytes(rows, cols, gated) / us / 1e3 > 2.0 * peaks()[0]:
            raise RuntimeError(f"GEMV timing for {name} exceeds twice the HBM peak: the capture did not record it")
        b = gemv_bytes(rows, cols, gated)
        out[name] = {"rows": rows, "cols": cols, "gated": gated, "us_per_launch": round(us, 3),
                     "bytes_per_launch": b, "gbs": round(b / us / 1e3, 1), "launches_per_token": per_tok}
        tot_b += b * per_tok
        tot_t += us * per_tok
        launches += n + 5
        del codes, scl
    return out, tot_b, tot_t, launches


SWEEP_SHAPES = [(3840, 3840), (15360, 3840), (3840, 15360), (262144, 3840)]
SWEEP_M = [1, 4, 16, 2048]


def gemm_sweep(spb, device, stream, int8_peak_tops, hbm_gbs, iters=20):
    """the OK_Q4B matmul alone (spb_q4b_matmul on a prepared matrix: the
    activation quantizer, then the dequant-GEMV for 1-16 token rows or the tcgen05 GEMM for
    2048), 4 weight shapes x M in {1, 4, 16, 2048}, random codes and seeded block scales with
    one exponent per matrix (two digit planes). CUDA events on the launching stream over
    `iters` launches; weight sets rotated so every launch reads from HBM for the small M.
    GB/s counts the algorithmic bytes (codes, scales, int8 activations, f32 outputs); TOP/s
    counts 2 x M x rows x K exact integer multiply-adds."""
    import ctypes as C
    import torch
    import spb200
    L2 = 126 * 2 ** 20
    P = lambda t: C.c_void_p(t.data_ptr())
    out = []
    for rows, cols in SWEEP_SHAPES:
        wbytes = rows * cols // 2 + rows * (cols // 32) * 2
        copies = max(1, -(-3 * L2 // wbytes))
        codes = [torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device=device) for _ in range(copies)]
        e = (int(np.floor(np.log2(1.0 / (8.0 * np.sqrt(cols))))) + 15) << 10
        scl = [(torch.randint(0, 1024, (rows * (cols // 32),), dtype=torch.int16, device=device) | e)
               for _ in range(copies)]
        mats = [spb200.PreparedQ4B(P(c), P(sc_), rows, cols, stream.cuda_stream) for c, sc_ in zip(codes, scl)]
        for M in SWEEP_M:
            x = torch.randn(M, cols, device=device)
            y = torch.empty(M, rows, dtype=torch.float32, device=device)
            n = iters if M < 2048 else max(3, iters // 4)
            for i in range(3):
                mats[i % copies].matmul(P(x), M, P(y), stream.cuda_stream)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(n):
                mats[i % copies].matmul(P(x), M, P(y), stream.cuda_stream)
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / n
            byts = wbytes + M * cols + M * (cols // 32) * 4 + M * rows * 4
            ops = 2.0 * M * rows * cols
            r = {"rows": rows, "cols": cols, "m": M, "us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
                 "tops": round(ops / us / 1e6, 2)}
            if M >= 1024:
                r["frac_int8"] = round(ops / us / 1e6 / int8_peak_tops, 4)
                r["kernel"] = "k_gemm_tc (tcgen05.mma kind::i8, 2 digit planes)" if mats[0].info()["planes"] else "k_gemm"
            else:
                r["frac_hbm"] = round(byts / us / 1e3 / hbm_gbs, 4)
                r["kernel"] = "k_gemv"
            out.append(r)
            del x, y
        for mm in mats:
            mm.release()
        del codes, scl
        torch.cuda.empty_cache()
    return out


def measure_batch(m, cfg, B, K, W, seed, max_over_ranks):
    """B independent sessions (seeded ragged contexts, U[128, 512] tokens each) decoding
    greedily together through spb_batch_decode_step: B*K tokens over the time of K steps
    (each call puts the B tokens H2D and reads the B argmaxes D2H; max over ranks)."""
    import torch
    import spb200
    import spmodel
    rng = np.random.default_rng(seed + 999)
    ctx = rng.integers(128, 513, size=B)
    pmax = int(ctx.max()) + W + K + 8
    sessions, toks = [], []
    t0 = time.perf_counter()
    for i in range(B):
        s = m.session(pmax)
        t = spmodel.gen_tokens(seed + 2000 + i, int(ctx[i]), cfg.n_vocab)
        s.prefill(t, logits=False)
        sessions.append(s)
        toks.append(int(t[-1]))
    prefill_s = time.perf_counter() - t0
    for _ in range(W):
        _, am = spb200.batch_decode(sessions, toks, logits=False)
        toks = am
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    torch.cuda.nvtx.range_push("b64_step")   # selects these launches for an ncu launch list
    for _ in range(K):
        _, am = spb200.batch_decode(sessions, toks, logits=False)
        toks = am
    torch.cuda.nvtx.range_pop()
    dt = max_over_ranks((time.perf_counter() - t0) * 1e3) / 1e3
    for s in sessions:
        s.close()
    return {"value": B * K / dt, "unit": "tokens/s", "sessions": B, "steps": K, "warmup": W,
            "ms_per_step": round(dt / K * 1e3, 3), "ctx": "seeded U[128, 512] tokens per session",
            "timing": "wall clock around K synchronous spb_batch_decode_step calls (B tokens H2D, "
                      "B argmaxes D2H per step)", "prefill_s_untimed": round(prefill_s, 2)}


def measure_qwen8b(args, local, rank, max_over_ranks, barrier, hbm_gbs):
    """BASELINE configs[3] on one GPU: the Qwen3-8B shape (36 layers, d 4096, 32/8 heads of 128,
    SwiGLU FFN 12288, vocab 151936, CORDIC-RoPE), random-init OK_Q4B from a seed; prefill
    --q8-prefill tokens (CUDA events), then --q8-steps greedy decode steps on the device (CUDA
    events on the session stream). frac: the bytes a decode token must read (every OK_Q4B
    weight, and the K/V rows of every layer at the step's context) over the step time, against
    the measured HBM peak."""
    import torch
    import spb200
    import spmodel
    cfg = spmodel.CONFIGS["qwen8b"]
    P, K = args.q8_prefill, args.q8_steps
    m = spb200.Model.synthetic(cfg, seed=args.seed + 8 + rank, device=local)
    s = m.session(P + K + 8)
    stream = torch.cuda.ExternalStream(s.stream(), device=torch.device("cuda", local))
    toks = spmodel.gen_tokens(args.seed + 300 + rank, P, cfg.n_vocab)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(stream)
    s.prefill(toks, logits=False)
    e1.record(stream)
    s.greedy(int(toks[-1]), 4)                          # warm-up (builds the step graph)
    barrier()
    e2.record(stream)
    s.greedy(int(toks[-1]), K)
    e3 = torch.cuda.Event(enable_timing=True)
    e3.record(stream)
    e3.synchronize()
    pre_s = e0.elapsed_time(e1) / 1e3
    ms = max_over_ranks(e2.elapsed_time(e3))
    wbytes = m.weight_bytes()
    ctx_mean = P + 4 + K / 2.0
    kv_bytes = 2 * cfg.n_layers * cfg.n_head_kv * cfg.head_dim * 4 * ctx_mean
    step_s = ms / K / 1e3
    s.close()
    m.free()
    return {"workload": f"qwen8b: prefill {P} + {K} greedy decode steps, B=1 (BASELINE configs[3])",
            "decode_tokens_per_s": round(K / (ms / 1e3), 2), "ms_per_step": round(ms / K, 4),
            "prefill_s": round(pre_s, 4), "prefill_tokens_per_s": round(P / pre_s, 1),
            "bytes_per_token": {"weights": wbytes, "kv_mean": int(kv_bytes)},
            "frac_hbm": round((wbytes + kv_bytes) / step_s / 1e9 / hbm_gbs, 4),
            "timing": "CUDA events on the session stream; inputs resident (device greedy loop)"}


SPEC_PG = 128


def measure_spec(m, cfg, S, steps, seed, max_over_ranks, barrier):
    """BASELINE configs[4], one GPU's share: S sessions (the 64 sessions spread over 8 GPUs are 8
    per GPU) with seeded ragged contexts U[128, 8192] in a paged, copy-on-write K/V pool. Each
    step: clone every session (O(1): the clone shares the pages), draft 4 greedy tokens on the
    clones as 4 batched decode steps (the first write into a shared page copies it), rewind a
    seeded 0-4 rejected tokens, close the parent. Timed: `steps` such steps, wall clock from the
    host (the clones, rewinds and closes included), max over ranks."""
    import torch
    import spb200
    import spmodel
    rng = np.random.default_rng(seed + 4242)
    ctx = rng.integers(128, 8193, size=S)
    pmax = int(ctx.max()) + 4 * (steps + 2) + 8
    need = sum(-(-(int(c) + 4 * (steps + 2) + 8) // SPEC_PG) for c in ctx) + 2 * S
    pool = spb200.KvPool(m, SPEC_PG, need)
    t0 = time.perf_counter()
    sess, nxt = [], []
    for i in range(S):
        s = pool.session(pmax)
        t = spmodel.gen_tokens(seed + 5000 + i, int(ctx[i]), cfg.n_vocab)
        s.prefill(t, logits=False)
        sess.append(s)
        nxt.append(int(t[-1]))
    prefill_s = time.perf_counter() - t0

    def spec_step(sess, nxt):
        clones = [s.clone() for s in sess]
        toks, outs = list(nxt), []
        for _ in range(4):
            _, am = spb200.batch_decode(clones, toks, logits=False)
            outs.append([int(a) for a in am])
            toks = outs[-1]
        rej = rng.integers(0, 5, size=S)
        for i in range(S):
            clones[i].rewind(int(rej[i]))
            if rej[i] < 4:
                nxt[i] = outs[3 - int(rej[i])][i]
            sess[i].close()
        return clones, int((4 - rej).sum())

    sess, _ = spec_step(sess, nxt)            # warm-up step
    barrier()
    t0 = time.perf_counter()
    accepted = 0
    for _ in range(steps):
        sess, a = spec_step(sess, nxt)
        accepted += a
    dt = max_over_ranks((time.perf_counter() - t0) * 1e3) / 1e3
    for s in sess:
        s.close()
    pool.free()
    return {"value": round(accepted / dt, 2), "unit": "accepted tokens/s (this GPU's sessions)",
            "drafted_tokens_per_s": round(4 * S * steps / dt, 2), "sessions": S, "steps": steps,
            "ms_per_step": round(dt / steps * 1e3, 3), "ctx": "seeded U[128, 8192] tokens per session",
            "kv": f"paged pool, {SPEC_PG}-position pages, copy-on-write; {need} pages",
            "timing": "wall clock around the steps (clone + 4 batched draft steps + rewind + close)",
            "prefill_s_untimed": round(prefill_s, 2)}


def kv_bytes_per_token(cfg, ctx, row_bytes):
    """K+V bytes one decode token reads at context ctx: every layer's window of positions x KV
    heads x 2 rows of row_bytes (sliding-window layers read at most the window)."""
    tot = 0
    for L in range(cfg.n_layers):
        glob = cfg.arch != spmodel_arch_gemma() or cfg.sliding_window <= 0 or (L % cfg.swa_period) == cfg.swa_period - 1
        n = ctx if glob else min(ctx, cfg.sliding_window)
        tot += n * cfg.n_head_kv * 2 * row_bytes
    return tot


def spmodel_arch_gemma():
    import spmodel
    return spmodel.ARCH_GEMMA3


def measure_spinor(m, cfg, args, max_over_ranks, barrier, hbm_gbs):
    """B=1 greedy decode with the K/V cache kept as Spinor blocks (SPB_KV_SPINOR): the same
    prefill length (its attention per row: the row tiles read int32 rows only) and K timed steps."""
    import torch
    import spmodel
    K, W = args.steps, args.warmup
    s = m.session(args.prefill + W + K + 8, spinor=True)
    stream = torch.cuda.ExternalStream(s.stream())
    toks = spmodel.gen_tokens(args.seed + 300, args.prefill, cfg.n_vocab)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    s.prefill(toks, logits=False)
    p1.record(stream)
    p1.synchronize()
    tok = int(toks[-1])
    s.greedy(tok, W)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s.greedy(tok, K)
    e1.record(stream)
    e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    s.close()
    hd = cfg.head_dim
    rb = (1 if hd <= 55 else (hd + 54) // 55) * 63
    ctx = args.prefill + W + K // 2
    kv_spin, kv_i32 = kv_bytes_per_token(cfg, ctx, rb), kv_bytes_per_token(cfg, ctx, hd * 4)
    step_b = m.weight_bytes() + kv_spin
    return {"value": round(K / (ms / 1e3), 3), "unit": "tokens/s (B=1, K/V as Spinor blocks)",
            "ms_per_step": round(ms / K, 4), "prefill_s": round(p0.elapsed_time(p1) / 1e3, 4),
            "kv_row_bytes": rb, "kv_row_bytes_int32": hd * 4, "ctx_mid": ctx,
            "kv_bytes_per_token": kv_spin, "kv_bytes_per_token_int32": kv_i32,
            "step_bytes_frac_of_hbm": round(step_b / (ms / K / 1e3) / 1e9 / hbm_gbs, 4),
            "note": "every K/V row encoded by the kernel producing it, decoded inside the attention"}


def measure_spinor_batch(m, cfg, args, max_over_ranks, hbm_gbs):
    """Long-context batch decode, K/V as int32 rows against Spinor blocks: one session prefills a
    --spin-ctx prefix, --spin-batch - 1 clones fork it (a shared prompt), and the sessions decode
    together through spb_batch_decode_step (distinct tokens per row). At this context the
    attention reads more bytes than the weights, which is where the 3.25x smaller rows pay."""
    import torch
    import spb200
    import spmodel
    S, L, K, W = args.spin_batch, args.spin_ctx, args.spin_batch_steps, 2
    out = {"sessions": S, "ctx": L, "steps": K, "warmup": W,
           "timing": "wall clock around K synchronous spb_batch_decode_step calls (S tokens H2D, S argmaxes D2H)"}
    hd = cfg.head_dim
    rb = (1 if hd <= 55 else (hd + 54) // 55) * 63
    for name, spin in (("int32", False), ("spinor", True)):
        s0 = m.session(L + W + K + 8, spinor=spin)
        toks = spmodel.gen_tokens(args.seed + 400, L, cfg.n_vocab)
        t0 = time.perf_counter()
        s0.prefill(toks, logits=False)
        torch.cuda.synchronize()
        pre = time.perf_counter() - t0
        sessions = [s0] + [s0.clone() for _ in range(S - 1)]
        cur = [int(t) for t in spmodel.gen_tokens(args.seed + 401, S, cfg.n_vocab)]
        for _ in range(W):
            _, am = spb200.batch_decode(sessions, cur, logits=False)
            cur = am
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(K):
            _, am = spb200.batch_decode(sessions, cur, logits=False)
            cur = am
        dt = max_over_ranks((time.perf_counter() - t0) * 1e3) / 1e3
        for s in sessions:
            s.close()
        kvb = S * kv_bytes_per_token(cfg, L + W + K // 2, rb if spin else hd * 4)
        out[name] = {"value": round(S * K / dt, 2), "unit": "tokens/s", "ms_per_step": round(dt / K * 1e3, 3),
                     "kv_bytes_per_step": kvb, "prefill_s_untimed": round(pre, 2),
                     "step_bytes_frac_of_hbm": round((m.weight_bytes() + kvb) / (dt / K) / 1e9 / hbm_gbs, 4)}
    out["spinor_over_int32"] = round(out["spinor"]["value"] / out["int32"]["value"], 3)
    return out


def measure_tp(cfg, args, rank, local, world, max_over_ranks, barrier, p2p=True):
    """One session of the model split over the group (spb_model_synthetic_tp): K greedy steps
    timed with CUDA events on the session stream, max over ranks; every rank produces the
    whole model's tokens."""
    import torch
    import spb200
    import spmodel
    uid = spb200.tp_uid_from_dist()
    tp = spb200.TensorParallel(uid, rank, world, device=local)
    if p2p:
        tp.enable_p2p(16 * cfg.n_embd)
    K, W = args.steps, args.warmup
    m = spb200.Model.synthetic_tp(cfg, tp, seed=args.seed)
    s = m.session(args.prefill + W + K + 8)
    stream = torch.cuda.ExternalStream(s.stream(), device=torch.device("cuda", local))
    toks = spmodel.gen_tokens(args.seed + 100, args.prefill, cfg.n_vocab)
    s.prefill(toks, logits=False)
    tok = int(toks[-1])
    tok = int(s.greedy(tok, W)[-1])
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s.greedy(tok, K)
    e1.record(stream)
    e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    s.close()
    m.free()
    tp.close()
    return {"model": cfg.name, "value": round(K / (ms / 1e3), 3), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "ms_per_step": round(ms / K, 4), "scaling": "strong",
            "parallelism": f"tp{world}: heads, FFN columns and LM-head rows split; int64 all-reduce after "
                           f"the attention output and FFN down projections, quantizer-max and argmax-key "
                           f"max-reduces ({'one-shot kernel over peer memory' if p2p else 'NCCL'}); "
                           f"logits all-gathered by NCCL"}


# ----------------------------------------------------------------------------- arms
def run_spb(args):
    import torch
    import torch.distributed as dist
    import spb200
    import spmodel

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    spb = spb200.load()
    cfg = bench_config(args)
    K, W = args.steps, args.warmup
    pmax = args.prefill + W + K + 8
    m = spb200.Model.synthetic(cfg, seed=args.seed + rank, device=local)
    s = m.session(pmax)
    stream = torch.cuda.ExternalStream(s.stream(), device=torch.device("cuda", local))
    toks = spmodel.gen_tokens(args.seed + 100 + rank, args.prefill, cfg.n_vocab)
    t0 = time.perf_counter()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    torch.cuda.nvtx.range_push("prefill")   # selects these launches for an ncu launch list
    s.prefill(toks, logits=False)
    torch.cuda.nvtx.range_pop()
    p1.record(stream)
    p1.synchronize()
    prefill_s = time.perf_counter() - t0
    prefill_dev_s = p0.elapsed_time(p1) / 1e3
    tok = int(toks[-1])
    s.greedy(tok, W)

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    smi_index = vis.split(",")[local] if vis else str(local)
    clocks = ClockSampler(smi_index)
    clocks.start()
    time.sleep(0.3)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # value: K greedy steps, inputs resident on the device
    pos0 = s.position()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    torch.cuda.nvtx.range_push("decode_steps")   # selects these launches for an ncu launch list
    generated = s.greedy(tok, K)
    torch.cuda.nvtx.range_pop()
    e1.record(stream)
    e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()

    # e2e: the same positions again through the host-buffer API
    s.rewind(s.position() - pos0)
    host_logits = torch.empty(cfg.n_vocab, dtype=torch.float32).pin_memory()
    import numpy as np
    lg_np = host_logits.numpy()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_e2e = tok
    e2.record(stream)
    e2e_tokens = []
    for _ in range(K):
        _, t_e2e = s.step_argmax(t_e2e, out=lg_np)
        e2e_tokens.append(t_e2e)
    e3.record(stream)
    e3.synchronize()
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    assert e2e_tokens == generated.tolist(), "host-API trajectory differs from the device-resident one"
    barrier()

    roof = None
    if not args.no_roofline:
        shapes, tot_b, tot_us, gl = gemv_roofline(cfg, spb, torch.device("cuda", local), stream)
        peak, peak_kind = peaks()
        achieved = tot_b / tot_us / 1e3
        # DRAM bytes per launch from one ncu capture of the 12B-width decode GEMVs
        # (profiles/k_gemv_decode_gemma12b_width.md); the LM head was not in that capture and is
        # counted at its algorithmic bytes. Per token, like `achieved`.
        traffic = None
        if cfg.name == "gemma12b":
            per_launch = {"qkv": 17.72e6, "o": 8.87e6, "gate_up": 66.70e6, "down": 33.22e6}
            traffic = int(sum(per_launch[n] * k for n, r, c, g, k in gemv_shapes(cfg) if n in per_launch) +
                          gemv_bytes(cfg.n_vocab, cfg.n_embd, False))
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "traffic_source": "ncu dram bytes per launch (profiles/k_gemv_decode_gemma12b_width.md), "
                                  "x launches per token; LM head at its algorithmic bytes",
                "peak_source": f"{peak_kind} hbm_gbs (burst copy)", "kernel": "k_gemv (OK_Q4B dequant-GEMV, M=1)",
                "algorithmic_bytes_per_token": int(tot_b), "gemv_us_per_token": round(tot_us, 1),
                "per_shape": shapes}
    clk = clocks.stop()

    b64 = None
    if args.batch > 0:
        b64 = measure_batch(m, cfg, args.batch, args.batch_steps, 3, args.seed + rank, max_over_ranks)
        b64["value"] = round(world * b64["value"], 3)

    spec = None
    if args.spec_sessions > 0:
        spec = measure_spec(m, cfg, args.spec_sessions, args.spec_steps, args.seed + rank, max_over_ranks, barrier)
        spec["value"] = round(world * spec["value"], 2)
        spec["unit"] = "accepted tokens/s (all GPUs' sessions)"
        spec["sessions_total"] = world * args.spec_sessions

    spin = None
    if args.spinor:
        spin = measure_spinor(m, cfg, args, max_over_ranks, barrier, peaks()[0])
        spin["value"] = round(world * spin["value"], 3)

    spin_b = None
    if args.spin_batch > 0:
        spin_b = measure_spinor_batch(m, cfg, args, max_over_ranks, peaks()[0])

    q8 = None
    if args.q8_prefill > 0:
        q8 = measure_qwen8b(args, local, rank, max_over_ranks, barrier, peaks()[0])
        q8["decode_tokens_per_s_all_gpus"] = round(world * q8["decode_tokens_per_s"], 2)

    tpr = None
    if world > 1 and not args.no_tp:
        tpr = measure_tp(cfg, args, rank, local, world, max_over_ranks, barrier, p2p=True)
        tpr["nccl_only"] = measure_tp(cfg, args, rank, local, world, max_over_ranks, barrier, p2p=False)
        if args.q8_prefill > 0:
            import spmodel
            tpr["qwen8b"] = measure_tp(spmodel.CONFIGS["qwen8b"], args, rank, local, world, max_over_ranks,
                                       barrier, p2p=True)

    cpu = None
    config1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, ORACLE)
        import cpu_baseline
        r = cpu_baseline.measure(cfg, procs=min(os.cpu_count() or 1, 32), steps=1)
        if r:
            cpu = {"value": round(r["value"], 5), "unit": "tokens/s", "cores": r["cores"], "kind": "reference",
                   "sample": r["sample"], "scaled": True, "scale": round(r["scale"], 3),
                   "sample_step_s": round(r["sample_step_s_median"], 4),
                   "per_core_tokens_per_s": round(r["per_core_tokens_per_s"], 6)}
        # BASELINE configs[0], unscaled, CPU beside GPU
        config1 = {"workload": "tiny (BASELINE configs[0]): prefill 64 + 64 greedy decode steps",
                   "gpu": measure_config1_gpu(local),
                   "cpu_reference": cpu_baseline.config1_e2e("reference"),
                   "cpu_xref": cpu_baseline.config1_e2e("xref")}

    # embed; per layer norm, QKV, attention (QK-norm + RoPE + KV store fused; a separate
    # k_rope_kv with SPB_ROPE_FUSED=0), quantize, O, norm, gate/up, quantize, down; final norm,
    # LM head, argmax take, position advance
    per_layer = 10 if os.environ.get("SPB_ROPE_FUSED") == "0" else 9
    kernels_per_step = 1 + per_layer * cfg.n_layers + 4
    # prefill on the tensor cores: the layer matmuls' int8 MACs (no LM head: no logits asked;
    # the attention dots are exact int64 work, not tensor work), against an int8 dense peak of
    # twice the measured bf16 GEMM burst (B200 tensor cores run dense int8 at 2x bf16)
    layer_params = sum(r * c * (2 if gated else 1) for name, r, c, gated, n in gemv_shapes(cfg)
                       if name != "lm_head")
    prefill_ops = 2.0 * args.prefill * cfg.n_layers * layer_params
    bf16 = None
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        bf16 = json.load(open(pk)).get("bf16_tflops")
    int8_peak = 2.0 * (bf16 or 1590.0)
    prefill = {"tokens": args.prefill, "s": round(prefill_dev_s, 4),
               "tokens_per_s": round(args.prefill / prefill_dev_s, 1),
               "int8_ops": prefill_ops, "achieved_tops": round(prefill_ops / prefill_dev_s / 1e12, 2),
               "peak_tops": round(int8_peak, 1),
               "peak_source": ("2 x measured" if bf16 else "2 x fallback") + " bf16 dense TF/s (int8 dense = 2 x bf16)",
               "frac": round(prefill_ops / prefill_dev_s / 1e12 / int8_peak, 4),
               "kernel": "k_gemm_tc (tcgen05.mma kind::i8 over 8-bit digit planes of the block-scaled weights, "
                         "TMA-staged activations, 256-row prefill chunks); CUDA events around "
                         "spb_session_prefill on the session stream (attention, norms and the rest included)"}
    sweep = None
    if not args.no_sweep and world == 1:
        sweep = gemm_sweep(spb, torch.device("cuda", local), stream, int8_peak, peaks()[0])
    line = {
        "metric": METRIC, "value": round(world * K / (ms / 1e3), 3), "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms / K, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint4->int64 (exact)",
        "data": "synthetic (random-init OK_Q4B weights from a seed, uniform random tokens)",
        "config": line_config(cfg, args, world),
        "ctx_at_timing": [args.prefill + W, args.prefill + W + K],
        "weight_bytes_per_token": m.weight_bytes(), "prefill_s_untimed": round(prefill_s, 3),
        "e2e": {"value": round(world * K / (ms_e2e / 1e3), 3), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": cfg.n_vocab * 4 + 4 + 4},
        "gpu_launches": kernels_per_step * K,
        "clocks": clk,
        "roofline": roof,
        "cpu_baseline": cpu,
        "config1": config1,
        "b64": b64,
        "spec": spec,
        "qwen8b": q8,
        "spinor_kv": spin,
        "spinor_batch_long_ctx": spin_b,
        "prefill": prefill,
        "config2_sweep": sweep,
    }
    if tpr:
        line["tp"] = tpr
    s.close()
    m.free()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_probe(args):
    """--probe-gemm ROWS,COLS,M: one seeded rows x cols OK_Q4B matrix prepared once
    (spb_q4b_prepare: its digit planes precomputed), spb_q4b_matmul of M seeded token rows run
    twice untimed, then --probe-iters times between CUDA events; prints one JSON line. Not a bench
    line: it exists so a profiler can capture a few launches of one GEMM shape."""
    import ctypes as C
    import torch
    import spb200
    rows, cols, M = (int(v) for v in args.probe_gemm.split(","))
    spb = spb200.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    codes = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device=dev, generator=g)
    scl = torch.randint(0, 1024, (rows * (cols // 32),), dtype=torch.int16, device=dev, generator=g) | (5 << 10)
    x = torch.randn(M, cols, device=dev, generator=g)
    y = torch.empty(M, rows, device=dev)
    st = torch.cuda.current_stream()
    P = lambda t: C.c_void_p(t.data_ptr())
    h = C.c_void_p()
    assert spb.spb_q4b_prepare(P(codes), P(scl), rows, cols, C.c_void_p(st.cuda_stream), C.byref(h)) == 0, \
        spb.spb_last_error()

    def go():
        assert spb.spb_q4b_matmul(h, P(x), M, P(y), C.c_void_p(st.cuda_stream)) == 0, spb.spb_last_error()
    for _ in range(2):
        go()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.probe_iters):
        go()
    e1.record(st)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.probe_iters
    spb.spb_q4b_release(h)
    print(json.dumps({"probe": "spb_q4b_matmul", "rows": rows, "cols": cols, "m": M, "iters": args.probe_iters,
                      "us": round(us, 2), "tops": round(2 * M * rows * cols / us / 1e6, 2)}), flush=True)


def run_reference(args):
    """The reference arm: the reference's own CPU decode (oracle/_ref/libspref.so, compiled from
    the reference sources) on all host cores. Each of the K timed steps is one decode token of
    the 12B-width 1-layer sample in every process at once (ms_per_step = the slowest process's
    wall time of that step, measured); `value` is the full model's tokens/s, the sample scaled by
    streamed parameters (cpu_baseline.measure says what that leaves out). Rank 0 alone runs."""
    rank, _, world = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, ORACLE)
    import cpu_baseline
    import spmodel
    cfg = spmodel.CONFIGS[args.config]
    procs = os.cpu_count() or 1
    K, W = args.steps, args.warmup
    t0 = time.perf_counter()
    r = cpu_baseline.measure(cfg, procs=procs, steps=K, warmup=W)
    wall = time.perf_counter() - t0
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference library oracle/_ref/libspref.so not built"}))
        return
    v = round(r["value"], 5)
    c1 = {"reference": cpu_baseline.config1_e2e("reference"), "xref": cpu_baseline.config1_e2e("xref")}
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(1e3 * sum(r["step_wall_s"]) / K, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init OK_Q4B weights from a seed)",
        "config": line_config(cfg, args, 1),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": r["cores"], "kind": "reference",
                         "sample": r["sample"], "scaled": True, "scale": round(r["scale"], 3),
                         "sample_step_s_median": round(r["sample_step_s_median"], 4),
                         "per_core_tokens_per_s": round(r["per_core_tokens_per_s"], 6)},
        "step_definition": "one sample decode token (12B widths, 1 layer, vocab 2048) in each of "
                           f"{procs} concurrent processes; ms_per_step is measured, value is scaled",
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "config1_unscaled": c1,
        "wall_s": round(wall, 1)}), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.probe_gemm:
        run_probe(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_spb(a)
