"""Tensor parallel on 2, 4 and 8 GPUs against the unsplit model on one: every rank returns the
same full-vocabulary logits, argmaxes and greedy tokens as the whole model, byte for byte, through
prefill (token-batch GEMM chunks, with the int64 all-reduce after the K-split matmuls), decode
steps (the GEMV path) and on-device greedy decoding; both the counter-generated shards and
shards sliced from a host model; with the exchanges on NCCL and with the decode exchanges on
the peer-memory kernel; micro models at 2 ranks and the 12B / 8B widths (8 KV heads) at 4 and 8.
The split being checked is the per-layer loop of gemma3_forward (gemma3.c:39-148) and
qwen3_forward_ex2 (forward.c:87-291). Each case is skipped on boxes with fewer GPUs than ranks."""
import dataclasses
import os
import socket

import numpy as np
import pytest

import spb200
import spmodel

pytestmark = pytest.mark.gpu

N_PRE, N_DEC, N_GREEDY = 40, 6, 8

MODELS = dict(spmodel.CONFIGS)
MODELS["gemma12b_w2"] = dataclasses.replace(spmodel.CONFIGS["gemma12b"], name="gemma12b_w2", n_layers=2,
                                            n_vocab=4096, swa_period=2, sliding_window=24, max_context=96)
MODELS["qwen8b_w2"] = dataclasses.replace(spmodel.CONFIGS["qwen8b"], name="qwen8b_w2", n_layers=2,
                                          max_context=96)


def _n_gpus():
    return spb200.load().spb_device_count()


def run_model(m, cfg):
    """prefill logits, decode-step logits + argmaxes, greedy tokens of one model"""
    toks = spmodel.gen_tokens(51, N_PRE, cfg.n_vocab)
    s = m.session(cfg.max_context)
    pre = s.prefill(toks)
    tok = int(pre[-1].argmax())
    steps, ams = [], []
    for _ in range(N_DEC):
        lg, am = s.step_argmax(tok)
        steps.append(lg.copy())
        ams.append(am)
        tok = am
    greedy = s.greedy(tok, N_GREEDY)
    kv = s.kv(0, N_PRE - 1, 0)
    s.close()
    return {"pre": pre, "steps": np.stack(steps), "ams": np.array(ams), "greedy": np.asarray(greedy), "kv": kv}


def _rank(rank, world, port, out_dir, name, mode, p2p):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    uid = spb200.tp_uid_from_dist()
    cfg = MODELS[name]
    tp = spb200.TensorParallel(uid, rank, world, device=rank)
    if p2p:   # the decode exchanges over peer memory; prefill chunks stay above cap (NCCL)
        tp.enable_p2p(16 * cfg.n_embd)
    if mode == "synthetic":
        m = spb200.Model.synthetic_tp(cfg, tp, seed=3)
    else:
        m = spb200.Model.upload_tp(cfg, spmodel.gen_model(cfg, seed=3), tp)
    res = run_model(m, cfg)
    m.free()
    tp.close()
    dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)


@pytest.mark.parametrize("world,name,mode,p2p", [
    (2, "micro_gemma", "synthetic", False), (2, "micro_qwen", "synthetic", False),
    (2, "micro_gemma", "upload", False), (2, "micro_gemma", "synthetic", True), (2, "micro_qwen", "upload", True),
    (4, "gemma12b_w2", "synthetic", True), (8, "gemma12b_w2", "synthetic", True),
    (8, "gemma12b_w2", "synthetic", False), (4, "qwen8b_w2", "synthetic", True), (8, "qwen8b_w2", "synthetic", True)])
def test_tp_matches_single_gpu(cuda_ok, tmp_path, world, name, mode, p2p):
    if _n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.spawn(_rank, args=(world, port, str(tmp_path), name, mode, p2p), nprocs=world, join=True)
    cfg = MODELS[name]
    if mode == "synthetic":
        m = spb200.Model.synthetic(cfg, seed=3)
    else:
        m = spb200.Model.upload(cfg, spmodel.gen_model(cfg, seed=3))
    want = run_model(m, cfg)
    m.free()
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npz")
        for k in ("pre", "steps"):
            assert np.array_equal(got[k].view(np.uint32), want[k].view(np.uint32)), f"rank {r} {k}"
        assert np.array_equal(got["ams"], want["ams"]) and np.array_equal(got["greedy"], want["greedy"])
        # the rank's KV heads are its slice of the whole cache row
        kvd = cfg.n_head_kv // world * cfg.head_dim
        assert np.array_equal(got["kv"][:kvd], want["kv"][r * kvd:(r + 1) * kvd]), f"rank {r} kv"
