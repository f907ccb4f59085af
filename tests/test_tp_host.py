"""Tensor-parallel host logic on CPU: the shards of spb_tp_shard tile every matrix of the model
exactly once (query heads with their GQA KV heads, FFN columns in whole 32-column blocks,
LM-head rows), unsupported splits are refused, and a world-size-2 gloo group shares one NCCL
unique id and agrees on the tiling."""
import os

import numpy as np
import pytest

import spb200
import spmodel


def shards(cfg, world):
    return [spb200.tp_shard(cfg, r, world) for r in range(world)]


def assert_tiles(cfg, sh):
    G = cfg.n_head // cfg.n_head_kv
    covered = {"h": [], "kv": [], "f": [], "v": []}
    for h0, nh, kv0, nkv, f0, nff, v0, nv in sh:
        assert nh == G * nkv and h0 == G * kv0          # query heads carry their own KV heads
        assert nff % 32 == 0 and f0 % 32 == 0           # down-projection columns in whole blocks
        assert (nh * cfg.head_dim) % 32 == 0             # O-projection columns in whole blocks
        covered["h"] += range(h0, h0 + nh)
        covered["kv"] += range(kv0, kv0 + nkv)
        covered["f"] += range(f0, f0 + nff)
        covered["v"] += range(v0, v0 + nv)
    assert covered["h"] == list(range(cfg.n_head))
    assert covered["kv"] == list(range(cfg.n_head_kv))
    assert covered["f"] == list(range(cfg.n_ff))
    assert covered["v"] == list(range(cfg.n_vocab))


@pytest.mark.parametrize("name,worlds", [("gemma12b", (1, 2, 4, 8)), ("qwen8b", (1, 2, 4, 8)),
                                         ("micro_gemma", (1, 2)), ("micro_qwen", (1, 2)), ("tiny", (1, 2))])
def test_shards_tile_the_model(name, worlds):
    cfg = spmodel.CONFIGS[name]
    for w in worlds:
        assert_tiles(cfg, shards(cfg, w))


def test_shard_refusals():
    cfg = spmodel.CONFIGS["micro_gemma"]   # 2 KV heads
    with pytest.raises(spb200.SpbError) as e:
        spb200.tp_shard(cfg, 0, 4)
    assert e.value.args[0].startswith(f"spb rc={spb200.SPB_EUNSUPPORTED}")
    with pytest.raises(spb200.SpbError):
        spb200.tp_shard(cfg, 2, 2)          # rank outside the group
    import dataclasses
    odd_ff = dataclasses.replace(spmodel.CONFIGS["gemma12b"], n_ff=15360 + 32)
    with pytest.raises(spb200.SpbError):
        spb200.tp_shard(odd_ff, 0, 8)        # a rank's down-projection columns would split a block


def _gloo_rank(rank, world, port, out_dir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    uid = spb200.tp_uid_from_dist()
    sh = spb200.tp_shard(spmodel.CONFIGS["gemma12b"], rank, world)
    got = [None] * world
    dist.all_gather_object(got, (uid, sh))
    dist.destroy_process_group()
    np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([g[0] for g in got], dtype=object), allow_pickle=True)
    np.save(os.path.join(out_dir, f"s{rank}.npy"), np.array([g[1] for g in got]))


def test_gloo_group_shares_uid_and_tiling(tmp_path):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_gloo_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        uids = np.load(tmp_path / f"r{r}.npy", allow_pickle=True)
        assert len(uids[0]) == spb200.TP_ID_BYTES and uids[0] == uids[1]
        sh = np.load(tmp_path / f"s{r}.npy")
        assert_tiles(spmodel.CONFIGS["gemma12b"], [tuple(x) for x in sh])
