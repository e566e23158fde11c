"""Data-parallel host logic on CPU: shard placement and max-over-ranks timing,
single process and as two gloo ranks."""
import os
import socket

import numpy as np
import pytest


def test_image_shard_blocks(g4m):
    from importlib import import_module
    sh = import_module(g4m.__name__ + ".sharding")
    for n, world in [(64, 1), (64, 8), (10, 4), (3, 8)]:
        parts = [list(sh.image_shard(n, world, r)) for r in range(world)]
        flat = [i for p in parts for i in p]
        assert flat == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_encoder_rows_and_lpt(g4m, syn, oracle):
    from importlib import import_module
    sh = import_module(g4m.__name__ + ".sharding")
    lens = syn.audio_batch_lengths(1000, 128)
    rows = [sh.encoder_rows(int(n)) for n in lens]
    assert rows == [oracle.audio_soft_token_count(int(n)) for n in lens]
    for world in (1, 2, 4, 8):
        parts = sh.lpt_assign(rows, world)
        assert sorted(i for p in parts for i in p) == list(range(len(rows)))
        loads = [sum(rows[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(rows)  # LPT bound


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, rows, out_dir):
    import importlib
    import sys

    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sh = importlib.import_module("gemma-4-webgpu-kernels-multimodal_b200.sharding")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        mine = sh.lpt_assign(rows, world)[rank]
        imgs = list(sh.image_shard(64, world, rank))
        t = sh.max_over_ranks(1.0 + rank, dist)
        gathered = [None] * world
        dist.all_gather_object(gathered, {"clips": mine, "images": imgs})
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([t], np.float64))
        if rank == 0:
            import json
            json.dump(gathered, open(os.path.join(out_dir, "parts.json"), "w"))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(g4m, syn, tmp_path):
    import torch.multiprocessing as mp
    from importlib import import_module
    sh = import_module(g4m.__name__ + ".sharding")
    rows = [sh.encoder_rows(int(n)) for n in syn.audio_batch_lengths(7, 24)]
    mp.start_processes(_rank, args=(2, _free_port(), rows, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    import json
    parts = json.load(open(tmp_path / "parts.json"))
    assert sorted(parts[0]["clips"] + parts[1]["clips"]) == list(range(24))
    assert parts[0]["images"] + parts[1]["images"] == list(range(64))
    for r in range(2):
        assert float(np.load(tmp_path / f"r{r}.npy")[0]) == 2.0  # max over ranks of 1.0 + rank
