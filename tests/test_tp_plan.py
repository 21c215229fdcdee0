"""Tensor-parallel host logic on CPU, world size 2 over gloo: every rank derives
its shard from ti_tp_plan; gathered, the shards must tile each split dimension
exactly (no gap, no overlap), and the NCCL unique id made by rank 0 must reach
the other rank unchanged (the bench and the GPU tests pass it this way)."""
import os
import sys

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "tensor-inference_b200"))

import ti_b200 as ti  # noqa: E402

PRESETS = ["tinyllama", "llama3_8b", "qwen25_7b", "llama3_70b"]


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        out = {}
        for name in PRESETS:
            d = ti.model_desc(**ti.PRESETS[name])
            try:
                out[name] = ti.tp_plan(d, world, rank)
            except ti.TiError as e:  # a split the model does not allow: every rank must agree
                out[name] = ("error", e.status)
        shards = [None] * world
        dist.all_gather_object(shards, out)
        ids = [ti.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        mine = ids[0]
        all_ids = [None] * world
        dist.all_gather_object(all_ids, mine)
        if rank == 0:
            q.put((shards, all_ids))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report, never hang the parent
        q.put(("error", repr(e)))


def _tiles(parts, total):
    parts = sorted(parts)
    pos = 0
    for a, n in parts:
        if a != pos:
            return False
        pos += n
    return pos == total


def test_shards_tile_every_split_dimension_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0] != "error", res
    shards, ids = res
    assert len(ids[0]) == 128 and ids[0] == ids[1]
    for name in PRESETS:
        d = ti.PRESETS[name]
        per = [s[name] for s in shards]
        if isinstance(per[0], tuple):
            assert all(isinstance(p, tuple) for p in per), name
            continue
        assert _tiles([(p["q0"], p["nq"]) for p in per], d["n_heads"]), name
        assert _tiles([(p["kv0"], p["nkv"]) for p in per], d["n_kv_heads"]), name
        assert _tiles([(p["i0"], p["inter"]) for p in per], d["intermediate"]), name
        assert _tiles([(p["v0"], p["vocab"]) for p in per], d["vocab"]), name
        # q head g attends kv head g // group: the local q heads must use the local kv heads
        G = d["n_heads"] // d["n_kv_heads"]
        for p in per:
            assert p["q0"] // G == p["kv0"] and p["nq"] == p["nkv"] * G


@pytest.mark.parametrize("tp", [3, 16])
def test_invalid_splits_are_rejected(tp):
    d = ti.model_desc(**ti.PRESETS["llama3_8b"])
    with pytest.raises(ti.TiError):
        ti.tp_plan(d, tp, 0)
