"""Row-parallel projections of tensor parallelism, on the CPU over gloo (world
sizes 2 and 4).  Each rank takes its shard from ti_tp_plan and computes the
fp32 partial sums of o_proj (the input columns of its q heads) and down_proj
(its intermediate columns) with the oracle's matmul (restating ops.cu:94-148);
the ranks exchange them, and every rank sums them in rank order and adds the
residual as the engine's receive step does (csrc/small.cu, k_tp_recv_resid):
out = bf16(resid + bf16(sum_r partial_r)).  Every rank must get the same bits,
within the bf16 tolerance of the oracle's unsharded bf16(resid + bf16(x W^T))
(llama_model.cpp:186-187 and :199-201)."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "tensor-inference_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402
import ti_b200 as ti  # noqa: E402

SHAPE = dict(arch=ti.ARCH_LLAMA, hidden=512, n_layers=1, n_heads=8, n_kv_heads=4, head_dim=64, intermediate=1024,
             vocab=1024, rms_eps=1e-5, rope_theta=10000.0)
B = 3


def _inputs():
    H, I, QW = SHAPE["hidden"], SHAPE["intermediate"], SHAPE["n_heads"] * SHAPE["head_dim"]
    return {"x_o": oracle.fill_bf16("attn_out", (B, QW), 11, 1.0), "w_o": oracle.fill_bf16("wo", (H, QW), 11),
            "x_d": oracle.fill_bf16("act", (B, I), 11, 1.0), "w_d": oracle.fill_bf16("wdown", (H, I), 11),
            "resid": oracle.fill_bf16("resid", (B, H), 11, 1.0)}


def _partial(x, w, c0, c1):
    xs = np.ascontiguousarray(x[:, c0:c1])
    ws = np.ascontiguousarray(w[:, c0:c1])
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    oracle.lib().orc_matmul_t_bf16_f32out(oracle.ptr(xs), oracle.ptr(ws), oracle.ptr(out), x.shape[0], w.shape[0],
                                          c1 - c0)
    return out


def _receive(partials, resid):
    s = np.zeros_like(partials[0])
    for p in partials:  # rank order, fp32
        s = (s + p).astype(np.float32)
    v = oracle.bf16_to_f32(oracle.f32_to_bf16(s))
    return oracle.f32_to_bf16(oracle.bf16_to_f32(resid) + v)


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        sh = ti.tp_plan(ti.model_desc(**SHAPE), world, rank)
        d, hd = _inputs(), SHAPE["head_dim"]
        mine = {"o": _partial(d["x_o"], d["w_o"], sh["q0"] * hd, (sh["q0"] + sh["nq"]) * hd),
                "down": _partial(d["x_d"], d["w_d"], sh["i0"], sh["i0"] + sh["inter"])}
        out = {}
        for k, p in mine.items():
            parts = [torch.empty_like(torch.from_numpy(p)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(p))
            out[k] = _receive([t.numpy() for t in parts], d["resid"])
        got = [None] * world
        dist.all_gather_object(got, out)
        if rank == 0:
            q.put(got)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report, never hang the parent
        q.put(("error", repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_rank_ordered_partial_sums_match_unsharded_projection(world):
    oracle.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() + 7 * world) % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert not (isinstance(res, tuple) and res[0] == "error"), res
    d = _inputs()
    for k, (x, w) in {"o": (d["x_o"], d["w_o"]), "down": (d["x_d"], d["w_d"])}.items():
        for r in range(1, world):
            np.testing.assert_array_equal(res[r][k], res[0][k])  # identical bits on every rank
        full = _receive([_partial(x, w, 0, x.shape[1])], d["resid"])
        g, ref = oracle.bf16_to_f32(res[0][k]), oracle.bf16_to_f32(full)
        assert float(np.abs(g - ref).max() / np.abs(ref).max()) < 2e-2, k
        # the sharded sum differs from the unsharded one by fp32 reassociation only
        assert float(np.mean(res[0][k] != full)) < 0.05, k
