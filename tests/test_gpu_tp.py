"""Tensor parallelism (TP=2) against the CPU oracle, on 2 GPUs.

Row-parallel sums go through the fused peer-memory all-reduce by default and
through NCCL in one parametrisation.  The parent runs the oracle first (teacher-forced: each step feeds the oracle's
greedy token) and hands the token schedule to two child processes, one per
GPU and rank, which run the same steps through TP engines that share an NCCL
communicator.  Checks: both ranks agree on every greedy id; rank 0's gathered
logits are within the bf16 (2e-2) / Q4_0 (5e-2) tolerance of the oracle's; ids
equal the oracle's up to recorded near-ties.  Skipped on a box with one GPU.
NVLS is off in the children (a rank that fails an assertion leaves while its
peer may still be in a collective)."""
import os
import queue
import sys
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle
import ti_b200 as ti
from gpu_util import rel_err

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)


def _need(n):
    import torch

    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _oracle_schedule(kw, prompts, steps, seed, std, adapters=(), per_seq=None):
    m = oracle.Model(**kw)
    m.init_synthetic(seed, std)
    for i, (rank, alpha, mask, aseed, sa, sb) in enumerate(adapters):
        m.add_adapter(i, rank, alpha, mask, aseed, sa, sb)
    per_seq = per_seq or [-1] * len(prompts)
    feeds, ref = [], []
    seqs = [m.new_seq(128) for _ in prompts]
    last = []
    for s, p, ad in zip(seqs, prompts, per_seq):
        _, lf = s.forward(p, adapter=ad)
        last.append(lf)
    ref.append(np.stack(last))
    feed = [int(np.argmax(lf)) for lf in last]
    for _ in range(steps):
        feeds.append(list(feed))
        rows = [s.forward([t], adapter=ad)[1] for s, t, ad in zip(seqs, feed, per_seq)]
        ref.append(np.stack(rows))
        feed = [int(np.argmax(r)) for r in rows]
    return feeds, ref


def _rank(rank, world, nid, kw, prompts, feeds, seed, std, q, mode, adapters, per_seq, sampler=None):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["TI_TP_ALLREDUCE"] = mode
    sys.path.insert(0, os.path.join(ROOT, "tensor-inference_b200"))
    try:
        import ti_b200 as tl

        B = len(prompts)
        lo = dict(max_adapters=len(adapters), max_lora_rank=max(a[0] for a in adapters), lora_proj_mask=0x7F) \
            if adapters else {}
        eng = tl.Engine(tl.model_desc(**kw), device=rank, max_batch=B, max_seqs=B, max_seq_len=128, tp_size=world,
                        tp_rank=rank, nccl_id=nid, **lo)
        eng.init_synthetic(seed, std)
        for (arank, alpha, mask, aseed, sa, sb) in adapters:
            a = eng.adapter_create(arank, alpha, mask)
            eng.adapter_init_synthetic(a, aseed, sa, sb)
        per = per_seq or [-1] * B
        sids = [eng.seq_create() for _ in prompts]
        for sid in sids:
            if sampler:
                eng.set_sampler(sid, *sampler)  # every rank, every sequence: the same seeded sampler
        out_ids, out_logits = [], []
        ids0, lg0 = [], []
        for sid, p, ad in zip(sids, prompts, per):
            nxt, lb = eng.prefill(sid, p, adapter=ad, logits=tl.LOGITS_BF16)
            ids0.append(int(nxt))
            lg0.append(lb)
        out_ids.append(ids0)
        out_logits.append(np.stack(lg0))
        for f in feeds:
            nxt, lb = eng.decode(sids, f, adapters=per if adapters else None, logits=tl.LOGITS_BF16)
            out_ids.append([int(x) for x in nxt])
            out_logits.append(lb)
        eng.check()
        eng.close()
        q.put((rank, out_ids, out_logits if rank == 0 else None))
    except BaseException as e:
        q.put((rank, "error", repr(e)))
        # os._exit skips the queue's feeder thread: flush the message first
        q.close()
        q.join_thread()
        os._exit(1)


def _run_tp(kw, prompts, steps, tol, seed=0, std=0.02, world=2, mode="peer", adapters=(), per_seq=None,
            sampler=None):
    _need(world)
    feeds, ref = _oracle_schedule(kw, prompts, steps, seed, std, adapters, per_seq)
    nid = ti.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, nid, kw, prompts, feeds, seed, std, q, mode, list(adapters),
                                             per_seq, sampler)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.monotonic() + 300
    try:
        while len(res) < world:
            try:
                r = q.get(timeout=5)
            except queue.Empty:
                # a rank that died without reporting (exit code < 0: the signal) or ranks
                # that stall fail the test now instead of holding the GPUs
                gone = [(i, p.exitcode) for i, p in enumerate(procs) if p.exitcode not in (None, 0)]
                assert not gone, f"rank process(es) exited without a result: {gone}"
                assert time.monotonic() < deadline, f"ranks did not report within 300 s (have {sorted(res)})"
                continue
            assert r[1] != "error", r
            res[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    ids = [res[r][1] for r in range(world)]
    assert all(i == ids[0] for i in ids), "ranks disagree on the ids"
    if sampler:
        # each id: the exact form on rank 0's gathered logits with the sequence's draw
        kind, temperature, p, k, sseed = sampler
        u = oracle.sample_draws(sseed, steps + 1)
        if kind == ti.SAMPLE_TOP_K:
            u[:] = u[0]
        for step, lb in enumerate(res[0][2]):
            for b in range(len(prompts)):
                assert ids[0][step][b] == oracle.sample_exact(lb[b], kind, temperature, p, k, float(u[step])), \
                    (step, b)
        return
    flips = 0
    for step, (lb, lf) in enumerate(zip(res[0][2], ref)):
        for b in range(len(prompts)):
            g = oracle.bf16_to_f32(lb[b])
            err = rel_err(g, lf[b])
            assert err <= tol, (step, b, err)
            if ids[0][step][b] != int(np.argmax(lf[b])):
                s = np.sort(lf[b])
                assert s[-1] - s[-2] <= tol * np.abs(lf[b]).max(), (step, b)
                flips += 1
    assert flips <= max(1, (steps + 1) * len(prompts) // 10)


@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_tp2_llama_small_ragged(mode):
    # peer: the fused all-reduce over NVLink peer memory; nccl: ncclAllReduce (the baseline path)
    prompts = [oracle.fill_ids(f"tp{b}", n, b, SMALL["vocab"]) for b, n in enumerate((5, 11, 3))]
    _run_tp(SMALL, prompts, steps=4, tol=2e-2, mode=mode)


def test_tp2_tensor_core_batch16():
    prompts = [oracle.fill_ids(f"tq{b}", 2 + b % 4, b, SMALL["vocab"]) for b in range(16)]
    _run_tp(SMALL, prompts, steps=2, tol=2e-2)


def test_tp2_q4_0():
    kw = dict(SMALL, hidden=512, n_heads=8, intermediate=1024, weight_format=ti.WFMT_Q4_0)
    prompts = [oracle.fill_ids(f"tz{b}", n, b, kw["vocab"]) for b, n in enumerate((4, 7))]
    _run_tp(kw, prompts, steps=3, tol=5e-2)


def test_tp2_llama3_8b_shapes():
    kw = dict(ti.PRESETS["llama3_8b"], n_layers=2)
    _run_tp(kw, [oracle.fill_ids("t8", 6, 1, kw["vocab"])], steps=2, tol=2e-2)


def test_tp2_lora_all_projections_mixed_adapters():
    # row-parallel LoRA (o, down): partial x.A^T summed over ranks before the expansion
    ads = [(8, 16.0, 0x7F, 21, 0.05, 0.05), (4, 8.0, 0x7F, 22, 0.05, 0.05)]
    prompts = [oracle.fill_ids(f"tl{b}", n, b, SMALL["vocab"]) for b, n in enumerate((5, 8, 3, 6))]
    _run_tp(SMALL, prompts, steps=3, tol=2e-2, adapters=ads, per_seq=[0, 1, -1, 0])


def test_tp2_lora_tensor_core_batch():
    ads = [(8, 16.0, 0x7F, 31, 0.05, 0.05), (8, 8.0, 0x0F, 32, 0.05, 0.05)]
    prompts = [oracle.fill_ids(f"tm{b}", 2 + b % 3, b, SMALL["vocab"]) for b in range(12)]
    _run_tp(SMALL, prompts, steps=2, tol=2e-2, adapters=ads, per_seq=[b % 3 - 1 for b in range(12)])


@pytest.mark.parametrize("sampler", [(ti.SAMPLE_TOP_P, 0.8, 0.9, 0, 17), (ti.SAMPLE_TOP_K, 1.0, 0.0, 25, 18)])
def test_tp2_device_sampling(sampler):
    # vocabulary-parallel logits gathered from both ranks, sampled identically on each
    prompts = [oracle.fill_ids(f"ts{b}", n, b, SMALL["vocab"]) for b, n in enumerate((4, 9))]
    _run_tp(SMALL, prompts, steps=3, tol=2e-2, std=0.5, sampler=sampler)


def _rank_chain(rank, world, nid, kw, prompts, steps, sampler, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, os.path.join(ROOT, "tensor-inference_b200"))
    try:
        import ti_b200 as tl

        B = len(prompts)
        eng = tl.Engine(tl.model_desc(**kw), device=rank, max_batch=B, max_seqs=B, max_seq_len=128, tp_size=world,
                        tp_rank=rank, nccl_id=nid)
        eng.init_synthetic(0, 0.5)
        sids = [eng.seq_create() for _ in prompts]
        first = []
        for sid, p in zip(sids, prompts):
            eng.set_sampler(sid, *sampler)
            first.append(int(eng.prefill(sid, p)))
            eng.seq_reserve(sid, len(p) + steps + 1)
        eng.bind(sids, first)
        for _ in range(steps):
            eng.decode_device()
        last = [int(v) for v in eng.unbind(steps)]
        eng.check()
        eng.close()
        q.put((rank, first, last))
    except BaseException as e:
        q.put((rank, "error", repr(e)))
        q.close()
        q.join_thread()
        os._exit(1)


def test_tp2_sampled_device_chain_ranks_agree():
    # the chain's graph all-gathers the logits before the sampler: both ranks feed
    # themselves the same ids step after step
    _need(2)
    prompts = [oracle.fill_ids(f"tc{b}", n, b, SMALL["vocab"]) for b, n in enumerate((5, 8))]
    nid = ti.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    sampler = (ti.SAMPLE_TOP_P, 0.9, 0.9, 0, 77)
    procs = [ctx.Process(target=_rank_chain, args=(r, 2, nid, SMALL, prompts, 6, sampler, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        deadline = time.monotonic() + 300
        while len(res) < 2:
            try:
                r = q.get(timeout=5)
            except queue.Empty:
                gone = [(i, p.exitcode) for i, p in enumerate(procs) if p.exitcode not in (None, 0)]
                assert not gone, f"rank process(es) exited without a result: {gone}"
                assert time.monotonic() < deadline, "ranks did not report within 300 s"
                continue
            assert r[1] != "error", r
            res[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res[0][1:] == res[1][1:]
