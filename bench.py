"""Benchmark: Llama-3-8B-shape bf16 greedy decode on B200 (benchmark configuration 2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-b32] [--no-qwen]
                    [--no-70b] [--no-cpu-baseline] [--sampled] [--ttft]
    python bench.py --profile [--layers L] [--prompt P] [--batch B] [--kernel KIND] [--ctx C]
                    [--preset NAME] [--adapters A] [--lora-rank R] [--timeline trace.json]

Prints ONE JSON line (rank 0).  `value` is decode tokens/s at batch 1 measured
on the device (CUDA events around K chained decode steps, inputs resident in
HBM); `e2e` is the same metric through the public C ABI call
(ti_engine_decode) with host token buffers: the H2D copy of the step
descriptor and the D2H read of the greedy ids are inside the timed region.
Weights (15 GB) are far larger than L2 (126 MB), so every step streams them
from HBM; no L2 flush is needed.

Opt-in extra fields: --sampled (batch 1 with device top-p sampling), --ttft (time
to first token of a 512-token prompt).  --profile runs a short workload for ncu
(or, with --timeline, traces the decode graph's kernels through the PyTorch
profiler and prints their in-graph timeline); it never prints a bench line.

--impl reference times the reference's decode step on the host CPU: the
reference ships no CPU implementation (its every op is CUDA), so the CPU
restatement of its algorithm (oracle/) is timed, multi-threaded, at full depth
(32 layers + LM head, 512-token context) for the given steps.  Its line also
carries ref_gpu_b1: the reference's own unchanged CUDA path (oracle/_ref) on the
same GPU at batch 1 (--no-ref-gpu skips it).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tensor-inference_b200"))

METRIC = "decode tok/s at B=1/32 (8B shape) and % of HBM roofline at 1/2/4/8 B200"
PROMPT = 512
NOMINAL_HBM_GBS = 8000.0
# one gate|up GEMV launch of the 8B shape under ncu: dram__bytes_read.sum +
# dram__bytes_write.sum (profiles/gemv_weight_stream_8b.md)
GATEUP_TRAFFIC_BYTES = 273213184


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (SM clock, reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ reference arm / CPU baseline
def cpu_baseline(sample_layers=2, steps=2):
    """Oracle (CPU restatement of the reference) timed on the host cores on a
    bounded sample of the benchmark step: 8B shapes, `sample_layers` decoder
    layers + LM head at the benchmark's 512-token context (seeded synthetic K/V),
    extrapolated to 32 layers."""
    import numpy as np

    import oracle
    import ti_b200 as ti

    kw = dict(ti.PRESETS["llama3_8b"], n_layers=sample_layers)
    m = oracle.Model(**kw)
    m.init_synthetic(0, 0.02)
    s = m.new_seq(PROMPT + steps + 8)
    s.fill_synthetic(PROMPT, seed=1)
    t_step = []
    tok = 7
    for _ in range(steps):
        t0 = time.perf_counter()
        _, lf = s.forward([tok])
        t_step.append(time.perf_counter() - t0)
        tok = int(np.argmax(lf))
    # LM head + final norm alone
    H, V = kw["hidden"], kw["vocab"]
    x = np.zeros((1, H), np.uint16)
    w = m.get_weight("lm_head.weight", (V, H))
    out = np.empty(V, np.float32)
    t0 = time.perf_counter()
    oracle.lib().orc_matmul_t_bf16_f32out(oracle.ptr(x), oracle.ptr(w), oracle.ptr(out), 1, V, H)
    t_head = time.perf_counter() - t0
    t_sample = min(t_step)
    t_layer = max(1e-9, (t_sample - t_head) / sample_layers)
    t_full = t_head + 32 * t_layer
    return {"value": 1.0 / t_full, "unit": "tok/s", "cores": oracle.lib().orc_get_threads(), "kind": "port",
            "sample": f"Llama-3-8B shapes, {sample_layers} of 32 layers + LM head timed per decode step at a "
                      f"{PROMPT}-token context (best of {steps}), extrapolated linearly to 32 layers: "
                      f"{t_layer * 1e3:.1f} ms/layer, {t_head * 1e3:.1f} ms LM head"}


def reference_cpu_decode(steps, warmup):
    """The benchmark step on the host cores: the CPU restatement of the
    reference's decode path (oracle/; the reference ships no CPU implementation,
    its every op is CUDA) at full depth, Llama-3-8B shape, batch 1, greedy, after
    a 512-token context (seeded synthetic K/V instead of a CPU prefill);
    `warmup` untimed steps, then `steps` timed steps."""
    import numpy as np

    import oracle
    import ti_b200 as ti

    m = oracle.Model(**ti.PRESETS["llama3_8b"])
    m.init_synthetic(0, 0.02)
    s = m.new_seq(PROMPT + warmup + steps + 8)
    s.fill_synthetic(PROMPT, seed=1)
    tok = 7
    for _ in range(warmup):
        tok = int(np.argmax(s.forward([tok])[1]))
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = int(np.argmax(s.forward([tok])[1]))
    dt = (time.perf_counter() - t0) / max(1, steps)
    return dt, oracle.lib().orc_get_threads()


def write_aliased_checkpoint(d, kw):
    """A safetensors checkpoint of the model shape `kw` (Llama) whose layers all
    point at one layer's seeded N(0, 0.02) bytes: a 2.6 GB file for the 8B shape.
    The reference's loader copies every tensor into its own device buffer
    (llama_model.cpp:32-82), so the device streams a full-size model per step."""
    import struct

    import oracle

    H, I, hd, V = kw["hidden"], kw["intermediate"], kw["head_dim"], kw["vocab"]
    QW, KW = kw["n_heads"] * hd, kw["n_kv_heads"] * hd
    blobs = {"embed": ((V, H), "model.embed_tokens.weight"), "norm": ((H,), "model.norm.weight"),
             "head": ((V, H), "lm_head.weight"), "in_norm": ((H,), "input_layernorm"),
             "post_norm": ((H,), "post_attention_layernorm"), "q": ((QW, H), "self_attn.q_proj"),
             "k": ((KW, H), "self_attn.k_proj"), "v": ((KW, H), "self_attn.v_proj"), "o": ((H, QW), "self_attn.o_proj"),
             "gate": ((I, H), "mlp.gate_proj"), "up": ((I, H), "mlp.up_proj"), "down": ((H, I), "mlp.down_proj")}
    data, offs, off = [], {}, 0
    for key, (shape, name) in blobs.items():
        a = oracle.fill_bf16(name, shape, 0, 0.02)
        offs[key] = (shape, off, off + a.nbytes)
        off += a.nbytes
        data.append(a)
    header = {}
    for key, name in (("embed", "model.embed_tokens.weight"), ("norm", "model.norm.weight"), ("head", "lm_head.weight")):
        shape, b, e = offs[key]
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [b, e]}
    for i in range(kw["n_layers"]):
        for key in ("in_norm", "post_norm", "q", "k", "v", "o", "gate", "up", "down"):
            shape, b, e = offs[key]
            base = blobs[key][1]
            name = f"model.layers.{i}.{base}.weight"
            header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [b, e]}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(os.path.join(d, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in data:
            f.write(a.tobytes())
    cfg = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": H, "intermediate_size": I,
           "num_hidden_layers": kw["n_layers"], "num_attention_heads": kw["n_heads"],
           "num_key_value_heads": kw["n_kv_heads"], "vocab_size": V, "rms_norm_eps": kw["rms_eps"],
           "rope_theta": kw["rope_theta"], "max_position_embeddings": 8192, "bos_token_id": 1, "eos_token_id": 2,
           "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)


def reference_gpu_decode(steps, warmup):
    """The reference's own CUDA decode path on this GPU: its unchanged backend,
    parser and Llama model code (oracle/_ref/libref.so, compiled for sm_100a from
    its sources), Llama-3-8B shape, batch 1 (the reference has no batching): a
    512-token prompt in one forward call, then per token Model::forward and the
    reference's own Greedy::sample, host-timed (its ops synchronise)."""
    import ctypes as C
    import shutil
    import tempfile

    import numpy as np

    import ti_b200 as ti

    path = os.path.join(ROOT, "oracle", "_ref", "libref.so")
    if not os.path.exists(path):
        return {"unavailable": "oracle/_ref/libref.so not built (needs the reference sources at build time)"}
    ref = C.CDLL(path)
    ref.ref_time_decode.restype = C.c_int
    ref.ref_time_decode.argtypes = [C.c_char_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.POINTER(C.c_double), C.POINTER(C.c_int32), C.c_char_p, C.c_int]
    kw = dict(ti.PRESETS["llama3_8b"])
    root = "/dev/shm" if os.path.isdir("/dev/shm") else None
    d = tempfile.mkdtemp(prefix="ti_refckpt_", dir=root)
    try:
        write_aliased_checkpoint(d, kw)
        prompt = np.random.default_rng(0).integers(0, kw["vocab"], size=PROMPT, dtype=np.int32)
        ms, last = C.c_double(0), C.c_int32(0)
        err = C.create_string_buffer(512)
        # the reference's loader logs to stdout: keep this process's stdout for the JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            rc = ref.ref_time_decode(d.encode(), prompt.ctypes.data, PROMPT, warmup, steps,
                                     PROMPT + warmup + steps + 8, C.byref(ms), C.byref(last), err, 512)
        finally:
            os.dup2(saved, 1)
            os.close(saved)
        if rc != 0:
            return {"unavailable": f"reference decode failed: {err.value.decode()[:200]}"}
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"tok_s": round(1e3 / ms.value, 2), "ms_per_step": round(ms.value, 3), "steps": steps, "warmup": warmup,
            "config": "Llama-3-8B shape, batch 1, 512-token prompt, greedy; the reference's unchanged CUDA path "
                      "(cuBLAS GEMMs, per-op allocation) on this B200; layers share one layer's values on disk, "
                      "each is its own device buffer"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    dt, cores = reference_cpu_decode(args.steps, args.warmup)
    v = 1.0 / dt
    cb = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
          "sample": f"the whole benchmark step: Llama-3-8B shape, 32 layers + LM head, batch 1, "
                    f"{PROMPT}-token context (synthetic K/V), {args.steps} timed steps after {args.warmup} warm-up"}
    line = {"metric": METRIC, "impl": "reference", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "Llama-3-8B-shape bf16 greedy decode, batch 1, 512-token context "
                                   "(CPU restatement of the reference's path; the reference has no CPU backend)",
                       "batch": 1, "prompt": PROMPT, "layers": 32},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_ref_gpu:
        import torch

        if torch.cuda.is_available():
            try:
                line["ref_gpu_b1"] = reference_gpu_decode(max(4, args.steps), min(args.warmup, 3))
            except Exception as exc:  # noqa: BLE001 - the extra leg reports its failure; the line stands
                line["ref_gpu_b1"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    emit(line)


# ------------------------------------------------------------------ our arm
def prefill_lockstep(eng, sids, prompts, adapters=None):
    """run equal-length prompts through all sequences in lockstep decode steps"""
    import numpy as np

    nxt = None
    for t in range(prompts.shape[1]):
        nxt = eng.decode(sids, np.ascontiguousarray(prompts[:, t]), adapters=adapters)
    return nxt


def measure_batch(ti, torch, eng, B, steps, warmup, stream, peak, measure_e2e=True, prompt=None, adapters=None,
                  lora_bytes=0, world=1, sampler=None):
    """sampler: (kind, temperature, p, k, seed) set on every sequence (device
    sampling in the chain and in the e2e steps), None = greedy"""
    import numpy as np

    desc = eng.desc
    prompt = prompt or PROMPT
    sids = [eng.seq_create() for _ in range(B)]
    if sampler:
        for s in sids:
            eng.set_sampler(s, *sampler)
    prompts = np.random.default_rng(0).integers(0, desc.vocab, size=(B, prompt), dtype=np.int32)
    t0 = time.perf_counter()
    first = prefill_lockstep(eng, sids, prompts, adapters)
    t_prefill = time.perf_counter() - t0
    total = prompt + 2 * (warmup + steps) + 8
    for s in sids:
        eng.seq_reserve(s, total)

    # ---- device-resident chain (value)
    eng.bind(sids, first, adapters)
    for _ in range(warmup):
        eng.decode_device(stream)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = eng.seq_len(sids[0]) + warmup
    ev0.record(torch.cuda.current_stream())
    for _ in range(steps):
        eng.decode_device(stream)
    ev1.record(torch.cuda.current_stream())
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    last = eng.unbind(warmup + steps, stream)
    eng.check()
    ctx_avg = ctx0 + (steps - 1) / 2.0
    step_bytes = ti.algorithmic_bytes_per_step(desc, B, B * ctx_avg, lora_bytes)
    res = {"batch": B, "ms_per_step": ms, "tok_s": B * 1e3 / ms, "ctx_avg": ctx_avg, "prefill_s": t_prefill,
           "step_bytes": step_bytes, "step_gbs": step_bytes / (ms * 1e-3) / 1e9}
    # tensor parallel: the step's bytes are spread over `world` GPUs' HBM
    res["step_frac_measured"] = res["step_gbs"] / (peak * world)
    res["step_frac_nominal"] = res["step_gbs"] / (NOMINAL_HBM_GBS * world)

    # ---- end to end through the C ABI with host buffers
    if measure_e2e:
        feed = np.ascontiguousarray(last, np.int32)
        for _ in range(2):
            feed = eng.decode(sids, feed, adapters=adapters, stream=stream)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev0.record(torch.cuda.current_stream())
        for _ in range(steps):
            feed = eng.decode(sids, feed, adapters=adapters, stream=stream)
        ev1.record(torch.cuda.current_stream())
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / steps
        e2e_ms = max(ev0.elapsed_time(ev1) / steps, wall * 1e3)
        MB = eng.opts.max_batch
        res["e2e"] = {"value": B * 1e3 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": (4 + 7 * MB) * 4,
                      "d2h_bytes_per_step": (MB + 1) * 4, "ms_per_step": e2e_ms}
    for s in sids:
        eng.seq_free(s)
    return res


def measure_tinyllama(ti, torch, stream, peak, dev=0, warmup=8, steps=128, prompt=128):
    """Benchmark configuration 1, the shape the reference's run_llama tool
    decodes: TinyLlama-1.1B shape (22 layers), seeded N(0, 0.02) bf16 weights, a
    128-token prompt of ids uniform in [0, 32000), greedy decode of 128 tokens at
    batch 1, device-timed over those 128 steps (after `warmup` untimed steps)"""
    desc = ti.model_desc(**ti.PRESETS["tinyllama"])
    eng = ti.Engine(desc, device=dev, max_batch=1, max_seqs=1, max_seq_len=prompt + 2 * (warmup + steps) + 16)
    try:
        eng.init_synthetic(0, 0.02)
        r = measure_batch(ti, torch, eng, 1, steps, warmup, stream, peak, measure_e2e=False, prompt=prompt)
    finally:
        eng.close()
    return {"tok_s": round(r["tok_s"], 1), "ms_per_step": round(r["ms_per_step"], 4),
            "step_gbs": round(r["step_gbs"], 1), "frac_measured": round(r["step_frac_measured"], 4),
            "frac_nominal_8tbs": round(r["step_frac_nominal"], 4), "bytes_per_step": r["step_bytes"],
            "ctx_avg": r["ctx_avg"],
            "config": "TinyLlama-1.1B shape, 22 layers, 128-token prompt, 128 greedy steps, batch 1"}


def measure_qwen_lora(ti, torch, stream, peak, wf, steps, warmup, dev=0):
    """Benchmark configuration 3: Qwen2.5-7B shape, rank-16 LoRA on q/k/v/o (A ~ N(0, 0.02),
    B ~ N(0, 0.001), alpha 32), batch 8, 256-token prompts; weights bf16 or GGUF Q4_0"""
    B, P, R = 8, 256, 16
    desc = ti.model_desc(**dict(ti.PRESETS["qwen25_7b"], weight_format=wf))
    eng = ti.Engine(desc, device=dev, max_batch=B, max_seqs=B, max_seq_len=P + 2 * (warmup + steps) + 64,
                    max_adapters=1, max_lora_rank=R, lora_proj_mask=0x0F)
    try:
        eng.init_synthetic(0, 0.02)
        ad = eng.adapter_create(R, 32.0, 0x0F)
        eng.adapter_init_synthetic(ad, 1, 0.02, 0.001)
        H, hd = desc.hidden, desc.head_dim
        qw, kw = desc.n_heads * hd, desc.n_kv_heads * hd
        lora_bytes = desc.n_layers * 2 * R * (3 * H + (qw + 2 * kw) + qw + H)
        r = measure_batch(ti, torch, eng, B, steps, warmup, stream, peak, measure_e2e=False, prompt=P,
                          adapters=[ad] * B, lora_bytes=lora_bytes)
    finally:
        eng.close()
    return {"tok_s": round(r["tok_s"], 1), "ms_per_step": round(r["ms_per_step"], 3),
            "step_gbs": round(r["step_gbs"], 1), "frac_measured": round(r["step_frac_measured"], 4),
            "bytes_per_step": r["step_bytes"], "ctx_avg": r["ctx_avg"]}


def measure_70b_tp(ti, torch, stream, peak, world, rank, dev, steps, warmup=3):
    """Benchmark configuration 5: Llama-3-70B shape, tensor-parallel over the job's GPUs,
    batch 64 at 4096 tokens of context (cached K/V filled with seeded synthetic
    values instead of a 4096-step prefill), 16 rank-64 LoRA adapters (alpha = rank,
    scale 1) on all seven projections, assigned to sequences round-robin"""
    import numpy as np
    import torch.distributed as dist

    B, CTX, R, NAD = 64, 4096, 64, 16
    box = [ti.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    desc = ti.model_desc(**ti.PRESETS["llama3_70b"])
    eng = ti.Engine(desc, device=dev, max_batch=B, max_seqs=B, max_seq_len=CTX + warmup + steps + 32,
                    tp_size=world, tp_rank=rank, nccl_id=box[0], max_adapters=NAD, max_lora_rank=R,
                    lora_proj_mask=0x7F)
    try:
        eng.init_synthetic(0, 0.02)
        ads = []
        for i in range(NAD):
            a = eng.adapter_create(R, float(R), 0x7F)
            eng.adapter_init_synthetic(a, 100 + i, 0.02, 0.001)
            ads.append(a)
        sids = [eng.seq_create() for _ in range(B)]
        for i, sid in enumerate(sids):
            eng.seq_fill_synthetic(sid, CTX - 1, seed=i, std=1.0)
            eng.seq_reserve(sid, CTX + warmup + steps + 8)
        per = [ads[i % NAD] for i in range(B)]
        first = np.random.default_rng(0).integers(0, desc.vocab, size=B, dtype=np.int32)
        eng.bind(sids, first, per)
        for _ in range(warmup):
            eng.decode_device(stream)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(torch.cuda.current_stream())
        for _ in range(steps):
            eng.decode_device(stream)
        ev1.record(torch.cuda.current_stream())
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / steps
        eng.unbind(warmup + steps, stream)
        eng.check()
    finally:
        eng.close()
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    H, I, hd = desc.hidden, desc.intermediate, desc.head_dim
    qw, kw = desc.n_heads * hd, desc.n_kv_heads * hd
    ins_outs = [(H, qw), (H, kw), (H, kw), (qw, H), (H, I), (H, I), (I, H)]
    lora_bytes = NAD * desc.n_layers * sum(2 * R * (i + o) for i, o in ins_outs)
    ctx_avg = CTX - 1 + warmup + (steps - 1) / 2.0
    step_bytes = ti.algorithmic_bytes_per_step(desc, B, B * ctx_avg, lora_bytes)
    gbs = step_bytes / (ms * 1e-3) / 1e9
    return {"tok_s": round(B * 1e3 / ms, 1), "ms_per_step": round(ms, 3), "step_gbs": round(gbs, 1),
            "frac_measured": round(gbs / (peak * world), 4), "bytes_per_step": step_bytes, "ctx_avg": ctx_avg,
            "config": f"Llama-3-70B shape, tp{world}, batch 64, context 4096, 16 rank-64 LoRA adapters on all "
                      "7 projections (round-robin); K/V context synthetic"}


def measure_ttft(ti, torch, prompt_len=512, chunks=(16, 64, 128), dev=0, reps=3):
    """Time to first token of a `prompt_len`-token prompt on the Llama-3-8B shape:
    ti_engine_prefill_chunked (batched prefill, `chunk` tokens per step) against
    one decode step per prompt token; host-timed around the whole call (it
    returns the first generated id), best of `reps`."""
    import numpy as np

    desc = ti.model_desc(**ti.PRESETS["llama3_8b"])
    mb = max(chunks)
    eng = ti.Engine(desc, device=dev, max_batch=mb, max_seqs=2, max_seq_len=prompt_len + 16)
    out = {"prompt": prompt_len}
    try:
        eng.init_synthetic(0, 0.02)
        ids = np.random.default_rng(1).integers(0, desc.vocab, size=prompt_len, dtype=np.int32)
        for chunk in (1,) + tuple(chunks):
            best = None
            for _ in range(reps + 1):  # the first run captures this chunk's graphs
                sid = eng.seq_create()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                if chunk == 1:
                    eng.prefill(sid, ids)
                else:
                    eng.prefill(sid, ids, chunk=chunk)
                dt = time.perf_counter() - t0
                eng.seq_free(sid)
                best = dt if best is None or dt < best else best
            out[f"chunk{chunk}_ms"] = round(best * 1e3, 2)
        eng.check()
    finally:
        eng.close()
    return out


def kernel_roofline(ti, torch, eng, stream, peak, iters=64):
    """dominant kernel (gate|up GEMV, 2 x 14336 x 4096 bf16 = 235 MB per launch)
    timed alone with CUDA events on its launch stream, cycling layers so every
    launch streams its weights from HBM"""
    desc = eng.desc
    tp = max(1, eng.opts.tp_size)
    nbytes = 2 * (desc.intermediate // tp) * desc.hidden * 2 + desc.hidden * 2 * 2  # this rank's shard
    for i in range(4):
        eng.launch_kernel(ti.KERNEL_GATEUP, i % desc.n_layers, 1, stream)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(torch.cuda.current_stream())
    for i in range(iters):
        eng.launch_kernel(ti.KERNEL_GATEUP, i % desc.n_layers, 1, stream)
    ev1.record(torch.cuda.current_stream())
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / iters
    gbs = nbytes / (ms * 1e-3) / 1e9
    # DRAM bytes (read + write) of one launch of this kernel, from an ncu capture
    # (dram__bytes_read.sum + dram__bytes_write.sum); a constant of this build,
    # not measured by this run.  It includes the L2 warm-up of the next kernel's rows.
    traffic = GATEUP_TRAFFIC_BYTES if tp == 1 else None
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
            "traffic": traffic,
            "traffic_source": "ncu capture of this kernel (profiles/gemv_weight_stream_8b.md), stated constant",
            "kernel": "k_gemv<1,kEpiGlu> (gate|up + RMSNorm + SiLU*up, 8B layer)",
            "bytes_per_launch": nbytes, "us_per_launch": round(ms * 1e3, 2)}


def measure_pkm(ti, torch, stream, iters=20):
    """Benchmark configuration 4: 65,536 queries of 512 fp32 against two 512 x 256 codebooks,
    4,096 registered adapters; queries resident on the device"""
    import numpy as np

    rng = np.random.default_rng(0)
    c1 = rng.standard_normal((512, 256), dtype=np.float32)
    c2 = rng.standard_normal((512, 256), dtype=np.float32)
    cents = rng.standard_normal((4096, 512), dtype=np.float32)
    q = torch.randn(65536, 512, device="cuda", dtype=torch.float32)
    addr = torch.empty(65536, device="cuda", dtype=torch.int32)
    ad = torch.empty(65536, device="cuda", dtype=torch.int32)
    p = ti.Pkm(c1, c2)
    p.register(cents, np.arange(4096, dtype=np.int32))
    for _ in range(3):
        p.query(q.data_ptr(), 65536, addr.data_ptr(), ad.data_ptr(), stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(torch.cuda.current_stream())
    for _ in range(iters):
        p.query(q.data_ptr(), 65536, addr.data_ptr(), ad.data_ptr(), stream)
    e1.record(torch.cuda.current_stream())
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    p.close()
    gemm_flop = 2.0 * 65536 * 2 * 512 * 256  # the GEMM-equivalent count the benchmark quotes (34.4 GFLOP)
    instr = 2.0 * 65536 * 2 * 512 * 256      # one sub + one fma per (query, code, dim)
    return {"queries": 65536, "ms": round(ms, 4), "queries_per_s": round(65536 / (ms * 1e-3), 1),
            "gemm_equiv_tflops": round(gemm_flop / (ms * 1e-3) / 1e12, 2), "fp32_instr_per_s": instr / (ms * 1e-3)}


def timeline_summary(trace_path, steps):
    """Kernel events of a torch.profiler (CUPTI) trace of graph replays: per
    kernel, launches, mean duration and mean contribution to the step.  With
    programmatic dependent launch a kernel starts while its predecessor runs,
    so durations overlap; every instant the GPU is busy is charged to the
    running kernel that finishes first (the one the chain is waiting on), so the
    contributions add up to the busy time and busy + idle = the span."""
    import heapq
    import json
    from collections import defaultdict

    with open(trace_path) as f:
        ev = [e for e in json.load(f)["traceEvents"] if e.get("cat") == "kernel" and e.get("ph") == "X"]
    if not ev:
        return ["timeline: no kernel events recorded"]
    iv = sorted((e["ts"], e["ts"] + e["dur"], e["name"].split("(")[0]) for e in ev)
    span = max(b for _, b, _ in iv) - iv[0][0]
    contrib = defaultdict(float)
    times = sorted({t for a, b, _ in iv for t in (a, b)})
    active, nxt, busy = [], 0, 0.0
    for t0, t1 in zip(times, times[1:]):
        while nxt < len(iv) and iv[nxt][0] <= t0:
            heapq.heappush(active, (iv[nxt][1], nxt))
            nxt += 1
        while active and active[0][0] <= t0:
            heapq.heappop(active)
        if active:
            contrib[iv[active[0][1]][2]] += t1 - t0
            busy += t1 - t0
    count, dur = defaultdict(int), defaultdict(float)
    for a, b, name in iv:
        count[name] += 1
        dur[name] += b - a
    lines = [f"timeline: {len(iv)} kernels over {steps} steps, {span / steps:.1f} us/step, "
             f"idle {(span - busy) / steps:.1f} us/step",
             "kernel | launches/step | mean duration us | mean contribution us | contribution us/step | share"]
    for name in sorted(count, key=lambda k: -contrib[k]):
        n = count[name]
        lines.append(f"{name} | {n / steps:.1f} | {dur[name] / n:.2f} | {contrib[name] / n:.2f} | "
                     f"{contrib[name] / steps:.1f} | {contrib[name] / max(span, 1e-9):.3f}")
    return lines


def run_profile(args):
    """Short, self-contained workload for ncu: a few decode steps (or repeated
    launches of one kernel) of the 8B shape with `--layers` layers after a
    `--prompt`-token prefill (`--preset` picks another model shape, `--adapters`
    adds LoRA adapters on all projections, tokens assigned round-robin).  Prints
    timing only; never a bench number."""
    import numpy as np
    import torch

    import ti_b200 as ti

    torch.cuda.set_device(0)
    ts = torch.cuda.Stream()
    torch.cuda.set_stream(ts)
    if args.preset == "pkm":
        # configuration 4 alone: `--steps` queries of 65,536 (NVTX range "kernels")
        r = measure_pkm(ti, torch, ts.cuda_stream, iters=args.steps)
        print(f"profile: pkm {r['ms']:.4f} ms per 65,536 queries")
        return
    wf = {"bf16": ti.WFMT_BF16, "q4_0": ti.WFMT_Q4_0, "q8_0": ti.WFMT_Q8_0}[args.wfmt]
    desc = ti.model_desc(**dict(ti.PRESETS[args.preset], n_layers=args.layers, weight_format=wf))
    ctx = args.ctx or args.prompt
    lora = dict(max_adapters=args.adapters, max_lora_rank=args.lora_rank, lora_proj_mask=0x7F) \
        if args.adapters else {}
    eng = ti.Engine(desc, device=0, max_batch=args.batch, max_seqs=args.batch,
                    max_seq_len=ctx + args.warmup + args.steps + 64, **lora)
    eng.init_synthetic(0, 0.02)
    per = None
    if args.adapters:
        # the config-5 mix: adapters on all projections, tokens assigned round-robin
        ads = []
        for i in range(args.adapters):
            a = eng.adapter_create(args.lora_rank, float(args.lora_rank), 0x7F)
            eng.adapter_init_synthetic(a, 100 + i, 0.02, 0.001)
            ads.append(a)
        per = [ads[b % len(ads)] for b in range(args.batch)]
    sids = [eng.seq_create() for _ in range(args.batch)]
    if args.ctx:
        # synthetic cached context instead of a prefill (long-context kernels)
        for i, s in enumerate(sids):
            eng.seq_fill_synthetic(s, ctx - 1, seed=i)
        first = np.random.default_rng(0).integers(0, desc.vocab, size=args.batch, dtype=np.int32)
    else:
        prompts = np.random.default_rng(0).integers(0, desc.vocab, size=(args.batch, args.prompt), dtype=np.int32)
        first = prefill_lockstep(eng, sids, prompts, per)
    for s in sids:
        eng.seq_reserve(s, ctx + args.warmup + args.steps + 8)
    eng.bind(sids, first, per)
    for _ in range(args.warmup):
        eng.decode_device(ts.cuda_stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    if args.timeline:
        # in-graph kernel timeline through the PyTorch profiler's CUPTI tracing
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(args.steps):
                eng.decode_device(ts.cuda_stream)
            torch.cuda.synchronize()
        prof.export_chrome_trace(args.timeline)
        print("\n".join(timeline_summary(args.timeline, args.steps)))
    elif args.kernel is None:
        # NVTX range "step" around the first timed step (ncu --nvtx --nvtx-include "step/")
        for i in range(args.steps):
            if i == 0:
                torch.cuda.nvtx.range_push("step")
            eng.decode_device(ts.cuda_stream)
            if i == 0:
                torch.cuda.nvtx.range_pop()
    else:
        # NVTX range so a profiler can select exactly these launches (ncu --nvtx --nvtx-include "kernels/")
        torch.cuda.nvtx.range_push("kernels")
        for i in range(args.steps):
            eng.launch_kernel(args.kernel, i % args.layers, args.batch, ts.cuda_stream)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / args.steps
    eng.unbind(args.warmup + (args.steps if args.kernel is None or args.timeline else 0), ts.cuda_stream)
    eng.check()
    print(f"profile: layers={args.layers} batch={args.batch} kernel={args.kernel} {dt * 1e3:.3f} ms/iter")
    eng.close()


def run_ours(args, rank, world):
    import torch

    import ti_b200 as ti

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", dev))
    peak, peak_src = measured_peaks()
    ts = torch.cuda.Stream()
    torch.cuda.set_stream(ts)  # kernels and events share this stream
    stream = ts.cuda_stream
    max_b = 32 if args.b32 else 1
    desc = ti.model_desc(**ti.PRESETS["llama3_8b"])
    nid = None
    if world > 1:
        # tensor parallel over the job's GPUs: rank 0 makes the NCCL id, all ranks share it
        import torch.distributed as dist

        box = [ti.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        nid = box[0]
    eng = ti.Engine(desc, device=dev, max_batch=max_b, max_seqs=max_b,
                    max_seq_len=PROMPT + 2 * (args.warmup + args.steps) + 64, tp_size=world, tp_rank=rank,
                    nccl_id=nid)
    eng.init_synthetic(0, 0.02)
    launches = eng.launches_per_step(1)

    with ClockSampler(dev) as clk:
        r1 = measure_batch(ti, torch, eng, 1, args.steps, args.warmup, stream, peak, world=world)
    roof = kernel_roofline(ti, torch, eng, stream, peak)

    def extra(fn, *a, **kw):
        # an extra leg that fails reports its error in the line; the headline stands
        try:
            return fn(*a, **kw)
        except Exception as exc:  # noqa: BLE001 - any failure of an extra leg is reported, not raised
            return {"error": f"{type(exc).__name__}: {exc}"[:300]}

    pkm = extra(measure_pkm, ti, torch, stream) if world == 1 else None
    tiny = extra(measure_tinyllama, ti, torch, stream, peak, dev) if world == 1 else None
    r32 = None
    if args.b32:
        r32 = measure_batch(ti, torch, eng, 32, max(2, args.steps // 4), min(args.warmup, 3), stream, peak,
                            measure_e2e=False, world=world)
    sampled = None
    if args.sampled and world == 1:
        # the same batch-1 step with a seeded top-p sampler (the reference's TopP defaults, t=0.8)
        rs = extra(measure_batch, ti, torch, eng, 1, args.steps, args.warmup, stream, peak,
                   sampler=(ti.SAMPLE_TOP_P, 0.8, 0.95, 0, 1234))
        sampled = rs if "error" in rs else {
            "tok_s": round(rs["tok_s"], 2), "ms_per_step": round(rs["ms_per_step"], 4),
            "e2e_tok_s": round(rs["e2e"]["value"], 2), "greedy_ms_per_step": round(r1["ms_per_step"], 4),
            "config": "config 2 at batch 1, top-p 0.95, temperature 0.8, seeded; sampled on the device"}
    qwen = None
    if args.qwen and world == 1:
        eng.close()  # the 8B engine's 15 GB is not needed for the Qwen legs
        qwen = {name: extra(measure_qwen_lora, ti, torch, stream, peak, wf, max(4, args.steps // 4), 3, dev)
                for name, wf in (("bf16", ti.WFMT_BF16), ("q4_0", ti.WFMT_Q4_0))}
    ttft = None
    if args.ttft and world == 1:
        eng.close()
        ttft = extra(measure_ttft, ti, torch, dev=dev)
    r70 = None
    if args.big and world > 1:
        eng.close()
        r70 = measure_70b_tp(ti, torch, stream, peak, world, rank, dev, max(4, args.steps // 8))

    # the ranks of the tensor-parallel group step together; the job's time is the slowest rank's
    ms = r1["ms_per_step"]
    e2e_ms = r1["e2e"]["ms_per_step"]
    ms32 = r32["ms_per_step"] if r32 else 0.0
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms, e2e_ms, ms32], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, ms32 = float(t[0]), float(t[1]), float(t[2])
        if r32:
            r32["ms_per_step"] = ms32
            r32["tok_s"] = 32 * 1e3 / ms32
            r32["step_gbs"] = r32["step_bytes"] / (ms32 * 1e-3) / 1e9
            r32["step_frac_measured"] = r32["step_gbs"] / (peak * world)
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(1e3 / ms, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) bf16 weights, uniform random 512-token prompts)",
            "config": {"workload": "Llama-3-8B-shape bf16 greedy decode, batch 1, 512-token prompt",
                       "batch": 1, "prompt": PROMPT, "ctx_avg": r1["ctx_avg"],
                       "parallelism": "single" if world == 1 else
                       f"tp{world} (all-reduce after o/down: " +
                       ("NCCL)" if os.environ.get("TI_TP_ALLREDUCE") == "nccl" else
                        "fused into the projection epilogue over NVLink peer memory)"),
                       "l2": "weights (15 GB) >> L2 (126 MB): every step streams from HBM; no flush"},
            "e2e": {k: (round(v, 3) if isinstance(v, float) else v) for k, v in r1["e2e"].items()},
            "roofline": roof,
            "step_roofline": {"achieved_gbs": round(r1["step_gbs"], 1), "bytes_per_step": r1["step_bytes"],
                              "frac_measured": round(r1["step_frac_measured"], 4),
                              "frac_nominal_8tbs": round(r1["step_frac_nominal"], 4), "peak_source": peak_src},
            "gpu_launches": launches * args.steps,
            "launches_per_step": launches,
            "clocks": clk.summary(),
        }
        if world > 1:
            line["e2e"]["value"] = round(1e3 / e2e_ms, 2)
            line["e2e"]["ms_per_step"] = round(e2e_ms, 3)
        if r32:
            line["b32"] = {"tok_s": round(r32["tok_s"], 1), "ms_per_step": round(r32["ms_per_step"], 3),
                           "step_gbs": round(r32["step_gbs"], 1), "frac_measured": round(r32["step_frac_measured"], 4),
                           "ctx_avg": r32["ctx_avg"]}
        if qwen:
            line["qwen7b_lora_b8"] = dict(qwen, config="Qwen2.5-7B shape, rank-16 LoRA q/k/v/o, batch 8, 256-token prompt")
        if tiny:
            line["tinyllama_b1"] = tiny
        if r70:
            line["llama70b_tp_b64_lora"] = r70
        if ttft:
            line["ttft_8b"] = ttft
        if sampled:
            line["sampled_b1"] = sampled
        if pkm and "error" not in pkm:
            # FP32 issue peak: 148 SMs x 128 lanes x SM clock during the run
            clk = (line["clocks"].get("sm_mhz") or 1965.0) * 1e6
            pkm["fp32_pipe_frac"] = round(pkm.pop("fp32_instr_per_s") / (148 * 128 * clk), 4)
            line["pkm"] = pkm
        elif pkm:
            line["pkm"] = pkm
        if cb:
            line["cpu_baseline"] = cb
        emit(line)
    eng.close()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


# The JSON line goes to the process's original stdout; everything else the run prints
# (NCCL's version banner, the reference's loader) goes to stderr, so stdout holds
# exactly one line.
_JSON_FD = None


def emit(line):
    text = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(text.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, text)


def main():
    global _JSON_FD
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-b32", dest="b32", action="store_false")
    ap.add_argument("--no-qwen", dest="qwen", action="store_false", help="skip the Qwen-7B LoRA legs (config 3)")
    ap.add_argument("--no-70b", dest="big", action="store_false",
                    help="skip the Llama-3-70B tensor-parallel leg (config 5, N >= 2 only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", dest="no_ref_gpu", action="store_true",
                    help="reference arm: skip the reference's own CUDA path on this GPU (the line's ref_gpu_b1)")
    ap.add_argument("--sampled", action="store_true",
                    help="also measure batch-1 decode with device top-p sampling: the line's sampled_b1 field")
    ap.add_argument("--ttft", action="store_true",
                    help="also time a 512-token prefill (batched, chunks of 16/64/128, and token by token) on the 8B "
                         "shape: the line's ttft_8b field")
    ap.add_argument("--profile", action="store_true", help="short ncu workload (see run_profile)")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--kernel", type=int, default=None, help="profile: launch only this kernel kind")
    ap.add_argument("--ctx", type=int, default=0, help="profile: synthetic cached context of this length")
    ap.add_argument("--preset", default="llama3_8b",
                    help="profile: model shape (ti_b200.PRESETS), or pkm for the PKM router workload alone")
    ap.add_argument("--wfmt", default="bf16", choices=["bf16", "q4_0", "q8_0"],
                    help="profile: storage format of the layers' linear weights")
    ap.add_argument("--adapters", type=int, default=0, help="profile: LoRA adapters on all projections")
    ap.add_argument("--lora-rank", type=int, default=64, help="profile: rank of those adapters")
    ap.add_argument("--timeline", default=None,
                    help="profile: trace the decode steps with the PyTorch profiler (CUPTI), write the Chrome trace "
                         "here and print each kernel's in-graph duration, chain contribution and the idle gaps")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not args.profile:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
    if args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world)


if __name__ == "__main__":
    main()
