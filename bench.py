"""Benchmark: batch-1 greedy decode of the Qwen3-0.6B-shaped q4 stack on B200.

One step = one generated token: all 28 layers at the current position plus the
f16 LM head and argmax (one CUDA-graph launch), positions cycling over the
8-token-prompt + 24-token decode of the batch-1 workload (positions 7..30, the
same token flow every cycle). Weights are seeded synthetic (seed 2) in the
reference's runtime layout.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload b1|b64]

N > 1 (torchrun): N independent replicas, one per GPU (batch-1 decode does not
shard); value = total tokens over all ranks / max over ranks of the device time.

--workload b64: batched decode, 64 independent sequences per GPU, each over a
2048-position f16 KV context built from seeded synthetic hidden states (seed 3)
pushed through every layer's input norm, k/v projections, k-norm and RoPE; one
step = one greedy token for all 64 sequences (one CUDA graph). With N GPUs each
rank holds its own 64 sequences (weak scaling, no collective).
"""
from __future__ import annotations

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

import numpy as np  # noqa: E402

from kernel_optimization_webgpu_b200 import synth  # noqa: E402

PROMPT_LEN, NEW_TOKENS = 8, 24
# DRAM bytes (read + write) of one k_decode_persistent token launch, measured by ncu
# on the default workload (428.79 MB read + 4.31 MB written): the layers' weights (the
# packed O and down slices carry ~18 MB more than the row records they come from) and,
# for a greedy token, the int8 copy of the LM head table (156 MB) in place of the f16
# table (311 MB) plus the f16 rows of the few candidates.
B1_TRAFFIC = 433105408
WORKLOAD = ("batch-1 greedy decode, Qwen3-0.6B shape (28 layers, hidden 1024, 16q/8kv heads x 128, "
            "SwiGLU 3072, q4 MatMulNBits block 32 with f16 scales, tied f16 LM head 151936x1024, f16 KV), "
            "8-token prompt + 24 generated, seed 2")
METRIC, UNIT = "decode tok/s", "tok/s"
B64, B64_CTX, B64_SEED = 64, 2048, 3
PF_PROMPTS, PF_LEN, PF_NEW, PF_SEED = 32, 512, 16, 4
B64_STEPS, PF_STEPS = 128, 10   # steps of the config-3 / config-4 objects of the default line
WORKLOAD_PF = ("prefill, Qwen3-0.6B shape: 32 prompts x 512 random ids (seed 4) as tcgen05 dequant-GEMMs over all "
               "prompt rows with causal GQA attention (mma.sync), then 16 greedy decode tokens per prompt")
WORKLOAD_B64 = ("batched greedy decode, Qwen3-0.6B shape, 64 independent sequences per GPU, each over a "
                "2048-position f16 KV context from seeded synthetic hidden states (seed 3), tcgen05 GEMMs")


def b1_config(world: int) -> dict:
    """The config object of the batch-1 line (the GPU arm and the reference arm alike)."""
    return {"workload": WORKLOAD, "global_batch": world, "seq_len": PROMPT_LEN + NEW_TOKENS,
            "parallelism": f"replicas x{world} (batch-1 decode does not shard)",
            "l2": "inputs larger than L2 (559 MB of weights streamed per token, L2 126 MB)"}


def prompt_ids():
    rng = np.random.Generator(np.random.PCG64(2))
    return rng.integers(0, synth.QWEN3_0_6B.vocab, size=PROMPT_LEN).tolist()


def runtime_dir() -> str:
    return os.environ.get("QDECODE_BENCH_RUNTIME", "/tmp/qdecode_runtime_qwen3_seed2")


def token_bytes(shape: synth.Shape, position: int, kv_bytes: int = 2) -> int:
    """Algorithmic HBM bytes of one batch-1 token at `position` (weights read once,
    KV rows 0..position read, one KV row written, logits written, id read back)."""
    H, I = shape.hidden, shape.intermediate
    QS, KV = shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    params = H * (QS + 2 * KV) + QS * H + 2 * H * I + I * H           # q4 weights per layer
    per_layer = params // 2 + (params // 32) * 2 + (2 * H + 2 * shape.head_dim) * 2
    kv_row = 2 * KV * kv_bytes                                          # K and V, one position
    return (shape.layers * per_layer + H * 2 + shape.vocab * H * 2 + H * 2
            + shape.layers * kv_row * (position + 1) + shape.layers * kv_row + shape.vocab * 4)


def batch_step_bytes(shape: synth.Shape, positions) -> int:
    """Algorithmic HBM bytes of one batched step: weights and the LM head table read
    once for all sequences, every sequence's KV rows 0..pos read and row pos written."""
    H, I = shape.hidden, shape.intermediate
    QS, KV = shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    params = H * (QS + 2 * KV) + QS * H + 2 * H * I + I * H
    per_layer = params // 2 + (params // 32) * 2 + (2 * H + 2 * shape.head_dim) * 2
    kv_row = 2 * KV * 2
    weights = shape.layers * per_layer + H * 2 + shape.vocab * H * 2
    kv = sum(shape.layers * kv_row * (p + 2) for p in positions)
    return weights + kv + len(positions) * H * 2


def prefill_flops(shape: synth.Shape, prompts: int, n: int) -> float:
    """Algorithmic FLOPs of a prefill: 2 * rows * (q4 projection weights) + causal QK^T and P*V."""
    H, I = shape.hidden, shape.intermediate
    QS, KV = shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    params = H * (QS + 2 * KV) + QS * H + 2 * H * I + I * H
    linear = 2.0 * prompts * n * params * shape.layers
    attn = shape.layers * prompts * shape.heads * 4.0 * shape.head_dim * (n * (n + 1) / 2)
    return linear + attn


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # the sampler is running before the timed region starts (its first row takes ~0.1-0.3 s)
            deadline = time.monotonic() + 5.0
            while not self.rows and time.monotonic() < deadline:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        self.t0 = time.monotonic()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append((time.monotonic(), parts))

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        # the rows read inside the timed region (plus one sampling interval of delivery lag)
        self.rows = [r for t, r in self.rows if self.t0 <= t <= self.t1 + 0.05]

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl" if _cuda() else "gloo", timeout=datetime.timedelta(seconds=120),
                                device_id=None)
    return world, rank, local


def _cuda():
    import torch
    return torch.cuda.is_available()


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def shard_range(total: int, world: int, rank: int):
    """Contiguous share [lo, hi) of `total` independent units for `rank` (no remainder allowed)."""
    if total % world:
        raise ValueError(f"{total} units do not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if _cuda() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _min_over_ranks(x: float, world: int) -> float:
    return -max_over_ranks(-x, world)


def prepare_runtime(world: int, rank: int) -> str:
    d = runtime_dir()
    if rank == 0:
        synth.ensure_runtime(d, synth.QWEN3_0_6B, seed=2)
    barrier(world)
    return d


# ---- CPU oracle timing (reference arm and the cpu_baseline object) -----------------

def time_cpu_decode(rt: str, steps: int, warmup: int):
    """Oracle decode tokens per second on the host cores: prefill once, then
    `warmup` + `steps` decode steps cycling over positions 7..30."""
    from oracle import oracle as O
    model = O.Model(rt)
    sess = model.session(max_seq=64, kv_f16=True)
    ids = prompt_ids()
    for i, t in enumerate(ids[:-1]):
        sess.forward(t, i)
    tok, pos, done, t_total = ids[-1], PROMPT_LEN - 1, 0, 0.0
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        sess.forward(tok, pos)
        tok, _, _ = sess.next_token()
        dt = time.perf_counter() - t0
        if i >= warmup:
            t_total += dt
            done += 1
        pos += 1
        if pos == PROMPT_LEN - 1 + NEW_TOKENS:
            pos, tok = PROMPT_LEN - 1, ids[-1]
    return done / t_total, O.lib().qo_num_threads(), done


def run_reference(args, world, rank):
    """The reference's CPU path: its WGSL math restated in C (oracle), all host threads."""
    if rank != 0:
        return 0
    # torchrun sets OMP_NUM_THREADS=1 for every rank; this arm runs on rank 0 alone and
    # uses every host thread
    from oracle import oracle as O
    O.lib().qo_set_num_threads(len(os.sched_getaffinity(0)))
    rt = runtime_dir()
    synth.ensure_runtime(rt, synth.QWEN3_0_6B, seed=2)
    # the GPU arm's steps and warm-up (each step is one ~30 ms oracle token: a
    # default-length run stays within a few minutes)
    steps, warm = max(1, min(args.steps, 2000)), max(args.warmup, 3)
    tps, cores, n = time_cpu_decode(rt, steps, warm)
    sample = (f"{n} decode tokens of the batch-1 workload (positions 7..30, after an 8-token prefill), "
              f"on rank 0's host cores")
    line = {"metric": METRIC, "value": round(tps, 4), "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": n, "warmup": warm, "ms_per_step": round(1000.0 / tps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, reference runtime layout)",
            "config": b1_config(world),
            "cpu_baseline": {"value": round(tps, 4), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tps, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference runs only through WebGPU (no graphics stack here: unavailable on this box); "
                    "this arm times its WGSL math restated in C on the host cores"}
    print(json.dumps(line), flush=True)
    return 0


# ---- GPU arm --------------------------------------------------------------------------

def _timed_chain(torch, stream, enqueue, n):
    """Device time of n back-to-back launches: a sleep kernel holds the stream
    while the host enqueues them, so host launch overhead cannot show up as gaps."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(50_000_000)
        e0.record(stream)
        for i in range(n):
            enqueue(i)
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1000.0 / n


def kernel_rooflines(torch, R, peak):
    """q4 matvec (gate 1024->3072, 128 distinct weight copies = 228 MB > L2) and the LM head
    (311 MB table per launch), each timed over back-to-back launches."""
    out = {}
    stream = torch.cuda.Stream()
    x, w, s = synth.matvec_case(3072, 1024, seed=0)
    copies = 128
    xs = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(w.view(np.int32)).cuda()
    sd = torch.from_numpy(s.astype(np.float16)).cuda()
    wcs = [wd.clone() for _ in range(copies)]
    scs = [sd.clone() for _ in range(copies)]
    ys = torch.empty(copies, 3072, device="cuda")
    per = 4 * 1024 + 3072 * 1024 // 2 + 3072 * 32 * 2 + 3072 * 4
    run = lambda i: R.q4_matvec(xs, wcs[i % copies], scs[i % copies], ys[i % copies], stream=stream)  # noqa: E731
    _timed_chain(torch, stream, run, copies)
    t = _timed_chain(torch, stream, run, 4 * copies)
    # the same kernel and launch path on a 1-row matvec (576 bytes): the per-launch floor
    x1, w1, s1 = synth.matvec_case(1, 1024, seed=0)
    w1d = torch.from_numpy(w1.view(np.int32)).cuda()
    s1d = torch.from_numpy(s1.astype(np.float16)).cuda()
    y1 = torch.empty(1, device="cuda")
    run1 = lambda i: R.q4_matvec(xs, w1d, s1d, y1, stream=stream)  # noqa: E731
    _timed_chain(torch, stream, run1, copies)
    t1 = _timed_chain(torch, stream, run1, 4 * copies)
    out["q4_matvec_gate_1024x3072"] = {"us_per_launch": round(t * 1e6, 3), "bytes": per,
                                       "achieved_gbs": round(per / t / 1e9, 1),
                                       "frac": round(per / t / 1e9 / peak, 4),
                                       "launch_floor_us": round(t1 * 1e6, 3),
                                       "frac_above_floor": round(per / max(t - t1, 1e-9) / 1e9 / peak, 4),
                                       "note": "isolated launches back to back (PDL), distinct weights; "
                                               "launch_floor_us: the same launches of a 1-row matvec"}
    del wcs, scs
    table, xh, eps = synth.lm_head_case()
    tb = torch.from_numpy(table.view(np.uint16)).cuda().view(torch.float16)
    xd = torch.from_numpy(xh).cuda()
    nw = torch.ones(1024, device="cuda")
    logits = torch.empty(151936, device="cuda")
    ws = R.LmHeadWorkspace(151936, "cuda")
    res = torch.zeros(2, dtype=torch.int32, device="cuda")
    per = 151936 * 1024 * 2 + 1024 * 4 * 2 + 151936 * 4 + 8
    run = lambda i: R.lm_head_argmax(xd, tb, nw, eps, logits, ws, res, stream=stream)  # noqa: E731
    _timed_chain(torch, stream, run, 3)
    t = _timed_chain(torch, stream, run, 30)
    out["lm_head_argmax_151936x1024"] = {"us_per_launch": round(t * 1e6, 3), "bytes": per,
                                         "achieved_gbs": round(per / t / 1e9, 1),
                                         "frac": round(per / t / 1e9 / peak, 4)}
    return out


def run_ours(args, world, rank, local):
    import torch

    from kernel_optimization_webgpu_b200 import runtime as R
    torch.cuda.set_device(local)
    rt = prepare_runtime(world, rank)
    peak, peak_kind = peaks()
    ids = prompt_ids()
    eng = R.Engine(rt, device=local, max_seq=64)
    step_kernels = eng.step_kernels
    eng_kernel = eng.token_kernel
    token_kernel_desc = {
        1: "decode token: k_decode_persistent, one launch per token (28 layers + LM head/argmax)",
    }.get(eng.token_kernel, f"decode token: one CUDA graph of {step_kernels} kernels (28 layers + LM head/argmax)")
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    shape = synth.QWEN3_0_6B
    cycle = NEW_TOKENS  # positions 7..30

    # warm-up (untimed): a full prompt + decode cycle at least
    eng.decode_begin(ids, NEW_TOKENS)
    pos_in_cycle, seeks = 0, 0
    for _ in range(max(args.warmup, 3)):
        if pos_in_cycle == cycle:
            eng.decode_seek(PROMPT_LEN - 1)
            pos_in_cycle = 0
        eng.decode_step()
        pos_in_cycle += 1
    eng.decode_sync(0)

    # timed: exactly K steps
    positions = []
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)
        e0.record(stream)
        for _ in range(args.steps):
            if pos_in_cycle == cycle:
                eng.decode_seek(PROMPT_LEN - 1)
                pos_in_cycle = 0
                seeks += 1
            positions.append(PROMPT_LEN - 1 + pos_in_cycle)
            eng.decode_step()
            pos_in_cycle += 1
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    eng.decode_sync(0)
    t_local = e0.elapsed_time(e1) / 1000.0
    t_max = max_over_ranks(t_local, world)
    value = world * args.steps / t_max
    ms_per_step = t_max * 1000.0 / args.steps
    bytes_avg = sum(token_bytes(shape, p) for p in positions) / len(positions)
    achieved = bytes_avg / (t_local / args.steps) / 1e9

    if args.decode_only:
        eng.close()
        if rank == 0:
            print(json.dumps({"decode_only": True, "tok_s": round(value, 2), "ms_per_step": ms_per_step}))
        return 0

    # e2e: the public C-ABI call with host buffers (prompt in, generated ids out)
    n_e2e = max(1, args.steps // NEW_TOKENS)
    eng.generate_greedy(ids, NEW_TOKENS)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(n_e2e):
        gen, _ = eng.generate_greedy(ids, NEW_TOKENS)
    f1.record(stream)
    f1.synchronize()
    t_e2e = max(f0.elapsed_time(f1) / 1000.0, time.perf_counter() - t0)
    t_e2e = max_over_ranks(t_e2e, world)
    e2e = world * n_e2e * NEW_TOKENS / t_e2e

    eng.close()
    sub = {}
    if not args.b1_only:
        # configs 3 and 4 in the same run (every rank takes part: collectives inside)
        sub["b64"] = measure_b64(args, world, rank, local, B64_STEPS, 3)
        if world > 1:
            sub["b64_vocab_shard"] = measure_b64(args, world, rank, local, B64_STEPS, 3, vocab_shard=True,
                                                 with_cpu=False)
        sub["prefill"] = measure_prefill(args, world, rank, local, PF_STEPS, 3)

    extra = {}
    cpu = None
    if rank == 0 and world == 1:
        extra = kernel_rooflines(torch, R, peak)
        if not args.no_cpu:
            tps, cores, n = time_cpu_decode(rt, args.cpu_steps, 1)
            cpu = {"value": round(tps, 4), "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"{n} decode tokens of the batch-1 workload (positions 7..30) on the host "
                             f"cores, WGSL math restated in C (OpenMP)"}
    if rank == 0:
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, reference runtime layout)",
            "config": b1_config(world),
            "roofline": {"bound": "hbm", "kernel": token_kernel_desc,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": B1_TRAFFIC if eng_kernel == 1 else None,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one token launch "
                                           "of this workload" if eng_kernel == 1 else None,
                         "bytes_note": "bytes_per_step is the reference token's algorithmic bytes (f16 LM head); "
                                       "for greedy tokens the kernel reads an int8 copy of the table and "
                                       "recomputes only the candidate rows in f16, so traffic is lower",
                         "bytes_per_step": int(bytes_avg), "peak_source": peak_kind},
            "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": PROMPT_LEN * 4,
                    "d2h_bytes_per_step": NEW_TOKENS * 4,
                    "step": "one qd_generate_greedy call: 8 prompt ids in, 24 generated ids out (prefill included)"},
            "gpu_launches": args.steps * step_kernels + seeks,
            "clocks": clocks,
            "kernels": extra,
            "generated_ids_sample": gen[:8],
        }
        if cpu:
            line["cpu_baseline"] = cpu
        line.update({k: v for k, v in sub.items() if v is not None})
        print(json.dumps(line), flush=True)
    return 0


def measure_b64(args, world, rank, local, steps, warmup, vocab_shard=False, with_cpu=True):
    """Config 3: 64 sequences per GPU over a 2048-position context, `steps` greedy
    steps; the line's fields (rank 0) or None. With vocab_shard the LM head is split
    by vocabulary over the ranks (two NCCL all-gathers per step); the sharded ids of
    the first steps are checked against the replicated head's on the same batch."""
    import torch

    from kernel_optimization_webgpu_b200 import runtime as R
    torch.cuda.set_device(local)
    rt = prepare_runtime(world, rank)
    peak, peak_kind = peaks()
    shape = synth.QWEN3_0_6B
    warm = max(warmup, 3)
    parity_steps = 4 if vocab_shard else 0
    max_seq = B64_CTX + warm + steps + parity_steps + 1
    nb = args.batch
    eng = R.Engine(rt, device=local, max_seq=64)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)  # batches enqueue on the engine's stream
    bt = R.Batch(eng, nb, max_seq)
    rng = np.random.Generator(np.random.PCG64(B64_SEED + 1000 * rank))
    tokens = rng.integers(0, shape.vocab, size=nb).astype(np.int32)
    t0 = time.perf_counter()
    bt.fill_context(B64_CTX, B64_SEED + rank)
    fill_s = time.perf_counter() - t0
    gather = None
    shard_parity, allgather_ms = None, None
    if vocab_shard:
        import torch.distributed as dist

        bufs = bt.set_vocab_shard(rank, world)

        def gather(out, inp):
            if world > 1:
                dist.all_gather_into_tensor(out, inp)
            elif out.data_ptr() != inp.data_ptr():
                out.view(inp.shape).copy_(inp)

        # parity: the same steps with the replicated LM head, then sharded
        bt.set_tokens(tokens, [B64_CTX] * nb)
        want = bt.decode(parity_steps)
        bt.set_tokens(tokens, [B64_CTX] * nb)
        with torch.cuda.stream(stream):
            got = bt.decode_sharded(parity_steps, gather)
        same = float(np.array_equal(want, got))
        shard_parity = bool(_min_over_ranks(same, world) == 1.0)
    bt.set_tokens(tokens, [B64_CTX] * nb)
    if vocab_shard:
        with torch.cuda.stream(stream):
            bt.decode_sharded(warm, gather)
    else:
        bt.decode(warm, want_ids=False)
    step_kernels = bt.step_kernels

    # timed: exactly `steps` steps, device time with events on the engine's stream
    positions = [B64_CTX + warm + i for i in range(steps)]
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)  # hold the stream while the host enqueues
        e0.record(stream)
        if vocab_shard:
            with torch.cuda.stream(stream):
                bt.decode_sharded(steps, gather)
        else:
            bt.decode(steps, want_ids=False)
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier(world)
    t_local = e0.elapsed_time(e1) / 1000.0
    t_max = max_over_ranks(t_local, world)
    value = world * nb * steps / t_max
    step_bytes = sum(batch_step_bytes(shape, [p] * nb) for p in positions) / len(positions)
    if vocab_shard:  # each rank reads only its slice of the LM-head table
        step_bytes -= shape.vocab * shape.hidden * 2 * (world - 1) / world
    achieved = step_bytes / (t_local / steps) / 1e9

    if vocab_shard:
        # the step's two collectives alone, same sizes, same stream
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            a0.record(stream)
            for _ in range(steps):
                for key in ("gather_hi", "gather_lo"):
                    gather(bufs[key], bufs[key][rank * nb:(rank + 1) * nb])
                gather(bufs["pairs_all"], bufs["pairs_local"])
            a1.record(stream)
        a1.synchronize()
        allgather_ms = max_over_ranks(a0.elapsed_time(a1) / steps, world)

    # e2e: host tokens and positions in, host ids out, through the public calls
    bt.set_tokens(tokens, [B64_CTX] * nb)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    bt.set_tokens(tokens, [B64_CTX] * nb)
    if vocab_shard:
        with torch.cuda.stream(stream):
            ids = bt.decode_sharded(steps, gather)
    else:
        ids = bt.decode(steps)
    t_e2e = max_over_ranks(time.perf_counter() - t0, world)
    e2e = world * nb * steps / t_e2e

    cpu = None
    if rank == 0 and world == 1 and with_cpu and not args.no_cpu:
        cpu = time_cpu_batched(rt, bt)
    bt.close()
    eng.close()
    if rank != 0:
        return None
    par = (f"sequences sharded: {nb} per GPU x {world}; LM head split by vocabulary over the {world} ranks "
           f"(NCCL all-gathers of the final-norm rows and of the (index, max) pairs)") if vocab_shard else \
        f"sequences sharded: {nb} per GPU x {world} (no collective)"
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": round(t_max * 1000.0 / steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init weights and context, reference runtime layout)",
        "config": {"workload": WORKLOAD_B64 if nb == B64 else WORKLOAD_B64.replace("64 independent", f"{nb} independent"),
                   "global_batch": nb * world, "seq_len": max_seq, "parallelism": par,
                   "l2": "inputs larger than L2 (about 15.5 GB of KV plus 559 MB of weights per step)",
                   "context_fill_s": round(fill_s, 3)},
        "roofline": {"bound": "hbm", "kernel": f"decode step of {nb} sequences (one CUDA graph: 28 layers x "
                                               "10 kernels + LM head/argmax)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "bytes_per_step": int(step_bytes), "peak_source": peak_kind},
        "e2e": {"value": round(e2e, 2), "unit": UNIT, "h2d_bytes_per_step": round(2 * nb * 4 / steps, 2),
                "d2h_bytes_per_step": nb * 4,
                "step": f"qd_batch_set_tokens ({nb} ids + positions in) + qd_batch_decode({steps}) "
                        "with every generated id copied out"},
        "gpu_launches": steps * step_kernels,
        "clocks": clk.summary(),
        "generated_ids_sample": ids[:2, :4].tolist(),
    }
    if vocab_shard:
        line["shard_parity"] = shard_parity
        line["shard_parity_steps"] = parity_steps
        line["allgather_ms_per_step"] = round(allgather_ms, 5)
    if cpu:
        line["cpu_baseline"] = cpu
    return line


def run_b64(args, world, rank, local):
    line = measure_b64(args, world, rank, local, args.steps, args.warmup, args.vocab_shard)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def measure_prefill(args, world, rank, local, steps, warmup, with_cpu=True):
    """Config 4: 32 prompts x 512 ids prefilled together (split over the ranks), then
    16 tokens; the line's fields (rank 0) or None."""
    import torch

    from kernel_optimization_webgpu_b200 import runtime as R
    torch.cuda.set_device(local)
    rt = prepare_runtime(world, rank)
    _, peak_kind = peaks()
    tflops_peak = _bf16_peak()
    shape = synth.QWEN3_0_6B
    lo, hi = shard_range(PF_PROMPTS, world, rank)
    mine = hi - lo
    rng = np.random.Generator(np.random.PCG64(PF_SEED))
    all_ids = rng.integers(0, shape.vocab, size=(PF_PROMPTS, PF_LEN)).astype(np.int32)
    ids = np.ascontiguousarray(all_ids[lo:hi])
    eng = R.Engine(rt, device=local, max_seq=64)
    stream = torch.cuda.Stream()
    eng.set_stream(stream)
    bt = R.Batch(eng, mine, PF_LEN + PF_NEW)
    warm = max(warmup, 3)
    for _ in range(warm):
        bt.prefill(ids)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)
        e0.record(stream)
        for _ in range(steps):
            first = bt.prefill(ids)
        e1.record(stream)
        e1.synchronize()
    barrier(world)
    t_local = e0.elapsed_time(e1) / 1000.0 / steps
    t_max = max_over_ranks(t_local, world)
    value = PF_PROMPTS * PF_LEN / t_max
    flops_local = prefill_flops(shape, mine, PF_LEN)
    achieved = flops_local / t_local / 1e12
    # decode tail: 15 more greedy tokens after the prefilled first one
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    more = bt.decode(PF_NEW - 1)
    d1.record(stream)
    d1.synchronize()
    tail_s = max_over_ranks(d0.elapsed_time(d1) / 1000.0, world)
    # e2e: host prompt ids in, first ids out, through qd_batch_prefill
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        bt.prefill(ids)
    t_e2e = max_over_ranks((time.perf_counter() - t0) / steps, world)
    bt.close()
    eng.close()
    if rank == 0:
        line = {
            "metric": "prefill tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(t_max * 1000.0, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (f16 hi/lo tensor-core operands)",
            "data": "synthetic (seeded random-init weights and prompt ids, reference runtime layout)",
            "config": {"workload": WORKLOAD_PF, "global_batch": PF_PROMPTS, "seq_len": PF_LEN,
                       "parallelism": f"prompts sharded: {mine} per GPU x {world} (no collective)",
                       "l2": "inputs larger than L2 (16384 prompt rows, 248 MB of q4 weights per pass)",
                       "decode_tail": {"tokens_per_prompt": PF_NEW, "ms": round(tail_s * 1000, 3),
                                       "tok_s": round(PF_PROMPTS * (PF_NEW - 1) / tail_s, 1)}},
            "roofline": {"bound": "tensor", "kernel": "prefill pass (28 layers: 4 q4 GEMMs, causal attention, "
                                                      "fused norms) + LM head",
                         "achieved": round(achieved, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                         "frac": round(achieved / tflops_peak, 4), "traffic": None,
                         "flops_per_step": flops_local, "peak_source": peak_kind,
                         "note": "algorithmic FLOPs; the GEMMs run 3 f16 MMAs per k-step (hi/lo splits) to keep "
                                 "f32 accuracy, so tensor-pipe work is about 1.5x this"},
            "e2e": {"value": round(PF_PROMPTS * PF_LEN / t_e2e, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": mine * PF_LEN * 4, "d2h_bytes_per_step": mine * 4,
                    "step": "one qd_batch_prefill call: the prompts' ids in, each prompt's first id out"},
            "gpu_launches": steps * (shape.layers * 8 + 3),  # per layer: 2 norms, 4 GEMMs, RoPE, attention
            "clocks": clk.summary(),
            "generated_ids_sample": [int(first[0])] + more[:3, 0].tolist(),
        }
        if world == 1 and with_cpu and not args.no_cpu:
            line["cpu_baseline"] = time_cpu_prefill(rt, all_ids[0])
        return line
    return None


def run_prefill(args, world, rank, local):
    line = measure_prefill(args, world, rank, local, args.steps, args.warmup)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def _bf16_peak() -> float:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def time_cpu_batched(rt, bt, steps=3):
    """Oracle decode of one sequence of the batched workload (its 2048 cached rows
    copied from the GPU context) on the host cores."""
    from oracle import oracle as O
    model = O.Model(rt)
    sess = model.session(max_seq=B64_CTX + steps + 1, kv_f16=True)
    for layer in range(len(model.layers)):
        k, v = bt.read_kv(layer, 0, 0, B64_CTX)
        sess.set_kv(layer, 0, k, v)
    tok, t_total = 1, 0.0
    for i in range(steps):
        t0 = time.perf_counter()
        sess.forward(tok, B64_CTX + i)
        tok, _, _ = sess.next_token()
        t_total += time.perf_counter() - t0
    tps = steps / t_total
    return {"value": round(tps, 4), "unit": UNIT, "cores": O.lib().qo_num_threads(), "kind": "port",
            "sample": f"{steps} decode tokens of one sequence at positions 2048.. over its 2048-row context "
                      "(the oracle has no batching: 64 sequences cost 64x this), WGSL math restated in C (OpenMP)"}


def time_cpu_prefill(rt, ids, n_tokens=256):
    """Oracle prefill of the first n_tokens ids of one prompt (positions 0..n-1, one
    forward per token: the oracle has no batched prefill) on the host cores."""
    from oracle import oracle as O
    model = O.Model(rt)
    sess = model.session(max_seq=n_tokens + 1, kv_f16=True)
    t0 = time.perf_counter()
    for i in range(n_tokens):
        sess.forward(int(ids[i]), i)
    dt = time.perf_counter() - t0
    return {"value": round(n_tokens / dt, 4), "unit": "tok/s", "cores": O.lib().qo_num_threads(), "kind": "port",
            "sample": f"prompt positions 0..{n_tokens - 1} of the first prompt, one token per forward "
                      "(the oracle has no batching or batched prefill), WGSL math restated in C (OpenMP)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (b1: 1000, b64: 128)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (b1: 24, b64: 3)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=24)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="b1", choices=["b1", "b64", "prefill"])
    ap.add_argument("--batch", type=int, default=B64, help="b64 workload: sequences per GPU (profiling cases)")
    ap.add_argument("--vocab-shard", action="store_true",
                    help="b64 workload: split the LM head by vocabulary over the ranks (NCCL all-gathers)")
    ap.add_argument("--b1-only", action="store_true",
                    help="default workload: skip the b64 / prefill objects of the line")
    ap.add_argument("--decode-only", action="store_true",
                    help="prefill + warm-up + timed decode steps only (for profiler launch lists)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"b64": 128, "prefill": 10}.get(args.workload, 1000)
    if args.warmup is None:
        args.warmup = 24 if args.workload == "b1" else 3
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            rc = run_reference(args, world, rank)
        elif args.workload == "b64":
            rc = run_b64(args, world, rank, local)
        elif args.workload == "prefill":
            rc = run_prefill(args, world, rank, local)
        else:
            rc = run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
