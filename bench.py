"""Benchmark of the B200 Q8_0 hot path (talker-shaped decode step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload talker|talker-1.7b] [--batch M]

Default workload: one talker-shaped decode step at M = 1
token -- 28 layers of the Qwen3-TTS 0.6B talker's Q8_0 projections (q 2048x1024,
k/v 1024x1024, o 1024x2048, gate/up 3072x1024, down 1024x3072) chained with the
decoder layer's dataflow, plus a Q8_0 GET_ROWS from a [3072, 1024] table.  The
metric is decode tokens/s (one token = one stream advanced one step).  With
N > 1 every GPU runs its own replica on its own streams (weights replicated,
no collectives on the data path): weak scaling, value = all ranks' tokens / the
slowest rank's time.

Synthetic data: weights 0.02*N(0,1), activations N(0,1), both from the seeded
normal stream of the reference (src/random-stream.cpp); 468 MB of weights per
step exceeds the 126 MB L2, so no flush is needed between steps.

--impl reference times the reference's CPU algorithm for the same step (the
oracle port of ggml-cpu's Q8_0 MUL_MAT; ggml itself is not in the reference
tree) on the host cores, rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="talker", choices=["talker", "talker-1.7b", "dp-sweep", "pack-1.7b", "gemv", "gemv-large", "mul-mat", "int8-peaks",
                             "frame"],
                    help="talker: BASELINE config 2 (config 3 with --batch 16/64/256); talker-1.7b: config 4 shapes; "
                         "dp-sweep: config 5, 512 streams split over the ranks in M=64 batches (one launch per op); "
                         "pack-1.7b: config 4 packing of all 1.4 B weights (synthesize-quantize); "
                         "gemv / gemv-large: config 1 GEMV (and a 142 MB one) as an HBM bandwidth measurement; "
                         "mul-mat: one MUL_MAT of --n x --k at M = --batch")
    ap.add_argument("--n", type=int, default=4096, help="mul-mat: weight rows")
    ap.add_argument("--k", type=int, default=1024, help="mul-mat: K")
    ap.add_argument("--batch", type=int, default=1, help="tokens (streams) per step per GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chain", default="auto", choices=["auto", "per-op"],
                    help="auto: single-launch persistent step for M <= 2, tensor-core GEMM chain from M = 3; "
                         "per-op: CUDA graph of per-op GEMVs up to M = 8")
    return ap.parse_args()


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic(key):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary, if one exists."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(key)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu_index)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def physical_gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def cpu_chain_tokens_per_s(O, mats, norms, table, shape, threads, budget_s, max_steps, x, ids):
    """Oracle decode chain (ggml-cpu's Q8_0 arithmetic restated in C, OpenMP over rows) on the host cores:
    steps until budget_s runs out (at most max_steps); returns (tokens/s, steps, seconds)."""
    m = x.shape[0]
    kw = dict(hidden=shape.hidden, n_head=shape.n_head, n_kv=shape.n_kv, head_dim=shape.head_dim,
              inter=shape.inter, eps=shape.eps, threads=threads)
    O.decoder_chain(mats, norms, table, ids, x, **kw)  # warm-up
    t0 = time.perf_counter()
    O.decoder_chain(mats, norms, table, ids, x, **kw)
    one = time.perf_counter() - t0
    n = max(1, min(max_steps, int(budget_s / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(n):
        O.decoder_chain(mats, norms, table, ids, x, **kw)
    dt = time.perf_counter() - t0
    return n * m / dt, n, dt


def host_threads() -> int:
    """Every host core this process may run on.  torchrun exports
    OMP_NUM_THREADS=1 to its ranks; the CPU arm passes its thread count
    explicitly, so that setting does not shrink it."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_info() -> dict:
    """The host CPU model and core counts (nproc = the cores this process may use)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": host_threads(), "logical_cpus": os.cpu_count()}


def default_threads(n: int) -> int:
    """The reference's default synthesis thread count for n available cores, min(n/2, n-1) and at least 1
    (src/cpu-parallelism.cpp:93-99)."""
    return 1 if n <= 2 else min(n // 2, n - 1)


def load_shapes():
    """The workload geometry (synthesize.cpp_b200/shapes.py), loaded by file path: pure arithmetic, so the CPU
    reference arm states the same workload without importing the product package or any native library."""
    import importlib.util

    name = "b200q8_workload_shapes"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "synthesize.cpp_b200", "shapes.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def talker_shape(args):
    S = load_shapes()
    return S.TALKER_17B if args.workload == "talker-1.7b" else S.TALKER_06B


def talker_sizes(args, world: int, rank: int):
    """(first stream, [batch sizes]) this rank runs per step."""
    if args.workload == "dp-sweep":
        # 512 independent streams split evenly over the ranks, run as M=64 batches.  One
        # launch per op serves all of a rank's batches: the tensor-core GEMM takes the tokens in chunks of at
        # most 64 (the batches), so every weight tile is read once per step and applied to each batch's records
        first, batches = load_shapes().partition_streams(512, world, rank, 64)
        return first, [sum(batches)]
    return rank * args.batch, [args.batch]


def talker_config(args, shape, sizes, world: int) -> dict:
    """The workload's config dict; both arms print exactly this."""
    dp = args.workload == "dp-sweep"
    if dp:
        n = sum(sizes)
        workload = (f"{shape.name} decode, BASELINE config 5: 512 streams over {world} GPU(s), {n} per GPU per "
                    f"step as {(n + 63) // 64} M<=64 batches, one launch per op for all of them")
    else:
        cfg = "4" if args.workload == "talker-1.7b" else ("2" if args.batch == 1 else "3")
        workload = f"{shape.name} decode step (BASELINE config {cfg}), M={args.batch} per GPU"
    return {"workload": workload, "layers": shape.n_layers, "batch_per_gpu": sum(sizes),
            "global_batch": 512 if dp else world * args.batch,
            "parallelism": f"replicas x{world} (no collectives)",
            "l2": "inputs larger than L2: weights streamed every step exceed 126 MB",
            "weight_bytes_per_step": shape.weight_bytes() * len(sizes),
            "algorithmic_bytes_per_step": sum(shape.step_bytes(m) for m in sizes),
            "int8_ops_per_step": sum(shape.step_flops(m) for m in sizes)}


def config3_outliers(args) -> bool:
    """BASELINE config 3 (the 0.6B talker at M > 1) scales 1 % of the activation entries by 20."""
    return args.workload == "talker" and args.batch > 1


def oracle_stream_inputs(O, m: int, hidden: int, table_rows: int, first_stream: int = 0, outliers: bool = False):
    """The streams' N(0,1) activations and token ids, drawn by the oracle's restatement of the reference's
    stream (the same values the product's host library draws), with config 3's outliers when asked."""
    import numpy as np

    S = load_shapes()
    x = np.stack(O.normal_many([S.STREAM_SEED + first_stream + s for s in range(m)], [1.0] * m,
                               [hidden] * m)).astype(np.float32)
    if outliers:
        x.reshape(-1)[S.outlier_positions(m, hidden, first_stream)] *= np.float32(S.OUTLIER_SCALE)
    return x, np.asarray(S.stream_ids(m, table_rows, first_stream), dtype=np.int32)


def oracle_model(O, shape, seed: int = 1000, threads: int = 0):
    """The talker model on the host, drawn and packed by the oracle: seeds as the device workload uses them
    (base + 16*layer + index), 0.02*N(0,1) weights packed by quantize_row_q8_0_ref, 1 + 0.1*N(0,1) norms."""
    import numpy as np

    mats, norms = [], []
    shp = shape.matrices()
    for l in range(shape.n_layers):
        seeds = [seed + 16 * l + j for j in range(7)] + [seed + 16 * l + 8, seed + 16 * l + 9]
        vals = O.normal_many(seeds, [0.02] * 7 + [0.1, 0.1], [n * k for n, k in shp] + [shape.hidden] * 2, threads)
        for j, (n, k) in enumerate(shp):
            mats.append(O.quantize_rows_mt(vals[j].reshape(n, k), threads=threads))
        norms += [1.0 + vals[7], 1.0 + vals[8]]
    tab = O.normal_many([seed - 1], [0.02], [shape.table_rows * shape.hidden])[0]
    table = O.quantize_rows_mt(tab.reshape(shape.table_rows, shape.hidden), threads=threads)
    return mats, np.stack(norms).astype(np.float32), table


def cpu_chain_baseline(O, mats, norms, table, shape, m, budget_s, max_steps, first_stream=0, outliers=False):
    """The oracle chain at the reference's default thread count and at every host core, each on a bounded
    sample; returns the cpu_baseline dict (value = all cores)."""
    x, ids = oracle_stream_inputs(O, m, shape.hidden, shape.table_rows, first_stream, outliers)
    info = cpu_info()
    runs = {}
    for key, threads in (("default", default_threads(info["nproc"])), ("all", info["nproc"])):
        tps, n, dt = cpu_chain_tokens_per_s(O, mats, norms, table, shape, threads, budget_s, max_steps, x, ids)
        runs[key] = {"threads": threads, "value": tps, "steps": n, "seconds": round(dt, 2)}
    return {"value": runs["all"]["value"], "unit": "tok/s", "cores": runs["all"]["threads"], "kind": "port",
            "sample": (f"{runs['all']['steps']} steps of the full {shape.n_layers}-layer step at M={m} "
                       f"({runs['all']['seconds']} s; oracle C port of ggml-cpu Q8_0, OpenMP {info['nproc']} threads); "
                       f"reference default min(n/2, n-1) = {runs['default']['threads']} threads: "
                       f"{runs['default']['value']:.1f} tok/s over {runs['default']['steps']} steps"),
            **info, "threads": runs}


def step_parity(O, ch, dm, shape, ids, x, got, threads):
    """One step of the device chain against the oracle on the same weights and inputs; raises on a mismatch,
    else returns (summary, host copies of the weights).

    Every layer is held to 2e-3 (rel L2 over the batch; 1e-2 per token) against the oracle's layer on the
    device's own input to it (the chain's per-layer buffers): a layer may differ only by the rare activation-code
    flip an ulp of fp32 summation order causes.  The whole step is held against the oracle's own chain with the bound the quantized
    chain's sensitivity allows at this depth (over 28 layers such flips compound to about 1 %)."""
    import numpy as np

    from synthesize_cpp_b200.workloads import host_copy

    mats, norms, table = host_copy(dm)
    kw = dict(hidden=shape.hidden, n_head=shape.n_head, n_kv=shape.n_kv, head_dim=shape.head_dim,
              inter=shape.inter, eps=shape.eps, threads=threads)
    m = x.shape[0]
    emb, _ = O.get_rows(table, shape.hidden, ids)
    h = (x + emb).astype(np.float32)
    zero = np.zeros((1, shape.hidden // 32 * 34), np.uint8)
    worst = 0.0
    for l in range(shape.n_layers):
        out = got if l == shape.n_layers - 1 else ch.buffer(l, "h", m).cpu().numpy()
        ref = O.decoder_chain(mats[7 * l: 7 * l + 7], norms[2 * l: 2 * l + 2], zero, np.zeros(m, np.int32), h, **kw)
        rel_all = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        rel = float((np.linalg.norm(out - ref, axis=1) / np.linalg.norm(ref, axis=1)).max())
        if not (rel_all < 2e-3 and rel < 1e-2):
            raise RuntimeError(f"layer {l} differs from the oracle's layer on the same input: rel L2 {rel_all:.3e} "
                               f"(worst token {rel:.3e})")
        worst = max(worst, rel)
        h = out
    ref = O.decoder_chain(mats, norms, table, ids, x, **kw)
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    cos = float(np.sum(got.astype(np.float64) * ref) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    if not (rel < 5e-2 and cos > 0.998):
        raise RuntimeError(f"step output differs from the oracle's chain: rel L2 {rel:.3e}, cosine {cos:.6f}")
    return ({"layer_token_rel_l2_max": worst, "layer_bound": "rel L2 < 2e-3 per layer, < 1e-2 per token", "step_rel_l2": rel, "step_cosine": cos,
             "step_bound": "rel L2 < 5e-2 and cosine > 0.998 over 28 layers"}, (mats, norms, table))


def frame_positions(i: int, prompt: int, window: int) -> int:
    """Talker position of frame i in the frame workload: frames cycle over positions prompt .. prompt+window-1."""
    return prompt + i % window


FRAME_PROMPT, FRAME_WINDOW = 64, 256


def oracle_frames_per_s(O, tref, pref, ptables, fs, m, threads, budget_s, max_frames):
    """Greedy frames of the oracle restatement (ggml-cpu's Q8_0 arithmetic and the reference's attention in C) on
    the host cores, at talker positions cycling like the GPU arm's; returns (frames/s, frames, seconds)."""
    import numpy as np

    KV, G = fs.talker.kv_dim, fs.groups
    n_ctx = FRAME_PROMPT + FRAME_WINDOW
    state = dict(tk=np.zeros((fs.talker.n_layers, m, n_ctx, KV), np.float32),
                 tv=np.zeros((fs.talker.n_layers, m, n_ctx, KV), np.float32),
                 pk=np.zeros((fs.predictor.n_layers, m, G, KV), np.float32),
                 pv=np.zeros((fs.predictor.n_layers, m, G, KV), np.float32), history={})
    rng = np.random.default_rng(0)
    text = rng.standard_normal((m, fs.talker.hidden)).astype(np.float32)
    prev = np.zeros((m, G), np.int32)
    slots = np.arange(m, dtype=np.int32)

    def one(i):
        nonlocal prev
        pos = np.full(m, frame_positions(i, FRAME_PROMPT, FRAME_WINDOW), np.int32)
        prev = O.frame(tref, pref, ptables, G, text, prev, pos, slots, state, threads=threads)[0]

    one(0)
    t0 = time.perf_counter()
    one(1)
    per = time.perf_counter() - t0
    n = max(1, min(max_frames, int(budget_s / max(per, 1e-6))))
    t0 = time.perf_counter()
    for i in range(n):
        one(2 + i)
    dt = time.perf_counter() - t0
    return n * m / dt, n, dt


def run_reference_frame(args, rank):
    """Reference arm of the frame workload: the oracle's greedy frames (the reference's own CPU code path for a
    frame is ggml-cpu, absent from its tree) on all host threads, rank 0 only."""
    import torch

    import __graft_entry__ as g

    g.load_package()
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from synthesize_cpp_b200.workloads import FRAME_06B, build_frame_model, frame_host_copy

    if not torch.cuda.is_available():
        raise RuntimeError("the frame workload builds its weights on the device")
    fm = build_frame_model(FRAME_06B, torch.device("cuda", 0))
    tref, pref, ptables = frame_host_copy(fm)
    threads = host_threads()
    value, n, dt = oracle_frames_per_s(O, tref, pref, ptables, FRAME_06B, args.batch, threads, 120.0, args.steps)
    sample = (f"{n} of {args.steps} greedy frames at M={args.batch} (28-layer talker + 15 predictor calls; oracle C "
              f"port, OpenMP {threads} threads)")
    line = {
        "impl": "reference", "metric": "Qwen3-TTS decode frames (talker + code predictor, greedy)", "value": value,
        "unit": "frames/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / n, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xint8->int32, f32 scale; f32 attention",
        "data": "synthetic (seeded N(0,1) stream of src/random-stream.cpp)",
        "config": {"workload": f"qwen3-tts-0.6b decode frame, M={args.batch}", "batch": args.batch},
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_frame(args, rank, local_rank):
    """A Qwen3-TTS decode frame on the device (b200q8_frame_run): the 28-layer talker step with the reference's
    attention, its codec head and greedy choice, then the code predictor's prefill and 14 steps (5 layers each,
    one head and one codec table per group), for M streams per GPU; replicas across GPUs."""
    import torch

    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import chain as chain_mod
    from synthesize_cpp_b200 import dp as dpu
    from synthesize_cpp_b200 import frame as frame_mod
    from synthesize_cpp_b200 import q8
    from synthesize_cpp_b200.workloads import FRAME_06B, build_frame_model, frame_host_copy

    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dpu.init("nccl", timeout_s=300.0, device=dev)
    fs, m = FRAME_06B, args.batch
    fm = build_frame_model(fs, dev)
    n_ctx = FRAME_PROMPT + FRAME_WINDOW
    mk = lambda dm, out, max_m, ctx: chain_mod.DecodeChain(
        dm.layers, dm.table, hidden=dm.shape.hidden, n_head=dm.shape.n_head, n_kv=dm.shape.n_kv,
        head_dim=dm.shape.head_dim, inter=dm.shape.inter, eps=dm.shape.eps, max_m=max_m,
        attention=dict(rope_theta=fs.rope_theta, n_ctx=ctx, n_slots=m), output=out)
    talker = mk(fm.talker, fm.t_out, max(8, m), n_ctx)
    pred = mk(fm.predictor, fm.p_out, max(8, 2 * m), fs.groups)
    fr = frame_mod.Frame(talker, pred, fm.ptables)
    G, H = fs.groups, fs.talker.hidden
    rng = torch.Generator().manual_seed(1234 + rank)
    text_host = torch.randn((m, H), generator=rng).pin_memory()
    text = text_host.to(dev)
    codes = [torch.zeros((m, G), dtype=torch.int32, device=dev) for _ in range(2)]
    codes_host = torch.empty((m, G), dtype=torch.int32).pin_memory()
    pos = torch.full((m,), FRAME_PROMPT, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    state = {"i": 0}

    def frame(e2e=False):
        i = state["i"]
        if i % FRAME_WINDOW == 0:
            pos.fill_(FRAME_PROMPT)
        else:
            pos.add_(1)
        if e2e:
            text.copy_(text_host, non_blocking=True)
        fr.run(codes[(i + 1) & 1], text=text, prev=codes[i & 1], pos=pos)
        if e2e:
            codes_host.copy_(codes[(i + 1) & 1], non_blocking=True)
        state["i"] = i + 1

    def barrier_sync():
        torch.cuda.synchronize(dev)
        dpu.barrier(dev)
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        frame()
    barrier_sync()
    if q8.device_status(local_rank) != 0:
        raise RuntimeError("device status set during warm-up")
    first = state["i"]
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    barrier_sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        frame()
    e1.record(stream)
    barrier_sync()
    t_dev = dpu.max_over_ranks(e0.elapsed_time(e1) / 1e3, dev)
    clocks = sampler.stop()
    barrier_sync()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        frame(e2e=True)
    f1.record(stream)
    barrier_sync()
    t_e2e = dpu.max_over_ranks(f0.elapsed_time(f1) / 1e3, dev)
    if q8.device_status(local_rank) != 0:
        raise RuntimeError("device status set during the timed region")

    positions = [frame_positions(i, FRAME_PROMPT, FRAME_WINDOW) for i in range(first, first + args.steps)]
    mean_pos = sum(positions) / len(positions)
    frames = world * m * args.steps
    frame_s = t_dev / args.steps
    peaks, peak_kind = measured_peaks()
    fbytes = fs.frame_bytes(m, mean_pos)
    achieved = fbytes / frame_s / 1e9

    def chain_launches(layers, mm):
        # the persistent step is one launch up to 2 tokens; from 3 on, per layer a stage and a GEMM for each of
        # qkv, o, gate|up and down plus the attention kernel, then the output stage and head
        return 1 + (1 if mm <= 2 else 9 * layers + 3)

    per_frame = (2 + chain_launches(fs.talker.n_layers, m) + 2 + chain_launches(fs.predictor.n_layers, 2 * m) + 1 +
                 (G - 2) * (chain_launches(fs.predictor.n_layers, m) + 1))
    line = {
        "metric": "Qwen3-TTS decode frames (talker + code predictor, greedy)", "value": frames / t_dev,
        "unit": "frames/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": 1e3 * frame_s, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8xint8->int32, f32 scale (Q8_0 x F32); f32 attention",
        "data": "synthetic (seeded N(0,1) stream of src/random-stream.cpp; weights 0.02*N, packed on device)",
        "config": {"workload": f"qwen3-tts-0.6b decode frame: 28-layer talker + {G - 1} code-predictor calls "
                               f"(5 layers), greedy, M={m} streams per GPU, talker positions "
                               f"{FRAME_PROMPT}..{FRAME_PROMPT + FRAME_WINDOW - 1} cycling (mean {mean_pos:.0f})",
                   "batch_per_gpu": m, "global_batch": world * m, "groups": G,
                   "parallelism": f"replicas x{world} (no collectives)",
                   "l2": "inputs larger than L2: 1.76 GB of weights streamed per frame",
                   "weight_bytes_per_frame": fs.weight_bytes(), "algorithmic_bytes_per_frame": fbytes,
                   "int8_ops_per_frame": fs.frame_ops(m),
                   "position_update": "one torch fill_/add_ of the [M] position vector per frame"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": ncu_traffic(f"frame-m{m}"),
                     "kernel": "the frame's CUDA graph (GEMV/GEMM + attention + selection kernels)",
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "int8_tops": fs.frame_ops(m) / frame_s / 1e12},
        "e2e": {"value": frames / t_e2e, "unit": "frames/s", "h2d_bytes_per_step": m * H * 4,
                "d2h_bytes_per_step": m * G * 4},
        "gpu_launches": per_frame * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        tref, pref, ptables = frame_host_copy(fm)
        threads = host_threads()
        v, n, dt = oracle_frames_per_s(O, tref, pref, ptables, fs, min(m, 8), threads, 12.0, 400)
        line["cpu_baseline"] = {"value": v, "unit": "frames/s", "cores": threads, "kind": "port",
                                "sample": f"{n} greedy frames at M={min(m, 8)} ({dt:.1f} s; oracle C port, OpenMP)"}
    fr.close()
    talker.close()
    pred.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, rank):
    """The reference's CPU path for the same step, rank 0 only: the oracle's restatement of ggml-cpu's Q8_0
    arithmetic (ggml itself is absent from the reference tree) on every host core.  Nothing from the product
    package or its native libraries is imported: the weights are drawn and packed by the oracle, and the
    workload geometry comes from the pure-arithmetic shapes module."""
    if rank != 0:
        return
    if args.workload == "frame":
        run_reference_frame(args, rank)
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    world = int(os.environ.get("WORLD_SIZE", "1"))
    shape = talker_shape(args)
    first, sizes = talker_sizes(args, world, 0)
    m = sizes[0]
    info = cpu_info()
    threads = info["nproc"]
    mats, norms, table = oracle_model(O, shape, threads=threads)
    x, ids = oracle_stream_inputs(O, m, shape.hidden, shape.table_rows, first, config3_outliers(args))
    kw = dict(hidden=shape.hidden, n_head=shape.n_head, n_kv=shape.n_kv, head_dim=shape.head_dim,
              inter=shape.inter, eps=shape.eps, threads=threads)
    for _ in range(max(1, min(args.warmup, 3))):
        O.decoder_chain(mats, norms, table, ids, x, **kw)
    t0 = time.perf_counter()
    O.decoder_chain(mats, norms, table, ids, x, **kw)
    one = time.perf_counter() - t0
    # each of the K steps is the full step when K steps fit in ~150 s, else the
    # run is cut to the steps that fit (stated in the sample string)
    n = max(1, min(args.steps, int(150.0 / max(one, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(n):
        O.decoder_chain(mats, norms, table, ids, x, **kw)
    dt = time.perf_counter() - t0
    # the per-step rate of this sample: one batch of m streams (a dp-sweep rank runs len(sizes) such batches)
    value = n * m / dt
    d_threads = default_threads(threads)
    tps_d, n_d, dt_d = cpu_chain_tokens_per_s(O, mats, norms, table, shape, d_threads, 20.0, args.steps, x, ids)
    sample = (f"{n} of {args.steps} steps of the full {shape.n_layers}-layer step at M={m} "
              f"(oracle C port of ggml-cpu Q8_0 MUL_MAT, OpenMP {threads} threads); reference default "
              f"min(n/2, n-1) = {d_threads} threads: {tps_d:.1f} tok/s over {n_d} steps")
    line = {
        "impl": "reference", "metric": "talker-shaped Q8_0 decode throughput", "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / n,
        "higher_is_better": True, "scaling": "strong" if args.workload == "dp-sweep" else "weak",
        "vs_baseline": None, "dtype": "int8xint8->int32, f32 scale (Q8_0 x F32)",
        "data": "synthetic (seeded N(0,1) stream of src/random-stream.cpp; weights 0.02*N, packed by the oracle)",
        "config": talker_config(args, shape, sizes, world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample, **info,
                         "threads": {"default": {"threads": d_threads, "value": tps_d, "steps": n_d},
                                     "all": {"threads": threads, "value": value, "steps": n}}},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_pack(args, rank, local_rank):
    """BASELINE config 4 packing: F32 -> Q8_0 of every 1.7B-shaped matrix (1,415,577,600 weights)."""
    import numpy as np
    import torch

    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import host, q8
    from synthesize_cpp_b200.workloads import TALKER_17B

    if rank != 0:
        return
    shape = TALKER_17B
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    mats = [(n, k) for _ in range(shape.n_layers) for (n, k) in shape.matrices()] + [(3072, shape.hidden)]
    weights = sum(n * k for n, k in mats)
    f32 = [np.empty(n * k, np.float32) for n, k in mats]
    host.normal_many([2000 + i for i in range(len(mats))], [0.02] * len(mats), f32)
    src_dev = [torch.from_numpy(a).to(dev) for a in f32]
    dst_dev = [torch.empty((n, k // 32 * 34), dtype=torch.uint8, device=dev) for n, k in mats]

    def step():
        for a, d, (n, k) in zip(src_dev, dst_dev, mats):
            q8.quantize_rows(a.view(n, k), out=d)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    t_dev = e0.elapsed_time(e1) / 1e3 / args.steps
    clocks = sampler.stop()
    # e2e: the quantize tool's own call, host F32 in, host Q8_0 out (its staging
    # is created by a first small call, as a quantize run's first tensor would)
    dst_host = [np.empty(n * (k // 32 * 34), np.uint8) for n, k in mats]
    q8.quantize_chunk_host(f32[0], dst_host[0], 0, 1, mats[0][1], device=local_rank)
    t0 = time.perf_counter()
    for a, d, (n, k) in zip(f32, dst_host, mats):
        q8.quantize_chunk_host(a, d, 0, n, k, device=local_rank)
    t_e2e = time.perf_counter() - t0
    # parity: every tensor's bytes, from the device buffers and from the host call, against the oracle's
    # restatement of quantize_row_q8_0_ref (OpenMP over rows); the reference tool's own entry point
    # (ggml_quantize_chunk) on the largest tensor; then that tool's rate (one thread, as ggml_quantize_chunk)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    for i, (a, (n, k)) in enumerate(zip(f32, mats)):
        ref = O.quantize_rows_mt(a.reshape(n, k)).ravel()
        if not (np.array_equal(ref, dst_host[i]) and np.array_equal(ref, dst_dev[i].cpu().numpy().ravel())):
            raise AssertionError(f"pack-1.7b: tensor {i} ({n} x {k}) differs from the oracle")
    n0, k0 = mats[4]
    ref, _ = O.quantize_chunk(f32[4], 0, n0, k0)
    assert np.array_equal(ref, dst_host[4]) and np.array_equal(ref, dst_dev[4].cpu().numpy().ravel())
    cpu_w = 0
    c0 = time.perf_counter()
    for a, (n, k) in zip(f32[:14], mats[:14]):
        O.quantize_chunk(a, 0, n, k)
        cpu_w += n * k
    cpu_t = time.perf_counter() - c0
    peaks, peak_kind = measured_peaks()
    bytes_step = weights * (4 + 34 / 32)
    line = {
        "metric": "Q8_0 packing throughput (synthesize-quantize, BASELINE config 4)", "value": weights / t_dev / 1e9,
        "unit": "Gweight/s", "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": 1e3 * t_dev, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 -> q8_0", "data": "synthetic (seeded 0.02*N(0,1) stream of src/random-stream.cpp)",
        "config": {"workload": f"pack all {len(mats)} 1.7B-shaped matrices + 3072x2048 head, {weights} weights",
                   "l2": "inputs larger than L2 (5.66 GB of F32 per step)"},
        "roofline": {"bound": "hbm", "achieved": bytes_step / t_dev / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": bytes_step / t_dev / 1e9 / peaks["hbm_gbs"], "traffic": None,
                     "kernel": "quantize_dense_kernel", "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
        "e2e": {"value": weights / t_e2e / 1e9, "unit": "Gweight/s", "h2d_bytes_per_step": weights * 4,
                "d2h_bytes_per_step": weights * 34 // 32},
        "gpu_launches": len(mats) * args.steps,
        "clocks": clocks,
        "parity": {"tensors_byte_equal": len(mats), "weights_checked": weights,
                   "against": "oracle quantize_row_q8_0_ref (device buffers and host-call output)"},
        "cpu_baseline": {"value": cpu_w / cpu_t / 1e9, "unit": "Gweight/s", "cores": 1, "kind": "port",
                         "sample": f"{cpu_w} weights (first 2 layers) through the oracle's quantize_row_q8_0_ref, "
                                   "one thread like ggml_quantize_chunk"},
    }
    print(json.dumps(line), flush=True)


def run_mul_mat(args, rank, local_rank):
    """One MUL_MAT(Q8_0 W [N, K], F32 x [K, M]) per step, W rotated over copies totalling > 2x L2, steps captured
    as CUDA graphs of back-to-back calls.  gemv: BASELINE config 1 (N=3072, K=1024, M=1); gemv-large: a 142 MB
    M=1 product (N=32768, K=4096); mul-mat: --n/--k/--batch (config 3 op shapes)."""
    import numpy as np
    import torch

    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import host, q8

    if rank != 0:
        return
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if args.workload == "gemv":
        n, k, m = 3072, 1024, 1
    elif args.workload == "gemv-large":
        n, k, m = 32768, 4096, 1
    else:
        n, k, m = args.n, args.k, args.batch
    rb = k // 32 * 34
    w_bytes = n * rb
    copies = max(2, int(2 * 126e6 // w_bytes) + 1)
    # weights: the seeded 0.02*N(0,1) stream packed on the device; copies differ by their seed
    ws = []
    for c in range(copies):
        f = np.empty(n * k, np.float32)
        host.normal_many([c], [0.02], [f])
        ws.append(q8.quantize_rows(torch.from_numpy(f).to(dev).view(n, k)))
    x_np = np.empty(m * k, np.float32)
    host.normal_many([1], [1.0], [x_np])
    x_np = x_np.reshape(m, k)
    x = torch.from_numpy(x_np).to(dev)
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    wsp = torch.empty(max(1, q8.workspace_size(k, n, m)), dtype=torch.uint8, device=dev)
    calls_per_graph = copies * max(1, 64 // copies)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for i in range(calls_per_graph):  # warm-up outside capture
            q8.mul_mat(ws[i % copies], k, x, out=y, workspace=wsp)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(calls_per_graph):
            q8.mul_mat(ws[i % copies], k, x, out=y, workspace=wsp)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(1, args.steps // calls_per_graph)
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(dev)
    e0.record(cur)
    for _ in range(reps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    calls = reps * calls_per_graph
    t_call = e0.elapsed_time(e1) / 1e3 / calls
    if q8.device_status(local_rank) != 0:
        raise RuntimeError("device status set during the timed region")
    # parity spot check against the oracle on copy 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    y0 = q8.mul_mat(ws[0], k, x, workspace=wsp).cpu().numpy()
    y_ref, bound = O.mul_mat(ws[0].cpu().numpy(), k, x_np)
    assert np.all(np.abs(y0 - y_ref) <= 1e-5 * bound + 1e-30)
    # e2e: host x in, host y out around each call
    x_host = torch.from_numpy(x_np).pin_memory()
    y_host = torch.empty((m, n), dtype=torch.float32).pin_memory()
    x_dev = torch.empty_like(x)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(cur)
    e2e_calls = min(calls, 2000)
    for i in range(e2e_calls):
        x_dev.copy_(x_host, non_blocking=True)
        q8.mul_mat(ws[i % copies], k, x_dev, out=y, workspace=wsp)
        y_host.copy_(y, non_blocking=True)
    f1.record(cur)
    torch.cuda.synchronize(dev)
    t_e2e = f0.elapsed_time(f1) / 1e3 / e2e_calls
    bytes_call = w_bytes + 4 * k * m + 4 * n * m
    ops_call = 2 * n * k * m
    peaks, peak_kind = measured_peaks()
    # CPU: the oracle port on a bounded sample, all host threads
    threads = host_threads()
    wq0 = ws[0].cpu().numpy()
    O.mul_mat(wq0, k, x_np, threads=threads)
    c0, cn = time.perf_counter(), 0
    while time.perf_counter() - c0 < 3.0:
        O.mul_mat(wq0, k, x_np, threads=threads)
        cn += 1
    cpu_t = (time.perf_counter() - c0) / cn
    name = {"gemv": "BASELINE config 1 GEMV", "gemv-large": "large GEMV"}.get(args.workload, "MUL_MAT")
    line = {
        "metric": f"Q8_0 MUL_MAT HBM GB/s ({'decode GEMV, ' if m == 1 else ''}M={m})",
        "value": bytes_call / t_call / 1e9, "unit": "GB/s",
        "n_gpus": 1, "steps": calls, "warmup": max(args.warmup, 3), "ms_per_step": 1e3 * t_call,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->int32, f32 scale",
        "data": "synthetic (seeded 0.02*N(0,1) weights packed on device, N(0,1) x)",
        "config": {"workload": f"{name} N={n} K={k} M={m}, {copies} rotating weight copies "
                               f"({copies * w_bytes / 1e6:.0f} MB > L2), CUDA graph of {calls_per_graph} calls",
                   "l2": "weights rotated over copies totalling more than 2x L2"},
        "roofline": {"bound": "hbm", "achieved": bytes_call / t_call / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": bytes_call / t_call / 1e9 / peaks["hbm_gbs"], "traffic": ncu_traffic(args.workload),
                     "kernel": "stage_rows_kernel + gemm_q8_0_kernel (int8 mma.sync, TMA tensor-map weight boxes)",
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "int8_tops": ops_call / t_call / 1e12},
        "e2e": {"value": bytes_call / t_e2e / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * k * m,
                "d2h_bytes_per_step": 4 * n * m},
        "gpu_launches": 2 * calls,
        "clocks": clocks,
        "cpu_baseline": {"value": bytes_call / cpu_t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{cn} calls on copy 0 (cache-resident on the host; oracle C port, OpenMP)"},
    }
    print(json.dumps(line), flush=True)


def run_int8_peaks(args, rank, local_rank):
    """Measured int8 ceilings of this B200 (libb200q8_peaks.so): tcgen05.mma kind::i8 (128 x 256 x 32 per MMA,
    one issuing thread per SM, TMEM accumulators), mma.sync m16n8k32 s8 (the legacy tensor path the Q8_0 GEMM
    uses) and the per-block fp32 rescale a Q8_0 GEMM does on the CUDA cores after every K = 32 block, as
    int8-op-equivalent rates.  The tcgen05 MMA is first checked on known operands against exact int32 products."""
    import ctypes

    import numpy as np
    import torch

    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import build

    if rank != 0:
        return
    torch.cuda.set_device(local_rank)
    L = ctypes.CDLL(build.PEAKS_LIB)
    L.b200q8p_tcgen05_check.argtypes = [ctypes.c_void_p]
    L.b200q8p_run.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
    L.b200q8p_tcgen05_latency.argtypes = [ctypes.c_void_p]
    out = np.empty((128, 256), np.int32)
    rc = L.b200q8p_tcgen05_check(out.ctypes.data)
    a = (np.arange(128)[:, None] % 7 - 3) * np.ones((1, 32), np.int64)
    b = (np.arange(256)[:, None] + 2 * np.arange(32)[None, :]) % 5 - 2
    want = (a @ b.T).astype(np.int32)
    if rc != 0 or not np.array_equal(out, want):
        raise RuntimeError(f"tcgen05 kind::i8 check failed (rc {rc}, {int((out != want).sum())} of 32768 differ)")
    # the round trips the tcgen05 GEMM's pipeline is built from (one CTA, SM clock cycles)
    lat = np.zeros(6, np.int64)
    rc = L.b200q8p_tcgen05_latency(lat.ctypes.data)
    if rc != 0:
        raise RuntimeError(f"tcgen05 latency probe: rc {rc}")
    latency = {"tcgen05_ld_16_columns_and_wait": {"best": int(lat[0]), "mean": int(lat[1])},
               "tcgen05_st_32_columns_and_wait": {"best": int(lat[2]), "mean": int(lat[3])},
               "mma_128x128x32_issue_to_commit": int(lat[4]),
               "mma_128x128x32_back_to_back_each": round((int(lat[5]) - int(lat[4])) / 31, 1)}
    sms = torch.cuda.get_device_properties(local_rank).multi_processor_count
    peaks, peak_kind = measured_peaks()
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    res = {}
    # (kind, iters per launch, int8 ops per launch)
    plan = {"tcgen05_kind_i8": (0, 8192, lambda it: sms * it * 2 * 128 * 256 * 32),
            "mma_sync_m16n8k32_s8": (1, 8192, lambda it: sms * 8 * it * 8 * 2 * 16 * 8 * 32),
            "q8_0_block_rescale_fp32": (2, 8192, lambda it: sms * 256 * it * 16 * 64)}
    for name, (kind, iters, ops) in plan.items():
        ms = ctypes.c_float()
        rc = L.b200q8p_run(kind, sms, iters, max(3, args.steps), ctypes.byref(ms))
        if rc != 0:
            raise RuntimeError(f"{name}: rc {rc}")
        res[name] = {"tops": ops(iters) / (ms.value * 1e-3) / 1e12, "ms_per_launch": ms.value, "iters": iters}
    clocks = sampler.stop()
    t = res["tcgen05_kind_i8"]["tops"]
    line = {
        "metric": "int8 tensor ceilings and the Q8_0 per-block rescale bound (TOPS)", "value": t, "unit": "TOPS",
        "n_gpus": 1, "steps": max(3, args.steps), "warmup": 1,
        "ms_per_step": res["tcgen05_kind_i8"]["ms_per_launch"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "s8 x s8 -> s32; fp32 rescale", "data": "synthetic register/shared operands",
        "config": {"workload": f"int8 peaks, one CTA per SM ({sms} SMs)",
                   "tcgen05": "M=128 N=256 K=32 kind::i8, one elected thread, two TMEM accumulators",
                   "mma_sync": "8 warps x 8 independent m16n8k32 s8 chains",
                   "rescale": "per 2 block-outputs: fadd2 (bias) + fmul2 (dw*dx) + ffma2; 64 int8 ops each"},
        "peaks": res,
        "tcgen05_check": "one MMA on known operands equals the exact int32 products",
        "tcgen05_latency_cycles": latency,
        "bf16_tflops_measured": peaks.get("bf16_tflops"), "peak_source": peak_kind,
        "gpu_launches": 3 * (max(3, args.steps) + 1) + 3,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "pack-1.7b":
        run_pack(args, rank, local_rank)
        return
    if args.workload == "int8-peaks":
        run_int8_peaks(args, rank, local_rank)
        return
    if args.workload in ("gemv", "gemv-large", "mul-mat"):
        run_mul_mat(args, rank, local_rank)
        return
    if args.workload == "frame":
        run_frame(args, rank, local_rank)
        return

    import torch
    import torch.distributed as dist

    import __graft_entry__ as g

    g.load_package()
    from synthesize_cpp_b200 import chain as chain_mod
    from synthesize_cpp_b200 import q8
    from synthesize_cpp_b200.workloads import build_model, host_copy, stream_inputs

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    from synthesize_cpp_b200 import dp as dpu

    if world > 1:
        dpu.init("nccl", timeout_s=300.0, device=dev)

    def barrier_sync():
        torch.cuda.synchronize(dev)
        dpu.barrier(dev)
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        return dpu.max_over_ranks(v, dev)

    shape = talker_shape(args)
    dp = args.workload == "dp-sweep"
    first, sizes = talker_sizes(args, world, rank)
    m_max = max(sizes)
    dm = build_model(shape, dev)
    os.environ["B200Q8_CHAIN_PER_OP"] = "1" if args.chain == "per-op" else "0"
    ch = chain_mod.DecodeChain(dm.layers, dm.table, hidden=shape.hidden, n_head=shape.n_head, n_kv=shape.n_kv,
                               head_dim=shape.head_dim, inter=shape.inter, eps=shape.eps, max_m=max(8, m_max))
    batches = []
    off = first
    for m in sizes:
        x_np, ids_np = stream_inputs(m, shape.hidden, shape.table_rows, first_stream=off,
                                     outliers=config3_outliers(args))
        off += m
        x_host = torch.from_numpy(x_np).pin_memory()
        ids_host = torch.from_numpy(ids_np).pin_memory()
        h_host = torch.empty((m, shape.hidden), dtype=torch.float32).pin_memory()
        batches.append((x_host, ids_host, h_host, x_host.to(dev), ids_host.to(dev),
                        torch.empty((m, shape.hidden), dtype=torch.float32, device=dev)))
    stream = torch.cuda.current_stream(dev)

    def step():
        for (_, _, _, x_dev, ids_dev, h_dev) in batches:
            ch.run(ids_dev, x_dev, h_dev)

    def step_e2e():
        for (x_host, ids_host, h_host, x_dev, ids_dev, h_dev) in batches:
            x_dev.copy_(x_host, non_blocking=True)
            ids_dev.copy_(ids_host, non_blocking=True)
            ch.run(ids_dev, x_dev, h_dev)
            h_host.copy_(h_dev, non_blocking=True)

    for _ in range(args.warmup):
        step()
    barrier_sync()
    if q8.device_status(local_rank) != 0:
        raise RuntimeError("device status set during warm-up")

    # ---- device-resident timing (inputs already in HBM)
    sampler = ClockSampler(physical_gpu_index(local_rank))
    sampler.start()
    time.sleep(0.3)
    barrier_sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier_sync()
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    clocks = sampler.stop()

    # ---- end to end through the C ABI with host buffers, host clock: every step copies its inputs in from
    # pinned host memory, runs, copies the result out and waits for it before the next step is issued (a
    # synthesis loop reads each step's output before it can form the next input, model.cpp:1402-1414)
    barrier_sync()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step_e2e()
        stream.synchronize()
    t_e2e = max_over_ranks(time.perf_counter() - t0)
    # the same copies enqueued back to back without the per-step wait (device clock)
    barrier_sync()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        step_e2e()
    f1.record(stream)
    barrier_sync()
    t_e2e_async = max_over_ranks(f0.elapsed_time(f1) / 1e3)
    if q8.device_status(local_rank) != 0:
        raise RuntimeError("device status set during the timed region")

    # ---- parity: one step of this rank's first batch against the oracle's chain on the same inputs and weights
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle as O

    x_host, ids_host, h_host, x_dev, ids_dev, h_dev = batches[0]
    h_dev.zero_()
    ch.run(ids_dev, x_dev, h_dev)
    torch.cuda.synchronize(dev)
    par, (mats, norms, table) = step_parity(O, ch, dm, shape, ids_host.numpy(), x_host.numpy(), h_dev.cpu().numpy(),
                      threads=max(1, host_threads() // world))
    par["checked"] = f"rank {rank}, batch of {sizes[0]} streams, one step"

    tokens = (512 if dp else world * args.batch) * args.steps
    value = tokens / t_dev
    step_s = t_dev / args.steps
    peaks, peak_kind = measured_peaks()
    config = talker_config(args, shape, sizes, world)
    step_bytes = config["algorithmic_bytes_per_step"]
    step_flops = config["int8_ops_per_step"]
    achieved = step_bytes / step_s / 1e9
    persistent = args.chain == "auto" and m_max <= 2
    per_batch = lambda m: (1 if persistent else
                           2 + 8 * shape.n_layers if m >= 3 and args.chain == "auto" or m > 8 else 1 + 4 * shape.n_layers)
    launches_per_step = sum(per_batch(m) for m in sizes)
    if persistent:
        kernel_name = "decode_step_kernel (the whole step in one persistent launch)"
    elif m_max > 8 or args.chain == "auto":
        kernel_name = "gemm_q8_0_kernel + stage_rows_kernel (int8 mma.sync GEMM per op, CUDA graph + PDL)"
    else:
        kernel_name = "gemv_q8_0_kernel (every launch of the step; 1 + 4*layers launches)"
    h2d = sum(m * shape.hidden * 4 + m * 4 for m in sizes)
    d2h = sum(m * shape.hidden * 4 for m in sizes)
    line = {
        "metric": "talker-shaped Q8_0 decode throughput", "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * step_s, "higher_is_better": True,
        "scaling": "strong" if dp else "weak", "vs_baseline": None, "dtype": "int8xint8->int32, f32 scale (Q8_0 x F32)",
        "data": "synthetic (seeded N(0,1) stream of src/random-stream.cpp; weights 0.02*N, packed on device)",
        "config": config,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": ncu_traffic(f"{shape.name}-m{m_max}"),
                     "kernel": kernel_name,
                     "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                     "int8_tops": step_flops / step_s / 1e12},
        "e2e": {"value": tokens / t_e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "clock": "host perf_counter over K steps, each copy-in + step + copy-out waited for before the next"},
        "e2e_async": {"value": tokens / t_e2e_async, "unit": "tok/s",
                      "clock": "CUDA events around K copy-in + step + copy-out sequences enqueued back to back"},
        "parity": par,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_chain_baseline(O, mats, norms, table, shape, min(m_max, 64), budget_s=8.0,
                                                  max_steps=400, first_stream=first, outliers=config3_outliers(args))
    ch.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
