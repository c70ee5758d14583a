"""Decode throughput benchmark (MiniCPM5-2B-shaped Q4_K_M greedy decode,
batch 1 per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --config 1        # config 1: isolated GEMV sweep, one JSON line per case
    python bench.py --config 2        # config 2: decode after an 8192-position prefill
    python bench.py --config 3        # config 3: batched decode, 64 sequences split over the GPUs
    python bench.py --config 4        # config 4: all-Q8_0 tensor-parallel batch-1 decode over the GPUs

A step is one greedy decode token.  Each rank prefills its own seeded 128-token prompt
(untimed), runs W warm-up tokens, then K timed tokens chained on the device (the argmax of
step t is the token of step t+1).  Ranks decode independent sequences (no collective in the
data path, weak scaling); `value` is the aggregate tokens/s over all ranks using the
slowest rank's device time.  Every token streams all 1.41 GB of weights, far larger than
L2, so no flush is needed between steps.

Prints one JSON line on rank 0.
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

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "minicpm5.cpp_b200"))

PROMPT = 128
METRIC = "decode tokens/s (batch 1 per GPU, MiniCPM5-2B Q4_K_M shape)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prefill length (untimed)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, default=0, choices=[0, 1, 2, 3, 4],
                    help="0: batch-1 decode (headline); 1: GEMV sweep; 2: long-context decode; 3: batched decode; "
                         "4: all-Q8_0 tensor-parallel decode")
    ap.add_argument("--comm", default="p2p", choices=["p2p", "nccl"], help="config 4: exchange of partial sums")
    ap.add_argument("--seqs", type=int, default=64, help="config 3: sequences in total (64 = the config; fewer for a "
                    "smaller case, e.g. one data-parallel rank's share on one GPU)")
    ap.add_argument("--batch-gemm", default="tcgen05", choices=["mma", "tcgen05"],
                    help="config 3: batched GEMM kernel (tcgen05, the default, or int8 mma.sync in the batch-1 order)")
    ap.add_argument("--case", default=None,
                    help="config 1: only the cases whose 'name type' contains this text, e.g. 'gate+up 12288x2048 Q4_K'")
    ap.add_argument("--kv-type", default="f32", choices=["f32", "f16"],
                    help="configs 0 and 2: KV-cache element type (f32 = the reference's cache; f16 halves its bytes)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def max_over_ranks(x: float, pg, device: str = "cuda") -> float:
    """Largest value of `x` over the ranks of process group `pg` (x itself without one).
    Timings are reduced this way: the job is as slow as its slowest rank."""
    import torch
    t = torch.tensor([x], dtype=torch.float64, device=device)
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic(avg_positions: float):
    """DRAM bytes (read + write) per decode launch from the committed ncu summary.

    The summary records one captured launch at `positions` attended positions; the K/V
    cache read grows by KV_BYTES_PER_POSITION per position, so the figure is moved to the
    benchmark's mean position by that amount (weights dominate: 1.41 GB vs 86 KB/position).
    """
    from mcpm import spec
    p = os.path.join(REPO, "profiles", "decode_kernel_traffic.txt")
    vals = {}
    try:
        with open(p) as f:
            for line in f:
                if "=" in line and not line.startswith("#"):
                    k, v = line.split("=", 1)
                    vals[k.strip()] = v.strip()
        b = float(vals["bytes_per_launch"])
        if "positions" in vals:
            b += (avg_positions - float(vals["positions"])) * spec.KV_BYTES_PER_POSITION
        return int(b)
    except (OSError, KeyError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 20 ms during the timed region (a
    config-0 run times 256 tokens, about 0.3 s)."""

    def __init__(self, device: int):
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(device), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "20"],
                                      stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.out.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.out.name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(model_path: str, n_prompt: int = 16, n_gen: int = 32, port_only: bool = False, n_skip: int = 0):
    """Reference CPU build (oracle/_ref, AVX2 + OpenMP) on a bounded sample of the same
    workload, in a child process so OMP settings apply; falls back to the C restatement
    (always for the all-Q8_0 model, which the reference build cannot run).  The prompt is
    prefilled token by token (untimed, as the reference's chat loop does), `n_skip` greedy
    tokens follow untimed (the GPU arm's warm-up), then `n_gen` greedy tokens are timed."""
    cores = os.cpu_count() or 1
    code = f"""
import sys, time, json, numpy as np
sys.path.insert(0, {os.path.join(REPO, 'oracle')!r}); sys.path.insert(0, {os.path.join(REPO, 'minicpm5.cpp_b200')!r})
import oracle as O
from mcpm import synth
kind = 'reference' if (O.have_ref() and not {port_only!r}) else 'port'
if kind == 'reference':
    e = O.RefEngine(O.Ref(), {model_path!r}, {n_prompt + n_skip + n_gen + 1})
else:
    e = O.OracleModel(O.Oracle(), {model_path!r}, {n_prompt + n_skip + n_gen + 1})
p = synth.prompt_ids({n_prompt}, seed=1234)
tok = 0
for pos in range({n_prompt}):
    tok = e.forward(int(p[pos]), pos)
for pos in range({n_prompt}, {n_prompt + n_skip}):
    tok = e.forward(tok, pos)
t0 = time.perf_counter()
for pos in range({n_prompt + n_skip}, {n_prompt + n_skip + n_gen}):
    tok = e.forward(tok, pos)
dt = time.perf_counter() - t0
print(json.dumps({{"kind": kind, "tok_s": {n_gen} / dt}}))
"""
    env = dict(os.environ, OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="close")
    try:
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
        d = json.loads(r.stdout.strip().splitlines()[-1])
    except Exception as ex:  # noqa: BLE001
        return {"value": None, "unit": "tokens/s", "cores": cores, "kind": "reference", "sample": f"failed: {ex}"}
    return {"value": round(d["tok_s"], 3), "unit": "tokens/s", "cores": cores, "kind": d["kind"],
            "sample": f"{n_prompt}-token prompt, {n_skip} untimed greedy tokens, then {n_gen} greedy tokens timed "
                      f"(positions {n_prompt + n_skip}..{n_prompt + n_skip + n_gen - 1}, decode only), "
                      f"OMP_NUM_THREADS={cores}"}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU implementation on rank 0's host cores."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    from mcpm import spec, synth
    tp = args.config == 4   # all-Q8_0: the reference build cannot run it, so its C restatement is timed
    path = synth.ensure_model("q8_0" if tp else "q4_k_m", 0)
    # the GPU arm's workload: its prompt, its warm-up tokens untimed, its timed steps (the
    # all-Q8_0 restatement is slower, so its prompt is bounded to keep the run within minutes)
    n_prompt = 32 if tp else args.prompt
    steps = args.steps
    cb = cpu_baseline(path, n_prompt=n_prompt, n_gen=steps, port_only=tp, n_skip=args.warmup)
    value = cb["value"]
    batch = args.config == 3   # the reference decodes one sequence at a time: its batch rate is its batch-1 rate
    if tp:
        line = {"impl": "reference", "metric": TP_METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / value, 3) if value else None,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
                "data": "synthetic",
                "config": {"workload": "config4: all-Q8_0 MiniCPM5-2B greedy decode, batch 1, CPU restatement "
                                       "(the reference build cannot run an all-Q8_0 model)",
                           "prompt": n_prompt, "parallelism": "openmp"},
                "cpu_baseline": cb,
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    line = {"impl": "reference", "metric": BATCH_METRIC if batch else METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 / value, 3) if value else None, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / fp32", "data": "synthetic",
            "config": ({"workload": "config3: 64 sequences decoded one at a time, CPU reference", "prompt": n_prompt,
                        "parallelism": "openmp"} if batch else
                       {"workload": "config0: MiniCPM5-2B Q4_K_M greedy decode, batch 1 per GPU", "prompt": n_prompt,
                        "positions": [n_prompt + args.warmup, n_prompt + args.warmup + steps - 1],
                        "parallelism": "openmp (the reference CPU build on the host cores)"}),
            "cpu_baseline": cb,
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


GEMV_CASES = [   # (name, ggml type, rows, cols): the config-1 shapes (rows x cols = out x in)
    ("o_proj 2048x2048", 12, 2048, 2048), ("k/v 256x2048", 12, 256, 2048), ("v 256x2048", 14, 256, 2048),
    ("gate+up 12288x2048", 12, 12288, 2048), ("down 2048x6144", 12, 2048, 6144), ("down 2048x6144", 14, 2048, 6144),
    ("lm_head 130560x2048", 14, 130560, 2048),
    ("o_proj 2048x2048", 8, 2048, 2048), ("k/v 256x2048", 8, 256, 2048), ("gate+up 12288x2048", 8, 12288, 2048),
    ("down 2048x6144", 8, 2048, 6144), ("lm_head 130560x2048", 8, 130560, 2048),
]
TYPE_NAME = {8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}


def run_gemv_sweep(args):
    """Config 1: each GEMV alone, weights rotated over enough copies that every launch reads
    them from HBM (> 256 MB in flight), timed with CUDA events; the reference build's GEMV on
    the host cores is timed on the same matrix for comparison (fp32 activations for Q8_0,
    Q8_K activations otherwise, as the reference's matmul / matmul_q8k)."""
    import numpy as np
    import torch
    from mcpm import engine as E, spec, synth
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    torch.cuda.set_device(0)
    peak, peak_kind = measured_peaks()
    ref = O.Ref() if (O.have_ref() and not args.no_cpu_baseline) else None
    orc = O.Oracle()
    cases = [(n, t, r, c, o) for n, t, r, c in GEMV_CASES for o in ((None,) if t == 8 else ("block", "avx2"))]
    for name, t, rows, cols, order in cases:
        if args.case and args.case not in f"{name} {TYPE_NAME[t]}" + (f" {order}" if order else ""):
            continue
        w = synth.tensor_bytes(spec.TensorInfo("w", t, (cols, rows)), np.random.Generator(np.random.PCG64([rows, cols, t])))
        nbytes = w.size
        copies = max(1, -(-(256 << 20) // nbytes))
        wd = torch.from_numpy(w).cuda().repeat(copies)
        x = np.random.default_rng(cols).normal(0, 1, cols).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        xq = orc.quantize_q8k(x, 0, 1)
        xqd = torch.from_numpy(xq.view(np.uint8).copy()).cuda()
        yd = torch.zeros(rows, dtype=torch.float32, device="cuda")

        def launch(i, stream=0):
            ptr = wd.data_ptr() + (i % copies) * nbytes
            if t == 8:
                E.gemv_q8_0(ptr, xd.data_ptr(), yd.data_ptr(), rows, cols, stream)
            elif order == "block":   # the decode kernel's order (engine default)
                E.gemv_q8k_block(t, ptr, xqd.data_ptr(), yd.data_ptr(), rows, cols, stream)
            else:                    # the reference's eight-lane AVX2 order
                E.gemv_q8k(t, ptr, xqd.data_ptr(), yd.data_ptr(), rows, cols, stream)
        for i in range(max(3, args.warmup)):
            launch(i)
        torch.cuda.synchronize()
        # the timed launches replay as one CUDA graph, so host launch cost does not show
        reps = max(20, min(args.steps, 200))
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for i in range(reps):
                launch(i, side.cuda_stream)
        graph.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):   # replay() launches on the current stream
            ev0.record()
            graph.replay()
            ev1.record()
        ev1.synchronize()
        ms = ev0.elapsed_time(ev1) / reps
        del graph
        act = cols * 4 if t == 8 else (cols // 256) * 292
        gbs = (nbytes + act + rows * 4) / (ms * 1e-3) / 1e9
        cpu = None
        if ref is not None:
            nrep = 3 if nbytes > (64 << 20) else 20
            t0 = time.perf_counter()
            for _ in range(nrep):
                if t == 8:
                    ref.gemv_f32(8, w, x, rows, cols)
                else:
                    ref.gemv_q8k(t, w, xq, rows, cols)
            cpu_ms = (time.perf_counter() - t0) / nrep * 1e3
            cpu = {"value": round(nbytes / (cpu_ms * 1e-3) / 1e9, 2), "unit": "GB/s", "cores": ref.threads(),
                   "kind": "reference", "sample": f"{nrep} calls of the reference build's GEMV on the same matrix"}
        print(json.dumps({
            "metric": "GEMV weight-stream GB/s (batch 1)", "config": {"workload": "config1", "case": name,
                                                                      "type": TYPE_NAME[t], "rows": rows, "cols": cols,
                                                                      "order": order or "q8_0 (reference order)",
                                                                      "l2": f"{copies} weight copies rotated", "timing": "CUDA graph of repeated launches"},
            "value": round(gbs, 1), "unit": "GB/s", "us_per_launch": round(ms * 1e3, 2), "higher_is_better": True,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_kind": peak_kind},
            "cpu_baseline": cpu}), flush=True)
        del wd


BATCH_TOTAL = 64
BATCH_PROMPT = 256
BATCH_METRIC = "decode tokens/s (64 sequences, MiniCPM5-2B Q4_K_M shape)"
BATCH_LAUNCHES_PER_STEP = 1 + 10 * 42 + 2   # embed; per layer 4 GEMMs + 6 small kernels; LM GEMM, argmax


def run_batch(args, rank, world, local):
    """Config 3: 64 independent sequences split data-parallel over the ranks (64/N each, no
    collective in the data path).  Every sequence has its own seeded 256-token prompt; the
    prefill runs as batched steps (untimed), then W warm-up and K timed steps, each step one
    greedy token for every sequence, chained on the device.  `value` = 64 * K tokens over the
    slowest rank's device time (strong scaling: the total work is fixed)."""
    import numpy as np
    import torch
    from mcpm import engine as E, spec, synth
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        pg = dist
    total = args.seqs
    n = total // world
    n_prompt = BATCH_PROMPT if args.prompt == PROMPT else args.prompt   # --prompt: a smaller case for profiling
    path = synth.ensure_model("q4_k_m", 0)
    if pg:
        pg.barrier()
    max_seq = n_prompt + args.warmup + args.steps + 80
    eng = E.MiniCPM5Engine(device=local, max_seq=64,
                           batch_gemm=E.GEMM_TCGEN05 if args.batch_gemm == "tcgen05" else E.GEMM_MMA)
    if not eng.load_model(path):
        raise SystemExit("load_model failed")
    eng.batch_init(n, max_seq)
    stream = torch.cuda.ExternalStream(eng.stream)
    prompts = np.stack([synth.prompt_ids(n_prompt, seed=5000 + rank * n + i) for i in range(n)]).astype(np.int32)
    for pos in range(n_prompt):   # prefill (untimed)
        eng.batch_step_async(prompts[:, pos], np.full(n, pos, np.int32))
    for _ in range(args.warmup):
        eng.batch_step_async()
    eng.batch_read()
    first_pos = n_prompt + args.warmup
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local) if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        eng.batch_step_async()
    ev1.record(stream)
    ev1.synchronize()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.stop() if clk else None
    eng.batch_read()
    ms_max = max_over_ranks(ms, pg)
    # e2e: host tokens in, greedy tokens out, every step
    e2e_steps = min(args.steps, 32)
    am, _ = eng.batch_read()
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        am, _ = eng.batch_step(am)
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg)
    if rank == 0:
        wbytes = spec.weight_bytes_per_token(spec.q4km_table())["total"]
        kv = spec.KV_BYTES_PER_POSITION
        mean_pos = first_pos + (args.steps - 1) / 2 + 1
        bytes_per_step = wbytes + n * kv * mean_pos   # per GPU: the weights once, each sequence's K/V
        peak, peak_kind = measured_peaks()
        per_step_ms = ms_max / args.steps
        achieved = bytes_per_step / (per_step_ms * 1e-3) / 1e9
        value = total * args.steps / (ms_max * 1e-3)
        cb = None if args.no_cpu_baseline else cpu_baseline(path)
        if cb is not None:
            cb["sample"] += "; the reference decodes one sequence at a time, so its batch rate is its batch-1 rate"
        line = {
            "metric": BATCH_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": ("int8 tcgen05" if args.batch_gemm == "tcgen05" else "int8 mma") + " / fp32",
            "data": "synthetic (seeded random-init GGUF, Q4_K_M layout)",
            "config": {"workload": f"config3: MiniCPM5-2B Q4_K_M batched greedy decode, {total} sequences",
                       "sequences_per_gpu": n, "prompt": n_prompt, "gemm": args.batch_gemm,
                       "positions": [first_pos, first_pos + args.steps - 1],
                       "parallelism": f"dp{world} (sequences split over GPUs)",
                       "l2": "inputs larger than L2 (1.41 GB of weights + K/V per step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "kernel": "batched step (k_b_gemm + attention units)",
                         "algorithmic_bytes_per_step": int(bytes_per_step)},
            "cpu_baseline": cb,
            "e2e": {"value": round(total * e2e_steps / e2e_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 4 * n},
            "gpu_launches": BATCH_LAUNCHES_PER_STEP * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()

TP_METRIC = "decode tokens/s (batch 1, all-Q8_0 MiniCPM5-2B shape, tensor parallel over the GPUs)"
TP_PROMPT = 512
TP_LAUNCHES_PER_STEP = 6 * 42 + 2   # per layer QKV, attention units, combine, o_proj, Gate+Up, down; LM head, pick


def tp_bytes_per_step(world: int, n_pos: float) -> int:
    """Weight + KV bytes one rank reads per token (its shards, the replicated norms and one
    embedding row, the K/V rows of its KV head(s) at n_pos positions)."""
    from mcpm import spec
    rb = spec.N_EMBD // 32 * 34
    hq, nf, ng = spec.N_HEAD // world, spec.N_FF // world, (2 if world == 1 else 1)
    nq, nkv = hq * spec.HEAD_DIM, ng * spec.HEAD_DIM
    layer = ((nq + 2 * nkv) * rb + spec.N_EMBD * (hq * spec.HEAD_DIM // 32 * 34) + 2 * nf * rb
             + spec.N_EMBD * (nf // 32 * 34) + 2 * 4 * spec.N_EMBD)
    kv = 2 * nkv * 4 * n_pos
    return int(spec.N_LAYER * (layer + kv) + spec.N_VOCAB // world * rb + 4 * spec.N_EMBD + rb)


def run_tp(args, rank, world, local):
    """Config 4: one all-Q8_0 sequence decoded tensor-parallel over the ranks (every rank
    holds 1/N of each matrix; the o_proj and down partial sums are exchanged after every
    layer).  Seeded 512-token prompt (untimed, token by token as the reference does), W
    warm-up tokens, then K timed greedy tokens chained on the device.  `value` = K tokens over
    the slowest rank's device time (strong scaling: the same sequence at every N)."""
    import datetime
    import numpy as np
    import torch
    from mcpm import synth
    from mcpm.tp import TPEngine
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))   # setup exchange, timing max
        pg = dist
    n_prompt = TP_PROMPT if args.prompt == PROMPT else args.prompt
    path = synth.ensure_model("q8_0", 0)
    if pg:
        pg.barrier()
    max_seq = n_prompt + args.warmup + args.steps + 80 + 64 + 8
    eng = TPEngine(local, rank, world, max_seq, args.comm)
    eng.load(path)
    eng.connect(pg)
    prompt = synth.prompt_ids(n_prompt, seed=2468)
    tok = 0
    for pos in range(n_prompt):   # prefill (untimed)
        tok, _ = eng.forward(int(prompt[pos]), pos, logits=False)
    eng.generate_async(args.warmup)
    eng.sync()
    first_pos = n_prompt + args.warmup
    if pg:
        pg.barrier()
    stream = torch.cuda.ExternalStream(eng.stream)
    torch.cuda.synchronize()
    clk = ClockSampler(local) if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    eng.generate_async(args.steps)
    ev1.record(stream)
    ev1.synchronize()
    eng.sync()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.stop() if clk else None
    ms_max = max_over_ranks(ms, pg, device="cpu")
    toks = eng.read_tokens(first_pos, args.steps)
    # per-token exchange cost: a kernel-by-kernel run with timing of the collectives / waits
    prof_steps = min(16, args.steps)
    ms_tok_eager, ms_comm = eng.profile(prof_steps)
    ms_comm_max = max_over_ranks(ms_comm, pg, device="cpu")
    ms_tok_eager = max_over_ranks(ms_tok_eager, pg, device="cpu")
    # e2e: the C-ABI call with host buffers (token in, greedy token out), synchronous per step
    e2e_steps = min(args.steps, 64)
    pos = first_pos + args.steps + prof_steps
    tok = int(eng.read_tokens(pos - 1, 1)[0])
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok, _ = eng.forward(tok, pos, logits=False)
        pos += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg, device="cpu")
    same = True
    if pg:   # every rank must have produced the same greedy stream
        digest = torch.tensor([int(np.sum(toks.astype(np.int64) * np.arange(1, len(toks) + 1)))], dtype=torch.int64)
        lo, hi = digest.clone(), digest.clone()
        pg.all_reduce(lo, op=pg.ReduceOp.MIN)
        pg.all_reduce(hi, op=pg.ReduceOp.MAX)
        same = bool(lo.item() == hi.item())
    if rank == 0:
        mean_pos = first_pos + (args.steps - 1) / 2 + 1
        bytes_per_step = tp_bytes_per_step(world, mean_pos)
        peak, peak_kind = measured_peaks()
        per_step_ms = ms_max / args.steps
        achieved = bytes_per_step / (per_step_ms * 1e-3) / 1e9
        value = args.steps / (ms_max * 1e-3)
        cb = None if (args.no_cpu_baseline or world > 1) else cpu_baseline(path, port_only=True)
        if cb is not None:
            cb["sample"] += "; C restatement (the reference build cannot run an all-Q8_0 model)"
        line = {
            "metric": TP_METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32 (Q8_0 weights)",
            "data": "synthetic (seeded random-init all-Q8_0 GGUF)",
            "config": {"workload": "config4: all-Q8_0 MiniCPM5-2B greedy decode, batch 1, tensor parallel",
                       "prompt": n_prompt, "positions": [first_pos, first_pos + args.steps - 1],
                       "parallelism": f"tp{world}", "exchange": args.comm,
                       "l2": f"inputs larger than L2 ({bytes_per_step / 1e6:.0f} MB per GPU per token)"},
            "per_token_latency_ms": round(per_step_ms, 4),
            "comm": {"ms_per_token": round(ms_comm_max, 4), "eager_ms_per_token": round(ms_tok_eager, 4),
                     "fraction": round(ms_comm_max / ms_tok_eager, 4) if ms_tok_eager else None,
                     "how": ("device time of the NCCL collectives" if args.comm == "nccl" else
                             "time the consuming kernels waited for the exchanged partial sums") +
                            f" over {prof_steps} kernel-by-kernel steps, max over ranks",
                     "ranks_agree": same},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "kernel": "token sequence (k_tp_gemv, attention)",
                         "algorithmic_bytes_per_step_per_gpu": bytes_per_step},
            "cpu_baseline": cb,
            "e2e": {"value": round(e2e_steps / e2e_s, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 32},
            "gpu_launches": TP_LAUNCHES_PER_STEP * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()   # no rank frees its receive buffer while a peer may still store into it
    eng.close()
    if pg:
        pg.destroy_process_group()


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.config == 1:
        if rank == 0:
            run_gemv_sweep(args)
        return
    if args.config == 3:
        run_batch(args, rank, world, local)
        return
    if args.config == 4:
        run_tp(args, rank, world, local)
        return
    if args.config == 2 and args.prompt == PROMPT:   # config 2: 8192-position context
        args.prompt = 8192
        if args.steps == 256:
            args.steps = 128
    import numpy as np
    import torch
    from mcpm import engine as E, spec, synth

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        pg = dist
    path = synth.ensure_model("q4_k_m", 0)
    if pg:
        pg.barrier()
    max_seq = args.prompt + args.warmup + args.steps + 80
    kv16 = args.kv_type == "f16"
    eng = E.MiniCPM5Engine(device=local, max_seq=max_seq, kv_type=E.KV_F16 if kv16 else E.KV_F32)
    if not eng.load_model(path):
        raise SystemExit("load_model failed")
    stream = torch.cuda.ExternalStream(eng.stream)
    prompt = synth.prompt_ids(args.prompt, seed=1234 + rank)
    # prefill: batched steps of up to 64 positions (mcpm_prefill), timed apart from decode
    eng.prefill(prompt[:1], 0, logits=False)   # first call allocates the row buffers
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.prefill(prompt, 0, logits=False)
    prefill_s = time.perf_counter() - t0
    pos = args.prompt
    for _ in range(args.warmup):
        eng.forward_async(-1, pos)
        pos += 1
    eng.sync()
    first_pos = pos
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local) if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        eng.forward_async(-1, pos)
        pos += 1
    ev1.record(stream)
    ev1.synchronize()
    eng.sync()
    ms = ev0.elapsed_time(ev1)
    clocks = clk.stop() if clk else None
    ms_max = max_over_ranks(ms, pg)

    # e2e: the reference-facing call with host buffers (token in, argmax out), synchronous per step
    e2e_steps = min(args.steps, 64)
    tok = eng.forward_greedy(-1, pos)
    pos += 1
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok = eng.forward_greedy(tok, pos)
        pos += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0, pg)

    if rank == 0:
        tensors = spec.q4km_table()
        wbytes = spec.weight_bytes_per_token(tensors)["total"]
        kv = spec.KV_BYTES_PER_POSITION // (2 if kv16 else 1)
        n_pos = [p + 1 for p in range(first_pos, first_pos + args.steps)]
        bytes_per_tok = wbytes + kv * (sum(n_pos) / len(n_pos))
        peak, peak_kind = measured_peaks()
        per_launch_ms = ms_max / args.steps
        achieved = bytes_per_tok / (per_launch_ms * 1e-3) / 1e9
        value = world * args.steps / (ms_max * 1e-3)
        # config 2: the reference's CPU prefill of 8192 positions alone takes minutes; no CPU line
        cb = None if (args.no_cpu_baseline or args.config == 2 or kv16) else cpu_baseline(
            path, n_prompt=args.prompt, n_gen=args.steps, n_skip=args.warmup)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_launch_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / fp32",
            "data": "synthetic (seeded random-init GGUF, Q4_K_M layout)",
            "config": {"workload": ("config2: MiniCPM5-2B Q4_K_M greedy decode after a long prefill, batch 1 per GPU"
                                    if args.config == 2 else
                                    "config0: MiniCPM5-2B Q4_K_M greedy decode, batch 1 per GPU"),
                       "prompt": args.prompt, "positions": [first_pos, first_pos + args.steps - 1],
                       "parallelism": f"dp{world} (independent sequences)", "kv_cache": args.kv_type,
                       "l2": "inputs larger than L2 (1.41 GB of weights per token)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None if kv16 else profiled_traffic(sum(n_pos) / len(n_pos)),
                         "peak_kind": peak_kind, "kernel": "k_decode",
                         "algorithmic_bytes_per_launch": int(bytes_per_tok)},
            "cpu_baseline": cb,
            "e2e": {"value": round(world * e2e_steps / e2e_s, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 16},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "prefill": {"tokens": args.prompt, "ms": round(prefill_s * 1e3, 2),
                        "tokens_per_s": round(args.prompt / prefill_s, 1),
                        "how": "mcpm_prefill: batched steps of up to 64 positions sharing the KV cache, host "
                               "wall clock around the synchronous call (token ids in, last logits kept on the device)"},
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
