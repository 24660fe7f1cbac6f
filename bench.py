"""Decode benchmark of the B200 quantized-matmul path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (the configuration the headline metric is quoted on): a
Qwen3-1.7B-shaped model with Q8_0 weights (random-init N(0, 0.02) from a
seed, generated on the device; synthetic, there is no checkpoint), a 512-token
seeded prompt prefilled first (untimed), then greedy decode at batch 1.
One step = one decode token (TransformerGraph.forward + argmax).  W warm-up
steps, then K timed steps; each step streams 1.83 GB of weights, far more
than the 126 MB L2, so no L2 flush is needed between steps.

Printed JSON line (rank 0):
  value      decode tok/s, device-resident, CUDA events on the launching stream
  e2e        the same metric through the C ABI call a host caller makes per
             token (brew_model_forward: token+position H2D, argmax D2H)
  roofline   the decode matvec kernel timed alone (gate matrices of all 28
             layers in rotation, 375 MB) against the measured HBM copy peak
  cpu_baseline  the oracle (CPU restatement of the reference's Java path,
             row-parallel over all host cores) on a bounded sample

N > 1: one independent model replica per GPU (decode at batch 1 does not
shard without a per-layer exchange); value = tokens of all ranks / max time.

--impl reference: times the CPU restatement of the reference path (the Java
reference cannot run here: no JDK) on the same config and metric.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from brewference_b200 import config as C  # noqa: E402

METRIC = "decode tok/s (bs1, 1/2/4/8 B200); quant matvec HBM GB/s vs peak"
SEED = 1234
PROMPT_LEN = 512


def workload_cfg():
    return C.qwen3_1_7b()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init(n_gpus):
    import torch
    import torch.distributed as dist
    if n_gpus <= 1 or "RANK" not in os.environ:
        return 0, 1, None
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    import datetime
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, dist


def max_over_ranks(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    import torch
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


# --------------------------------------------------------------------------
# CPU baseline: the oracle (CPU restatement of the reference path)
# --------------------------------------------------------------------------
def cpu_decode_rate(cfg, n_tokens: int, position: int):
    """Times `n_tokens` decode forwards of the oracle at positions near
    `position` (cost is that of a decode step at that context length; the
    cache contents do not change the work).  Returns (tok/s, threads, seconds)."""
    import oracle
    threads = oracle.get_threads()
    om = oracle.OracleModel(cfg, SEED)
    om.forward(1, position)            # warm caches / page in weights
    t0 = time.perf_counter()
    for i in range(n_tokens):
        om.forward(1 + i, position + 1 + i)
    dt = time.perf_counter() - t0
    om.close()
    return n_tokens / dt, threads, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = workload_cfg()
    # each step is one oracle decode token; bound the run to a few minutes
    per_tok = None
    steps = args.steps
    import oracle
    t0 = time.perf_counter()
    om = oracle.OracleModel(cfg, SEED)
    synth_s = time.perf_counter() - t0
    for i in range(max(1, min(args.warmup, 1))):
        ts = time.perf_counter()
        om.forward(1, PROMPT_LEN + i)
        per_tok = time.perf_counter() - ts
    budget = 150.0
    steps = max(3, min(steps, int(budget / max(per_tok, 1e-3))))
    t0 = time.perf_counter()
    for i in range(steps):
        om.forward(2 + i, PROMPT_LEN + 1 + i)
    dt = time.perf_counter() - t0
    v = steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": steps,
        "warmup": args.warmup, "ms_per_step": 1000 * dt / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-init weights, seeded token ids)",
        "config": {"workload": f"{cfg.name} Q8_0 decode at batch 1, context {PROMPT_LEN}+",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": oracle.get_threads(), "kind": "port",
                         "sample": f"{steps} decode tokens at positions {PROMPT_LEN + 1}..{PROMPT_LEN + steps} "
                                   f"(C restatement of the reference Java path, row-parallel; no JDK on this host)"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": f"weights synthesized in {synth_s:.1f}s (untimed)",
    }
    om.close()
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------
def kernel_roofline(dm, cfg, iters: int):
    """Times the decode matvec kernel alone: the gate matrices of all layers
    in rotation (inputs far larger than L2), batch 1, CUDA events on the
    launching stream.  Returns per-launch algorithmic bytes and mean ms."""
    import torch
    from brewference_b200.api import Linear
    K, Nr = cfg.dim, cfg.hidden_dim
    w = dm.tensor(C.W_GATE)
    x = torch.randn(K, device="cuda", dtype=torch.float32)
    y = torch.empty(Nr, device="cuda", dtype=torch.float32)
    prep = torch.empty(Linear.prep_bytes(K, 1) + 256, dtype=torch.uint8, device="cuda")
    pp = (prep.data_ptr() + 15) // 16 * 16
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    s = st.cuda_stream
    Linear.prepare_input_device(x.data_ptr(), K, 1, pp, s)
    for l in range(4):
        Linear.matmul_prepared_device(y.data_ptr(), pp, w, l * K * Nr, K, Nr, 1, s)
    torch.cuda.synchronize()
    # the launches are captured in a CUDA graph so host launch cost does not
    # enter the kernel time
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            Linear.matmul_prepared_device(y.data_ptr(), pp, w, (i % cfg.n_layers) * K * Nr, K, Nr, 1,
                                          torch.cuda.current_stream().cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    wbytes = Nr * K // 32 * 34
    alg = wbytes + 4 * K + 4 * Nr
    return alg, ms, wbytes


def run_gpu(args):
    import torch
    from brewference_b200 import _native as N
    from brewference_b200.api import DeviceModel

    rank, world, dist = dist_init(args.gpus)
    dev = torch.cuda.current_device() if world > 1 else 0
    torch.cuda.set_device(dev)
    N.init(dev)
    cfg = workload_cfg()
    t0 = time.perf_counter()
    dm = DeviceModel.synthesize(cfg, SEED)
    synth_s = time.perf_counter() - t0
    if args.profile_decode:
        # a short prompt, then a few decode steps (profiling entry: the decode
        # kernel of the steps after the prompt)
        rng = np.random.default_rng(SEED)
        prompt = rng.integers(0, cfg.vocab_size, args.prompt_len).astype(np.int32)
        dm.prefill(prompt)
        toks = dm.decode(args.steps)
        print(json.dumps({"profile_decode": True, "prompt": args.prompt_len, "steps": args.steps, "tokens": toks[:4]}))
        dm.close()
        return 0
    if args.kernel_only:
        # the decode matvec alone (profiling entry: a few launches, no decode)
        alg, kms, _ = kernel_roofline(dm, cfg, iters=args.steps)
        peak, peak_kind = measured_peaks()
        print(json.dumps({"kernel": "mv_kernel Q8_0 batch 1, 6144x2048", "ms_per_launch": kms,
                          "GBps": alg / (kms / 1000.0) / 1e9, "peak": peak, "peak_kind": peak_kind}), flush=True)
        dm.close()
        return 0
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, cfg.vocab_size, args.prompt_len).astype(np.int32)
    # a dedicated stream: the library enqueues the decode on it and the CUDA
    # events below are recorded on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    s = stream.cuda_stream
    dm.prefill(prompt, s)
    dm.decode(args.warmup, s, want_tokens=False)
    barrier(dist)

    clocks = ClockSampler(dev)
    clocks.start()
    k0 = N.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    e0.record(stream)
    dm.decode(args.steps, s, want_tokens=False)
    e1.record(stream)
    barrier(dist)
    launches = N.kernel_launches() - k0
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(dist, ms)
    value = world * args.steps / (ms_max / 1000.0)

    # end to end through the per-token C ABI call with host buffers
    e2e_steps = min(args.steps, 64)
    pos0 = args.prompt_len + args.warmup + args.steps
    tok = np.array([int(prompt[-1])], np.int32)
    torch.cuda.synchronize()
    barrier(dist)
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        _, am = dm.forward(tok, np.array([pos0 + i], np.int32), want_logits=False)
        tok = am
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(dist, e2e_s)
    e2e = world * e2e_steps / e2e_s

    # roofline of the dominant kernel (decode matvec) timed alone
    alg, kms, wbytes = kernel_roofline(dm, cfg, iters=112)
    peak, peak_kind = measured_peaks()
    achieved = alg / (kms / 1000.0) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init N(0,0.02) weights quantized to Q8_0 on the device, seeded prompt ids)",
        "config": {"workload": f"{cfg.name} Q8_0 greedy decode at batch 1 after a {args.prompt_len}-token prompt",
                   "model": cfg.name, "global_batch": world, "seq_len": cfg.seq_len,
                   "positions": [args.prompt_len + args.warmup, args.prompt_len + args.warmup + args.steps - 1],
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (1.83 GB of weights per step vs 126 MB L2)"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
                "call": "brew_model_forward per token, host token/position in, host argmax out"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": "mv_kernel Q8_0 batch 1, gate matrix 6144x2048 (13.37 MB), layers rotated",
                     "bytes_per_launch": alg, "ms_per_launch": kms},
        "weight_stream": {"bytes_per_step": cfg.decode_weight_bytes(),
                          "GBps": cfg.decode_weight_bytes() / (ms_max / args.steps / 1000.0) / 1e9},
        "clocks": clk,
        "setup_s": {"synthesize": round(synth_s, 2)},
    }
    if rank == 0 and not args.no_cpu_baseline:
        tps, thr, dt = cpu_decode_rate(cfg, args.cpu_tokens, args.prompt_len)
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": thr, "kind": "port",
                                "sample": f"{args.cpu_tokens} decode tokens at positions {args.prompt_len + 1}.."
                                          f"{args.prompt_len + args.cpu_tokens} of the same model, oracle (C "
                                          f"restatement of the reference Java path), {dt:.1f}s"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dm.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt-len", type=int, default=PROMPT_LEN)
    ap.add_argument("--cpu-tokens", type=int, default=48)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel-only", action="store_true", help="time the decode matvec kernel alone")
    ap.add_argument("--profile-decode", action="store_true", help="prompt + a few decode steps, no timing")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
