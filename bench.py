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
             token (brew_model_forward: token+position in, argmax id out)
  roofline   the dominant kernel, the persistent decode kernel (one launch
             per token): weight + KV bytes per step over its time, against
             the measured HBM copy peak; `traffic` is the DRAM bytes per
             launch from the committed ncu summary of the same kernel
  matvec_sweep  the packed-block matvec kernel alone on the decode shapes,
             Q8_0 and Q4_0, batch 1 and 8, layers rotated (inputs > L2)
  cpu_baseline  the oracle (CPU restatement of the reference's Java path,
             row-parallel over all host cores) on a bounded sample

N > 1: one independent model replica per GPU (decode at batch 1 does not
shard without a per-layer exchange); value = tokens of all ranks / max time.

workloads (sub-records, N = 1): the other named single-GPU workloads on the
same persistent decode kernel, each with its roofline fraction and an oracle
CPU sample: SmolLM2-135M-shaped (32-token prompt, 128 decode tokens) and
Gemma-3-1B-shaped (Q4_0 layers, Q8_0 embedding; 1024-token prompt, 256 decode
tokens).

tp (sub-record, every N including 1): the Qwen2.5-7B-shaped K-quant config
decoding 32 sequences, every matrix row-sharded over the N ranks, each
projection's slices gathered by peer stores into every rank's tagged slots
over NVLink (strong scaling), with a bit-for-bit check of the sharded
first-step logits against the unsharded model on one GPU (N > 1).

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


def q4_cfg(cfg):
    """The same shapes with Q4_0 layer matrices and a Q4_0 classifier (the
    Q4_0 half of the matvec sweep)."""
    q4 = C.TYPE_Q4_0
    return cfg.replace(type_embed=q4, type_output=q4, type_q=q4, type_k=q4, type_v=q4, type_o=q4, type_gate=q4,
                       type_up=q4, type_down=q4)


TRAFFIC_PROFILE = "decode_kernel_qwen3-1.7b_q8_0.md"


def measured_peaks(kind: str = "hbm_gbs"):
    """(peak, "measured" | "fallback"): HBM copy GB/s (`hbm_gbs`) or dense
    bf16 TFLOP/s (`bf16_tflops`) from MEASURED_PEAKS.json, else the
    fallback figures."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if kind in d:
            return float(d[kind]), "measured"
    return (6650.0 if kind == "hbm_gbs" else 1590.0), "fallback"


class ClockSampler:
    """SM clocks and throttle reasons sampled every 20 ms during the timed
    region, through NVML (nvidia-smi as the fallback).  Reads only."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, torch_device: int):
        self.dev = torch_device
        self.samples, self.reasons, self.smax = [], set(), None
        self.stop_ev = threading.Event()
        self.thread = None
        self.nvml = None
        self.handle = None

    def _open(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        self.nvml = pynvml
        prop = torch.cuda.get_device_properties(self.dev)
        bus = "%08x:%02x:%02x.0" % (getattr(prop, "pci_domain_id", 0), prop.pci_bus_id, prop.pci_device_id)
        self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))

    def _reasons(self):
        n = self.nvml
        f = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(f(self.handle))

    def _run(self):
        n = self.nvml
        while not self.stop_ev.is_set():
            try:
                self.samples.append(float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)))
                r = self._reasons()
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:   # noqa: BLE001 - sampling must not break the benchmark
                pass
            self.stop_ev.wait(0.02)

    def start(self):
        try:
            self._open()
        except Exception as e:   # noqa: BLE001
            self.nvml = None
            self.err = str(e)
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def stop(self):
        if self.nvml is None:
            return _nvidia_smi_clocks(self.dev)
        self.stop_ev.set()
        self.thread.join(timeout=2)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.smax,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml, 20 ms"}


def _nvidia_smi_clocks(dev: int):
    fields = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        out = subprocess.run(["nvidia-smi", "-i", str(dev), f"--query-gpu={fields}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=10).stdout.strip().split(",")
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        return {"sm_mhz": float(out[0]), "sm_max_mhz": float(out[1]),
                "reasons": [n for n, v in zip(names, out[2:6]) if v.strip().lower() == "active"],
                "samples": 1, "source": "nvidia-smi after the timed region"}
    except Exception:   # noqa: BLE001
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}


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


def named_workloads():
    """The other single-GPU workloads of the benchmarked configurations:
    (model config, prompt tokens, decode tokens, oracle sample tokens)."""
    return [(C.smollm2_135m(), 32, 128, 64), (C.gemma3_1b(), 1024, 256, 12)]


def workload_measure(cfg, plen, n_dec, cpu_tokens, peak, peak_kind, with_cpu=True):
    """One named workload on this GPU: a seeded prompt of `plen` tokens
    prefilled through the batched prefill (token by token where its tiles do
    not fit the shapes), 3 untimed decode steps, then
    `n_dec` greedy decode steps at batch 1 with the tokens fed back on the
    device (brew_session_decode).  CUDA events on the session's stream time
    the prompt and the decode; value = decode tok/s.  The roofline counts the
    packed weight bytes and the K/V rows each step reads.  The CPU baseline
    is the oracle decoding `cpu_tokens` tokens at the same positions on all
    host threads."""
    import torch
    from brewference_b200.api import PREFILL_BATCHED, DeviceModel

    t0 = time.perf_counter()
    dm = DeviceModel.synthesize(cfg, SEED)
    synth_s = time.perf_counter() - t0
    kernels = dm.step_kernels(1)
    mode = "batched"
    try:
        dm.set_prefill(PREFILL_BATCHED)
    except Exception:   # noqa: BLE001 - shapes the tcgen05 prefill does not tile: token by token
        mode = "token by token"
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab_size, plen).astype(np.int32)
    stream = torch.cuda.Stream()
    prev = torch.cuda.current_stream()
    torch.cuda.set_stream(stream)
    s = stream.cuda_stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    k0 = N_launches()
    ev[0].record(stream)
    dm.prefill(prompt, s)
    ev[1].record(stream)
    dm.decode(3, s, want_tokens=False)
    ev[2].record(stream)
    dm.decode(n_dec, s, want_tokens=False)
    ev[3].record(stream)
    stream.synchronize()
    launches = N_launches() - k0
    prefill_ms = ev[0].elapsed_time(ev[1])
    ms = ev[2].elapsed_time(ev[3])
    torch.cuda.set_stream(prev)
    dm.close()
    positions = list(range(plen + 3, plen + 3 + n_dec))
    wbytes = cfg.decode_weight_bytes()
    kvb = kv_bytes_per_step(cfg, positions)
    achieved = (wbytes + kvb) / (ms / n_dec / 1000.0) / 1e9
    rec = {"workload": f"{cfg.name}: {plen}-token seeded prompt ({mode} prefill), then {n_dec} greedy decode "
                       f"tokens at batch 1", "value": n_dec / (ms / 1000.0), "unit": "tok/s",
           "ms_per_step": ms / n_dec, "steps": n_dec, "warmup": 3, "prefill_ms": prefill_ms,
           "prefill_tok_s": plen / (prefill_ms / 1000.0), "kernels_per_step": kernels,
           "gpu_launches": int(launches),
           "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "peak_kind": peak_kind, "weight_bytes": wbytes, "kv_bytes": kvb},
           "l2": f"{wbytes / 1e6:.0f} MB of weights streamed per step vs 126 MB L2 (no flush between steps)",
           "setup_s": {"synthesize": round(synth_s, 2)}}
    if with_cpu:
        tps, thr, dt = cpu_decode_rate(cfg, cpu_tokens, plen)
        rec["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": thr, "kind": "port",
                               "sample": f"{cpu_tokens} decode tokens at positions {plen + 1}..{plen + cpu_tokens}, "
                                         f"oracle (C restatement of the reference Java path), {dt:.1f}s"}
    return rec


def N_launches():
    from brewference_b200 import _native as N
    return N.kernel_launches()


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
def time_matvec(w, K, Nr, layers, batch, iters):
    """Times the packed-block matvec kernel alone on tensor `w` ([layers][Nr][K]),
    rotating over the layers so the inputs exceed L2 (a single matrix larger
    than L2 needs no rotation).  The x records are prepared once; the timed
    launches run from a CUDA graph on a dedicated stream, CUDA events on that
    stream.  Returns (algorithmic bytes per launch, ms per launch)."""
    import torch
    from brewference_b200.api import Linear
    x = torch.randn(batch, K, device="cuda", dtype=torch.float32)
    y = torch.empty(batch, Nr, device="cuda", dtype=torch.float32)
    prep = torch.empty(Linear.prep_bytes(K, batch) + 256, dtype=torch.uint8, device="cuda")
    pp = (prep.data_ptr() + 15) // 16 * 16
    st = torch.cuda.Stream()
    prev = torch.cuda.current_stream()
    torch.cuda.set_stream(st)
    s = st.cuda_stream
    Linear.prepare_input_device(x.data_ptr(), K, batch, pp, s)
    for l in range(min(layers, 4)):
        Linear.matmul_prepared_device(y.data_ptr(), pp, w, l * K * Nr, K, Nr, batch, s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            Linear.matmul_prepared_device(y.data_ptr(), pp, w, (i % layers) * K * Nr, K, Nr, batch,
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
    torch.cuda.set_stream(prev)
    qt = w.type
    eb, bb = C.TYPE_BLOCK[qt]
    wbytes = Nr * K // eb * bb
    alg = wbytes + 4 * K * batch + 4 * Nr * batch
    return alg, ms


def time_gemm(w, K, Nr, layers, T, iters):
    """Times the tcgen05 GEMM through GEMM plans (the matrix repacked once) of
    up to 4 layers of tensor `w`, run in turn from a CUDA graph on a
    dedicated stream with CUDA events on it; x [T][K] and y [T][N] stay on
    the device.  Returns (weight bytes per run, ms per run)."""
    import torch
    from brewference_b200.api import GemmPlan
    nl = min(layers, 4)
    plans = [GemmPlan(w, l * K * Nr, K, Nr) for l in range(nl)]
    x = torch.randn(T, K, device="cuda", dtype=torch.float32)
    y = torch.empty(T, Nr, device="cuda", dtype=torch.float32)
    st = torch.cuda.Stream()
    prev = torch.cuda.current_stream()
    torch.cuda.set_stream(st)
    for pl in plans:   # sizes each plan's scratch before the capture
        pl.run(y.data_ptr(), x.data_ptr(), T, st.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(iters):
            plans[i % nl].run(y.data_ptr(), x.data_ptr(), T, torch.cuda.current_stream().cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    del g
    torch.cuda.set_stream(prev)
    for pl in plans:
        pl.free()
    eb, bb = C.TYPE_BLOCK[w.type]
    return Nr * K // eb * bb, ms


def matvec_sweep(models, cfg, peak):
    """The quant-matvec half of the metric on the decode shapes (W = N x K)
    for each weight type: HBM GB/s of the matvec kernel at batch 1 / 8, and
    the tcgen05 GEMM at 64 / 512 token vectors (weight GB/s and
    TFLOP/s-equivalent of the fp32 product)."""
    bf16_peak = measured_peaks(kind="bf16_tflops")[0]
    shapes = [("2048x2048 (wq)", C.W_Q, cfg.n_heads * cfg.head_size, cfg.dim, cfg.n_layers),
              ("6144x2048 (gate)", C.W_GATE, cfg.hidden_dim, cfg.dim, cfg.n_layers),
              ("2048x6144 (down)", C.W_DOWN, cfg.dim, cfg.hidden_dim, cfg.n_layers),
              ("151936x2048 (classifier)", C.W_OUTPUT, cfg.vocab_size, cfg.dim, 1)]
    out = []
    for tname, dm in models:
        for name, which, Nr, K, layers in shapes:
            w = dm.tensor(which)
            if which == C.W_OUTPUT and tname != C.TYPE_NAMES[w.type]:
                continue   # the tied classifier keeps the embedding's type
            for batch in (1, 8):
                alg, ms = time_matvec(w, K, Nr, layers, batch, iters=56 if layers > 1 else 16)
                gbs = alg / (ms / 1000.0) / 1e9
                out.append({"type": tname, "shape": name, "batch": batch, "path": "matvec", "GBps": round(gbs, 1),
                            "frac": round(gbs / peak, 4), "us": round(ms * 1000.0, 2)})
            for T in (64, 512):
                wb, ms = time_gemm(w, K, Nr, layers, T, iters=24 if layers > 1 else 8)
                tflops = 2.0 * Nr * K * T / (ms / 1000.0) / 1e12
                out.append({"type": tname, "shape": name, "batch": T, "path": "gemm",
                            "GBps": round(wb / (ms / 1000.0) / 1e9, 1), "TFLOPs": round(tflops, 1),
                            "tensor_frac": round(tflops / bf16_peak, 4) if bf16_peak else None,
                            "us": round(ms * 1000.0, 2)})
    return out


def kv_bytes_per_step(cfg, positions):
    """fp32 K/V cache bytes one decode step moves at each position: the rows
    of every earlier position read (K and V, all layers) plus the new row
    written.  Mean over the timed positions."""
    kvd = cfg.n_kv_heads * cfg.head_size
    row = 2 * kvd * 4 * cfg.n_layers
    tot = []
    for p in positions:
        seen = min(p, cfg.sliding_window - 1) if cfg.sliding_window else p
        tot.append(seen * row + row)
    return float(np.mean(tot))


def profiled_traffic(name: str):
    """DRAM bytes per launch recorded in a committed ncu summary
    (line `dram_bytes_per_launch: <n>`), or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for ln in f:
                if ln.strip().startswith("dram_bytes_per_launch:"):
                    return float(ln.split(":", 1)[1].split()[0])
    except (OSError, ValueError, IndexError):
        pass
    return None


def tp_measure(rank, world, dist, dev, steps, warmup, B, plen, check_parity=True, layers=0):
    """Tensor-parallel decode of the Qwen2.5-7B-shaped K-quant config (Q4_K
    attention/FFN, Q6_K down and classifier, QKV bias): every matrix
    row-sharded over the `world` ranks with one NCCL all-gather per
    projection; B concurrent sequences prefilled with seeded prompts
    (untimed), then decode steps fed back on the device.  Returns a dict:
    value = tokens of all B sequences per second (the ranks cooperate on the
    same tokens: strong scaling), ms_per_step (max over ranks), and, with
    check_parity at world > 1, whether rank 0's sharded logits of the first
    step equal those of the same model unsharded on one GPU bit for bit."""
    import ctypes
    import torch
    from brewference_b200 import _native as N
    from brewference_b200.api import Communicator, DeviceModel, comm_unique_id

    cfg = C.qwen25_7b()
    if layers:   # a shallower model of the same shapes (profiler captures)
        cfg = cfg.replace(n_layers=layers)
    box = [comm_unique_id() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(box, src=0)
    comm = Communicator(box[0], world, rank)
    t0 = time.perf_counter()
    dm = DeviceModel.synthesize(cfg, SEED, max_batch=B)
    dm.set_tp(comm)
    synth_s = time.perf_counter() - t0
    rng = np.random.default_rng(SEED)
    prompts = rng.integers(0, cfg.vocab_size, (B, plen)).astype(np.int32)
    # first step from a reset state, logits kept for the parity check
    lg_tp, _ = dm.forward(prompts[:, 0], np.zeros(B, np.int32), want_logits=True)
    dm.reset()
    t0 = time.perf_counter()
    for i in range(plen):
        dm.forward(prompts[:, i], np.full(B, i, np.int32), want_logits=False)
    prefill_s = time.perf_counter() - t0
    stream = torch.cuda.Stream()
    prev = torch.cuda.current_stream()
    torch.cuda.set_stream(stream)
    s = stream.cuda_stream
    tok = torch.from_numpy(prompts[:, -1].copy()).cuda()
    n_pos = warmup + steps
    pos = torch.arange(plen, plen + n_pos, dtype=torch.int32, device="cuda").repeat_interleave(B).view(n_pos, B)
    lib = N.lib()

    def step(k):
        N.check(lib.brew_model_forward_dev(dm.handle, ctypes.c_void_p(tok.data_ptr()),
                                           ctypes.c_void_p(pos[k].data_ptr()), B, None,
                                           ctypes.c_void_p(tok.data_ptr()), ctypes.c_void_p(s)), "forward_dev")

    for k in range(warmup):
        step(k)
    barrier(dist)
    k0 = N.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist)
    e0.record(stream)
    for k in range(warmup, n_pos):
        step(k)
    e1.record(stream)
    barrier(dist)
    launches = N.kernel_launches() - k0
    ms = max_over_ranks(dist, e0.elapsed_time(e1))
    torch.cuda.synchronize()
    torch.cuda.set_stream(prev)
    dm.close()
    parity = None
    parity_rel = None
    if check_parity and world > 1:
        ok = 1.0
        if rank == 0:   # the same seeded model unsharded on this GPU, same first step
            ref = DeviceModel.synthesize(cfg, SEED, max_batch=B)
            lg_1, _ = ref.forward(prompts[:, 0], np.zeros(B, np.int32), want_logits=True)
            ref.close()
            rel = float(max(np.linalg.norm(lg_tp[b].astype(np.float64) - lg_1[b]) /
                            np.linalg.norm(lg_1[b].astype(np.float64)) for b in range(B)))
            same = bool(np.array_equal(np.argmax(lg_tp, axis=1), np.argmax(lg_1, axis=1)))
            ok = 1.0 if (rel <= 1e-5 and same) else 0.0
            parity_rel = rel
        # rank 0 decides: the minimum over ranks (the others report 1)
        parity = bool(1.0 - max_over_ranks(dist, 1.0 - ok) > 0.5) if dist is not None else bool(ok)
    comm.close()
    value = B * steps / (ms / 1000.0)
    return {"value": value, "unit": "tok/s", "ms_per_step": ms / steps, "n_gpus": world, "steps": steps,
            "warmup": warmup, "sequences": B, "prompt_tokens": plen, "gpu_launches": int(launches),
            "collective": ("peer stores of each projection's slice (q|k|v, wo, gate|up, down, logits) into every "
                           "rank's tagged slots over NVLink (CUDA IPC), NCCL all-gather of the argmax keys"
                           if world > 1 and not os.environ.get("BREW_TP_NCCL") else
                           "NCCL all-gather per projection (q|k|v, wo, gate|up, down, logits) + argmax key reduction"),
            "parity": parity,
            "parity_rel_l2": parity_rel,
            "parity_check": "rank 0: first-step logits of the sharded model within 1e-5 relative L2 of the unsharded "
                            "1-GPU model, same argmax for every sequence (bit for bit with BREW_TP_EXACT=1, which "
                            "splits K as on one GPU)"
                            if world > 1 else "single GPU (no sharding)",
            "model": cfg.name, "weight_bytes_per_step": cfg.decode_weight_bytes(),
            "setup_s": {"synthesize": round(synth_s, 2), "prefill": round(prefill_s, 2)}}


def run_tp(args):
    """--tp: the tensor-parallel decode of the Qwen2.5-7B-shaped config as the
    headline line (see tp_measure)."""
    import torch
    from brewference_b200 import _native as N

    rank, world, dist = dist_init(args.gpus)
    dev = torch.cuda.current_device() if world > 1 else 0
    torch.cuda.set_device(dev)
    N.init(dev)
    clocks = ClockSampler(dev)
    clocks.start()
    r = tp_measure(rank, world, dist, dev, args.steps, args.warmup, args.batch, args.prompt_len, layers=args.layers)
    clk = clocks.stop()
    peak, peak_kind = measured_peaks()
    cfg = C.qwen25_7b()
    if args.layers:
        cfg = cfg.replace(n_layers=args.layers)
    per_gpu = cfg.decode_weight_bytes() / world / (r["ms_per_step"] / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32 (K-quant dequant in registers)",
        "data": "synthetic (seeded random-init N(0,0.02) weights quantized to Q4_K/Q6_K on the device, seeded prompts)",
        "config": {"workload": f"{cfg.name} Q4_K/Q6_K decode, {args.batch} concurrent sequences after "
                               f"{args.prompt_len}-token prompts, tensor-parallel over {world} GPU(s)",
                   "model": cfg.name, "global_batch": args.batch, "seq_len": cfg.seq_len,
                   "parallelism": f"tp{world} (row-sharded matrices, peer-store gather per projection)",
                   "l2": "inputs larger than L2 (4.6 GB of weights per step)"},
        "gpu_launches": r["gpu_launches"],
        "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": "per-GPU weight stream of the forward (weight bytes / P per step)"},
        "clocks": clk, "tp_parity": r["parity"], "setup_s": r["setup_s"],
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def decode_trace_table(dm, cfg, reps=3):
    """Runs `reps` traced decode steps and summarises the last along the
    critical path.  Per phase (Q|K|V, attention, wo, gate|up, down), means
    over the layers, in microseconds after the previous phase's last
    producing CTA finished its work (E_prev): when the phase's input landed
    in its first and in its last CTA, the prep time (mean over CTAs), the
    multiply + epilogue time (mean), and the span E - E_prev, where E is the
    phase's own last producing CTA.  The spans add up to the layer time."""
    L, G = cfg.n_layers, None
    slots = 1 + 5 * (5 * L + 1) + 3 * 32
    names = ["qkv", "attn", "wo", "gate_up", "down"]
    for _ in range(reps):
        dm.decode(1)
        T = np.array(dm.trace(), dtype=np.int64).reshape(-1, slots).astype(np.float64) / 1000.0
    G = T.shape[0]
    tiles = [(cfg.q_width + 2 * cfg.kv_dim) // 16, cfg.dim // 16, cfg.hidden_dim // 8, cfg.dim // 16]
    owns = [np.array([(c + 1) * t // G - c * t // G > 0 for c in range(G)]) for t in tiles]
    mph = [0, None, 1, 2, 3]
    rows = {n: [] for n in names}
    prev_e = None
    with np.errstate(all="ignore"):
        import warnings
        warnings.simplefilter("ignore")
        for l in range(L):
            for p in range(5):
                b = 1 + 5 * (5 * l + p)
                st = T[:, b:b + 5]
                act = st[:, 0] > 0 if p == 1 else owns[mph[p]]
                w = st[act]
                e = float(np.max(w[:, 3]))
                if prev_e is not None:
                    land = np.where(w[:, 0] > 0, w[:, 0], np.nan) - prev_e
                    rows[names[p]].append([np.nanmin(land), np.nanmax(land), np.nanmean(w[:, 1] - w[:, 0]),
                                           np.nanmean(w[:, 3] - w[:, 1]), e - prev_e])
                prev_e = e
        b = 1 + 5 * (5 * L)
        cls_end = float(np.max(T[:, b + 3]))
        out = {"step_us": round(float(np.max(T[:, b + 4]) - np.min(T[:, 0])), 2), "layers": L,
               "columns": ["input landed, first CTA", "input landed, last CTA", "prep", "multiply + epilogue",
                           "span"],
               "classifier_span_us": round(cls_end - prev_e, 2), "phases_mean_over_layers": {}}
        per_layer = 0.0
        for n in names:
            a = np.nanmean(np.array(rows[n]), axis=0)
            if n == "attn":   # no prep / multiply stamps: the attention reports its span only
                a[2] = a[3] = np.nan
            out["phases_mean_over_layers"][n] = [None if np.isnan(x) else round(float(x), 2) for x in a]
            per_layer += float(a[4])
        out["layer_us"] = round(per_layer, 2)
    return out


def run_gpu(args):
    import torch
    from brewference_b200 import _native as N
    from brewference_b200.api import PREFILL_BATCHED, DeviceModel

    rank, world, dist = dist_init(args.gpus)
    dev = torch.cuda.current_device() if world > 1 else 0
    torch.cuda.set_device(dev)
    N.init(dev)
    cfg = workload_cfg()
    if args.profile_decode and (args.layers or args.vocab):
        # a smaller model of the same shapes for detailed profiler captures
        cfg = cfg.replace(n_layers=args.layers or cfg.n_layers, vocab_size=args.vocab or cfg.vocab_size)
    t0 = time.perf_counter()
    dm = DeviceModel.synthesize(cfg, SEED)
    synth_s = time.perf_counter() - t0
    if args.profile_decode:
        # a short prompt, then a few decode steps (profiling entry: the decode
        # kernel of the steps after the prompt)
        rng = np.random.default_rng(SEED)
        prompt = rng.integers(0, cfg.vocab_size, args.prompt_len).astype(np.int32)
        if args.batched_prefill:
            dm.set_prefill(PREFILL_BATCHED)
        dm.prefill(prompt)
        toks = dm.decode(args.steps)
        print(json.dumps({"profile_decode": True, "prompt": args.prompt_len, "steps": args.steps, "tokens": toks[:4]}))
        dm.close()
        return 0
    if args.trace_decode:
        # per-phase timing of one decode step from the kernel's %globaltimer
        # stamps (BREW_TRACE=1 must be set before the model is created)
        from brewference_b200.api import PREFILL_BATCHED as _PB
        rng = np.random.default_rng(SEED)
        prompt = rng.integers(0, cfg.vocab_size, args.prompt_len).astype(np.int32)
        dm.set_prefill(_PB)
        dm.prefill(prompt)
        dm.decode(4)
        dm.set_trace(True)
        print(json.dumps(decode_trace_table(dm, cfg)), flush=True)
        dm.close()
        return 0
    if args.kernel_only:
        # the matvec kernel alone (profiling entry: a few launches, no decode)
        alg, kms = time_matvec(dm.tensor(C.W_GATE), cfg.dim, cfg.hidden_dim, cfg.n_layers, 1, iters=args.steps)
        peak, peak_kind = measured_peaks()
        print(json.dumps({"kernel": "mv_kernel Q8_0 batch 1, 6144x2048", "ms_per_launch": kms,
                          "GBps": alg / (kms / 1000.0) / 1e9, "peak": peak, "peak_kind": peak_kind}), flush=True)
        dm.close()
        return 0
    if args.gemm_only:
        # the prefill GEMM alone on the gate|up-sized projection (profiling
        # entry: activation limb split + tcgen05 GEMM per run, layers rotated)
        T = args.gemm_tokens
        wb, ms = time_gemm(dm.tensor(C.W_GATE), cfg.dim, cfg.hidden_dim, cfg.n_layers, T, iters=args.steps)
        tflops = 2.0 * cfg.hidden_dim * cfg.dim * T / (ms / 1000.0) / 1e12
        bf16_peak = measured_peaks(kind="bf16_tflops")[0]
        print(json.dumps({"kernel": f"gemm_limbs_kernel + gemm_q8_kernel, Q8_0 {cfg.hidden_dim}x{cfg.dim}, {T} tokens",
                          "us_per_run": ms * 1000.0, "TFLOPs_equivalent": tflops,
                          "tensor_frac": tflops / bf16_peak if bf16_peak else None,
                          "weight_GBps": wb / (ms / 1000.0) / 1e9}), flush=True)
        dm.close()
        return 0
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, cfg.vocab_size, args.prompt_len).astype(np.int32)
    if args.prefill_only:
        # the batched prefill of the prompt, twice (profiling entry: the
        # second prefill's launches follow the first's one-time set-up)
        dm.set_prefill(PREFILL_BATCHED)
        stream = torch.cuda.Stream()   # the library enqueues the prefill on it
        ms = []
        for _ in range(2):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dm.prefill(prompt, stream.cuda_stream)
            e1.record(stream)
            stream.synchronize()
            ms.append(e0.elapsed_time(e1))
        print(json.dumps({"prefill_only": True, "prompt": args.prompt_len, "ms": ms}), flush=True)
        dm.close()
        return 0
    # a dedicated stream: the library enqueues the decode on it and the CUDA
    # events below are recorded on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    s = stream.cuda_stream
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    dm.prefill(prompt, s)   # token by token, the reference's order (untimed for the decode metric)
    p1.record(stream)
    dm.decode(args.warmup, s, want_tokens=False)
    stream.synchronize()
    prefill_tokens_ms = p0.elapsed_time(p1)
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

    # the same prompt through the batched prefill (tcgen05 GEMM), after the
    # decode measurements (it rewrites the session's cache)
    prefill = {"prompt_tokens": int(args.prompt_len), "token_by_token_ms": prefill_tokens_ms}
    if not args.no_prefill:
        t0 = time.perf_counter()
        dm.set_prefill(PREFILL_BATCHED)
        setup_ms = 1000.0 * (time.perf_counter() - t0)
        runs = []
        for _ in range(4):
            p0.record(stream)
            dm.prefill(prompt, s)
            p1.record(stream)
            stream.synchronize()
            runs.append(p0.elapsed_time(p1))
        bms = float(np.median(runs[1:]))
        prefill.update({"batched_ms": bms, "batched_setup_ms": setup_ms, "speedup": prefill_tokens_ms / bms,
                        "batched_tok_per_s": args.prompt_len / (bms / 1000.0),
                        "kernels": "gemm_q8_kernel (tcgen05.mma kind::i8, TMEM accumulators), prefill_attn_kernel, "
                                   "prefill_qk_kernel, norms"})

    # roofline of the dominant kernel: the persistent decode kernel is one
    # launch per token and carries the whole forward; its algorithmic bytes
    # are the packed weights plus the KV rows of the timed positions
    peak, peak_kind = measured_peaks()
    positions = list(range(args.prompt_len + args.warmup, args.prompt_len + args.warmup + args.steps))
    kvb = kv_bytes_per_step(cfg, positions)
    wbytes = cfg.decode_weight_bytes()
    alg = wbytes + kvb
    achieved = alg / (ms_max / args.steps / 1000.0) / 1e9
    sweep = []
    if not args.no_sweep:
        dm4 = DeviceModel.synthesize(q4_cfg(cfg), SEED)
        sweep = matvec_sweep([("Q8_0", dm), ("Q4_0", dm4)], cfg, peak)
        dm4.close()

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "s8 MMA, f32 accumulate",
        "data": "synthetic (seeded random-init N(0,0.02) weights quantized to Q8_0 on the device, seeded prompt ids)",
        "config": {"workload": f"{cfg.name} Q8_0 greedy decode at batch 1 after a {args.prompt_len}-token prompt",
                   "model": cfg.name, "global_batch": world, "seq_len": cfg.seq_len,
                   "positions": [args.prompt_len + args.warmup, args.prompt_len + args.warmup + args.steps - 1],
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (1.83 GB of weights per step vs 126 MB L2)"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "call": "brew_model_forward per token: host token and position in (8 bytes, launch parameters of "
                        "the decode kernel), host argmax id out with the device error word (4 + 4 bytes, written by "
                        "the kernel into mapped pinned host memory)"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": profiled_traffic(TRAFFIC_PROFILE), "peak_kind": peak_kind,
                     "traffic_source": f"profile: profiles/{TRAFFIC_PROFILE} (ncu dram__bytes_read.sum + "
                                       f"dram__bytes_write.sum of one launch; the command is in the file)",
                     "kernel": "decode_kernel (persistent; one launch = one decode step, timed with the step's "
                               "1-launch token update)",
                     "bytes_per_launch": alg, "weight_bytes": wbytes, "kv_bytes": kvb,
                     "ms_per_launch": ms_max / args.steps},
        "matvec_sweep": sweep,
        "prefill": prefill,
        "clocks": clk,
        "setup_s": {"synthesize": round(synth_s, 2)},
    }
    dm.close()
    if not args.no_tp:
        # the sharded 7B config at the same N (tensor parallelism over the
        # ranks; strong scaling): a sub-record of the line
        line["tp"] = tp_measure(rank, world, dist, dev, args.tp_steps, 3, args.batch, args.tp_prompt_len)
    if world == 1 and not args.no_workloads:
        # the other named single-GPU workloads (one GPU only: the ranks of a
        # multi-GPU run would wait for them at the closing barrier)
        line["workloads"] = [workload_measure(c, pl, nd, ct, peak, peak_kind, with_cpu=not args.no_cpu_baseline)
                             for c, pl, nd, ct in named_workloads()]
    if rank == 0 and not args.no_cpu_baseline:
        tps, thr, dt = cpu_decode_rate(cfg, args.cpu_tokens, args.prompt_len)
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": thr, "kind": "port",
                                "sample": f"{args.cpu_tokens} decode tokens at positions {args.prompt_len + 1}.."
                                          f"{args.prompt_len + args.cpu_tokens} of the same model, oracle (C "
                                          f"restatement of the reference Java path), {dt:.1f}s"}
    if rank == 0:
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--prompt-len", type=int, default=None,
                    help=f"prompt tokens (default {PROMPT_LEN}; 256 with --tp)")
    ap.add_argument("--cpu-tokens", type=int, default=224, help="decode tokens of the CPU-baseline sample (~13 s)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the matvec sweep")
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched-prefill timing")
    ap.add_argument("--tp", action="store_true",
                    help="tensor-parallel decode of the Qwen2.5-7B-shaped K-quant config over --gpus ranks")
    ap.add_argument("--batch", type=int, default=32, help="concurrent sequences of the --tp workload")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel 7B sub-record")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the SmolLM2-135M / Gemma-3-1B workload sub-records")
    ap.add_argument("--tp-steps", type=int, default=16, help="timed steps of the tensor-parallel sub-record")
    ap.add_argument("--tp-prompt-len", type=int, default=256, help="prompt tokens of the tensor-parallel sub-record")
    ap.add_argument("--kernel-only", action="store_true", help="time the decode matvec kernel alone")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time the prefill GEMM alone (gate|up-sized projection, --gemm-tokens tokens, --steps runs)")
    ap.add_argument("--gemm-tokens", type=int, default=512, help="--gemm-only: token vectors per GEMM")
    ap.add_argument("--prefill-only", action="store_true", help="batched prefill of the prompt, twice, then exit")
    ap.add_argument("--profile-decode", action="store_true", help="prompt + a few decode steps, no timing")
    ap.add_argument("--layers", type=int, default=0, help="--profile-decode / --tp: layers of the model (default: all)")
    ap.add_argument("--vocab", type=int, default=0, help="--profile-decode: vocabulary size (default: the config's)")
    ap.add_argument("--batched-prefill", action="store_true", help="--profile-decode: prefill the prompt batched")
    ap.add_argument("--trace-decode", action="store_true",
                    help="per-phase %%globaltimer table of one decode step (run with BREW_TRACE=1)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        args.prompt_len = args.prompt_len or PROMPT_LEN
        return run_reference(args)
    if args.tp:
        args.prompt_len = args.prompt_len or 256
        return run_tp(args)
    args.prompt_len = args.prompt_len or PROMPT_LEN
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
