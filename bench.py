#!/usr/bin/env python3
"""Benchmark of the batched programmable bootstrap (PBS/s) and of encrypted MLP inference
(samples/s) on B200.

Workload: the PBS microbenchmark -- a batch of 4096 LWE ciphertexts under
n=834, k=1, N=2048, PBS gadget (2^23, 1), keyswitch gadget (2^3, 5), Gaussian noise at the
set's std, uniform 4-bit messages (2 message + 2 carry bits) and a random 16-entry LUT.  One
step = keyswitch + blind rotation + sample extraction of the whole batch (the work the
reference does with one shortint apply_lookup_table call per ciphertext,
runtime/src/ops/activation.rs:115).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl reference]

Per-configuration legs, at the end of the same line (the driver keeps the line's tail):
  "mlp"  -- configuration 4: the 6-bit MLP 784-128-128-10 (graph quantized by the reference
            quantizer, tests/golden/cfg4_mlp.json) evaluated end to end under encryption --
            every Linear on the tensor cores, every Requant an exact bootstrap program -- on a
            fixed global batch of `--mlp-batch` (1024) synthetic samples sharded over the GPUs
            (strong scaling);
  "cnn"  -- configuration 5: the small CNN (tests/golden/cfg5_cnn.json) on `--cnn-batch` (64)
            samples per GPU, so 8 GPUs evaluate the configuration's 512-sample batch;
  "n8192" -- configuration 3 on the 6-bit N=8192 set: PBS/s, the Linear 784->128 contraction
            over 8193-word ciphertexts (15.3 GB at 256 samples) against the HBM roofline, and
            the Linear + ReLU-Requant graph end to end, every sample decrypt-checked;
  "linear_requant" -- the same Linear + Requant graph on the N=2048 set;
  "contraction"    -- the encrypted Linear 784->128 (int4 weights, 256 samples of 784
                      ciphertexts) on the tensor cores against the HBM roofline;
  "noise"          -- the single-level bootstrap's output noise over ~1e5 bootstraps beside its
                      analytic value and the CPU restatements' (95% intervals);
  "pbs_by_key_set", "pbs_batch_sweep" -- PBS/s of the multi-level key sets, and across batch
                      sizes 1 to 65536.
Every graph leg decrypts every sample on rank 0 and compares it with the cleartext graph.

N > 1 runs one process per GPU under torchrun; in the PBS leg each rank bootstraps its own 4096
ciphertexts against its own key replica and one all-gather per step (the library's
pnb_allgather over NCCL) reassembles the layer's outputs on every rank (weak scaling), time =
max over ranks.  The graph legs shard samples over ranks and reassemble the output ciphertexts
with one pnb_allgather.
`--impl reference` times the CPU restatement of the same PBS (the oracle's unvectorised f64 FFT
path, the algorithm tfhe-rs runs on the CPU) on all host cores; it needs no GPU.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "penumbra-fhe_b200")

SEED = 20241201
FLOP_PER_PBS = 834 * (4 * 51200 + 32768)  # 1.981e8 FFT-equivalent FP64 flop (n=834, N=2048)


FP64_PEAK = [None]  # TFLOP/s, measured once per run by the PBS leg


def flop_per_pbs(n=834, N=2048, k=1, levels=1):
    """FFT-equivalent FP64 flop of one bootstrap: n CMux steps of (k+1) l forward and k+1 inverse
    transforms of N/2 complex points (5 (N/2) log2(N/2) each) and (k+1)^2 l pointwise complex
    multiply-adds (8 flop each)."""
    import math
    h = N // 2
    return n * (((k + 1) * levels + (k + 1)) * 5 * h * int(math.log2(h)) +
                (k + 1) ** 2 * levels * h * 8)
WORKLOAD = ("pbs_microbenchmark: n=834 k=1 N=2048 pbs=(2^23,1) ks=(2^3,5) gaussian noise, "
            "uniform 4-bit messages, random 16-entry LUT")
# DRAM bytes (read + write) of one blind-rotation launch over 4096 ciphertexts: a one-pass ncu
# capture of the timed launch of this workload (191.4 MB read: the 54.7 MB Fourier key about
# three times over the launch's seven block waves plus the small ciphertexts; 58.3 MB written).
BR_TRAFFIC_PER_LAUNCH = 191380000 + 58270000
# DRAM bytes (read + write) of one contract_tc_kernel launch of the contraction leg at 256
# samples: the 32-sample ncu capture (411.8 MB read + 53.5 MB written, every input ciphertext
# read once and every output written once) scaled by the 8x sample count.
CONTRACT_TRAFFIC = 8 * (411782400 + 53461248)


def load_package():
    if "penumbra_b200" in sys.modules:
        return sys.modules["penumbra_b200"]
    spec = importlib.util.spec_from_file_location(
        "penumbra_b200", os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["penumbra_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                     "--format=csv,noheader,nounits"], capture_output=True, text=True,
                    timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for s in self.samples:
            for name, v in zip(names, s[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def pbs_config(batch: int, world: int) -> dict:
    """The PBS microbenchmark's `config` (both arms print the same one)."""
    return {"workload": WORKLOAD, "batch_per_gpu": batch, "global_batch": batch * world,
            "parallelism": (f"ciphertexts sharded over {world} GPUs, outputs all-gathered "
                            "(pnb_allgather over NCCL) every step" if world > 1 else "one GPU"),
            "l2": "flushed (256 MB write) between timed steps"}


def cpu_reference_run(args, samples_per_step: int, warmup: int, steps: int):
    """Time the oracle's f64-FFT PBS on all host cores; returns (PBS/s, info)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    threads = os.cpu_count() or 1
    p = O.default_params()
    keys = O.OracleKeys(p, SEED)
    _ = keys.fbsk
    rng = np.random.default_rng(SEED)
    lut = rng.integers(0, 16, 16)
    tv = keys.test_vector(lut)
    msgs = rng.integers(0, 16, samples_per_step)
    ct = keys.encrypt_big(msgs, seed=SEED + 1)
    for _ in range(warmup):
        keys.pbs_fft(ct, tv, threads=threads)
    t0 = time.perf_counter()
    out = None
    for _ in range(steps):
        out = keys.pbs_fft(ct, tv, threads=threads)
    dt = time.perf_counter() - t0
    ok = bool(np.array_equal(keys.decode(keys.phase_big(out)), lut[msgs]))
    return samples_per_step * steps / dt, {"threads": threads, "decrypt_ok": ok,
                                           "seconds": dt}


def run_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    steps, warm = args.steps, max(args.warmup, 0)
    per_step = args.ref_samples
    v, info = cpu_reference_run(args, per_step, warm, steps)
    line = {
        "impl": "reference", "metric": "pbs_per_second", "value": v, "unit": "PBS/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warm,
        "ms_per_step": 1e3 * per_step / v, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": pbs_config(args.batch, args.gpus),
        "cpu_baseline": {"value": v, "unit": "PBS/s", "cores": info["threads"], "kind": "port",
                         "sample": f"each step bootstraps a bounded sample of {per_step} of the "
                                   f"batch's ciphertexts, x {steps} steps, on {info['threads']} "
                                   "host threads (the oracle's unvectorised f64-FFT PBS "
                                   "restatement; tfhe-rs itself cannot be built here)"},
        "e2e": {"value": v, "unit": "PBS/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "decrypt_ok": info["decrypt_ok"],
    }
    print(json.dumps(line), flush=True)
    return 0


def device_timed(fn, flush, steps, stream):
    """Device time of `steps` launches of fn(), each after an L2 flush, from CUDA events around
    each launch.  A device-side spin queued first lets the host enqueue every step before the
    GPU reaches them, so host-side launch latency never lands inside an event pair."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(50_000_000)  # ~25 ms of GPU cycles ahead of the first step
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def contraction_leg(args, pnb, local, dev, flush):
    """Encrypted Linear 784 -> 128 (int4 weights, 256 samples) on the tensor cores.

    HBM-bound: every input ciphertext is read once and every output written once, so the
    roofline is algorithmic bytes / time against the measured copy bandwidth."""
    import numpy as np
    import torch
    M, K, B = 128, 784, args.contract_batch
    L = 2049
    LD = 2050  # the graph evaluator's row pitch: 16-byte aligned rows, read by TMA tiles
    rng = np.random.default_rng(SEED + 3)
    W = torch.tensor(rng.integers(-8, 8, (M, K)).astype(np.int8), device=dev)
    bias = torch.tensor(rng.integers(-100, 100, M), device=dev)
    X = torch.randint(-(1 << 62), 1 << 62, (B, K, LD), dtype=torch.int64, device=dev)
    Y = torch.empty((B, M, LD), dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 1)):
        pnb.lwe_contract_ld(W, bias, 1 << 40, X, L, out=Y)
    ms = device_timed(lambda: pnb.lwe_contract_ld(W, bias, 1 << 40, X, L, out=Y), flush,
                      args.steps, stream)
    avg = sum(ms) / len(ms)
    algo_bytes = B * K * L * 8 + B * M * L * 8 + M * K + M * 8
    peak = _measured_hbm()
    gbs = algo_bytes / (avg * 1e-3) / 1e9
    macs = M * K * B * L
    return {
        "metric": "contraction_u64_macs_per_second", "value": macs / (avg * 1e-3),
        "unit": "u64 MAC/s", "ms": avg, "ms_median": statistics.median(ms), "ms_min": min(ms),
        "config": {"workload": f"Linear {K}->{M}, int4 weights U[-8,7], {B} samples of {K} "
                               f"ciphertexts (kN+1 = {L} words at a {LD}-word row pitch)",
                   "l2": "inputs (%.2f GB) exceed L2; flushed between steps" %
                         (B * K * L * 8 / 1e9)},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak["value"], "unit": "GB/s",
                     "frac": gbs / peak["value"], "peak_source": peak["source"],
                     "kernel": "contract_tc_kernel<2> (TMA operand tiles)",
                     "algorithmic_bytes": algo_bytes,
                     "traffic": CONTRACT_TRAFFIC},
    }


def n8192_leg(args, pnb, world, rank, local, dist, dev, flush, comm=None):
    """Configuration 3 on the 6-bit set at N = 8192 (pnb_params_n8192): the bootstrap's PBS/s
    (keyswitch + blind rotation, 64-entry LUT, decryption-checked), the Linear 784 -> 128
    contraction over 8193-word ciphertexts against the HBM roofline (the 15.3 GB workload at 256
    samples), and the Linear + ReLU-Requant graph end to end on `--n8k-batch` samples per GPU."""
    import numpy as np
    import torch
    p = pnb.params_n8192()
    keys = pnb.keygen(p, seed=SEED, device=local)
    rng = np.random.default_rng(SEED + 81)
    B = args.n8k_pbs_batch
    lut = rng.integers(0, 64, 64)
    msgs = rng.integers(0, 64, B)
    tv = pnb.test_vector(keys, lut)
    ct = pnb.encrypt(keys, torch.tensor(msgs), seed=SEED + 82)
    small = torch.empty((B, p.n + 1), dtype=torch.int64, device=dev)
    ks_ws = torch.empty(pnb.keyswitch_workspace_bytes(keys, B), dtype=torch.uint8, device=dev)
    o = torch.empty_like(ct)
    stream = torch.cuda.current_stream(dev)
    pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
    pnb.blind_rotate(keys, tv, small, out=o)
    ok = bool(np.array_equal(pnb.decrypt_vec(keys, o).cpu().numpy(), lut[msgs]))
    ms = []
    for _ in range(3):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
        pnb.blind_rotate(keys, tv, small, out=o)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    pbs = {"batch": B, "pbs_per_second": B / (sum(ms) / len(ms) * 1e-3), "decrypt_ok": ok,
           "params": {"n": p.n, "N": p.N, "pbs": [p.pbs_base_log, p.pbs_level],
                      "ks": [p.ks_base_log, p.ks_level], "msg_bits": p.msg_bits,
                      "carry_bits": p.carry_bits}}
    del ct, small, ks_ws, o
    keys.free()
    # the contraction at d = 8192
    M, K, Bc, L, LD = 128, 784, args.n8k_contract_batch, 8193, 8194
    if Bc <= 0:
        return {"pbs": pbs, "contraction": None, "linear_requant": None}
    Wt = torch.tensor(rng.integers(-8, 8, (M, K)).astype(np.int8), device=dev)
    bias = torch.tensor(rng.integers(-100, 100, M), device=dev)
    X = torch.randint(-(1 << 62), 1 << 62, (Bc, K, LD), dtype=torch.int64, device=dev)
    Y = torch.empty((Bc, M, LD), dtype=torch.int64, device=dev)
    pnb.lwe_contract_ld(Wt, bias, 1 << 40, X, L, out=Y)
    cms = device_timed(lambda: pnb.lwe_contract_ld(Wt, bias, 1 << 40, X, L, out=Y), flush, 5,
                       stream)
    del X, Y
    avg = sum(cms) / len(cms)
    algo = Bc * K * L * 8 + Bc * M * L * 8 + M * K + M * 8
    peak = _measured_hbm()
    gbs = algo / (avg * 1e-3) / 1e9
    contraction = {"workload": f"Linear {K}->{M}, int4 weights, {Bc} samples of {K} "
                               f"ciphertexts of {L} words at a {LD}-word pitch",
                   "ms": avg, "ms_median": statistics.median(cms), "algorithmic_bytes": algo,
                   "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak["value"],
                                "unit": "GB/s", "frac": gbs / peak["value"],
                                "peak_source": peak["source"],
                                "floor_ms": algo / (peak["value"] * 1e9) * 1e3}}
    graph = None
    if args.n8k_batch > 0:
        graph = graph_leg(args, pnb, world, rank, local, dist, dev, linear_requant_graph(),
                          args.n8k_batch * world, SEED + 400,
                          "Linear 784->128 (int4 weights U[-8,7]) + ReLU-Requant to 2 bits, "
                          "6-bit inputs, 6-bit N=8192 parameter set",
                          "encrypted_linear_requant_n8192_samples_per_second", "weak",
                          params=p, comm=comm)
    return {"pbs": pbs, "contraction": contraction, "linear_requant": graph}


def _measured_hbm():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        for k in ("hbm_gbs", "hbm_GBps", "hbm"):
            if k in d:
                v = d[k]
                v = v.get("value", v) if isinstance(v, dict) else v
                return {"value": float(v), "source": "MEASURED_PEAKS.json " + k + " (of measured)"}
    except Exception:
        pass
    return {"value": 6650.0, "source": "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"}


def batch_sweep(pnb, keys, dev, flush, batches=(1, 16, 256, 1024, 4096, 16384, 65536)):
    """[batch, PBS/s] (keyswitch + blind rotation, device-timed, inputs resident) across batch
    sizes."""
    import numpy as np
    import torch
    rng = np.random.default_rng(SEED + 21)
    tv = pnb.test_vector(keys, rng.integers(0, 16, 16))
    stream = torch.cuda.current_stream(dev)
    out = []
    for B in batches:
        ct = pnb.encrypt(keys, torch.tensor(rng.integers(0, 16, B)), seed=SEED + 22)
        small = torch.empty((B, keys.params.n + 1), dtype=torch.int64, device=dev)
        ks_ws = torch.empty(pnb.keyswitch_workspace_bytes(keys, B), dtype=torch.uint8, device=dev)
        o = torch.empty_like(ct)
        reps = 3 if B >= 4096 else 5
        pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
        pnb.blind_rotate(keys, tv, small, out=o)
        ms = 0.0
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
            pnb.blind_rotate(keys, tv, small, out=o)
            b.record(stream)
            torch.cuda.synchronize(dev)
            ms += a.elapsed_time(b)
        ms /= reps
        out.append([B, round(B / (ms * 1e-3))])
        del ct, small, ks_ws, o
    return out


def key_set_leg(pnb, dev, flush, sets=((15, 2), (11, 3), (10, 4), (7, 6), (5, 9)), B=4096,
                fp64_peak=None):
    """PBS/s of the multi-level key sets the graph planner uses (keyswitch + blind rotation,
    device-timed at batch B, L2 flushed between repetitions), each checked by decryption, with
    its FFT-equivalent FP64 rate against the FP64 peak measured in the run."""
    import numpy as np
    import torch
    rng = np.random.default_rng(SEED + 31)
    stream = torch.cuda.current_stream(dev)
    out = []
    for base_log, levels in sets:
        p = pnb.default_params()
        p.pbs_base_log, p.pbs_level = base_log, levels
        keys = pnb.keygen(p, seed=SEED, device=dev.index)
        lut = rng.integers(0, 16, 16)
        msgs = rng.integers(0, 16, B)
        tv = pnb.test_vector(keys, lut)
        ct = pnb.encrypt(keys, torch.tensor(msgs), seed=SEED + 32)
        small = torch.empty((B, keys.params.n + 1), dtype=torch.int64, device=dev)
        ks_ws = torch.empty(pnb.keyswitch_workspace_bytes(keys, B), dtype=torch.uint8, device=dev)
        o = torch.empty_like(ct)
        pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
        pnb.blind_rotate(keys, tv, small, out=o)
        ok = bool(np.array_equal(pnb.decrypt_vec(keys, o).cpu().numpy(), lut[msgs]))
        ph = pnb.phase(keys, o).cpu().numpy().view(np.uint64)
        err = (ph - lut[msgs].astype(np.uint64) * np.uint64(keys.params.delta())).view(np.int64)
        log2_std = float(np.log2(err.astype(np.float64).std()))
        reps, ms = 3, 0.0
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
            pnb.blind_rotate(keys, tv, small, out=o)
            b.record(stream)
            torch.cuda.synchronize(dev)
            ms += a.elapsed_time(b)
        ms /= reps
        rate = B / (ms * 1e-3)
        tflops = flop_per_pbs(levels=levels) * rate / 1e12
        out.append({"key": [base_log, levels], "pbs_per_second": round(rate),
                    "fp64_tflops": round(tflops, 2),
                    "fp64_frac": round(tflops / fp64_peak, 3) if fp64_peak else None,
                    "decrypt_ok": ok, "log2_noise_std": round(log2_std, 3)})
        del ct, small, ks_ws, o
        keys.free()
    return out


def _ratio_ci(a, b, reps=2000, seed=0):
    """Variance ratio var(a)/var(b) of paired error samples with a 95% percentile interval from
    resampling the pairs."""
    import numpy as np
    rng = np.random.default_rng(seed)
    n = a.size
    r = []
    for _ in range(reps):
        i = rng.integers(0, n, n)
        r.append(a[i].var() / b[i].var())
    lo, hi = np.percentile(r, [2.5, 97.5])
    return [float(a.var() / b.var()), float(lo), float(hi)]


def fft_product_error(pnb, dev, base_log, polys=256):
    """Variance of the f64-FFT negacyclic product's error per coefficient: random balanced
    digits of the gadget (|d| <= 2^(base_log-1)) times uniform torus polynomials through the
    blind rotation's transform (pnb_fft_negacyclic_mul), against the exact product mod 2^64."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    rng = np.random.default_rng(SEED + 41)
    N = 2048
    h = 1 << (base_log - 1)
    a = rng.integers(-h, h, (polys, N), dtype=np.int64)
    b = rng.integers(0, 1 << 64, (polys, N), dtype=np.uint64)
    got = pnb.fft_negacyclic_mul(torch.tensor(a, device=dev),
                                 torch.tensor(b.view(np.int64), device=dev))
    got = got.cpu().numpy().view(np.uint64)
    want = np.stack([O.negacyclic_mul(a[i].view(np.uint64), b[i]) for i in range(polys)])
    e = (got - want).view(np.int64).astype(np.float64)
    return float(e.var())


def noise_leg(pnb, keys, dev, cpu_count=8192, exact_count=512, total=100352):
    """Output noise of the single-level bootstrap over ~1e5 bootstraps (phase - LUT*delta),
    beside the analytic model and the CPU restatements run on the same keys and ciphertexts:
    the f64-FFT restatement (the algorithm tfhe-rs runs) on the first `cpu_count` bootstraps
    and the exact-arithmetic restatement (no FFT error) on the first `exact_count`."""
    import numpy as np
    import torch
    rng = np.random.default_rng(SEED + 9)
    B = 4096
    lut = rng.integers(0, 16, 16)
    tv = pnb.test_vector(keys, lut)
    errs, cts, ms = [], [], []
    n = 0
    while n < total:
        msgs = rng.integers(0, 16, B)
        ct = pnb.encrypt(keys, torch.tensor(msgs), seed=SEED + 50 + n)
        out = pnb.pbs_batch(keys, tv, ct)
        ph = pnb.phase(keys, out).cpu().numpy()
        want = (lut[msgs].astype(np.uint64) * np.uint64(keys.params.delta()))
        errs.append((ph.view(np.uint64) - want).view(np.int64).astype(np.float64))
        if n < max(cpu_count, exact_count):
            cts.append(ct.cpu().numpy().view(np.uint64))
            ms.append(msgs)
        n += B
    e = np.concatenate(errs)
    p = keys.params
    # analytic variance: key noise through the gadget digits, gadget rounding, and the f64
    # product's rounding error; the last two sit on the mask polynomial too, where the secret
    # key multiplies them (1 + kN/2 terms)
    s = p.glwe_std * 2.0 ** 64
    Bb = 2.0 ** p.pbs_base_log
    v1 = p.n * (p.k + 1) * p.pbs_level * p.N * (Bb * Bb / 12 + 1 / 6) * s * s
    eps = 2.0 ** (64 - p.pbs_base_log * p.pbs_level)
    v2 = (p.n / 2) * (1 + p.k * p.N / 2) * eps * eps / 12
    vprod = fft_product_error(pnb, dev, p.pbs_base_log)
    v3 = p.n * (1 + p.k * p.N / 2) * (p.k + 1) * p.pbs_level * vprod
    res = {"bootstraps": int(e.size), "log2_std": float(np.log2(e.std())),
           "mean_over_std": float(e.mean() / e.std()),
           "decrypt_errors": int(np.sum(np.abs(e) >= p.delta() / 2)),
           "analytic_log2_std": float(0.5 * np.log2(v1 + v2 + v3)),
           "analytic_terms_log2_std": {"key": float(0.5 * np.log2(v1)),
                                       "gadget_rounding": float(0.5 * np.log2(v2)),
                                       "fft_product": float(0.5 * np.log2(v3))},
           "fft_product_error_log2_std": float(0.5 * np.log2(vprod)),
           "variance_over_analytic": float(e.var() / (v1 + v2 + v3))}
    if cpu_count > 0:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        ok = O.OracleKeys(O.default_params(), SEED)
        allc, allm = np.concatenate(cts), np.concatenate(ms)
        threads = os.cpu_count() or 1

        def cpu_err(fn, cnt):
            ref = fn(allc[:cnt], ok.test_vector(lut), threads=threads)
            w = lut[allm[:cnt]].astype(np.uint64) * np.uint64(keys.params.delta())
            return (ok.phase_big(ref) - w).view(np.int64).astype(np.float64)

        e_fft = cpu_err(ok.pbs_fft, cpu_count)
        res["vs_cpu_fft_restatement"] = {
            "bootstraps": cpu_count, "cpu_log2_std": float(np.log2(e_fft.std())),
            "variance_ratio_ci95": _ratio_ci(e[:cpu_count], e_fft)}
        if exact_count > 0:
            e_ex = cpu_err(ok.pbs_exact, exact_count)
            res["vs_cpu_exact_restatement"] = {
                "bootstraps": exact_count, "cpu_log2_std": float(np.log2(e_ex.std())),
                "variance_ratio_ci95": _ratio_ci(e[:exact_count], e_ex),
                "cpu_variance_over_analytic_without_fft_term": float(e_ex.var() / (v1 + v2))}
    return res


def program_cpu_baseline(plan, graph, per_level: int = 32):
    """CPU restatement of the same encrypted program (a graph whose first node is a Linear
    layer), timed on a bounded sample.

    Every key set the program uses gets `per_level` oracle f64-FFT bootstraps (keyswitch +
    blind rotation + extraction, all host threads); the first layer's contraction is timed on
    one sample.  Samples/s = 1 / (sum over key sets of count x seconds per bootstrap +
    contraction seconds)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(SEED + 11)
    sec = 0.0
    timed = []
    for base_log, level, count in plan.key_sets():
        p = O.default_params()
        p.pbs_base_log, p.pbs_level = base_log, level
        keys = O.OracleKeys(p, SEED)
        _ = keys.fbsk
        ct = keys.encrypt_big(rng.integers(0, 16, per_level), seed=SEED + 12)
        tv = keys.test_vector(rng.integers(0, 16, 16))
        keys.pbs_fft(ct[:2], tv, threads=threads)
        t0 = time.perf_counter()
        keys.pbs_fft(ct, tv, threads=threads)
        t = (time.perf_counter() - t0) / per_level
        sec += count * t
        timed.append(f"({base_log},{level}): {count} x {1e3 * t:.2f} ms")
    W = np.array(graph["nodes"][0]["op"]["weights"], dtype=np.int64)
    X = rng.integers(0, 1 << 63, (1, W.shape[1], 2049), dtype=np.uint64)
    t0 = time.perf_counter()
    O.contract(W, None, 0, X, threads=threads)
    tc = time.perf_counter() - t0
    sec += tc
    return {"value": 1.0 / sec, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{per_level} oracle bootstraps per key set, extrapolated by the "
                      f"program's counts [{'; '.join(timed)}] + the {W.shape[1]}->{W.shape[0]} "
                      f"contraction of one sample ({1e3 * tc:.1f} ms)"}


def graph_leg(args, pnb, world, rank, local, dist, dev, graph, global_batch, seed, workload,
              metric, scaling, cpu_baseline=None, params=None, comm=None):
    """Encrypted inference of `graph` over `global_batch` samples sharded over the ranks
    (contiguous shards, `pnb.shard`): each rank encrypts and evaluates its shard on its own GPU
    (identical key replicas from one seed), one pnb_allgather reassembles the output
    ciphertexts on every rank.  `value` = global_batch / (max over ranks of the device time of
    evaluation + all-gather); `e2e` adds this rank's host->device input copy and rank 0's
    device->host copy of the gathered outputs.  Rank 0 decrypts EVERY sample and compares it
    with the cleartext integer graph."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ir_eval
    plan = pnb.Plan(pnb.Graph(graph), params=params)
    ev = pnb.Evaluator(plan, device=local, seed=SEED)  # identical keys on every rank
    hi = (1 << graph["input_bits"]) - 1
    x_all = np.random.default_rng(seed).integers(0, hi + 1, (global_batch, plan.input_elems))
    a, b = pnb.shard(global_batch, world, rank)
    B = b - a
    # keystream indices follow the global sample index, so the ciphertexts of a sample are the
    # same whatever the number of ranks
    ct = ev.encrypt(x_all[a:b], seed=SEED + 7, first_index=a * plan.input_elems)
    ev.reserve(max(B, 1))
    ev.evaluate(ct[:1])  # warm-up
    h_in = ct.cpu().pin_memory()
    d_in = torch.empty_like(ct)
    h_out = torch.empty((global_batch, plan.output_elems, ct.shape[-1]),
                        dtype=torch.int64).pin_memory()
    stream = torch.cuda.current_stream(dev)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    evs[0].record(stream)
    d_in.copy_(h_in, non_blocking=True)
    evs[1].record(stream)
    out = ev.evaluate(d_in)
    evs[2].record(stream)
    gathered = pnb.gather_shards(out, global_batch, comm=comm) if dist is not None else out
    evs[3].record(stream)
    if rank == 0:
        h_out.copy_(gathered, non_blocking=True)
    evs[4].record(stream)
    torch.cuda.synchronize(dev)
    t_dev = evs[1].elapsed_time(evs[3])
    t_e2e = evs[0].elapsed_time(evs[4])
    t_gather = evs[2].elapsed_time(evs[3])
    if dist is not None:
        t = torch.tensor([t_dev, t_e2e, t_gather], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_dev, t_e2e, t_gather = float(t[0]), float(t[1]), float(t[2])
    checked, ok = 0, None
    if rank == 0:
        got = ev.decrypt(h_out.to(dev)).cpu().numpy()
        ok = True
        for i in range(global_batch):
            want = ir_eval.evaluate(graph, {graph["inputs"][0]: x_all[i].tolist()})
            ok = ok and got[i].tolist() == want[graph["outputs"][0]]
            checked += 1
    value = global_batch / (t_dev * 1e-3)
    roofline = None
    if FP64_PEAK[0]:
        # Samples/s bound of the bootstrap stages (97% of the device time; contractions and
        # keyswitches stay under 1% and are left out): every bootstrap's FFT-equivalent flop
        # at the FP64 peak measured in the run, on `world` GPUs.
        flop = sum(c * flop_per_pbs(n=plan.params.n, N=plan.params.N, levels=lv)
                   for _, lv, c in plan.key_sets())
        bound = world * FP64_PEAK[0] * 1e12 / flop
        roofline = {"bound": "fp64", "samples_per_second_bound": bound, "frac": value / bound,
                    "flop_per_sample": flop, "peak_tflops": FP64_PEAK[0],
                    "stages": "bootstraps only (FFT-equivalent flop per key set)"}
    return {
        "metric": metric, "value": value, "unit": "samples/s",
        "global_batch": global_batch, "samples_per_gpu": B, "scaling": scaling, "ms": t_dev,
        "roofline": roofline,
        "config": {"workload": workload,
                   "parallelism": f"samples sharded over {world} GPU(s), outputs all-gathered "
                                  "(pnb_allgather over NCCL)"},
        "bootstraps_per_sample": plan.pbs_per_sample,
        "bootstraps_by_key_set": [[bl, lv, c] for bl, lv, c in plan.key_sets()],
        "cpu_baseline": (cpu_baseline(plan, graph) if cpu_baseline is not None and rank == 0
                         and world == 1 and not args.no_cpu_baseline else None),
        "allgather_ms": t_gather,
        "e2e": {"value": global_batch / (t_e2e * 1e-3), "unit": "samples/s",
                "h2d_bytes_per_step": int(global_batch * plan.input_elems * ct.shape[-1] * 8),
                "d2h_bytes_per_step": int(h_out.numel() * 8)},
        "decrypt_ok": ok, "samples_checked": checked,
    }


def mlp_leg(args, pnb, world, rank, local, dist, dev, comm=None):
    """Encrypted MLP 784-128-128-10 (the reference quantizer's graph for that configuration) on
    a fixed global batch sharded over the ranks (strong scaling)."""
    with open(os.path.join(ROOT, "tests", "golden", "cfg4_mlp.json")) as f:
        graph = json.load(f)["graph"]
    return graph_leg(args, pnb, world, rank, local, dist, dev, graph, args.mlp_batch,
                     SEED + 100,
                     "MLP 784-128-128-10, ReLU fused in Requant, PTQ n_bits=6 (reference "
                     "quantizer graph), 6-bit inputs",
                     "encrypted_mlp_samples_per_second", "strong",
                     cpu_baseline=program_cpu_baseline, comm=comm)


def cnn_leg(args, pnb, world, rank, local, dist, dev, comm=None):
    """Encrypted small CNN (Conv 3x3x8 s1 -> ReLU -> avg pool 2x2 -> Conv 3x3x16 s2 -> ReLU ->
    Linear 576->10; the reference quantizer's graph) on `--cnn-batch` samples per GPU (weak
    scaling: 8 GPUs evaluate the configuration's 512-sample batch)."""
    with open(os.path.join(ROOT, "tests", "golden", "cfg5_cnn.json")) as f:
        graph = json.load(f)["graph"]
    return graph_leg(args, pnb, world, rank, local, dist, dev, graph, args.cnn_batch * world,
                     SEED + 300,
                     "CNN 1x28x28: Conv 3x3x8 s1, ReLU, avg pool 2x2, Conv 3x3x16 s2, ReLU, "
                     "Linear 576->10 (reference quantizer graph, n_bits=6), 6-bit inputs",
                     "encrypted_cnn_samples_per_second", "weak", comm=comm)


def linear_requant_graph():
    """Encrypted Linear 784 -> 128 with int4 weights U[-8, 7] from a seed and 6-bit inputs,
    followed by a ReLU-fused requantization to 2 bits (shift 11, round bias 1024)."""
    import numpy as np
    rng = np.random.default_rng(3)
    W = rng.integers(-8, 8, (128, 784)).tolist()
    nodes = [{"name": "fc", "inputs": ["x"], "outputs": ["acc"],
              "op": {"op_type": "Linear", "weights": W, "bias": [0] * 128, "weight_bits": 4}},
             {"name": "rq", "inputs": ["acc"], "outputs": ["y"],
              "op": {"op_type": "Requant", "shift": 11, "mult": 1, "round_bias": 1024,
                     "out_bits": 2, "clamp_lut": [0, 1, 2, 3]}}]
    return {"schema_version": "0.6.0", "num_blocks": 12, "input_bits": 6, "inputs": ["x"],
            "outputs": ["y"], "nodes": nodes}


def linear_requant_leg(args, pnb, world, rank, local, dist, dev, comm=None):
    """The Linear 784 -> 128 + Requant configuration end to end (contraction + bootstraps)."""
    return graph_leg(args, pnb, world, rank, local, dist, dev, linear_requant_graph(),
                     args.lr_batch * world, SEED + 200,
                     "Linear 784->128 (int4 weights U[-8,7]) + ReLU-Requant to 2 bits, 6-bit "
                     "inputs, N=2048 parameter set",
                     "encrypted_linear_requant_samples_per_second", "weak",
                     cpu_baseline=program_cpu_baseline, comm=comm)


def run_gpu(args):
    import numpy as np
    import torch
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    pnb = load_package()
    # the library's own communicator carries every output all-gather (pnb_allgather over NCCL)
    comm = pnb.Comm.from_process_group(local) if dist is not None else None
    B = args.batch
    keys = pnb.keygen(seed=SEED, device=local)  # identical replica on every rank
    rng = np.random.default_rng(SEED + rank)
    lut = rng.integers(0, 16, 16)
    msgs = rng.integers(0, 16, B)
    tv = pnb.test_vector(keys, lut)
    ct = pnb.encrypt(keys, torch.tensor(msgs), seed=SEED + 1 + rank)
    out = torch.empty_like(ct)
    small = torch.empty((B, keys.params.n + 1), dtype=torch.int64, device=dev)
    ks_ws = torch.empty(pnb.keyswitch_workspace_bytes(keys, B), dtype=torch.uint8, device=dev)
    pbs_ws = torch.empty(pnb.pbs_workspace_bytes(keys, B), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # warm-up (also verifies the result decrypts to the LUT)
    for _ in range(max(args.warmup, 0)):
        pnb.pbs_batch(keys, tv, ct, out=out, workspace=pbs_ws)
    torch.cuda.synchronize(dev)
    dec = pnb.decrypt_vec(keys, out).cpu().numpy()
    decrypt_ok = bool(np.array_equal(dec, lut[msgs]))

    # With N > 1 ranks each step is one sharded layer of bootstraps: every rank bootstraps its
    # own 4096 ciphertexts, then one all-gather (pnb_allgather) reassembles the layer's outputs
    # on every rank (the exchange step of the sample-sharded evaluation).
    gathered = (torch.empty((world * B, keys.big_dim + 1), dtype=torch.int64, device=dev)
                if dist is not None else None)
    if comm is not None:
        comm.allgather(out, world * B, out=gathered)  # warm the communicator

    # timed region: K steps, L2 flushed between steps (outside the step events)
    ev = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(4))
          for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush.zero_()
            e0, e1, e2, e3 = ev[i]
            e0.record(stream)
            pnb.keyswitch(keys, ct, out=small, workspace=ks_ws)
            e1.record(stream)
            pnb.blind_rotate(keys, tv, small, out=out)
            e2.record(stream)
            if comm is not None:
                comm.allgather(out, world * B, out=gathered)
            e3.record(stream)
        barrier()
    step_ms = [a.elapsed_time(d) for a, b, c, d in ev]
    br_ms = [b.elapsed_time(c) for a, b, c, d in ev]
    ks_ms = [a.elapsed_time(b) for a, b, c, d in ev]
    ag_ms = [c.elapsed_time(d) for a, b, c, d in ev]
    total_ms = sum(step_ms)
    if dist is not None:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = world * B * args.steps / (total_ms * 1e-3)

    # end-to-end: host ciphertexts in pinned memory -> device -> PBS -> host, every step, as a
    # caller streaming batches would run it: uploads and downloads on their own streams into
    # two device buffers, so step k's upload and step k-1's download overlap step k-1's and
    # step k's bootstraps; every byte still crosses the bus inside the timed region
    h_in = ct.cpu().pin_memory()
    h_outs = [torch.empty_like(h_in).pin_memory() for _ in range(2)]
    d_ins = [torch.empty_like(ct) for _ in range(2)]
    d_outs = [torch.empty_like(ct) for _ in range(2)]
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    barrier()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    up.wait_stream(stream)
    down.wait_stream(stream)
    computed, downloaded = [], []
    for k in range(args.steps):
        b = k % 2
        with torch.cuda.stream(up):
            if k >= 2:
                up.wait_event(computed[k - 2])  # d_ins[b] was read by step k-2's bootstraps
            d_ins[b].copy_(h_in, non_blocking=True)
            uploaded = torch.cuda.Event()
            uploaded.record(up)
        stream.wait_event(uploaded)
        if k >= 2:
            stream.wait_event(downloaded[k - 2])  # d_outs[b] was read by step k-2's download
        pnb.pbs_batch(keys, tv, d_ins[b], out=d_outs[b], workspace=pbs_ws)
        computed.append(torch.cuda.Event())
        computed[k].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(computed[k])
            h_outs[b].copy_(d_outs[b], non_blocking=True)
            downloaded.append(torch.cuda.Event())
            downloaded[k].record(down)
    stream.wait_stream(down)
    stream.wait_stream(up)
    e_end.record(stream)
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    if dist is not None:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h_out = h_outs[(args.steps - 1) % 2]
    e2e_ok = bool(np.array_equal(pnb.decrypt_vec(keys, h_out.to(dev)).cpu().numpy(),
                                 lut[msgs]))
    e2e_value = world * B * args.steps / (e2e_ms * 1e-3)

    # roofline of the dominant kernel (blind rotation): FP64-bound
    peak = pnb.measure_fp64_peak(local)
    FP64_PEAK[0] = peak
    br_avg = sum(br_ms) / len(br_ms)
    achieved = FLOP_PER_PBS * B / (br_avg * 1e-3) / 1e12
    roofline = {"bound": "fp64", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_source": "FP64 FMA probe measured in this run (no FP64 entry in "
                               "MEASURED_PEAKS.json)",
                "kernel": "blind_rotate_tm_kernel<4>",
                "traffic": BR_TRAFFIC_PER_LAUNCH}

    contraction = None if args.contract_batch <= 0 else contraction_leg(args, pnb, local, dev,
                                                                           flush)
    noise = (noise_leg(pnb, keys, dev, args.noise_cpu if world == 1 else 0,
                       args.noise_exact if world == 1 else 0)
             if (rank == 0 and args.noise) else None)
    sweep = batch_sweep(pnb, keys, dev, flush) if (rank == 0 and args.sweep) else None
    key_sets = (key_set_leg(pnb, dev, flush, fp64_peak=peak)
                if (rank == 0 and args.key_sets) else None)
    n8k = (n8192_leg(args, pnb, world, rank, local, dist, dev, flush, comm)
           if args.n8k else None)
    if n8k is not None:  # the N = 8192 bootstrap's FP64 rate against the same peak
        pp = n8k["pbs"]
        pp["fp64_tflops"] = round(flop_per_pbs(n=pp["params"]["n"], N=pp["params"]["N"]) *
                                  pp["pbs_per_second"] / 1e12, 2)
        pp["fp64_frac"] = round(pp["fp64_tflops"] / peak, 3)
    lin_rq = (None if args.lr_batch <= 0
              else linear_requant_leg(args, pnb, world, rank, local, dist, dev, comm))
    cnn = (None if args.cnn_batch <= 0
           else cnn_leg(args, pnb, world, rank, local, dist, dev, comm))
    mlp = (None if args.mlp_batch <= 0
           else mlp_leg(args, pnb, world, rank, local, dist, dev, comm))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, info = cpu_reference_run(args, args.ref_samples, 1, args.ref_steps)
        cpu = {"value": v, "unit": "PBS/s", "cores": info["threads"], "kind": "port",
               "sample": f"{args.ref_samples} PBS x {args.ref_steps} passes of the same "
                         f"workload (the oracle's unvectorised f64-FFT PBS restatement, "
                         f"{info['threads']} host threads)"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        clocks = clk.summary()
        # the large per-leg objects go last, in increasing order of importance, so that a
        # reader that keeps only the end of the line keeps the configuration legs
        line = {
            "metric": "pbs_per_second", "value": value, "unit": "PBS/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": pbs_config(B, world),
            "e2e": {"value": e2e_value, "unit": "PBS/s",
                    "h2d_bytes_per_step": int(h_in.numel() * 8),
                    "d2h_bytes_per_step": int(h_out.numel() * 8),
                    "pipelining": "upload and download streams, two device buffers"},
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": 3 * args.steps,
            "stage_ms": {"keyswitch": sum(ks_ms) / len(ks_ms), "blind_rotate": br_avg,
                         "allgather": sum(ag_ms) / len(ag_ms)},
            "decrypt_ok": decrypt_ok and e2e_ok,
            "pbs_batch_sweep": sweep,
            "pbs_by_key_set": key_sets,
            "noise": noise,
            "contraction": contraction,
            "n8192": n8k,
            "linear_requant": lin_rq,
            "cnn": cnn,
            "mlp": mlp,
        }
        print(json.dumps(line), flush=True)
    if comm is not None:
        torch.cuda.synchronize(dev)
        comm.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


LAUNCH_TIME_SCALE = {"ns": 1e-6, "nsecond": 1e-6, "us": 1e-3, "usecond": 1e-3, "ms": 1.0,
                     "msecond": 1.0, "s": 1e3, "second": 1e3}


def summarize_launches(path):
    """Per-kernel launches, total device time and share of an ncu launch list
    (`ncu --metrics gpu__time_duration.sum --csv --log-file <path>`; cold-cache, serialised)."""
    import collections
    import csv
    with open(path) as f:
        rows = list(csv.reader(f))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    hdr, data = rows[hi], rows[hi + 1:]
    ki, mi = hdr.index("Kernel Name"), hdr.index("Metric Name")
    vi, ui = hdr.index("Metric Value"), hdr.index("Metric Unit")
    agg = collections.defaultdict(lambda: [0, 0.0])
    for r in data:
        if len(r) <= vi or r[mi] != "gpu__time_duration.sum":
            continue
        name = r[ki].split("(")[0].strip()
        agg[name][0] += 1
        agg[name][1] += float(r[vi].replace(",", "")) * LAUNCH_TIME_SCALE[r[ui]]
    tot = sum(v[1] for v in agg.values())
    print(f"{'kernel':62s} {'launches':>8s} {'total ms':>10s} {'share':>7s}")
    for k, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1]):
        print(f"{k[:62]:62s} {n:8d} {t:10.2f} {100 * t / tot:6.2f}%")
    print(f"{'all':62s} {sum(v[0] for v in agg.values()):8d} {tot:10.2f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=4096)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-samples", type=int, default=1024)
    ap.add_argument("--ref-steps", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--contract-batch", type=int, default=256,
                    help="samples of the Linear 784->128 contraction leg (0 skips it)")
    ap.add_argument("--sweep", type=int, default=1,
                    help="PBS/s across batch sizes 1..65536 (rank 0)")
    ap.add_argument("--summarize-launches", metavar="CSV", default=None,
                    help="print the per-kernel table of an ncu launch list and exit")
    ap.add_argument("--key-sets", type=int, default=1,
                    help="PBS/s of the multi-level key sets at batch 4096 (rank 0)")
    ap.add_argument("--noise", type=int, default=1,
                    help="measure the bootstrap output noise over ~1e5 bootstraps (rank 0)")
    ap.add_argument("--lr-batch", type=int, default=32,
                    help="samples per GPU of the Linear 784->128 + Requant leg (0 skips it)")
    ap.add_argument("--mlp-batch", type=int, default=1024,
                    help="global batch of the encrypted MLP leg, sharded over the GPUs "
                         "(strong scaling; 0 skips it)")
    ap.add_argument("--n8k", type=int, default=1,
                    help="configuration 3 on the 6-bit N=8192 set (PBS/s, contraction, graph)")
    ap.add_argument("--n8k-batch", type=int, default=8,
                    help="samples per GPU of the N=8192 Linear 784->128 + Requant graph")
    ap.add_argument("--n8k-pbs-batch", type=int, default=2048,
                    help="bootstraps per launch of the N=8192 PBS measurement")
    ap.add_argument("--n8k-contract-batch", type=int, default=256,
                    help="samples of the N=8192 contraction (256: 15.3 GB of traffic)")
    ap.add_argument("--cnn-batch", type=int, default=64,
                    help="encrypted CNN samples per GPU (weak scaling; 0 skips the CNN leg)")
    ap.add_argument("--noise-cpu", type=int, default=8192,
                    help="bootstraps the f64-FFT CPU restatement repeats for the noise "
                         "comparison (one GPU only)")
    ap.add_argument("--noise-exact", type=int, default=512,
                    help="bootstraps the exact-arithmetic CPU restatement repeats for the noise "
                         "comparison (one GPU only)")
    args = ap.parse_args()
    if args.summarize_launches:
        summarize_launches(args.summarize_launches)
        return 0
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
