"""Benchmark: Q4_K decode matvec weight GB/s on B200 (Llama-3-8B FFN-down layer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--act x16|x8] [--copies C]

Workload (n x k = 4096 x 14336, the "4096x14336-class" Llama-3-8B down
projection, Q4_K, 33,030,144 weight bytes): one step = C matvecs, each over a
distinct resident copy of the weights (C * 33 MB > 2 x the 126 MB L2, so every
step streams its weights from HBM), x ~ N(0, 1) fp32, W ~ N(0, 0.02) packed to
Q4_K. value = weight bytes / device time (GB/s), all ranks summed; each rank
runs the same per-GPU work (weak scaling, no collective on the data path).

Rank 0 prints one JSON line. `--impl reference` times the reference engine's
own CPU op (oracle/_ref/libref_qm.so, compiled from its sources) on the host
cores over a bounded sample of the same workload.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_ROWS, K_DIM = 4096, 14336
QT_Q4_K = 12
METRIC = "Q4_K matvec weight GB/s (4096x14336 Llama-3-8B FFN-down layer)"


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _weights(seed: int = 0) -> np.ndarray:
    from cybel_b200 import quantize as Q

    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(N_ROWS, K_DIM)).astype(np.float32)
    return Q.quantize_q4_k(w)


def _peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def _traffic_per_launch():
    p = ROOT / "profiles" / "gemv_q4k_4096x14336_traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch"])
        except Exception:
            return None
    return None


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: through
    NVML in-process (a sample every ~0.5 ms, so even a region of a few
    milliseconds is covered), else nvidia-smi every 200 ms."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    # NVML clocks-event reason bits
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, device: int):
        self.device = device
        self.samples = []  # (sm_mhz, max_mhz, reasons set)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            try:
                uuid = str(torch.cuda.get_device_properties(device).uuid)
                h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device)
            get_r = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self._nvml = (pynvml, h, get_r, pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.source = "nvml"
        except Exception:
            self._nvml = None
            self.source = "nvidia-smi"

    def _sample_nvml(self):
        p, h, get_r, mx = self._nvml
        sm = p.nvmlDeviceGetClockInfo(h, p.NVML_CLOCK_SM)
        bits = int(get_r(h))
        return float(sm), float(mx), {n for n, b in self.REASON_BITS.items() if bits & b}

    def _sample_smi(self):
        out = subprocess.run(
            ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
            capture_output=True, text=True, timeout=5,
        ).stdout.strip()
        if not out:
            return None
        f = [x.strip() for x in out.split(",")]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm = float(f[1]) if f[1].replace(".", "").isdigit() else None
        mx = float(f[2]) if f[2].replace(".", "").isdigit() else None
        return sm, mx, {names[i] for i in range(4) if len(f) > 5 + i and f[5 + i] == "Active"}

    def sample_now(self):
        try:
            smp = self._sample_nvml() if self._nvml else None
            if smp is not None:
                self.samples.append(smp)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            try:
                smp = self._sample_nvml() if self._nvml else self._sample_smi()
                if smp is not None:
                    self.samples.append(smp)
            except Exception:
                pass
            self._stop.wait(0.0005 if self._nvml else 0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        t0 = time.perf_counter()  # sampling is running before the timed region opens
        while not self.samples and time.perf_counter() - t0 < 2.0:
            time.sleep(0.0005)
        return self

    def mark(self):
        """The timed region opens: keep only the samples taken from here on
        (the last earlier one stays as a fallback for a region shorter than
        one sample)."""
        self._before = self.samples[-1:] if self.samples else []
        self.samples = []

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples and getattr(self, "_before", None):
            self.samples = list(self._before)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "source": self.source}
        sm = [s[0] for s in self.samples if s[0] is not None]
        mx = [s[1] for s in self.samples if s[1] is not None]
        reasons = sorted(set().union(*(s[2] for s in self.samples)))
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(self.samples),
            "source": self.source,
        }


def _cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), or "unknown"."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_reference_sample(W: np.ndarray, x: np.ndarray, budget_s: float = 12.0):
    """The reference's compiled simd_matvec_q4k on the host cores: GB/s."""
    from oracle import oracle as O

    threads = len(os.sched_getaffinity(0))
    if O.ref_available():
        os.environ["ANVIL_NUM_THREADS"] = str(threads)
        O.ref_matvec(QT_Q4_K, W, x, K_DIM, N_ROWS)  # warm-up
        calls, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget_s or calls < 3:
            O.ref_matvec(QT_Q4_K, W, x, K_DIM, N_ROWS)
            calls += 1
        dt = time.perf_counter() - t0
        return {
            "value": round(W.nbytes * calls / dt / 1e9, 3),
            "unit": "GB/s",
            "cores": threads,
            "kind": "reference",
            "cpu_model": _cpu_model(),
            "sample": f"{calls} x simd_matvec_q4k {N_ROWS}x{K_DIM} (one weight copy) in {dt:.1f} s, ANVIL_NUM_THREADS={threads}",
        }
    # Fallback: the oracle's scalar restatement, single thread.
    n_rows = 256
    Ws = np.ascontiguousarray(W[:n_rows])
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or calls < 1:
        O.matvec_f64(Ws, QT_Q4_K, x, K_DIM, n_rows)
        calls += 1
    dt = time.perf_counter() - t0
    return {
        "value": round(Ws.nbytes * calls / dt / 1e9, 3),
        "unit": "GB/s",
        "cores": 1,
        "kind": "port",
        "cpu_model": _cpu_model(),
        "sample": f"{calls} x oracle matvec of {n_rows} rows of the {N_ROWS}x{K_DIM} layer in {dt:.1f} s",
    }


def run_reference(args, ws, rank):
    if rank != 0:
        return
    W = _weights()
    x = np.random.default_rng(1).standard_normal(K_DIM).astype(np.float32)
    samples = []
    for _ in range(args.warmup):
        _cpu_reference_sample(W, x, budget_s=0.5)
    for _ in range(args.steps):
        samples.append(_cpu_reference_sample(W, x, budget_s=2.0))
    vals = [s["value"] for s in samples]
    v = float(np.mean(vals))
    base = samples[-1]
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(v, 3),
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(W.nbytes * args.copies / (v * 1e9) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"q4k_matvec_{N_ROWS}x{K_DIM}", "copies": args.copies, "l2": "inputs > L2"},
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": base["cores"], "kind": base["kind"],
                         "cpu_model": base.get("cpu_model", _cpu_model()), "sample": base["sample"]},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _peak_bf16():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def _normal_w(seed: int, n: int, k: int) -> np.ndarray:
    """N(0, 0.02) fp32 weights [n][k] from default_rng(seed)."""
    return (np.random.default_rng(seed).standard_normal((n, k), dtype=np.float32) * np.float32(0.02))


def chain_time_us(dev, qt: int, W: np.ndarray, k: int, n: int, act: int, reps: int = 10,
                  min_bytes: float = 300e6) -> float:
    """Device time per matvec of a chain of C matvecs over C distinct resident
    copies of W (C * bytes > 2 x L2), one fp32 x, captured as one CUDA graph
    (PDL between launches) and replayed `reps` times after 3 warm-up replays."""
    import torch

    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    C = max(8, int(min_bytes // W.nbytes) + 1)
    mats = [DeviceMatrix(qt, k, n, W) for _ in range(C)]
    x = torch.from_numpy(np.random.default_rng(1).standard_normal(k).astype(np.float32)).to(dev)
    ys = [torch.empty(n, dtype=torch.float32, device=dev) for _ in range(C)]

    def step():
        for i in range(C):
            matmul_device(x, mats[i], out=ys[i], act_mode=act)

    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        for _ in range(3):
            step()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        step()
    for _ in range(3):
        g.replay()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / (reps * C)
    del g, mats, ys
    torch.cuda.empty_cache()
    return us


def _ref_call_time(fn, budget_s: float, min_calls: int = 2) -> tuple[float, int]:
    """Mean seconds per call of fn() over about budget_s (after one warm-up)."""
    fn()
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s or calls < min_calls:
        fn()
        calls += 1
    return (time.perf_counter() - t0) / calls, calls


def _ref_threads() -> int:
    threads = len(os.sched_getaffinity(0))
    os.environ["ANVIL_NUM_THREADS"] = str(threads)
    return threads


def c1_bench(dev, no_cpu: bool = False):
    """Q4_0 4096 x 4096 (W ~ N(0, 0.02) from default_rng(0), packed by the
    ggml Q4_0 layout; x from default_rng(1)) in both activation modes; the
    CPU baseline is gguf-py dequantize + a numpy fp32 product (the reference
    engine has no Q4_0 kernel)."""
    from cybel_b200 import _native
    from cybel_b200 import quantize as Q

    n = k = 4096
    w = np.random.default_rng(0).normal(0.0, 0.02, size=(n, k)).astype(np.float32)
    W = Q.quantize(w, 2)
    peak, _ = _peak_hbm()
    rec = {"workload": "q4_0_matvec_4096x4096", "weight_bytes": int(W.nbytes)}
    for name, act in (("x8", _native.ACT_X8), ("x16", _native.ACT_X16)):
        us = chain_time_us(dev, 2, W, k, n, act)
        gbs = W.nbytes / (us * 1e-6) / 1e9
        rec[name] = {"us_per_matvec": round(us, 2), "weight_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4)}
    if not no_cpu:
        try:
            import gguf

            x = np.random.default_rng(1).standard_normal(k).astype(np.float32)
            qt = gguf.GGMLQuantizationType.Q4_0

            def cpu():
                return gguf.dequantize(W, qt).reshape(n, k) @ x

            sec, calls = _ref_call_time(cpu, 2.0)
            rec["cpu_baseline"] = {"value": round(W.nbytes / sec / 1e9, 3), "unit": "GB/s", "cores": 1,
                                   "kind": "port", "cpu_model": _cpu_model(),
                                   "sample": f"{calls} x gguf-py dequantize + numpy fp32 matvec (no reference "
                                             f"Q4_0 kernel exists), {sec * 1e3:.1f} ms per call"}
        except ImportError:
            rec["cpu_baseline"] = None
    return rec


C2_SHAPES = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]  # (n, k), Llama-3-8B linears


def c2_bench(dev, no_cpu: bool = False):
    """Q8_0 and Q4_K matvec sweep at the Llama-3-8B linear shapes, x8 and
    x16, with the reference's simd_matvec_* on all host cores beside each."""
    from cybel_b200 import _native
    from cybel_b200 import quantize as Q

    peak, _ = _peak_hbm()
    out = []
    ref_ok = False
    if not no_cpu:
        from oracle import oracle as O

        ref_ok = O.ref_available()
        threads = _ref_threads()
    for i, (n, k) in enumerate(C2_SHAPES):
        w = _normal_w(i, n, k)
        x = np.random.default_rng(100 + i).standard_normal(k).astype(np.float32)
        for qt, name in ((12, "q4_k"), (8, "q8_0")):
            W = Q.quantize(w, qt)
            rec = {"qtype": name, "n": n, "k": k, "weight_bytes": int(W.nbytes)}
            for mode, act in (("x8", _native.ACT_X8), ("x16", _native.ACT_X16)):
                us = chain_time_us(dev, qt, W, k, n, act, min_bytes=270e6)
                gbs = W.nbytes / (us * 1e-6) / 1e9
                rec[mode] = {"us_per_matvec": round(us, 2), "weight_gbs": round(gbs, 1),
                             "hbm_frac": round(gbs / peak, 4)}
            if ref_ok:
                sec, calls = _ref_call_time(lambda: O.ref_matvec(qt, W, x, k, n), 0.6)
                rec["cpu_baseline"] = {"value": round(W.nbytes / sec / 1e9, 3), "unit": "GB/s", "cores": threads,
                                       "kind": "reference",
                                       "sample": f"{calls} x simd_matvec_{'q4k' if qt == 12 else 'q8_0'}"}
            out.append(rec)
    return out


TILE_SHAPES = [(14336, 4096), (4096, 14336)]  # (n, k): Llama-3-8B gate/up and down
TILE_MS = [8, 32, 128]


def tile_bench(dev, steps: int, warmup: int, shapes=TILE_SHAPES, ms=TILE_MS, copies: int = 8, no_cpu: bool = True):
    """Speculative-verify batched matmul on the tile path (tcgen05, fp16
    operands): per (shape, m), `copies` distinct resident Q4_K weight copies
    (> 2 x L2 in total) are multiplied by an m-row activation block, replayed
    as one CUDA graph; time per matmul from CUDA events on the replay
    stream. Returns one record per case."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import quantize as Q
    from cybel_b200.quantized_matmul import DeviceMatrix, matmul_device

    peak_hbm, _ = _peak_hbm()
    peak_tc, _ = _peak_bf16()
    out = []
    ref_ok = False
    if not no_cpu:
        from oracle import oracle as O

        ref_ok = O.ref_available()
        threads = _ref_threads()
    for n, k in shapes:
        rng = np.random.default_rng(n + k)
        W = Q.quantize_q4_k(rng.normal(0.0, 0.02, size=(n, k)).astype(np.float32))
        mats = [DeviceMatrix(QT_Q4_K, k, n, W) for _ in range(copies)]
        for m in ms:
            X = torch.from_numpy(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)).to(dev)
            ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _ in range(copies)]

            def step():
                for i in range(copies):
                    matmul_device(X, mats[i], out=ys[i], act_mode=_native.ACT_F16)

            cap = torch.cuda.Stream(dev)
            with torch.cuda.stream(cap):
                for _ in range(max(3, warmup)):
                    step()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                step()
            for _ in range(max(3, warmup)):
                g.replay()
            st = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(dev)
            e0.record(st)
            for _ in range(steps):
                g.replay()
            e1.record(st)
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) * 1e3 / (steps * copies)
            del g
            gbs = W.nbytes / (us * 1e-6) / 1e9
            tflops = 2.0 * m * n * k / (us * 1e-6) / 1e12
            rec = {
                "n": n, "k": k, "m": m,
                "us_per_matmul": round(us, 2),
                "weight_gbs": round(gbs, 1),
                "hbm_frac": round(gbs / peak_hbm, 4),
                "tflops": round(tflops, 1),
                "tensor_frac": round(tflops / peak_tc, 4),
            }
            if ref_ok:
                Xh = X.cpu().numpy()
                sec, calls = _ref_call_time(lambda: O.ref_matmul(12, W, Xh, k, n), 0.5)
                rec["cpu_baseline"] = {"us_per_matmul": round(sec * 1e6, 1), "tflops": round(2.0 * m * n * k / sec / 1e12, 4),
                                       "cores": threads, "kind": "reference",
                                       "sample": f"{calls} x simd_matmul_q4k m={m}"}
            out.append(rec)
        del mats
        torch.cuda.empty_cache()
    return out


def _cpu_layer_baseline(shape, layer, head, batch: int = 1, budget_s: float = 0.6):
    """The reference's CPU ops for one token's linears, timed per layer on all
    host cores: the 7 matvecs of one layer (simd_matvec_*; simd_matmul_* at
    batch > 1) times the layer count, plus the LM head. tok/s = batch / that."""
    from cybel_b200 import decode as D
    from oracle import oracle as O

    if not O.ref_available():
        return None
    threads = _ref_threads()
    q = shape.linear_qtype
    shapes = D.layer_matrix_shapes(shape)
    rng = np.random.default_rng(3)

    def run(W, qt, k, n):
        X = rng.standard_normal((batch, k)).astype(np.float32)
        if batch == 1:
            return _ref_call_time(lambda: O.ref_matvec(qt, W, X[0], k, n), budget_s / 8, 1)[0]
        return _ref_call_time(lambda: O.ref_matmul(qt, W, X, k, n), budget_s / 8, 1)[0]

    layer_s = sum(run(layer[name], q, k, n) for name, (n, k) in shapes.items())
    head_s = run(head, shape.head_qtype, shape.hidden, shape.vocab)
    tok_s = shape.layers * layer_s + head_s
    return {"ms_per_step": round(tok_s * 1e3, 2), "tok_s": round(batch / tok_s, 3), "cores": threads,
            "kind": "reference",
            "sample": f"one layer's 7 {'simd_matvec' if batch == 1 else f'simd_matmul (m={batch})'} calls x "
                      f"{shape.layers} layers + the LM head, {threads} threads"}


def decode_bench(dev, steps: int, warmup: int, shape_name: str = "llama3_8b", ctx: int = 2048,
                 no_cpu: bool = True):
    """Single-token decode of the Llama-3-8B-shaped stack at context `ctx`
    (KV cache prefilled with random values): one step = embedding, 32 layers
    of norm / qkv / rope / attention / o / norm / SwiGLU FFN, final norm and
    the Q6_K LM head, replayed as one CUDA graph. Weights: one random-init
    N(0, 0.02) layer quantized on the host and copied into each layer's own
    HBM buffers; the 128256-row embedding and head are a random 16032-row
    block repeated (every row still streams its own bytes). Also times the
    same step's quantized linears alone (the matvec share of a token)."""
    import torch

    from cybel_b200 import decode as D
    from cybel_b200.formats import Q4_K

    shape = {"llama3_8b": D.LLAMA3_8B, "llama3_70b": D.LLAMA3_70B}[shape_name]
    rng = np.random.default_rng(0)
    layer = D.random_layer(shape, rng)
    embed = D.random_rows(Q4_K, shape.vocab, shape.hidden, rng, block_rows=16032, std=1.0)
    head = D.random_rows(shape.head_qtype, shape.vocab, shape.hidden, rng, block_rows=16032)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    stack = D.DecodeStack(shape, ctx, [layer], embed, head, out_norm, act_mode=2)
    cpu = None if no_cpu else _cpu_layer_baseline(shape, layer, head)
    del layer, embed, head
    stack.k_cache.normal_()
    stack.v_cache.normal_()
    stack.set_token(128000 % shape.vocab)
    pos = ctx - 1
    res = {}
    for name, lin in (("step", False), ("linears", True)):
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap):
            for _ in range(max(3, warmup)):
                stack.step(pos, linears_only=lin)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            stack.step(pos, linears_only=lin)
        for _ in range(3):
            g.replay()
        st = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(st)
        for _ in range(steps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize(dev)
        res[name] = e0.elapsed_time(e1) / steps
        del g
    # Batched speculative verify (DecodeStack.verify): m drafted tokens in one
    # pass over the weights (m-row linears: GEMV below 8 rows, tcgen05 tile
    # kernel from 8), against m single-token steps.
    verify = []
    for m in (4, 8):
        toks = torch.full((m,), 128000 % shape.vocab, dtype=torch.int32, device=dev)
        pos0 = ctx - m
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap):
            for _ in range(max(3, warmup)):
                stack.verify(toks, pos0)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            stack.verify(toks, pos0)
        for _ in range(3):
            g.replay()
        st = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(st)
        for _ in range(steps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        del g
        verify.append({"m": m, "ms_per_pass": round(ms, 4), "ms_as_single_steps": round(m * res["step"], 4),
                       "tokens_checked_per_s": round(m * 1e3 / ms, 1),
                       "speedup_vs_single_steps": round(m * res["step"] / ms, 2)})
    peak, _ = _peak_hbm()
    wbytes = shape.token_weight_bytes()
    kv_bytes = 2 * shape.layers * shape.kv_heads * ctx * shape.head_dim * 2
    out = {
        "workload": f"{shape_name}_q4k_decode_ctx{ctx}",
        "weight_bytes_per_token": wbytes,
        "kv_bytes_per_token": kv_bytes,
        "ms_per_token": round(res["step"], 4),
        "tok_s": round(1e3 / res["step"], 1),
        "matvec_ms_per_token": round(res["linears"], 4),
        "matvec_tok_s": round(1e3 / res["linears"], 1),
        "matvec_weight_gbs": round(wbytes / (res["linears"] * 1e-3) / 1e9, 1),
        "matvec_hbm_frac": round(wbytes / (res["linears"] * 1e-3) / 1e9 / peak, 4),
        "step_hbm_frac": round((wbytes + kv_bytes) / (res["step"] * 1e-3) / 1e9 / peak, 4),
        "act_mode": "x16",
        "verify": verify,
        "cpu_baseline": cpu,
    }
    del stack
    torch.cuda.empty_cache()
    return out


def attention_bench(dev, steps: int, warmup: int, ctx: int = 2048):
    """The fused RoPE + KV-append + attention launch of the Llama-3-8B step
    (32 query / 8 kv heads, head_dim 128, batch 1) at context `ctx`, over
    the contiguous fp16 cache and the Q8 paged cache: 32 launches (one cache
    per layer, 32 x the KV bytes > L2) chained with PDL in one CUDA graph.
    Algorithmic bytes per launch: the cached K and V rows read
    (2 x 8 x ctx x 128 x 2 B fp16; 1 B + 4 B scale per row in Q8)."""
    import torch

    from cybel_b200 import _native
    from cybel_b200.kv_cache import PagedKVCache

    L = _native.lib()
    H, KV, HD, layers, pos = 32, 8, 128, 32, ctx - 1
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(H * HD, device=dev, generator=g)
    k = torch.randn(KV * HD, device=dev, generator=g)
    v = torch.randn(KV * HD, device=dev, generator=g)
    xq = torch.zeros(int(L.b200q_xq_row_bytes(H * HD, _native.ACT_X16)), dtype=torch.uint8, device=dev)
    peak, _ = _peak_hbm()
    out = []
    for kind in ("fp16_contiguous", "q8_paged"):
        if kind == "fp16_contiguous":
            kc = torch.randn((layers, KV, ctx, HD), device=dev, generator=g).half()
            vc = torch.randn((layers, KV, ctx, HD), device=dev, generator=g).half()

            def launch(i, st):
                _native.check(L.b200q_rope_attention_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, H, KV, HD,
                                                            pos, 5e5, kc[i].data_ptr(), vc[i].data_ptr(), ctx, None,
                                                            xq.data_ptr(), _native.ACT_X16, st), "attention")
            kv_bytes = 2 * KV * ctx * HD * 2
        else:
            cache = PagedKVCache(layers, KV, ctx, batch=1, q8=True, device=dev.index or 0)
            cache.ensure(0, pos)
            cache.k.copy_(torch.randint(-127, 128, cache.k.shape, device=dev, generator=g, dtype=torch.int32))
            cache.v.copy_(torch.randint(-127, 128, cache.v.shape, device=dev, generator=g, dtype=torch.int32))
            cache.ks.fill_(0.01)
            cache.vs.fill_(0.01)

            def launch(i, st):
                cache.attention(i, q.data_ptr(), k.data_ptr(), v.data_ptr(), pos, H, 5e5, None, xq.data_ptr(),
                                _native.ACT_X16, st)
            kv_bytes = 2 * KV * ctx * (HD + 4)
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap):
            for _ in range(max(1, warmup)):
                for i in range(layers):
                    launch(i, cap.cuda_stream)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap):
            for i in range(layers):
                launch(i, cap.cuda_stream)
        for _ in range(3):
            gr.replay()
        st = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(st)
        for _ in range(steps):
            gr.replay()
        e1.record(st)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1e3 / (steps * layers)
        _native.check_device(dev.index or 0, "attention bench")
        del gr
        out.append({"cache": kind, "ctx": ctx, "us_per_launch": round(us, 2), "kv_bytes_per_launch": kv_bytes,
                    "kv_gbs": round(kv_bytes / us / 1e3, 1), "hbm_frac": round(kv_bytes / us / 1e3 / peak, 4)})
    return out


def sharded_decode_bench(dev, ws, rank, local, steps: int, warmup: int, batch: int = 1, ctx: int = 2048,
                         shape_name: str = "llama3_70b", collective: str = "peer", no_cpu: bool = True):
    """Llama-3-70B-shaped Q4_K decode row-sharded over the ws ranks of this
    node (rank g holds rows [g n/ws, (g+1) n/ws) of every linear and the
    matching heads; all-gathers of the partial outputs by the peer-memory
    kernel or NCCL, --collective), `batch`
    sequences at context `ctx` (KV caches prefilled with random values).
    One step is captured as a CUDA graph (collectives included) and
    replayed; time = max over ranks of the CUDA-event time. Weights: each
    linear repeats one random N(0, 0.02) 2048-row block, embedding and head
    one 16032-row block (bytes per token are those of the full model)."""
    import torch

    from cybel_b200 import _native
    from cybel_b200 import decode as D
    from cybel_b200.formats import Q4_K
    from cybel_b200.sharded import GpuOps, ShardedDecode, ShardPlan, shard_layer, shard_rows

    shape = {"llama3_8b": D.LLAMA3_8B, "llama3_70b": D.LLAMA3_70B}[shape_name]
    plan = ShardPlan(shape, ws, rank)
    rng = np.random.default_rng(0)
    layer = D.random_layer(shape, rng, block_rows=2048)
    embed = D.random_rows(Q4_K, shape.vocab, shape.hidden, rng, block_rows=16032, std=1.0)
    head = D.random_rows(shape.head_qtype, shape.vocab, shape.hidden, rng, block_rows=16032)
    out_norm = (1 + 0.1 * rng.standard_normal(shape.hidden)).astype(np.float32)
    act = _native.ACT_X16 if batch < 8 else _native.ACT_X8
    ops = GpuOps(local, act_mode=act, world=ws, collective=collective, rank=rank)
    model = ShardedDecode(plan, ctx, batch, [shard_layer(layer, plan)], embed, shard_rows(head, plan, "head"),
                          out_norm, ops)
    cpu = None if (no_cpu or ws > 1 or rank != 0) else _cpu_layer_baseline(shape, layer, head, batch)
    del layer, embed, head
    model.k_cache.normal_()
    model.v_cache.normal_()
    model.tokens.fill_(128000 % shape.vocab)
    pos = ctx - 1

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        for _ in range(max(3, warmup)):
            model.step(pos)
    barrier()
    graph = torch.cuda.CUDAGraph()
    graphed = True
    try:
        with torch.cuda.graph(graph, stream=cap):
            model.step(pos)
    except Exception as e:  # collectives that cannot be captured: time the eager step
        graphed = False
        graph = None
        err = f"{type(e).__name__}: {e}"[:200]
    barrier()

    def run():
        if graphed:
            graph.replay()
        else:
            model.step(pos)

    for _ in range(3):
        run()
    barrier()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        run()
    e1.record(st)
    barrier()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t[0])
    del graph
    barrier()
    ops.close()
    wbytes = shape.token_weight_bytes()
    peak, _ = _peak_hbm()
    rec = {
        "workload": f"{shape_name}_q4k_decode_rowsharded_b{batch}_ctx{ctx}",
        "n_gpus": ws,
        "batch": batch,
        "ms_per_step": round(ms, 4),
        "tok_s": round(batch * 1e3 / ms, 1),
        "weight_bytes_per_token_all_gpus": wbytes,
        "weight_gbs_per_gpu": round(wbytes / ws / (ms * 1e-3) / 1e9, 1),
        "hbm_frac_per_gpu": round(wbytes / ws / (ms * 1e-3) / 1e9 / peak, 4),
        "collectives_per_step": 4 * shape.layers + 1 if ws > 1 else 0,
        "collective": (collective if ws > 1 else None),
        "cuda_graph": graphed,
        "act_mode": ("fp32 rows, Q4_K on the tile path (fp16 operands)" if model.tile
                     else ("x16" if act == _native.ACT_X16 else "x8")),
        "cpu_baseline": cpu,
    }
    if not graphed:
        rec["graph_error"] = err
    del model
    torch.cuda.empty_cache()
    return rec


def run_sharded_only(args, ws, rank, local):
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rec = sharded_decode_bench(dev, ws, rank, local, args.steps, args.warmup, args.batch, args.ctx, args.decode_shape,
                               args.collective)
    if rank == 0:
        print(json.dumps({"impl": "ours", **rec}), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_decode_only(args, ws, rank, local):
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    rec = decode_bench(dev, args.steps, args.warmup, args.decode_shape, args.ctx)
    if rank == 0:
        print(json.dumps({"impl": "ours", **rec}), flush=True)


def run_attention_only(args, ws, rank, local):
    """`--workload attention`: the fused decode attention alone, one JSON line."""
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    recs = attention_bench(dev, args.steps, args.warmup, ctx=args.ctx)
    if rank == 0:
        print(json.dumps({"workload": "llama3_8b_decode_attention", "impl": "ours", "cases": recs}), flush=True)


def run_tile_only(args, ws, rank, local):
    """`--workload tile`: the tile path alone (one shape/m or all), one JSON line."""
    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    shapes = TILE_SHAPES if args.tile_n is None else [(args.tile_n, args.tile_k)]
    ms = TILE_MS if args.tile_m is None else [args.tile_m]
    recs = tile_bench(dev, args.steps, args.warmup, shapes, ms, copies=args.copies)
    if rank == 0:
        print(json.dumps({"workload": "q4k_tile_matmul", "impl": "ours", "cases": recs}), flush=True)


def run_ours(args, ws, rank, local):
    import torch

    from cybel_b200 import _native
    from cybel_b200.quantized_matmul import DeviceMatrix, QuantizedMatrix, matmul_device

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    act = _native.ACT_X8 if args.act == "x8" else _native.ACT_X16
    W = _weights()
    x = np.random.default_rng(1).standard_normal(K_DIM).astype(np.float32)
    C = args.copies
    mats = [DeviceMatrix(QT_Q4_K, K_DIM, N_ROWS, W) for _ in range(C)]
    xt = torch.from_numpy(x).to(dev)
    ys = [torch.empty(N_ROWS, dtype=torch.float32, device=dev) for _ in range(C)]
    _native.lib().b200q_set_pdl(1 if args.pdl else 0)

    def step():
        for i in range(C):
            matmul_device(xt, mats[i], out=ys[i], act_mode=act)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    # One step (C matvecs; each one GEMV launch that quantizes x itself) is captured in a
    # CUDA graph, so the timed region measures the device, not Python launch
    # overhead. Warm-up on the capture stream sizes the library's scratch.
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        for _ in range(max(3, args.warmup)):
            step()
    barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        clk.mark()
        e0.record(st)
        for _ in range(args.steps):
            graph.replay()
        e1.record(st)
        clk.sample_now()  # the queued replays are still running on the device
        barrier()
    ms_total = e0.elapsed_time(e1)
    # One matvec alone (events around a single eager call, same stream).
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(4 * C)]
    for j, (a, b) in enumerate(evs):
        a.record(st)
        matmul_device(xt, mats[j % C], out=ys[j % C], act_mode=act)
        b.record(st)
    torch.cuda.synchronize(dev)
    launch_ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    del graph
    # The same chain in the other activation mode (x16 is the drop-ins'
    # default: int16 codes, within 1e-5 of the fp32-activation product).
    other = None
    if ws == 1:
        other_act = _native.ACT_X16 if act == _native.ACT_X8 else _native.ACT_X8

        def step_other():
            for i in range(C):
                matmul_device(xt, mats[i], out=ys[i], act_mode=other_act)

        with torch.cuda.stream(cap):
            for _ in range(3):
                step_other()
        barrier()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=cap):
            step_other()
        for _ in range(3):
            g2.replay()
        barrier()
        reps = max(10, args.steps // 2)
        e0.record(st)
        for _ in range(reps):
            g2.replay()
        e1.record(st)
        barrier()
        ms_o = e0.elapsed_time(e1) / (reps * C)
        gbs_o = W.nbytes / (ms_o / 1e3) / 1e9
        other = {"act_mode": "x16" if other_act == _native.ACT_X16 else "x8", "ms_per_matvec": round(ms_o, 5),
                 "weight_gbs": round(gbs_o, 1), "hbm_frac": round(gbs_o / _peak_hbm()[0], 4)}
        del g2

    t = torch.tensor([ms_total, launch_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_total, launch_ms = float(t[0]), float(t[1])

    # End to end through the public drop-in (host buffers, pinned).
    qms = [QuantizedMatrix(name=f"w{i}", qtype=QT_Q4_K, shape=(K_DIM, N_ROWS), data=W.copy()) for i in range(C)]
    xh = torch.from_numpy(x).pin_memory().numpy()
    yh = torch.empty(N_ROWS, dtype=torch.float32).pin_memory().numpy()
    import ctypes

    L = _native.lib()
    L.b200q_set_act_mode(act)
    fp = ctypes.POINTER(ctypes.c_float)
    xp, yp = xh.ctypes.data_as(fp), yh.ctypes.data_as(fp)
    ptrs = [q.ensure_packed().ctypes.data for q in qms]

    def e2e_step():
        for i in range(C):
            L.simd_matvec_q4k(xp, ptrs[i], yp, K_DIM, N_ROWS)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    assert L.b200q_last_error() == 0, L.b200q_last_error()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
    e2e_s = float(te[0])
    L.b200q_weight_cache_clear()

    wbytes = W.nbytes
    value = ws * wbytes * C * args.steps / (ms_total / 1e3) / 1e9
    e2e_val = ws * wbytes * C * args.steps / e2e_s / 1e9
    peak, peak_kind = _peak_hbm()
    # Average launch duration over the timed region (back-to-back launches,
    # overlapped by programmatic dependent launch when enabled).
    avg_launch_ms = ms_total / (C * args.steps)
    achieved = wbytes / (avg_launch_ms / 1e3) / 1e9
    cpu = _cpu_reference_sample(W, x) if (rank == 0 and ws == 1 and not args.no_cpu) else None
    del mats, ys
    torch.cuda.empty_cache()
    no_cpu = args.no_cpu or rank != 0
    c1 = c2 = None
    if ws == 1 and not args.no_sweep:
        c1 = c1_bench(dev, no_cpu)
        c2 = c2_bench(dev, no_cpu)
    tile = None
    if ws == 1 and not args.no_tile:
        tile = tile_bench(dev, max(10, args.steps // 2), args.warmup, no_cpu=no_cpu)
    decode = attention = None
    if ws == 1 and not args.no_decode:
        decode = decode_bench(dev, max(10, args.steps // 2), args.warmup, no_cpu=no_cpu)
        attention = attention_bench(dev, max(10, args.steps // 2), args.warmup)
    sharded = sharded8 = None
    if not args.no_decode:
        sharded = sharded_decode_bench(dev, ws, rank, local, 10, args.warmup, 1, 2048, "llama3_70b", "peer",
                                       no_cpu=no_cpu)
        sharded8 = sharded_decode_bench(dev, ws, rank, local, 10, args.warmup, 8, 2048, "llama3_70b", "peer",
                                        no_cpu=no_cpu)
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_total / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8 dp4a (x8)" if act == _native.ACT_X8 else "int16-in-int8x2 dp4a (x16)",
            "data": "synthetic",
            "config": {
                "workload": f"q4k_matvec_{N_ROWS}x{K_DIM}",
                "weight_bytes_per_matvec": wbytes,
                "copies_per_step": C,
                "l2": f"inputs > L2 ({C} distinct weight copies, {C * wbytes / 1e6:.0f} MB per step)",
                "act_mode": args.act,
                "pdl": bool(args.pdl),
                "step": f"{C} x GEMV (activation quantization fused in), replayed as one CUDA graph",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_source": peak_kind,
                "traffic": _traffic_per_launch(),
                # the reference engine's own byte counter adds the fp32 activation
                # and output bytes to the weight bytes (model_graph.cpp:377-389)
                "achieved_with_activation_bytes": round((wbytes + 4 * (K_DIM + N_ROWS)) / (avg_launch_ms / 1e3) / 1e9, 1),
                "avg_launch_ms": round(avg_launch_ms, 5),
                "isolated_launch_ms": round(launch_ms, 5),
            },
            "e2e": {
                "value": round(e2e_val, 2),
                "unit": "GB/s",
                "h2d_bytes_per_step": C * K_DIM * 4,
                "d2h_bytes_per_step": C * N_ROWS * 4,
            },
            "other_act_mode": other,
            "gpu_launches": C * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "c1_q4_0": c1,
            "c2_sweep": c2,
            "tile": tile,
            "decode": decode,
            "attention": attention,
            "sharded_decode": sharded,
            "sharded_decode_b8": sharded8,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--act", default="x8", choices=["x8", "x16"])
    ap.add_argument("--copies", type=int, default=8)
    ap.add_argument("--pdl", type=int, default=1)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-tile", action="store_true", help="skip the tile-path (batched matmul) summary")
    ap.add_argument("--no-decode", action="store_true", help="skip the Llama-3-8B / 70B decode-step summaries")
    ap.add_argument("--no-sweep", action="store_true", help="skip the Q4_0 and Q8_0/Q4_K shape-sweep records")
    ap.add_argument("--workload", default="gemv", choices=["gemv", "tile", "decode", "sharded", "attention"])
    ap.add_argument("--decode-shape", default=None, choices=["llama3_8b", "llama3_70b"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--collective", default="peer", choices=["peer", "nccl"])
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--tile-m", type=int, default=None)
    ap.add_argument("--tile-n", type=int, default=None)
    ap.add_argument("--tile-k", type=int, default=None)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = _dist()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if args.workload == "tile":
        run_tile_only(args, ws, rank, local)
        return
    if args.workload == "decode":
        args.decode_shape = args.decode_shape or "llama3_8b"
        run_decode_only(args, ws, rank, local)
        return
    if args.workload == "sharded":
        args.decode_shape = args.decode_shape or "llama3_70b"
        run_sharded_only(args, ws, rank, local)
        return
    if args.workload == "attention":
        run_attention_only(args, ws, rank, local)
        return
    run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
