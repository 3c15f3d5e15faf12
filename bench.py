"""Benchmark: fused GGML dequantize x matvec on B200 (the kernel microbench).

Workload (one "step"): the kernel microbench at
batch 1 -- y = W x for W in {Q8_0, Q4_K, Q5_K, Q6_K, IQ4_XS} x {4096x4096,
14336x4096, 4096x14336} (rows x cols), 15 matrices, quantized by the package's
quantizers (byte-identical to the reference's fixture encoders; IQ4_XS by the
package's own) from seeded N(0, 0.02) fp32 weights, x ~ N(0, 1) fp32.  A step
streams 492 MB of weights, far above the 126 MB L2, so every matrix is read
cold from HBM (inputs > L2; no flush needed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Metric: weight-stream throughput in GB/s (algorithmic bytes / time), summed
over ranks (weak scaling: every rank runs the whole step on its own GPU; the
path shards by independent rows / matrices with no data-path collective).
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s @bs1 + dequant-matvec HBM GB/s (% of B200 peak), 1/2/4/8 GPU"
TYPES = {"Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ4_XS": 23}
SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]  # rows x cols
SEED = 20251201


ONLY: tuple[str, int, int] | None = None  # --only TYPE:ROWSxCOLS (profiling one matrix)


def workload():
    wl = [(name, t, rows, cols) for (rows, cols) in SHAPES for name, t in TYPES.items()]
    if ONLY is not None:
        wl = [w for w in wl if (w[0], w[2], w[3]) == ONLY]
        if not wl:
            raise SystemExit(f"--only {ONLY} is not part of the workload")
    return wl


def row_bytes(t: int, cols: int) -> int:
    from pyrite_b200.ggml_types import spec  # a plain table: loads no library
    s = spec(t)
    return cols // s.block_size * s.bytes_per_block


def algo_bytes(t: int, rows: int, cols: int, ncols: int = 1) -> int:
    """Algorithmic bytes of one launch: weights once, x and y once."""
    return rows * row_bytes(t, cols) + ncols * (rows + cols) * 4


def gaussian_weights(rows: int, cols: int, seed: int) -> np.ndarray:
    """Seeded N(0, 0.02) fp32 weights (the same draw as pyrite_b200.quantize.gaussian_weights)."""
    return np.random.default_rng(seed).normal(0.0, 0.02, rows * cols).astype(np.float32)


def build_payloads(quantize=None) -> dict[tuple[int, int, int], bytes]:
    """The 15 payloads of the step.  quantize: the library's quantizer by
    default; the reference arm passes the numpy encoders (identical bytes,
    tests/test_quantize.py) so its process never loads libpyrite_b200.so."""
    if quantize is None:
        from pyrite_b200.quantize import quantize
    out = {}
    wl = workload()
    for (rows, cols) in SHAPES:
        if not any((r, c) == (rows, cols) for _, _, r, c in wl):
            continue
        w = gaussian_weights(rows, cols, SEED + rows * 31 + cols)
        for name, t, r, c in wl:
            if (r, c) == (rows, cols):
                out[(t, rows, cols)] = quantize(t, w)
    return out


def x_vectors() -> dict[int, np.ndarray]:
    rng = np.random.default_rng(SEED)
    return {cols: rng.normal(0.0, 1.0, cols).astype(np.float32) for cols in sorted({c for _, c in SHAPES})}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, polled through NVML
    (about every 2 ms) for the whole timed region."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, torch_device):
        self.dev = torch_device
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.dev)
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            busid = f"{getattr(props, 'pci_domain_id', 0):08x}:{bus:02x}:{getattr(props, 'pci_device_id', 0):02x}.0"
            try:
                return pynvml.nvmlDeviceGetHandleByPciBusId(busid)
            except pynvml.NVMLError:
                pass
        return pynvml.nvmlDeviceGetHandleByIndex(self.dev.index or 0)

    def _run(self):
        try:
            import pynvml
            h = self._handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            while not self._stop.is_set():
                clk = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                try:
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                except AttributeError:
                    rs = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((float(clk), int(rs)))
                time.sleep(0.002)
        except Exception as e:  # noqa: BLE001 - clocks are reported, not required
            self.err = repr(e)

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        time.sleep(0.05)  # first sample before the timed region starts
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self.thread.join(timeout=5)

    def summary(self) -> dict:
        sm = [c for c, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
               "reasons": reasons, "samples": len(sm), "source": "nvml"}
        if self.err:
            out["error"] = self.err
        return out


# ---------------------------------------------------------------- helpers
def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def ncu_traffic(kernel_key: str) -> float | None:
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.is_file():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_key)
    except ValueError:
        return None


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


# ---------------------------------------------------------------- our arm
def run_ours(args) -> None:
    import torch

    from pyrite_b200 import _lib
    from pyrite_b200.kernels import cuda as K

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    lib = _lib.require()
    payloads = build_payloads()
    xs = x_vectors()
    wl = workload()
    W = {key: torch.frombuffer(bytearray(p), dtype=torch.uint8).to(dev) for key, p in payloads.items()}
    X = {c: torch.from_numpy(v).to(dev) for c, v in xs.items()}
    Y = {(t, r, c): torch.empty(r, dtype=torch.float32, device=dev) for _, t, r, c in wl}
    step_bytes = sum(algo_bytes(t, r, c) for _, t, r, c in wl)
    stream = torch.cuda.Stream(device=dev)

    WS = {c: torch.empty(K.workspace_size(0, c) + 256, dtype=torch.uint8, device=dev) for c in X}

    def step():
        # one encoding of each activation, shared by the five formats of its shape
        # (as Q/K/V or gate/up share their input in a decode step)
        px = {c: K.prepare_x(X[c], workspace=WS[c]) for c in X}
        for _, t, r, c in wl:
            K.matvec_prepared(t, W[(t, r, c)], px[c], r, c, out=Y[(t, r, c)], static_weights=True)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    if K.status() != 0:
        raise SystemExit("device status word set: a kernel wait timed out")

    # capture one step in a CUDA graph (launch overhead out of the timed loop)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        step()  # warm (function attributes set before capture)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
    if pg:
        pg.barrier()
    ms = start.elapsed_time(end)
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * step_bytes / (ms_per_step * 1e-3) / 1e9

    strong = strong_leg(dev, W, X, Y, wl, stream, pg, world, rank, args.steps, args.warmup) if pg else None

    # ---- per-kernel live timing: each matrix alone, rotating over copies so every
    # launch reads cold HBM (copies total > 4 x L2), timed with events on its stream
    per_kernel = []
    if rank == 0:
        for name, t, r, c in wl:
            size = r * row_bytes(t, c)
            copies = max(3, -(-512 * 2**20 // size))
            src = W[(t, r, c)]
            bufs = [src.clone() for _ in range(copies)]
            reps = 2
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                px = K.prepare_x(X[c], workspace=WS[c])
                with torch.cuda.graph(g, stream=stream):
                    for _ in range(reps):
                        for b in bufs:
                            K.matvec_prepared(t, b, px, r, c, out=Y[(t, r, c)], static_weights=True)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
            gbs = algo_bytes(t, r, c) / (us * 1e-6) / 1e9
            per_kernel.append({"type": name, "rows": r, "cols": c, "us": round(us, 3), "GBps": round(gbs, 1)})
            del g, bufs
            torch.cuda.empty_cache()

    # ---- end to end through the reference-facing C ABI (pyrite_matvec):
    # host payload + host fp64 x in, host fp64 y out, H2D/D2H inside the timing
    e2e = None
    if rank == 0 and not args.no_e2e:
        import ctypes
        pd = ctypes.POINTER(ctypes.c_double)
        host = {key: torch.frombuffer(bytearray(p), dtype=torch.uint8).pin_memory() for key, p in payloads.items()}
        xd = {c: np.ascontiguousarray(v, dtype=np.float64) for c, v in xs.items()}
        yd = {(t, r, c): np.zeros(r) for _, t, r, c in wl}

        def e2e_step():
            for _, t, r, c in wl:
                hb = host[(t, r, c)]
                rc = lib.pyrite_matvec(t, hb.data_ptr(), hb.numel(), xd[c].ctypes.data_as(pd),
                                       yd[(t, r, c)].ctypes.data_as(pd), r, c)
                if rc != 0:
                    raise SystemExit(f"pyrite_matvec failed ({rc})")
        e2e_step()
        t0 = time.perf_counter()
        e2e_steps = max(1, min(args.steps, 5))
        for _ in range(e2e_steps):
            e2e_step()
        dt = (time.perf_counter() - t0) / e2e_steps
        h2d = sum(len(payloads[(t, r, c)]) + c * 8 for _, t, r, c in wl)
        d2h = sum(r * 8 for _, t, r, c in wl)
        e2e = {"value": round(step_bytes / dt / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "api": "pyrite_matvec (reference-compatible C ABI, fp64 host buffers, "
               "payload copied to HBM every call; pinned host payload)", "ms_per_step": round(dt * 1e3, 3),
               "steps": e2e_steps}

    ours_y = {k: v.cpu().numpy() for k, v in Y.items()} if rank == 0 else None
    cpu = (cpu_baseline(payloads, xs, wl, budget_s=args.cpu_seconds, ours=ours_y)
           if (rank == 0 and not args.no_cpu) else None)
    decode = decode_leg(dev) if (rank == 0 and not args.no_decode) else None
    batched = batched_leg(dev, W, X, wl, stream) if (rank == 0 and not args.no_batched) else None
    # one GPU only: under torchrun the other ranks already wait in the model
    # legs' first collective while rank 0 runs its single-GPU legs
    types = types_leg(dev, stream) if (rank == 0 and world == 1 and not args.no_types) else None
    del W, X, Y
    torch.cuda.empty_cache()
    models = None
    if not args.no_models:  # every rank takes part (tensor parallel when world > 1)
        models = {}
        for which in ("c3", "c4", "c5"):
            parity = golden_parity(dev, which, world, rank, pg)
            models[which] = model_leg(dev, which, world, rank, pg)
            models[which]["parity"] = parity
            torch.cuda.empty_cache()

    if rank == 0:
        peak, peak_kind = measured_peak()
        dom = max(per_kernel, key=lambda k: k["us"])
        dom_bytes = algo_bytes(TYPES[dom["type"]], dom["rows"], dom["cols"])
        achieved = dom_bytes / (dom["us"] * 1e-6) / 1e9
        key = f"mv_tile_kernel<{dom['type']}>@{dom['rows']}x{dom['cols']}"
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "u8 codes, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) fp32 weights quantized by pyrite_b200.quantize; x ~ N(0,1)",
            "config": {"workload": "configs[1] kernel microbench, batch 1: {Q8_0,Q4_K,Q5_K,Q6_K,IQ4_XS} x "
                                   "{4096x4096,14336x4096,4096x14336}, 15 matvecs per step",
                       "global_batch": 1, "ncols": 1, "step_bytes": step_bytes,
                       "l2": "inputs larger than L2 (492 MB of weights per step vs 126 MB L2)",
                       "parallelism": f"replica x{world} (weak)", "launch": "CUDA graph: 3 x-encodings + 15 matvecs, PDL"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                         "kernel": key, "algorithmic_bytes_per_launch": dom_bytes,
                         "traffic": ncu_traffic(key)},
            "whole_step_frac_of_peak": round(value / world / peak, 4),
            "strong": strong,
            "kernels": per_kernel,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "decode": decode,
            "batched": batched,
            "types": types,
            "models": models,
            "gpu_launches": args.steps * (len(wl) + len({c for _, _, _, c in wl})),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


# ---------------------------------------------------------------- strong-scaling leg (N > 1)
def strong_leg(dev, W, X, Y, wl, stream, pg, world: int, rank: int, steps: int, warmup: int) -> dict:
    """The same step with every matrix's rows split over the GPUs (rank k
    multiplies rows [k r / N, (k + 1) r / N), the row range of the reference's
    executor call, executor.py:481-509) and the outputs assembled on every GPU
    by one NCCL all_gather of all matrices' row slices: total work fixed as N
    grows.  Time: CUDA events around `steps` replays of one graph, max over
    ranks.  The gathered rows must equal the one-GPU rows bit for bit (any row
    partition gives the same bits)."""
    import torch

    from pyrite_b200.kernels import cuda as K
    offs, total, parts = {}, 0, {}
    for _, t, r, c in wl:
        offs[(t, r, c)] = total
        total += r // world
    local = torch.empty(total, device=dev)            # this rank's rows of every matrix
    gathered = torch.empty(world * total, device=dev)  # rank-major: every rank's rows
    for _, t, r, c in wl:
        rr, rb = r // world, row_bytes(t, c)
        o = offs[(t, r, c)]
        parts[(t, r, c)] = (W[(t, r, c)][rank * rr * rb:(rank + 1) * rr * rb], local[o:o + rr], rr)
    WS = {c: torch.empty(K.workspace_size(0, c) + 256, dtype=torch.uint8, device=dev) for c in X}

    def step():
        px = {c: K.prepare_x(X[c], workspace=WS[c]) for c in X}
        for _, t, r, c in wl:
            w, yl, rr = parts[(t, r, c)]
            K.matvec_prepared(t, w, px[c], rr, c, out=yl, static_weights=True)
        pg.all_gather_into_tensor(gathered, local)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    pg.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    g = gathered.view(world, total)
    same = int(all(torch.equal(g[:, offs[k]:offs[k] + k[1] // world].reshape(-1), Y[k]) for k in offs))
    same = torch.tensor([same], device=dev)
    pg.all_reduce(same, op=pg.ReduceOp.MIN)
    ms = float(t.item())
    step_bytes = sum(algo_bytes(t_, r, c) for _, t_, r, c in wl)
    del graph
    return {"value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 5),
            "n_gpus": world, "scaling": "strong", "steps": steps,
            "parallelism": f"rows of every matrix split over {world} GPUs, one NCCL all_gather of all row slices",
            "rows_bit_identical_to_one_gpu": bool(same.item())}


# ---------------------------------------------------------------- batched leg
def batched_leg(dev, W, X, wl, stream, ncols_list=(8, 64)) -> dict:
    """configs[1] at 8 and 64 columns: the tensor-core path (tcgen05).  Each
    matrix rotates over > 512 MB of weight copies inside one CUDA graph, so
    every launch reads cold HBM; timed with CUDA events on its stream.  Work
    per launch: 2 rows cols ncols flops (tensor roofline against the measured
    bf16 peak) and rows x row_bytes weight bytes."""
    import torch

    from pyrite_b200.kernels import cuda as K
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").is_file() else {}
    tflops_peak = float(peaks.get("bf16_tflops", 1590.0))
    tflops_kind = "measured bf16_tflops (burst)" if "bf16_tflops" in peaks else "fallback bf16 1590 TFLOP/s (burst)"
    rows_out, tot_flops, tot_us = [], 0.0, 0.0
    for ncols in ncols_list:
        for name, t, r, c in wl:
            src = W[(t, r, c)]
            copies = max(3, -(-512 * 2**20 // src.numel()))
            bufs = [src.clone() for _ in range(copies)]
            gen = torch.Generator(device=dev).manual_seed(ncols)
            x = torch.randn(ncols, c, device=dev, generator=gen)
            y = torch.empty(ncols, r, device=dev)
            ws = torch.empty(K.workspace_size(t, c, ncols) + 256, dtype=torch.uint8, device=dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                K.matvec(t, bufs[0], x, r, c, out=y, workspace=ws)
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=stream):
                    for b in bufs:
                        K.matvec(t, b, x, r, c, out=y, workspace=ws, static_weights=True)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(2):
                    g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (2 * copies)
            fl = 2.0 * r * c * ncols
            rows_out.append({"type": name, "rows": r, "cols": c, "ncols": ncols, "us": round(us, 2),
                             "TFLOPs": round(fl / us / 1e6, 1),
                             "weight_GBps": round(r * row_bytes(t, c) / us / 1e3, 1)})
            tot_flops += fl
            tot_us += us
            del g, bufs
            torch.cuda.empty_cache()
    if K.status() != 0:
        raise SystemExit("device status word set during the batched leg")
    dom = max((k for k in rows_out if k["ncols"] == max(ncols_list)), key=lambda k: k["us"])
    dom_tf = dom["TFLOPs"]
    return {"config": "configs[1] at ncols 8 and 64: 15 matrices each, tcgen05 split-bf16 path",
            "kernels": rows_out,
            "aggregate_TFLOPs": round(tot_flops / tot_us / 1e6, 1),
            "roofline": {"bound": "tensor", "kernel": f"mm_tc_kernel<{dom['type']}>@{dom['rows']}x{dom['cols']}"
                                                      f"x{dom['ncols']}",
                         "achieved": dom_tf, "peak": tflops_peak, "unit": "TFLOP/s",
                         "frac": round(dom_tf / tflops_peak, 4), "peak_kind": tflops_kind,
                         "flops": "2 rows cols ncols per launch (algorithmic; the split-bf16 scheme issues 4x)"}}


# ---------------------------------------------------------------- the other decodable types
OTHER_TYPES = {"Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_1": 9, "IQ4_NL": 20, "Q2_K": 10, "Q3_K": 11,
               "F16": 1, "BF16": 30, "F32": 0}


def other_payload(t: int, rows: int, cols: int, seed: int) -> bytes:
    """Seeded N(0, 0.02) weights in format t: the package's quantizer where it
    has one, a plain cast for the float formats, and seeded random blocks with
    finite scales (tests/payloads.py) for Q8_1, which has no encoder here (the
    bytes streamed per row are the same either way)."""
    from pyrite_b200.quantize import quantize, quantize_types
    w = gaussian_weights(rows, cols, seed)
    if t in quantize_types():
        return quantize(t, w)
    if t == 0:
        return w.tobytes()
    if t == 1:
        return w.astype(np.float16).tobytes()
    if t == 30:
        return (w.view(np.uint32) >> 16).astype(np.uint16).tobytes()
    from tests.payloads import random_payload
    return random_payload(t, rows, cols, seed=seed)


def types_leg(dev, stream, shapes=((14336, 4096), (4096, 14336))) -> dict:
    """Batch-1 throughput of every other decodable type on the large configs[1]
    shapes, timed like the step's per-kernel lines (each matrix rotating over
    > 512 MB of copies inside one CUDA graph, events on its stream).  Q4_0,
    Q4_1, Q5_0, Q5_1, Q8_1, IQ4_NL, Q2_K and Q3_K run the tile kernel; the
    float formats the warp-per-row kernel."""
    import torch

    from pyrite_b200.kernels import cuda as K
    out = []
    for (r, c) in shapes:
        x = torch.from_numpy(np.random.default_rng(SEED + c).normal(0.0, 1.0, c).astype(np.float32)).to(dev)
        y = torch.empty(r, dtype=torch.float32, device=dev)
        ws = torch.empty(K.workspace_size(0, c) + 256, dtype=torch.uint8, device=dev)
        for name, t in OTHER_TYPES.items():
            src = torch.frombuffer(bytearray(other_payload(t, r, c, SEED + 7 * t + r)), dtype=torch.uint8).to(dev)
            copies = max(3, -(-512 * 2**20 // src.numel()))
            bufs = [src.clone() for _ in range(copies)]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                px = K.prepare_x(x, workspace=ws)
                K.matvec_prepared(t, bufs[0], px, r, c, out=y, static_weights=True)
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=stream):
                    for _ in range(2):
                        for b in bufs:
                            K.matvec_prepared(t, b, px, r, c, out=y, static_weights=True)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (2 * copies)
            out.append({"type": name, "rows": r, "cols": c, "us": round(us, 3),
                        "GBps": round(algo_bytes(t, r, c) / (us * 1e-6) / 1e9, 1),
                        "kernel": "mv_tile_kernel" if t in (2, 3, 6, 7, 9, 10, 11, 20) else "mv_generic_kernel"})
            del g, bufs, src
            torch.cuda.empty_cache()
    if K.status() != 0:
        raise SystemExit("device status word set during the types leg")
    return {"config": "batch 1, every other decodable type at 14336x4096 and 4096x14336, cold HBM per launch",
            "kernels": out}


# ---------------------------------------------------------------- greedy parity of the model legs
# 2-layer full-width checkpoints, 120-token prompt + 8 greedy tokens (a 128-position window)
GOLDEN_2L = {"c3": "c3_2l_w128.json", "c4": "moe_c4_2l_w128.json", "c5": "moe_c5_2l_w128.json"}


def golden_parity(dev, which: str, world: int = 1, rank: int = 0, pg=None) -> dict:
    """The leg's architecture at full width with 2 layers, decoded on the same
    GPUs in the same way (tensor parallel when world > 1), against the greedy
    ids the reference executor produced for that checkpoint (tests/golden)."""
    from dataclasses import fields

    import torch

    from pyrite_b200.model import MixedDecoder
    from pyrite_b200.synthetic import DenseSpec, MoESpec
    g = json.loads((ROOT / "tests" / "golden" / GOLDEN_2L[which]).read_text())
    cls = MoESpec if g["spec"]["architecture"] == "qwen3moe" else DenseSpec
    spec = cls(**{k: v for k, v in g["spec"].items() if k in {f.name for f in fields(cls)}})
    if world > 1:
        from pyrite_b200.sharded import ShardedDecoder
        dec = ShardedDecoder.synthetic(spec, rank, world, device=dev, max_ctx=256)
    else:
        dec = MixedDecoder.synthetic(spec, device=dev, max_ctx=256)
    prompt, want = g["prompt"], g["generated"]
    got = dec.generate(prompt, len(want))[len(prompt):]
    dec.graph = None  # graphs holding NCCL calls go before the process group does
    if pg:
        pg.barrier()
        dec.close()
    del dec
    torch.cuda.empty_cache()
    return {"golden": f"tests/golden/{GOLDEN_2L[which]}", "layers": 2, "prompt_tokens": len(prompt),
            "generated_tokens": len(want), "greedy_ids_match": got == want,
            "decoded_as": f"tensor parallel x{world}" if world > 1 else "one GPU"}


# ---------------------------------------------------------------- model legs
def model_leg(dev, which: str, world: int = 1, rank: int = 0, pg=None) -> dict:
    """Batch-1 decode throughput of a full-depth configs[2] (Llama-3-8B Q4_K_M),
    configs[3] (Qwen3-30B-A3B Q4_K_M MoE) or configs[4] (Qwen3-235B-A22B
    Q4_K_M MoE, ~142 GB) model: the prompt is processed one
    token at a time (as the reference does), then greedy decode; one CUDA graph
    per step, CUDA events around the decode steps.  Layer weights: layers 0 and
    1 are generated from their seeds, every other layer holds its own HBM copy
    of layer (i % 2)'s bytes (generating 8-30 B seeded values on the host would
    take minutes; the bytes streamed per token are the same).  Parity for these
    architectures is tested on 2-layer full-width models against the reference.
    With several GPUs the model is split tensor-parallel over them
    (pyrite_b200.sharded: heads / rows / experts by id, a one-kernel NVLink sum
    after the output and down projections); the time is the max over ranks."""
    import time as _t

    import torch

    from pyrite_b200.model import MixedDecoder
    from pyrite_b200.synthetic import DenseSpec, MoESpec, prompt_ids

    if which == "c3":
        spec, prefill, new, ctx = DenseSpec.c3(), 512, 128, 4096
        cfg = ("configs[2]: Llama-3-8B-shaped, Q4_K_M mix, 32 layers, prefill 512 seeded tokens (blocks of 64 on one "
               "GPU, one per step tensor parallel), batch-1 decode of 128 tokens, KV ctx 4096")
    elif which == "c4":
        spec, prefill, new, ctx = MoESpec.c4(), 256, 128, 1024
        cfg = ("configs[3]: Qwen3-30B-A3B-shaped MoE, Q4_K_M mix, 48 layers, 128 experts top-8, prefill 256 "
               "seeded tokens (one per step), batch-1 decode of 128 tokens")
    else:
        spec, prefill, new, ctx = MoESpec.c5(), 1024, 256, 8192
        cfg = ("configs[4]: Qwen3-235B-A22B-shaped MoE, Q4_K_M mix (~142 GB), 94 layers, 64 q / 4 kv heads, "
               "128 experts top-8, expert ffn 1536, prefill 1024 seeded tokens (one per step), batch-1 decode of "
               "256 tokens, KV ctx 8192")
    t0 = _t.time()
    if world > 1:
        from pyrite_b200.sharded import ShardedDecoder
        dec = ShardedDecoder.synthetic(spec, rank, world, device=dev, max_ctx=ctx, replicate=True)
    else:
        dec = MixedDecoder.synthetic(spec, device=dev, max_ctx=ctx, replicate=True)
    built = _t.time() - t0
    prompt = prompt_ids(spec, n=prefill)
    dec.reset(prompt)
    dec.capture()
    dec.reset(prompt)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    batched = dec.batched_prefill  # dense, one GPU: the prompt in 64-position blocks on the tensor cores
    if batched:
        dec.prefill(prompt, 64)  # warm: buffers and kernel attributes
        torch.cuda.synchronize(dev)
    e0.record(stream)
    if batched:
        dec.prefill(prompt, 64)
    else:
        dec.run_steps(prefill - 1)
    e1.record(stream)
    dec.run_steps(new)
    e2.record(stream)
    torch.cuda.synchronize(dev)
    from pyrite_b200.kernels import cuda as K
    if K.status() != 0:
        raise SystemExit(f"device status word set during the {which} model leg")
    times = torch.tensor([e1.elapsed_time(e2), e0.elapsed_time(e1)], device=dev)
    h = spec.hidden_size
    per_layer = [ly.qk.data.numel() + ly.v.data.numel() + ly.o.data.numel() for ly in dec.layers]
    if dec.moe:  # the selected experts' slices (each GPU holds E / world of them)
        k = spec.num_experts_per_tok
        held = spec.num_experts // world
        per_layer = [a + ly.router.data.numel() // world
                     + k * sum(m.data.numel() for m in (ly.gate_exps, ly.up_exps, ly.gate_up_exps, ly.down_exps)
                               if m is not None) // (held * world)
                     for a, ly in zip(per_layer, dec.layers)]
    else:
        per_layer = [a + (ly.gate_up.data.numel() if ly.gate_up is not None else
                          ly.gate.data.numel() + ly.up.data.numel()) + ly.down.data.numel()
                     for a, ly in zip(per_layer, dec.layers)]
    mine = torch.tensor([float(sum(per_layer) + dec.lm_head.data.numel() + h * 4 // world)], device=dev,
                        dtype=torch.float64)
    if pg:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
        pg.all_reduce(mine)
    active = float(mine.item())
    ms_tok = float(times[0].item()) / new
    pre_ms = float(times[1].item())
    dec.graph = None  # graphs holding NCCL calls go before the process group does
    if pg:  # the NVLink sum's peer mappings, after every rank's last step
        pg.barrier()
        dec.close()
    batch16 = None
    if which == "c4" and world == 1:  # configs[3] also decodes 16 sequences at once
        del dec
        torch.cuda.empty_cache()
        batch16 = batch_leg(dev, spec, prefill, new)
    out = {"config": cfg, "decode_tok_s": round(1000.0 / ms_tok, 1), "ms_per_token": round(ms_tok, 4),
           "prefill_tok_s": round((prefill - 1) * 1000.0 / pre_ms, 1),
           "prefill": ("blocks of 64 positions, projections on the tensor cores (MixedDecoder.prefill)" if batched
                       else "one position per step, as the reference"),
           "n_gpus": world, "parallelism": f"tensor parallel x{world}" if world > 1 else "one GPU",
           "active_weight_bytes_per_token": int(active),
           "weight_GBps": round(active / (ms_tok * 1e-3) / 1e9, 1),
           "hbm_frac_of_measured": round(active / (ms_tok * 1e-3) / 1e9 / (measured_peak()[0] * world), 4),
           "weights": "layers 0-1 generated from seeds (N(0,0.02) quantized), deeper layers: own HBM copies of them",
           "host_build_seconds": round(built, 1)}
    if batch16 is not None:
        out["batch16"] = batch16
    else:
        del dec
    return out


def batch_leg(dev, spec, prefill: int, new: int, batch: int = 16) -> dict:
    """configs[3] at batch 16: 16 sequences (seeded prompts of `prefill` ids)
    decoded together (pyrite_b200.batch.BatchDecoder: one multi-column product
    per projection for all sequences, per-row routing, every (sequence,
    expert) selection in one launch); the prompts run one position per step for
    all sequences at once.  CUDA events around the decode steps."""
    import torch

    from pyrite_b200.batch import BatchDecoder
    dec = BatchDecoder.synthetic(spec, device=dev, max_ctx=prefill + new, batch=batch, replicate=True)
    rng = np.random.default_rng(SEED + batch)
    prompts = [list(map(int, rng.integers(0, spec.vocab_size, prefill))) for _ in range(batch)]
    dec.breset(prompts)
    dec.bcapture()
    dec.breset(prompts)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(stream)
    dec.brun_steps(prefill - 1)
    e1.record(stream)
    dec.brun_steps(new)
    e2.record(stream)
    torch.cuda.synchronize(dev)
    dec.check_status()
    ms_tok = e1.elapsed_time(e2) / new
    out = {"batch": batch, "decode_tok_s": round(batch * 1000.0 / ms_tok, 1), "ms_per_step": round(ms_tok, 4),
           "prefill_tok_s": round(batch * (prefill - 1) * 1000.0 / e0.elapsed_time(e1), 1),
           "note": "16 seeded prompts of equal length; tok/s counts every sequence's tokens"}
    del dec
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------- decode leg
def decode_leg(dev, reps: int = 5) -> dict:
    """configs[0] decode tok/s: the Qwen3-0.6B-shaped Q8_0 model, 16-token
    prompt processed one token at a time (as the reference does), then 8 greedy
    tokens; the step is one CUDA graph replayed per token.  Timed with CUDA
    events: decode = the 8 generated tokens' steps."""
    import torch

    from pyrite_b200.dense import DenseDecoder
    from pyrite_b200.synthetic import DenseSpec, prompt_ids

    spec = DenseSpec.c1()
    dec = DenseDecoder.synthetic(spec, device=dev, max_ctx=512)
    prompt, new = prompt_ids(spec), 8
    ids = dec.generate(prompt, new)  # capture + warm
    stream = torch.cuda.current_stream(dev)
    pre_ms, dec_ms = [], []
    for _ in range(reps):
        dec.reset(prompt)
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        dec.run_steps(len(prompt) - 1)   # prompt positions 0..14
        e1.record(stream)
        dec.run_steps(new)               # position 15 (first new token) .. 22
        e2.record(stream)
        torch.cuda.synchronize(dev)
        pre_ms.append(e0.elapsed_time(e1))
        dec_ms.append(e1.elapsed_time(e2))
    weights = sum(t.numel() for ly in dec.layers for t in (ly.qkv, ly.o, ly.gate_up, ly.down)) + dec.lm_head.numel()
    ms_tok = statistics.median(dec_ms) / new
    golden = ROOT / "tests" / "golden" / "c1_decode.json"
    ref = json.loads(golden.read_text()) if golden.is_file() else {}
    return {"config": "configs[0]: Qwen3-0.6B-shaped, 28 layers, Q8_0, vocab 151936 tied, 16-token prompt, "
                      "8 greedy tokens, KV 512, batch 1",
            "decode_tok_s": round(1000.0 / ms_tok, 1), "ms_per_token": round(ms_tok, 4),
            "prefill_tok_s": round((len(prompt) - 1) * 1000.0 / statistics.median(pre_ms), 1),
            "weight_bytes_per_token": weights,
            "weight_GBps": round(weights / (ms_tok * 1e-3) / 1e9, 1),
            "generated": ids[len(prompt):],
            "greedy_matches_reference": ids[len(prompt):] == ref.get("generated"),
            "reference_tok_s_cpu": round(ref["reference_tokens_per_second"], 3) if ref else None,
            "reference_note": "reference DenseExecutor (fp64 Python + native C kernels), 24 forward passes "
                              "incl. the sequential prompt, timed when the golden file was made "
                              "(tests/golden/make_c1_golden.py, 8-core build host)"}


# ---------------------------------------------------------------- CPU baseline
def _ref_kernel():
    from oracle import oracle as O
    if O.reference_lib() is None:
        try:
            O.build()
        except Exception:  # noqa: BLE001
            pass
    if O.reference_lib() is not None:
        return O.reference_matvec, "reference"
    return O.matvec, "port"


def cpu_baseline(payloads, xs, wl, budget_s: float = 12.0, threads: int = 1, ours=None) -> dict:
    """Reference C kernel (oracle/_ref, built from pyrite/kernels/native.c) on the
    host cores: a bounded sample -- the first rows of each of the 15 matrices,
    about budget_s / 15 seconds each -- timed single threaded (the reference
    kernel is scalar and single threaded).  ours: this build's outputs of the
    same step (rows x 1 arrays per matrix); the sampled rows are then also a
    parity check, reported as the largest error relative to sum |w x| (the
    oracle's decoded weights), outside any timed region."""
    from oracle import oracle as O
    fn, kind = _ref_kernel()
    total_b, total_t = 0, 0.0
    per = budget_s / len(wl)
    rows_done = {}
    worst, worst_at = 0.0, None
    for name, t, r, c in wl:
        rb = row_bytes(t, c)
        x64 = xs[c].astype(np.float64)
        # calibrate with 8 rows, then size the sample to ~per seconds
        t0 = time.perf_counter()
        fn(t, payloads[(t, r, c)][: 8 * rb], x64, 8, c)
        dt8 = max(time.perf_counter() - t0, 1e-6)
        n = int(min(r, max(8, 8 * per / dt8)))
        t0 = time.perf_counter()
        want = fn(t, payloads[(t, r, c)][: n * rb], x64, n, c)
        dt = time.perf_counter() - t0
        total_b += n * rb + (n + c) * 4
        total_t += dt
        rows_done[f"{t}:{r}x{c}"] = n
        if ours is not None:
            w = O.dequantize_rows(t, payloads[(t, r, c)][: n * rb], n, c)
            bound = np.abs(w) @ np.abs(x64)
            err = float(np.max(np.abs(np.asarray(ours[(t, r, c)][:n], dtype=np.float64) - want) /
                               np.maximum(bound, 1e-30)))
            if err >= worst:
                worst, worst_at = err, f"{name} {r}x{c}"
    full = all(rows_done[f"{t}:{r}x{c}"] == r for _, t, r, c in wl)
    what = ("all rows of all 15 matrices (the whole step)" if full else
            f"the first rows of each of the 15 matrices ({sum(rows_done.values())} rows, ~{per:.1f} s each)")
    out = {"value": round(total_b / total_t / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": kind,
           "sample": f"{what}, single thread, fp64 as the reference computes", "seconds": round(total_t, 2)}
    if ours is not None:
        out["parity"] = {"max_rel_err": worst, "worst_matrix": worst_at, "tolerance": 1e-4, "ok": worst <= 1e-4,
                         "against": f"{kind} kernel outputs on the sampled rows, relative to sum |w x|"}
    return out


def run_reference(args) -> None:
    """Reference arm: the reference's own CPU kernel (oracle/_ref, compiled from
    pyrite/kernels/native.c) on this box's host cores, over the same workload
    as ours -- every row of all 15 matrices per step -- with each matrix split
    into one contiguous row range per host thread (ctypes releases the GIL
    during the call).  Inputs come from the numpy encoders, so this process
    loads none of this build's libraries."""
    world, rank, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor

    from oracle import encoders
    fn, kind = _ref_kernel()
    payloads = build_payloads(encoders.quantize)
    xs = x_vectors()
    wl = workload()
    threads = os.cpu_count() or 1
    jobs = []
    for _, t, r, c in wl:
        rb = row_bytes(t, c)
        x64 = xs[c].astype(np.float64)
        buf = memoryview(payloads[(t, r, c)])
        for i in range(threads):
            a, b = r * i // threads, r * (i + 1) // threads
            if b > a:
                jobs.append((t, buf[a * rb:b * rb], x64, b - a, c))
    step_bytes = sum(algo_bytes(t, r, c) for _, t, r, c in wl)

    def step(pool):
        list(pool.map(lambda j: fn(*j), jobs))

    with ThreadPoolExecutor(threads) as pool:
        for _ in range(args.warmup):
            step(pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step(pool)
        dt = (time.perf_counter() - t0) / args.steps
    value = step_bytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp64", "data": "synthetic (the same payloads as ours)",
        "config": {"workload": "configs[1] kernel microbench, batch 1: {Q8_0,Q4_K,Q5_K,Q6_K,IQ4_XS} x "
                               "{4096x4096,14336x4096,4096x14336}, 15 matvecs per step, every row",
                   "global_batch": 1, "ncols": 1, "step_bytes": step_bytes, "same_config": True,
                   "parallelism": f"{threads} host threads, one contiguous row range per thread per matrix"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": "the whole step (all rows of the 15 matrices) every step"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the configs[0] decode tok/s leg")
    ap.add_argument("--no-batched", action="store_true", help="skip the 8- and 64-column tensor-core leg")
    ap.add_argument("--no-models", action="store_true", help="skip the configs[2] / configs[3] decode legs")
    ap.add_argument("--no-types", action="store_true", help="skip the batch-1 leg of the other decodable types")
    ap.add_argument("--only", help="profile one matrix of the workload, e.g. Q4_K:14336x4096")
    args = ap.parse_args()
    if args.only:
        global ONLY
        name, shape = args.only.split(":")
        r, c = shape.lower().split("x")
        ONLY = (name, int(r), int(c))
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
