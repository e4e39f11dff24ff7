"""Benchmark of the activation-compression hot path (one JSON line on stdout).

Workload (one B200 per rank, weak scaling): each rank
holds its own 16384-token shard of a LLaMA-7B-shaped MLP activation
X (16384 x 4096 bf16, rank-64 signal + 0.05 N(0,1) noise + 16 outlier
channels x30, seed = rank), compressed with r = 32, k = 16, int4, group 64.

One step = encode X + decode X^ (the channel-group kernels through the C ABI,
inputs resident in HBM).  ``value`` = algorithmic bytes of all ranks' steps /
max-over-ranks device time, in GB/s.  Per-component numbers (encode, decode,
fused SiLU backward on the 16384 x 11008 input, fused dequant-dW GEMM of
config 4 in TFLOP/s) ride along under "components".

``--impl reference`` times the reference's algorithm on the host cores
instead (the oracle port in oracle/, all threads, bounded sample).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "triton-kernel-test_b200"))

METRIC = "encode/decode GB/s of bf16 activation vs HBM peak; fused dequant-dW GEMM TFLOPS"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------- algorithmic work
def packed_bytes_per_row(H, bits, group, rank, k):
    """codes + float32 group scales + float32 projection L + bf16 outlier values."""
    return H * bits // 8 + (H // group) * 4 + 4 * rank + 2 * k


def basis_bytes(H, rank):
    """The bf16 basis, read once."""
    return rank * H * 2


def encode_bytes(T, H, bits, group, rank, k):
    """Read X once, write every packed buffer once, read the basis once."""
    return T * (2 * H + packed_bytes_per_row(H, bits, group, rank, k)) + basis_bytes(H, rank)


decode_bytes = encode_bytes  # the same buffers, the other way round


def consumer_bytes(T, H, bits, group, rank, k):
    """Read the packed activation and dY, write dX."""
    return T * (4 * H + packed_bytes_per_row(H, bits, group, rank, k)) + basis_bytes(H, rank)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 10 ms by a
    thread while the timed regions run.  Read-only NVML queries (nvidia-ml-py);
    the device is matched to the CUDA device by UUID.  Falls back to
    ``nvidia-smi -lms`` when NVML is not importable."""

    NAMES = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
             "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.samples = []  # (sm_mhz, reasons bitmask)
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._active = 0

    def __enter__(self):
        import threading

        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.device_index).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons",
                                  getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        except Exception:  # no NVML: nothing to sample with
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                if self._active:
                    try:
                        self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                             int(get_reasons(h)) if get_reasons else 0))
                    except Exception:
                        pass
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def timed(self):
        """Context manager marking a timed region (samples are kept only inside)."""
        sampler = self

        class _T:
            def __enter__(self_):
                sampler._active += 1

            def __exit__(self_, *exc):
                sampler._active -= 1

        return _T()

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        reasons = sorted(n for n, bit in self.NAMES.items() if any(r & bit for _, r in self.samples))
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------- distributed plumbing
def dist_setup(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gather_all(x, world):
    """x from every rank, in rank order (a list)."""
    import torch

    if world == 1:
        return [x]
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(v.item()) for v in out]


def allreduce_max(x, world):
    import torch

    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


class _Done:
    """A finished handle (wait() returns at once) for time_copy."""

    def wait(self):
        pass


# ---------------------------------------------------------------- timing
class L2Flush:
    """Between timed steps: a 256 MB write, then a 256 MB read of another
    buffer.  The write evicts every line of the step's inputs; the read then
    evicts the write's dirty lines, so that their write-back to HBM happens
    here and not inside the next timed step."""

    def __init__(self, dev):
        import torch

        self.w = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        self.r = torch.ones(64 * 1024 * 1024, dtype=torch.int32, device=dev)

    def __call__(self):
        self.w.zero_()
        self.r.max()


def time_steps(fn, steps, warmup, flush, world, clk=None, detail=None):
    """Warm up, then time exactly `steps` calls of fn, each bracketed by CUDA
    events on the current stream, with an L2 flush (L2Flush: a 256 MB write,
    then a 256 MB read) between calls outside the events.  Returns per-step ms
    (mean) as max over ranks."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    evs = []
    with (clk.timed() if clk is not None else contextlib.nullcontext()):
        for _ in range(steps):
            flush()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    ranks = gather_all(ms, world)
    if detail is not None:
        detail["per_rank_ms"] = ranks
    return max(ranks)


# ---------------------------------------------------------------- CPU baseline (oracle port)
def cpu_baseline(T_sample, H, bits, group, rank, k, reps_seconds=10.0, max_reps=40):
    """The reference's algorithm restated in oracle/ (C, OpenMP over tokens),
    encode + decode of a T_sample-token slice of the config-2 activation."""
    import numpy as np

    # all host cores (torchrun sets OMP_NUM_THREADS=1; the oracle's OpenMP reads it when it loads)
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count())
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import torch

    from actcomp import synthetic

    x, ch = synthetic.lowrank_activation(T_sample, H, n_outlier=k, seed=0)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    rng = np.random.default_rng(0)
    V = np.linalg.qr(rng.standard_normal((H, rank)))[0].astype(np.float32)
    prep = O.basis_prepare(V)
    idx = ch.numpy()
    times = []
    t_end = time.perf_counter() + reps_seconds
    while len(times) < max_reps and (len(times) < 2 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        enc = O.encode(xb, prep, idx, bits, group, False)
        O.decode(enc["codes"], enc["scales"], enc["lowrank"], prep[1], enc["outliers"], idx, H, bits, group,
                 False)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    work = encode_bytes(T_sample, H, bits, group, rank, k) + decode_bytes(T_sample, H, bits, group, rank, k)
    return {"value": work / t / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle encode+decode of {T_sample} x {H} tokens (config-2 parameters), "
                      f"median of {len(times)} runs ({sum(times):.1f} s of CPU work), {t:.3f} s each"}


def _synthetic_module():
    """actcomp/synthetic.py loaded by file path: the reference arm must not
    import the actcomp package (importing it maps libactcomp.so)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "_bench_synthetic", os.path.join(ROOT, "triton-kernel-test_b200", "actcomp", "synthetic.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    cfg = {"workload": "config-2 encode+decode, 16384 x 4096 bf16 per rank, r=32 k=16 int4 g64",
           "tokens_per_rank": args.tokens, "channels": 4096, "rank": 32, "n_outlier": 16, "bits": 4, "group": 64,
           "global_batch": args.tokens * args.gpus, "parallelism": f"token-shard x{args.gpus}"}
    if rank != 0:
        return
    T_sample = args.tokens  # the whole config-2 activation per step (about 0.3 s on 16 cores)
    H, bits, group, r, k = 4096, 4, 64, 32, 16
    # all host cores (torchrun sets OMP_NUM_THREADS=1; the oracle's OpenMP reads it when it loads)
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count())
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    import torch

    synthetic = _synthetic_module()
    x, ch = synthetic.lowrank_activation(T_sample, H, n_outlier=k, seed=0)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    V = np.linalg.qr(np.random.default_rng(0).standard_normal((H, r)))[0].astype(np.float32)
    prep = O.basis_prepare(V)
    idx = ch.numpy()

    def step():
        enc = O.encode(xb, prep, idx, bits, group, False)
        O.decode(enc["codes"], enc["scales"], enc["lowrank"], prep[1], enc["outliers"], idx, H, bits, group,
                 False)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    work = encode_bytes(T_sample, H, bits, group, r, k) + decode_bytes(T_sample, H, bits, group, r, k)
    v = work / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": f"oracle encode+decode of {T_sample} x {H} per step (the reference's "
                                       "algorithm restated in C, OpenMP over tokens; the reference itself is "
                                       "Triton/PyTorch and has no CPU path that runs here)"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def run_gpu(args):
    import torch

    import actcomp
    from actcomp import synthetic

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    T, H, H2, N = args.tokens, 4096, 11008, 11008
    bits, group, r, k = 4, 64, 32, 16
    pk, peak_kind = peaks()

    # calibration (off the timed path): basis and outlier channels from a seed-0 sample shared by all ranks
    xcal, ch = synthetic.lowrank_activation(min(T, 4096), H, n_outlier=k, seed=0, device=dev, outlier_seed=0)
    basis = actcomp.Basis.fit(xcal, r)
    idx = actcomp.select_outlier_channels(xcal, k)
    x, _ = synthetic.lowrank_activation(T, H, n_outlier=k, seed=rank, device=dev, outlier_seed=0)
    del xcal
    flush = L2Flush(dev)

    state = {}

    def step():
        c = actcomp.encode(x, basis, idx, bits=bits, group=group)
        state["xh"] = actcomp.decode(c)
        state["c"] = c

    def enc_only():
        state["c"] = actcomp.encode(x, basis, idx, bits=bits, group=group)

    step()
    c0 = state["c"]

    def dec_only():
        actcomp.decode(c0, out=state["xh"].view(1, T, H))

    clk = ClockSampler(torch.cuda.current_device()).__enter__()
    step_detail = {}
    ms_step = time_steps(step, args.steps, args.warmup, flush, world, clk, step_detail)
    ms_enc = time_steps(enc_only, args.steps, 1, flush, world, clk)
    ms_dec = time_steps(dec_only, args.steps, 1, flush, world, clk)

    eb = encode_bytes(T, H, bits, group, r, k)
    db = decode_bytes(T, H, bits, group, r, k)
    value = world * (eb + db) / (ms_step * 1e-3) / 1e9
    hbm = pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    enc_gbs = eb / (ms_enc * 1e-3) / 1e9
    dec_gbs = db / (ms_dec * 1e-3) / 1e9
    dom = ("encode", ms_enc, eb) if ms_enc >= ms_dec else ("decode", ms_dec, db)
    achieved = dom[2] / (dom[1] * 1e-3) / 1e9

    # error statistics of the reconstruction, all-reduced over ranks (the only collective)
    stats = actcomp.dist.reduce_error_stats(actcomp.error_stats(state["xh"], x))
    st = stats.cpu().tolist()

    components = {"encode": {"ms": ms_enc, "GB/s": enc_gbs, "frac_of_hbm": enc_gbs / hbm, "bytes": eb},
                  "decode": {"ms": ms_dec, "GB/s": dec_gbs, "frac_of_hbm": dec_gbs / hbm, "bytes": db}}

    if not args.skip_extra:
        # fused SiLU backward on the 16384 x 11008 SiLU input (config 2)
        x2, _ = synthetic.lowrank_activation(T, H2, n_outlier=k, seed=100 + rank, device=dev, outlier_seed=100)
        b2 = actcomp.Basis.fit(x2[: min(T, 4096)], r)
        i2 = actcomp.select_outlier_channels(x2, k)
        c2 = actcomp.encode(x2, b2, i2, bits=bits, group=group)
        del x2
        dy2 = synthetic.gradient((T, H2), seed=7 + rank, device=dev)
        ms_silu = time_steps(lambda: actcomp.silu_backward(c2, dy2), args.steps, 1, flush, world, clk)
        sb = consumer_bytes(T, H2, bits, group, r, k)
        components["silu_bwd_fused_16384x11008"] = {"ms": ms_silu, "GB/s": sb / (ms_silu * 1e-3) / 1e9,
                                                    "frac_of_hbm": sb / (ms_silu * 1e-3) / 1e9 / hbm, "bytes": sb}
        del c2, dy2
        # fused dequant + dW GEMM (config 4): dW (4096 x 11008) = Xhat^T dY, K = 16384 tokens
        dy = synthetic.gradient((T, N), seed=11 + rank, device=dev)
        ws = torch.empty(actcomp._lib.load().actcomp_cg_dw_workspace(__import__("ctypes").byref(c0.desc()), N),
                         dtype=torch.uint8, device=dev)
        ms_dw = time_steps(lambda: actcomp.weight_grad(c0, dy, torch.float32, ws), max(3, args.steps // 2), 1,
                           flush, world, clk)
        flops = 2.0 * H * N * T
        tf = flops / (ms_dw * 1e-3) / 1e12
        # error of dW = Xhat^T dY against the bf16 GEMM of the uncompressed X, and
        # against the float32 GEMM of Xhat (the fused path's own arithmetic)
        dw = actcomp.weight_grad(c0, dy, torch.float32, ws)
        dw_x = actcomp.gemm(x.mT, dy, torch.float32)
        dw_xh = actcomp.gemm(actcomp.decode(c0).mT, dy, torch.float32)
        components["dw_gemm_fused_4096x11008_k16384"] = {
            "path": "one C call: decode into a workspace, then the tcgen05 GEMM (actcomp_cg_dw)",
            "ms": ms_dw, "TFLOP/s": tf, "frac_of_bf16_peak": tf / pk.get("bf16_tflops", 1590.0), "flops": flops,
            "rel_err_vs_bf16_gemm_of_x": float((dw - dw_x).norm() / dw_x.norm()),
            "rel_err_vs_gemm_of_xhat": float((dw - dw_xh).norm() / dw_xh.norm())}
        # the same product with the dequantisation inside the GEMM's producer
        # (actcomp_cg_dw_fused: dW = Q^T dY + V (L^T dY), outlier rows O^T dY;
        # no T x H workspace), beside the decode-then-GEMM path above
        ms_dwf = time_steps(lambda: actcomp.weight_grad(c0, dy, torch.float32, fused=True), max(3, args.steps // 2),
                            1, flush, world, clk)
        dwf = actcomp.weight_grad(c0, dy, torch.float32, fused=True)
        tff = flops / (ms_dwf * 1e-3) / 1e12
        components["dw_gemm_dequant_in_producer_4096x11008_k16384"] = {
            "path": "dequantisation inside the GEMM's producer (actcomp_cg_dw_fused)",
            "ms": ms_dwf, "TFLOP/s": tff, "frac_of_bf16_peak": tff / pk.get("bf16_tflops", 1590.0), "flops": flops,
            "rel_err_vs_bf16_gemm_of_x": float((dwf - dw_x).norm() / dw_x.norm()),
            "rel_err_vs_gemm_of_xhat": float((dwf - dw_xh).norm() / dw_xh.norm()),
            "workspace_MB": actcomp._lib.load().actcomp_cg_dw_fused_workspace(
                __import__("ctypes").byref(c0.desc()), N) / 1e6}
        del dy, ws, dw, dw_x, dw_xh, dwf
        # config 5: GELU backward on a compressed 65536 x 5120 activation
        T5, H5 = 4 * T, 5120
        x5, _ = synthetic.lowrank_activation(T5, H5, n_outlier=k, seed=200 + rank, device=dev, outlier_seed=200)
        c5 = actcomp.encode(x5, actcomp.Basis.fit(x5[:4096], r), actcomp.select_outlier_channels(x5, k), bits=bits,
                            group=group)
        del x5
        dy5 = synthetic.gradient((T5, H5), seed=13 + rank, device=dev)
        ms_gelu = time_steps(lambda: actcomp.gelu_backward(c5, dy5), max(3, args.steps // 2), 1, flush, world, clk)
        gb = consumer_bytes(T5, H5, bits, group, r, k)
        components[f"gelu_bwd_fused_{T5}x{H5}"] = {"ms": ms_gelu, "GB/s": gb / (ms_gelu * 1e-3) / 1e9,
                                                  "frac_of_hbm": gb / (ms_gelu * 1e-3) / 1e9 / hbm, "bytes": gb}
        del c5, dy5
        # config 3: the rotated format -- 128-point Walsh-Hadamard before int4
        # group-128 quantisation, r = 16, no outlier channels -- on a 32768 x 5120
        # heavy-tailed activation: encode and decode (the inverse rotation fused)
        T3, H3, r3 = 2 * T, 5120, 16
        x3 = synthetic.heavy_tailed_activation(T3, H3, seed=400 + rank, device=dev)
        b3 = actcomp.Basis.fit(x3[:4096], r3)
        c3 = actcomp.encode(x3, b3, None, bits=4, group=128, wht=True)
        ms_e3 = time_steps(lambda: actcomp.encode(x3, b3, None, bits=4, group=128, wht=True), max(3, args.steps // 2),
                           1, flush, world, clk)
        ms_d3 = time_steps(lambda: actcomp.decode(c3), max(3, args.steps // 2), 1, flush, world, clk)
        wb = encode_bytes(T3, H3, 4, 128, r3, 0)
        for name, ms3 in ((f"encode_wht_{T3}x{H3}", ms_e3), (f"decode_wht_{T3}x{H3}", ms_d3)):
            components[name] = {"ms": ms3, "GB/s": wb / (ms3 * 1e-3) / 1e9,
                                "frac_of_hbm": wb / (ms3 * 1e-3) / 1e9 / hbm, "bytes": wb}
        # reconstruction error of the heavy-tailed activation with and without the rotation
        e_rot = actcomp.error_stats(actcomp.decode(c3), x3).cpu().tolist()
        c3p = actcomp.encode(x3, b3, None, bits=4, group=128, wht=False)
        e_plain = actcomp.error_stats(actcomp.decode(c3p), x3).cpu().tolist()
        components[f"encode_wht_{T3}x{H3}"]["rel_err_rotated"] = (e_rot[0] / e_rot[1]) ** 0.5
        components[f"encode_wht_{T3}x{H3}"]["rel_err_without_rotation"] = (e_plain[0] / e_plain[1]) ** 0.5
        del x3, b3, c3, c3p
        # config 5: softmax backward on compressed causal probabilities P (8, 32, 2048, 2048), one basis for all heads
        Bh, NH, S = 8, 32, 2048
        P = torch.empty((Bh * NH, S, S), dtype=torch.bfloat16, device=dev)
        for bi in range(Bh):
            P[bi * NH:(bi + 1) * NH] = synthetic.causal_softmax(1, NH, S, seed=300 + bi, device=dev)[0]
        pf = P[0].to(torch.float32)
        V = torch.linalg.eigh(pf.T @ pf)[1][:, -r:].flip(-1)
        del pf
        bP = actcomp.Basis.from_vectors(V.unsqueeze(0).expand(Bh * NH, S, r).contiguous())
        cP = actcomp.encode(P, bP, None, bits=bits, group=group)
        del P
        dP = synthetic.gradient((Bh * NH, S, S), seed=17 + rank, device=dev)
        ms_smax = time_steps(lambda: actcomp.softmax_backward(cP, dP, causal=True), max(3, args.steps // 4), 1, flush,
                             world, clk)
        sbytes = Bh * NH * (consumer_bytes(S, S, bits, group, r, 0))
        components["softmax_bwd_fused_8x32x2048x2048_causal"] = {
            "ms": ms_smax, "GB/s": sbytes / (ms_smax * 1e-3) / 1e9, "frac_of_hbm": sbytes / (ms_smax * 1e-3) / 1e9 / hbm,
            "bytes": sbytes}
        del cP, dP, bP
        # NF4 base weight of the reference's backward driver (d1 = 4096 in,
        # d2 = 14336 out, low_rank_system_profile_backward.py:21-22,31,58):
        # blocksize 64 with nested statistics (LinearNF4's default), dequantised
        # to bf16 every step; HBM-bound: n/2 + n/64 bytes in, 2n bytes out
        from actcomp import nf4 as NF4

        d1n, d2n = 4096, 14336
        nn4 = d1n * d2n
        gq = torch.Generator(device=dev).manual_seed(31)
        wq = torch.randint(0, 256, ((nn4 + 1) // 2, 1), dtype=torch.uint8, device=dev, generator=gq)
        st2 = NF4.QuantState(absmax=torch.rand(-(-nn4 // (64 * 256)), device=dev, generator=gq) * 0.1,
                             shape=torch.Size([-(-nn4 // (64 * 256))]),
                             code=torch.linspace(-1, 1, 256, device=dev), blocksize=256)
        stq = NF4.QuantState(absmax=torch.randint(0, 256, (nn4 // 64,), dtype=torch.uint8, device=dev, generator=gq),
                             shape=torch.Size([d2n, d1n]), code=NF4.nf4_code(dev), blocksize=64,
                             offset=torch.tensor(0.05, device=dev), state2=st2)
        wout = torch.empty((d2n, d1n), dtype=torch.bfloat16, device=dev)
        ms_nf4 = time_steps(lambda: NF4.dequantize_4bit(wq.t(), stq, out=wout), max(3, args.steps // 2), 1, flush,
                            world, clk)
        nb4 = (nn4 + 1) // 2 + nn4 // 64 + 2 * nn4
        components[f"nf4_dequant_{d2n}x{d1n}"] = {"ms": ms_nf4, "GB/s": nb4 / (ms_nf4 * 1e-3) / 1e9,
                                                  "frac_of_hbm": nb4 / (ms_nf4 * 1e-3) / 1e9 / hbm, "bytes": nb4}
        del wq, st2, stq, wout

        # the reference-named API (compat / reference_api) on its own speed-test
        # shapes: x (B=4, M, M), rank R=16, 1-bit encode with a dense outlier
        # matrix, 2-bit decode (low_rank_kernel_encode_speed_test.py:28-33,
        # low_rank_kernel_decode_speed_test.py:28-38).  The harness reports
        # 2 B M R M / t as TFLOPS; the kernels are HBM-bound, so GB/s is beside it.
        from actcomp import ops as AOPS
        from actcomp import reference_api as RA

        for Mrc in (4096, 16384):
            g = torch.Generator(device=dev).manual_seed(21)
            xr = torch.randn((4, Mrc, Mrc), device=dev, dtype=torch.bfloat16, generator=g)
            lr_ = torch.randn((Mrc, 16), device=dev, dtype=torch.bfloat16, generator=g)
            rr_ = torch.randn((16, Mrc), device=dev, dtype=torch.bfloat16, generator=g)
            sr_ = torch.randn((4, Mrc), device=dev, dtype=torch.bfloat16, generator=g) + 2
            # the kernel (dense o), and the named call (which converts o to COO, as the reference does)
            ms_e = time_steps(lambda: AOPS.rc_encode(lr_, rr_, xr, sr_, 1, 12.0, 0), max(3, args.steps // 4), 1,
                              flush, world, clk)
            ms_api = time_steps(lambda: RA.low_rank_addition_fuse_compression_quantization(lr_, rr_, xr, sr_, 1, 12.0),
                                3, 1, flush, world, clk)
            el = 4 * Mrc * Mrc
            rc_eb = el * 2 + el * 2 + el // 8  # x in, dense o out, 1-bit codes out
            components[f"rc_encode_1bit_B4_M{Mrc}"] = {
                "ms": ms_e, "GB/s": rc_eb / (ms_e * 1e-3) / 1e9, "frac_of_hbm": rc_eb / (ms_e * 1e-3) / 1e9 / hbm,
                "harness_TFLOPS": 2 * 4 * Mrc * 16 * Mrc / (ms_e * 1e-3) / 1e12, "bytes": rc_eb,
                "named_call_ms": ms_api}
            o_, q_ = AOPS.rc_encode(lr_, rr_, xr, sr_, 2, 12.0, 0)
            del xr
            ms_d = time_steps(lambda: RA.low_rank_addition_fuse_decompression_dequantization(lr_, rr_, q_, o_, sr_, 2),
                              max(3, args.steps // 4), 1, flush, world, clk)
            rc_db = el // 4 + el * 2 + el * 2  # 2-bit codes and dense o in, x out
            components[f"rc_decode_2bit_B4_M{Mrc}"] = {
                "ms": ms_d, "GB/s": rc_db / (ms_d * 1e-3) / 1e9, "frac_of_hbm": rc_db / (ms_d * 1e-3) / 1e9 / hbm,
                "harness_TFLOPS": 2 * 4 * Mrc * 16 * Mrc / (ms_d * 1e-3) / 1e12, "bytes": rc_db}
            del o_, q_, lr_, rr_, sr_

    # offload of the packed activation to pinned host memory and back (side stream, events)
    off = actcomp.Offloader(dev)

    def time_copy(fn, reps, release):
        ts = []
        for i in range(reps + 2):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            h = fn()
            h.wait()
            e1.record()
            torch.cuda.synchronize()
            if i >= 2:
                ts.append(e0.elapsed_time(e1))
            if release:
                off.release(h)
        return float(statistics.median(ts))

    nb_packed = c0.nbytes()
    ms_off = time_copy(lambda: off.offload(c0), max(3, args.steps // 2), True)
    h_keep = off.offload(c0)
    h_keep.wait()

    def reload_once():
        state["back"] = off.reload(h_keep)
        return h_keep

    ms_rel = time_copy(reload_once, max(3, args.steps // 2), False)
    torch.cuda.synchronize()
    assert torch.equal(state["back"].codes, c0.codes)
    # the host link's measured peak: one pinned 1 GiB copy each way
    big_d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    big_h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)

    def link(copy):
        ts = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            copy()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return (1 << 30) / (statistics.median(ts) * 1e-3) / 1e9

    d2h_peak = link(lambda: big_h.copy_(big_d, non_blocking=True))
    h2d_peak = link(lambda: big_d.copy_(big_h, non_blocking=True))
    del big_d, big_h
    components["offload_d2h"] = {"ms": ms_off, "GB/s": nb_packed / (ms_off * 1e-3) / 1e9, "bytes": nb_packed,
                                 "link_peak_GB/s": d2h_peak}
    components["reload_h2d"] = {"ms": ms_rel, "GB/s": nb_packed / (ms_rel * 1e-3) / 1e9, "bytes": nb_packed,
                                "link_peak_GB/s": h2d_peak}
    del state["back"]
    # offload overlapped with compute: the packed activation leaves on the side
    # stream while a GEMM of about the copy's length runs on the compute stream;
    # overlap = (t_copy + t_gemm - t_both) / min(t_copy, t_gemm)
    ga = torch.randn(8192, 8192, device=dev).to(torch.bfloat16)
    gb_ = torch.randn(8192, 8192, device=dev).to(torch.bfloat16)

    def both():
        h = off.offload(c0)
        actcomp.gemm(ga, gb_, torch.bfloat16)
        h.wait()
        return h

    ms_gemm = time_copy(lambda: (actcomp.gemm(ga, gb_, torch.bfloat16), _Done())[1], 3, False)
    ms_both = time_copy(both, 3, True)
    components["offload_overlap_with_gemm"] = {
        "copy_ms": ms_off, "gemm_ms": ms_gemm, "both_ms": ms_both,
        "overlap": (ms_off + ms_gemm - ms_both) / min(ms_off, ms_gemm)}
    del ga, gb_

    # end to end through the public API with host buffers: pinned X -> H2D -> encode -> decode -> D2H,
    # streamed in token chunks (every token row is encoded on its own, so chunking changes no bit):
    # chunk i's H2D, chunk i-1's encode + decode and chunk i-2's D2H run on three streams, so that
    # the two PCIe directions overlap
    E2E_CHUNKS = 9
    xh_host = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    x_host = x.cpu().pin_memory()
    x_dev = torch.empty_like(x)
    xd_dev = torch.empty_like(x)
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    # half-size first and last chunks: the pipeline fills and drains on one H2D / D2H of T/16 tokens
    cut = [0] + [(T // 16 + T * i // 8) // 128 * 128 for i in range(E2E_CHUNKS - 1)] + [T]

    def e2e_step():
        cur = torch.cuda.current_stream()
        for st_ in (s_in, s_cmp, s_out):
            st_.wait_stream(cur)
        for i in range(E2E_CHUNKS):
            sl = slice(cut[i], cut[i + 1])
            with torch.cuda.stream(s_in):
                x_dev[sl].copy_(x_host[sl], non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(e_in)
                c = actcomp.encode(x_dev[sl], basis, idx, bits=bits, group=group)
                actcomp.decode(c, out=xd_dev[sl])
                e_cmp = torch.cuda.Event()
                e_cmp.record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(e_cmp)
                xh_host[sl].copy_(xd_dev[sl], non_blocking=True)
        for st_ in (s_in, s_cmp, s_out):
            cur.wait_stream(st_)

    ms_e2e = time_steps(e2e_step, max(3, args.steps // 2), 2, flush, world, clk)
    # the same steps on the host clock, as a cross-check of the device events
    import time as _time

    torch.cuda.synchronize()
    t0 = _time.perf_counter()
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    ms_e2e_wall = (_time.perf_counter() - t0) / 3 * 1e3
    # the streamed result is the whole-tensor roundtrip, bit for bit
    assert torch.equal(xh_host, actcomp.decode(actcomp.encode(x, basis, idx, bits=bits, group=group)).cpu())
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    e2e_val = world * (eb + db) / (ms_e2e * 1e-3) / 1e9

    if rank == 0:
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get(dom[0])
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, config-2 generator)",
            "config": {"workload": "config-2 encode+decode, 16384 x 4096 bf16 per rank, r=32 k=16 int4 g64",
                       "tokens_per_rank": T, "channels": H, "rank": r, "n_outlier": k, "bits": bits,
                       "group": group, "global_batch": T * world, "parallelism": f"token-shard x{world}",
                       "l2": "256 MB write, then 256 MB read of another buffer, between timed steps (outside the events)"},
            "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": dom[2]},
            "clocks": clocks,
            "e2e": {"value": e2e_val, "unit": "GB/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2,
                    "pipeline": f"{E2E_CHUNKS} token chunks: H2D, encode + decode, D2H on three streams",
                    "ms_per_step": ms_e2e, "ms_per_step_host_clock": ms_e2e_wall},
            "gpu_launches": args.steps * launches_per_step(),
            "per_rank_ms_per_step": step_detail.get("per_rank_ms"),
            "components": components,
            "error": {"rel_fro": (st[0] / st[1]) ** 0.5 if st[1] else None, "max_abs": st[2],
                      "changed_values": st[3]},
        }
        if not args.no_cpu_baseline and world == 1:  # the CPU baseline is an N=1 figure
            line["cpu_baseline"] = cpu_baseline(T, H, bits, group, r, k)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def launches_per_step():
    """Kernels of this library launched by one encode + decode."""
    return 3  # the encode's projection and quantisation kernels, and the row decode


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="actcomp", choices=["actcomp", "reference"])
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per rank (profiling runs use fewer)")
    ap.add_argument("--skip-extra", action="store_true", help="only the encode/decode step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and not args.skip_extra:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    main()
