"""Benchmark of the recurrent hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

Headline workload: the fused selective scan at batch 8, seqlen 32768,
dim 4096, dstate 16, bf16 I/O with fp32 state (inputs 8.6 GB per rank, far
larger than L2, so no flush is needed between steps).  One step = one fused
scan pass (softplus(delta+bias), exp(delta*A), recurrence, C.h + D*u,
y*silu(z), final state) over the rank's batch.  Multi-GPU: every rank scans
its own batch (units are independent channels; no collective on the data
path) -> weak scaling; time = max over ranks of CUDA-event time.

Prints ONE JSON line (rank 0).  ``--impl reference`` times the reference's
own CPU path (its ``selective_scan_pytorch`` with the softplus / SiLU of
``MambaBlock.forward``, from the unmodified install in baseline/_ref; the C
restatement of that loop when the install is absent), all host threads, on a
bounded sample of the same workload, and prints the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "selective-scan HBM GB/s (fused scan, bf16 I/O, fp32 state)"
WORKLOAD = dict(batch=8, seqlen=32768, dim=4096, dstate=16)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profile_traffic(kernel_key):
    """DRAM bytes per launch from a committed ncu capture (profiles/traffic.json)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(kernel_key)
    return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 5 ms during the timed
    region, by NVML from a host thread (read-only queries; nvidia-smi's first sample
    takes longer than a short timed region).  Samples are kept from mark() on."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device):
        self.device = device
        self.samples = []  # (sm_mhz, reason bits)
        self.start = 0
        self.max_mhz = None
        self.handle = None
        self.nvml = None
        self.stop = threading.Event()
        self.thread = None

    def _handle(self, nv):
        try:
            props = torch.cuda.get_device_properties(self.device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.device.index)

    def _run(self):
        nv, h = self.nvml, self.handle
        while not self.stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                return
            time.sleep(0.005)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nvml, self.handle = nv, self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
        return self

    def mark(self):
        """Start of the timed region."""
        self.start = len(self.samples)

    def hold(self, seconds=0.25):
        """Wait (host side, the launches queued) until a sample inside the timed region exists."""
        t_end = time.time() + seconds
        while self.thread is not None and time.time() < t_end and len(self.samples) <= self.start:
            time.sleep(0.002)

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.nvml is not None:
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        got = self.samples[self.start:] or self.samples
        if not got:
            return None
        reasons = sorted(name for name, const in self.REASONS
                         if any(bits & getattr(self.nvml, const, 0) for _, bits in got))
        return {"sm_mhz": statistics.median(m for m, _ in got), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(got), "source": "NVML, every 5 ms over the timed region"}


def dist_setup(args):
    from hybrid_model_mamba_xlstm_b200 import dist as D
    world, rank, local = D.env_world()
    if world > 1:
        D.init("nccl", timeout_s=120.0)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    from hybrid_model_mamba_xlstm_b200 import dist as D
    D.barrier(world)


def max_over_ranks(x, world):
    from hybrid_model_mamba_xlstm_b200 import dist as D
    return D.max_over_ranks(x, world)


def ref_pkg():
    """The reference package installed unmodified in baseline/_ref (pip --target,
    no dependencies), or None.  Only the CPU baselines below import it."""
    d = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(d, "hybrid_xmamba")):
        return None
    if d not in sys.path:
        sys.path.insert(0, d)
    import importlib
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        # by module path: the package re-exports functions under the subpackages' names
        si = importlib.import_module("hybrid_xmamba.kernels.selective_scan.scan_interface")
        ti = importlib.import_module("hybrid_xmamba.kernels.tfla.tfla_interface")
    return {"scan": si, "tfla": ti}


def _cpu_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def _scan_bytes(batch, seqlen, dim, dstate, es=2):
    return batch * seqlen * dim * 4 * es + 2 * batch * seqlen * dstate * es + (dim * dstate + 2 * dim) * 4 + \
        batch * dim * dstate * 4


def cpu_scan_sample(seqlen, dim_sample, dstate, seed=0):
    """Bounded CPU sample of the headline workload (one batch row x dim_sample
    channels x seqlen steps): the reference's own path when baseline/_ref holds
    it — softplus(delta + bias), selective_scan_pytorch, y * silu(z), as
    MambaBlock runs them (mamba_block.py:115-130, scan_interface.py:103-152) —
    else the C restatement of that loop.  Returns (run -> seconds, bytes of the
    sample as the bf16 workload moves them, threads, kind, what ran)."""
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    inp = scan_inputs(1, seqlen, dim_sample, dstate, torch.float32, seed=seed)
    nbytes = _scan_bytes(1, seqlen, dim_sample, dstate)
    ref = ref_pkg()
    if ref is not None:
        threads = _cpu_threads()
        tr = lambda t: t.transpose(1, 2).contiguous()  # noqa: E731  (B, L, D) as the reference takes it
        u, raw, z, Bm, Cm = tr(inp.u), tr(inp.delta), tr(inp.z), tr(inp.B), tr(inp.C)

        def run():
            t0 = time.perf_counter()
            with torch.no_grad():
                dt = torch.nn.functional.softplus(raw + inp.delta_bias)
                y = ref["scan"].selective_scan_pytorch(u, dt, inp.A, Bm, Cm, inp.D)
                y = y * torch.nn.functional.silu(z)
            return time.perf_counter() - t0
        return run, nbytes, threads, "reference", "hybrid_xmamba selective_scan_pytorch + softplus / silu (torch, fp32)"
    import numpy as np
    from oracle import build as OC
    n = lambda t: t.numpy()  # noqa: E731
    args = (n(inp.u), n(inp.delta), n(inp.A), n(inp.B), n(inp.C), n(inp.D), n(inp.z), n(inp.delta_bias))
    sl = lambda a: np.ascontiguousarray(a[..., :64])  # noqa: E731
    OC.scan(sl(args[0]), sl(args[1]), args[2], sl(args[3]), sl(args[4]), args[5], sl(args[6]), args[7],
            softplus=True, z_mode=2, disc=0)  # warm the thread pool

    def run():
        t0 = time.perf_counter()
        OC.scan(*args, softplus=True, z_mode=2, disc=0)
        return time.perf_counter() - t0
    return run, nbytes, OC.lib().hxm_oracle_max_threads(), "port", "C restatement of the reference loop (fp32, OpenMP)"


REF_SAMPLE = dict(dim=4096, seqlen=4096)  # one batch row x 4096 channels x 4096 steps = 1/64 of the workload


def run_reference(args, world, rank):
    """Reference arm: the reference's own CPU path of the scan on the host cores
    (all threads), on a bounded sample of the headline workload per step."""
    if rank != 0:
        return
    S = REF_SAMPLE
    run, nbytes, threads, kind, what = cpu_scan_sample(S["seqlen"], S["dim"], WORKLOAD["dstate"])
    for _ in range(args.warmup):
        run()
    ts = [run() for _ in range(args.steps)]
    t = sum(ts) / len(ts)
    gbs = nbytes / t / 1e9
    sample = (f"1 batch row x {S['dim']} channels x {S['seqlen']} steps x dstate {WORKLOAD['dstate']} per step "
              f"(1/64 of the workload; {what})")
    out = {"metric": METRIC, "value": gbs, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "selective scan b8 l32768 d4096 n16 (bounded CPU sample)", **WORKLOAD},
           "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
           "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def _time_cuda(fn, steps, warmup, dev, world):
    """Mean ms per call over `steps` timed calls (CUDA events, max over ranks)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    barrier(world)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.synchronize(dev)
    return max_over_ranks(e0.elapsed_time(e1) / steps, world)


def roofline_obj(bound, achieved, unit, kernel_key, algorithmic, per_launch_scale=1.0):
    """A roofline object for a secondary workload: `achieved` against the
    measured peak of its bound (HBM GB/s or dense bf16 TFLOP/s, burst), and the
    DRAM traffic of one launch from the committed ncu captures
    (profiles/traffic.json, `kernel_key`), scaled by `per_launch_scale` when
    the capture ran a smaller case of the same kernel."""
    pk, kind = peaks()
    peak = pk["hbm_gbs"] if bound == "hbm" else pk["bf16_tflops"]
    t = profile_traffic(kernel_key)
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "peak_kind": kind, "traffic": None if t is None else t * per_launch_scale,
            "traffic_key": kernel_key, "algorithmic": algorithmic}


def secondary_metrics(args, dev, world, rank):
    """The other hot-path workloads, each timed on every rank (same order on all ranks)."""
    from hybrid_model_mamba_xlstm_b200.kernels.slstm import slstm_scan
    from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan
    from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_interface import mlstm_chunkwise_fwd
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs, ssd_inputs
    pk, pk_kind = peaks()
    tf_peak = pk["bf16_tflops"]
    out = {}
    steps = max(3, min(args.steps, 10))
    # mLSTM chunkwise, per-head gates (tcgen05): the large-batch d=256 case and the exact 2x4x2048x256 case
    # and the long-context case (batch 8, 8 heads, seqlen 32768, qk = v = 512: key-streaming kernel)
    # (the kernels run 128-step chunks; FLOPs are counted for the chunk that runs)
    for name, (b, h, L, d, c) in {"mlstm_b8_h8_l32768_d512": (8, 8, 32768, 512, 128),
                                  "mlstm_b8_h8_l8192_d256": (8, 8, 8192, 256, 128),
                                  "mlstm_b2_h4_l2048_d256": (2, 4, 2048, 256, 128)}.items():
        inp = mlstm_inputs(b, h, L, d, torch.bfloat16, seed=rank, device=dev, on_device=True)
        ms = _time_cuda(lambda: mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, chunk=c),
                        steps, 3, dev, world)
        fl = inp.flops(c)
        kern = "chunk_tc_kernel<%d, mLSTM>" % d if d <= 256 else "mlstm_stream_kernel<%d>" % d
        out[name] = {"metric": "mLSTM chunkwise TFLOP/s (algorithmic)", "value": world * fl / ms / 1e9,
                     "unit": "TFLOP/s", "ms": ms, "chunk": c, "frac_of_bf16_peak": fl / ms / 1e9 / tf_peak,
                     "peak_kind": pk_kind, "scaling": "weak", "kernel": kern,
                     "roofline": roofline_obj("tensor", fl / ms / 1e9, "TFLOP/s", f"{kern} {name}",
                                              {"flops": fl, "bytes": inp.bytes_moved()})}
        del inp
    # Mamba-2 SSD, batch 8, 32 heads x 64, dstate 128, seqlen 4096 (tcgen05)
    inp = ssd_inputs(8, 4096, 32, 64, 128, seed=rank, device=dev, on_device=True)
    ms = _time_cuda(lambda: ssd_chunk_scan(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D), steps, 3, dev, world)
    fl = inp.flops(128)
    out["ssd_b8_h32_p64_n128_l4096"] = {"metric": "SSD chunked scan TFLOP/s (algorithmic, for the 128-step chunk "
                                                  "that runs)",
                                        "value": world * fl / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "chunk": 128,
                                        "frac_of_bf16_peak": fl / ms / 1e9 / tf_peak, "peak_kind": pk_kind,
                                        "scaling": "weak", "kernel": "chunk_tc_kernel<128, SSD>",
                                        "roofline": roofline_obj("tensor", fl / ms / 1e9, "TFLOP/s",
                                                                 "chunk_tc_kernel<128, SSD> ssd_b8_h32_p64_n128_l4096",
                                                                 {"flops": fl, "bytes": inp.bytes_moved()})}
    del inp
    # sLSTM recurrence with block-diagonal R, the prefill's layer shape: batch 8, 4 heads x 256, seqlen 2048
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    gates = torch.randn(8, 2048, 4, 4, 256, generator=g, device=dev).mul_(0.5).to(torch.bfloat16)
    Rw = (torch.randn(4, 256, 1024, generator=g, device=dev) / 16).to(torch.bfloat16)
    w = torch.ones(256, device=dev)
    ms = _time_cuda(lambda: slstm_scan(gates, w, R=Rw), min(steps, 3), 2, dev, world)
    out["slstm_b8_h4_hd256_l2048"] = {"metric": "sLSTM recurrence us/step (sequential over seqlen)",
                                      "value": ms * 1e3 / 2048, "unit": "us/step", "ms": ms,
                                      "kernel": "slstm_cluster_kernel<bf16, 256>"}
    del gates, Rw
    # mLSTM backward at the 350M model's mLSTM layer shape (batch 8, 4 heads x 512, seqlen 2048,
    # per-channel gates): chunkwise, the chunk GEMMs on the tcgen05 chunk-GEMM kernel (bf16 high / low
    # split operands) around the hxm gate / chunk-scan kernels; these gates' 128-step chunk factors
    # exceed e^60, so the chunk that runs is 64 steps
    from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_bwd import _channel_chunk, mlstm_chunkwise_bwd
    b, h, L, d = 8, 4, 2048, 512
    g.manual_seed(7 + rank)
    q, k, v, dh = (torch.randn(b, h, L, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(4))
    q.mul_(d ** -0.5)
    li = torch.randn(b, h, L, d, generator=g, device=dev).mul_(0.5)
    lf = torch.nn.functional.logsigmoid(torch.randn(b, h, L, d, generator=g, device=dev))
    c = _channel_chunk(li, lf, 128)
    ms = _time_cuda(lambda: mlstm_chunkwise_bwd(q, k, v, li, lf, dh), min(steps, 3), 2, dev, world)
    ms_fast = _time_cuda(lambda: mlstm_chunkwise_bwd(q, k, v, li, lf, dh, precise=False), min(steps, 3), 2, dev,
                         world)
    ms_lib = _time_cuda(lambda: mlstm_chunkwise_bwd(q, k, v, li, lf, dh, chunk=64, tensor_cores=False, tf32=True),
                        min(steps, 3), 2, dev, world)
    w8 = (d + 1 + 7) // 8 * 8
    nch = L // c
    fl = b * h * nch * (3 * 2 * c * c * d + 3 * 2 * c * c * w8 + 6 * 2 * c * d * w8)  # the 8 products that run
    out["mlstm_bwd_b8_h4_l2048_d512_channel_gates"] = {
        "metric": "mLSTM backward ms (chunk GEMM TFLOP/s alongside)", "value": ms, "unit": "ms",
        "gemm_tflops": world * fl / ms / 1e9, "scaling": "weak", "higher_is_better": False,
        "chunk": c, "precise_false_ms": ms_fast, "library_tf32_ms": ms_lib,
        "kernels": "hxm mlstm_bwd prepare / normalizer / chunk_scan / chunk_dot / finalize + "
        "chunk_gemm_kernel (tcgen05, bf16 high / low split operands) chunk GEMMs",
        "accuracy": "default (precise): every fp32 operand split (~3e-5 vs float64); precise=False: gate-scaled "
                    "q, k split (~1e-3); library_tf32: cuBLAS TF32 chunk GEMMs at chunk 64 (~1e-3)"}
    del q, k, v, dh, li, lf
    # SSD backward at the SSD workload's shape (batch 8, 32 heads x 64, dstate 128, seqlen 4096)
    from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan_bwd
    inp = ssd_inputs(8, 4096, 32, 64, 128, seed=rank, device=dev, on_device=True)
    dy = torch.randn(8, 4096, 32, 64, generator=g, device=dev).to(torch.bfloat16)
    sargs = (inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D, dy)
    ms = _time_cuda(lambda: ssd_chunk_scan_bwd(*sargs), min(steps, 3), 2, dev, world)
    ms_fast = _time_cuda(lambda: ssd_chunk_scan_bwd(*sargs, precise=False), min(steps, 3), 2, dev, world)
    ms_lib = _time_cuda(lambda: ssd_chunk_scan_bwd(*sargs, tensor_cores=False, tf32=True), min(steps, 3), 2, dev,
                        world)
    out["ssd_bwd_b8_h32_p64_n128_l4096"] = {
        "metric": "SSD backward ms", "value": ms, "unit": "ms", "scaling": "weak", "higher_is_better": False,
        "chunk": 64, "precise_false_ms": ms_fast, "library_tf32_ms": ms_lib,
        "kernels": "chunk_gemm_kernel (tcgen05, bf16 high / low split operands) + hxm scale_split / chunk-state "
                   "scan (row mode) / ssd_bwd intra / rows (exact per-head chunk form)",
        "accuracy": "default (precise): ~1e-5 vs float64; precise=False ~1e-3; library_tf32: cuBLAS TF32 ~1e-3"}
    del inp, dy
    # selective-scan backward at the 350M model's Mamba layer shape (batch 8, seqlen 2048, d_inner 2048, N 16)
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan.scan_interface import selective_scan_bwd
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    sb, sl, sd = 8, 2048, 2048
    inp = scan_inputs(sb, sl, sd, 16, torch.bfloat16, seed=rank, device=dev, on_device=True)
    dout = torch.randn(sb, sd, sl, generator=g, device=dev).to(torch.bfloat16)
    tr = lambda x: x.transpose(1, 2)
    ms = _time_cuda(lambda: selective_scan_bwd(tr(dout), tr(inp.u), tr(inp.delta), inp.A, tr(inp.B), tr(inp.C),
                                               inp.D, tr(inp.z), z_mode="silu", delta_bias=inp.delta_bias,
                                               delta_softplus=True), min(steps, 3), 2, dev, world)
    nbytes = sb * sl * sd * (4 * 2 + 3 * 4) + sb * sl * 16 * (2 * 2 + 2 * 4)
    out["scan_bwd_b8_l2048_d2048_n16"] = {
        "metric": "selective-scan backward GB/s (one read of each bf16 input, one write of each fp32 gradient)",
        "value": world * nbytes / ms / 1e6, "unit": "GB/s", "ms": ms, "scaling": "weak",
        "kernel": "hxm::scanbwd::scan_bwd_kernel (checkpointed reverse recurrence, 2 lanes per channel here)",
        "roofline": roofline_obj("hbm", nbytes / ms / 1e6, "GB/s", "scan_bwd_kernel scan_bwd_b8_l2048_d2048_n16",
                                 {"bytes": nbytes})}
    del inp, dout
    torch.cuda.empty_cache()
    out["prefill"] = prefill_metric(args, dev, world, rank)
    return out


def prefill_metric(args, dev, world, rank):
    """Hybrid-350M prefill (24 layers [Mamba, Mamba, mLSTM, sLSTM], d 1024, vocab
    50304, bf16), data parallel over the ranks: batch 8 x seqlen 2048 per rank
    (weak scaling, the data-parallel serving throughput) and the global batch 8
    split over the ranks (strong scaling)."""
    import hybrid_model_mamba_xlstm_b200.layers as Lyr
    gb, seqlen = 8, 2048
    torch.manual_seed(1234)  # identical weights on every rank
    model = Lyr.HybridLanguageModel(Lyr.hybrid_350m_config()).to(dev).to(torch.bfloat16).eval()
    nparam = sum(p.numel() for p in model.parameters())
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    out = {}
    # algorithmic FLOPs of one forward token: 2 x every weight used per token (the token embedding is a
    # lookup, the LM head a GEMM) + the chunkwise mLSTM's intra-chunk terms (4 c d per head and token)
    cfg = model.config
    n_w = sum(p.numel() for n_, p in model.named_parameters() if "token_embedding" not in n_)
    n_mlstm = sum(1 for i in range(cfg.num_layers) if cfg.layer_pattern[i % len(cfg.layer_pattern)] == "mlstm")
    tied = model.lm_head.weight is model.embeddings.token_embedding.weight  # then n_w lacks the head's GEMM
    flop_tok = 2 * n_w + (2 * cfg.dim * cfg.vocab_size if tied else 0) + \
        n_mlstm * cfg.num_heads * 4 * 128 * cfg.head_dim
    for kind, per in (("weak", gb), ("strong", max(1, gb // world))):
        # finer wavefront pieces when one GPU holds up to four sequences (measured: batch 1
        # 11.2 ms with 8 pieces, 13.2 with 4, 14.0 with 16; batch 4 17.97 with 8, 18.43 with 4;
        # batch 8, 4 pieces 29.5-29.7 ms, 6 pieces 31.0, 8 pieces 31.9)
        pieces = 8 if per <= 4 else 4
        ids = torch.randint(0, 50304, (per, seqlen), generator=g, device=dev)
        with torch.no_grad():
            pg = Lyr.PrefillGraph(model, per, seqlen, pieces=pieces, device=dev)
            ms = _time_cuda(lambda: pg(ids), 3, 2, dev, world)
            ms_eager = _time_cuda(lambda: model(ids), 2, 1, dev, world)
        out[kind] = {"metric": "hybrid-350M prefill tokens/s", "value": world * per * seqlen / ms * 1e3,
                     "unit": "tok/s", "ms_per_step": ms, "batch_per_rank": per, "global_batch": world * per,
                     "seqlen": seqlen, "params": nparam,
                     "schedule": f"CUDA-graph wavefront: {pieces} sequence pieces x 24 layers, one stream per layer",
                     "single_stream_forward_ms": ms_eager,
                     "scaling": "weak (batch 8 per rank)" if kind == "weak" else "strong (global batch 8 split over ranks)",
                     "parallelism": f"dp{world}",
                     "roofline": roofline_obj("tensor", per * seqlen * flop_tok / ms / 1e9, "TFLOP/s",
                                              "prefill hybrid350m", {"flops_per_token": flop_tok})}
        del ids, pg
        torch.cuda.empty_cache()
    del model
    return out


def run_ours(args, world, rank, local):
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import selective_scan_fn
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    dev = torch.device("cuda", local if world > 1 else 0)
    W = WORKLOAD
    inp = scan_inputs(W["batch"], W["seqlen"], W["dim"], W["dstate"], torch.bfloat16, seed=1000 + rank,
                      device=dev, on_device=True)
    y = torch.empty_like(inp.u)
    stream = torch.cuda.current_stream(dev)

    def step():
        return selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z, delta_bias=inp.delta_bias,
                                 delta_softplus=True, return_last_state=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clk:
        torch.cuda.synchronize(dev)
        barrier(world)
        clk.mark()
        ev[0].record(stream)
        for i in range(args.steps):
            step()
            ev[i + 1].record(stream)
        clk.hold()  # the launches are queued: wait (host side) for a sample while they run
        torch.cuda.synchronize(dev)
        barrier(world)
    per = [ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    total_ms = max_over_ranks(total_ms, world)
    clocks = clk.summary()
    nbytes = inp.bytes_moved()
    value = world * nbytes * args.steps / (total_ms / 1e3) / 1e9
    pk, pk_kind = peaks()
    launch_ms = sum(per) / len(per)
    achieved = nbytes / (launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "peak_kind": pk_kind,
                "traffic": profile_traffic("scan_fwd_kernel bf16 b8 l32768 d4096 n16"),
                "kernel": "hxm::scan::scan_fast_kernel<bf16, 64, 32, silu, softplus>", "algorithmic_bytes": nbytes}

    # ---- verification (outside the timed region): every rank checks sampled channels of its own
    #      output against the C oracle over the full length; the errors are all-gathered (NCCL)
    from hybrid_model_mamba_xlstm_b200 import dist as D
    yv, hv = step()
    errs = verify_scan_channels(inp, yv, hv, [(0, 0), (3, 1234), (W["batch"] - 1, W["dim"] - 1)])
    gathered = D.gather_checksums(errs, world)
    verification = {"per_rank_max_rel_err_y_hT": gathered.tolist(), "tolerance": 2e-2,
                    "ok": bool((gathered <= 2e-2).all()),
                    "note": "3 (batch row, channel) pairs per rank, y over all 32768 steps and the final state, "
                            "against the C oracle (fp32) on the same bf16 inputs"}
    del yv, hv

    # ---- end to end through the public API with host buffers (bounded: 1 batch row per rank)
    e2e = e2e_scan(dev, args, world)

    secondary = None
    if not args.no_secondary:
        del inp, y
        torch.cuda.empty_cache()
        secondary = secondary_metrics(args, dev, world, rank)
        secondary["config5_sharded"] = config5_sharded(args, dev, world, rank, per_rank_gbs=achieved,
                                                       weak_mlstm=secondary.get("mlstm_b8_h8_l32768_d512"))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        S = REF_SAMPLE
        run, cb, threads, kind, what = cpu_scan_sample(S["seqlen"], S["dim"], W["dstate"])
        run()
        tcpu = min(run() for _ in range(2))
        cpu = {"value": cb / tcpu / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": f"1 batch row x {S['dim']} channels x {S['seqlen']} steps ({what})"}
        if secondary is not None:
            attach_cpu_baselines(secondary)
    if rank == 0:
        out = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
               "config": {"workload": "selective scan b8 l32768 d4096 n16 per rank", **W,
                          "l2": "inputs 8.6 GB per step > L2 (no flush needed)", "parallelism": f"dp{world}"},
               "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps,
               "clocks": clocks, "verification": verification, "secondary": secondary}
        print(json.dumps(out), flush=True)


def verify_scan_channels(inp, y, hT, pairs):
    """Max normwise relative error of y[b, d, :] and hT[b, d, :] against the C
    oracle for each (batch row, channel) pair; inputs taken from `inp` (the
    same bf16 values the kernel read), as (err_y, err_hT)."""
    import numpy as np
    from oracle import build as OC
    ey, eh = 0.0, 0.0
    for b, d in pairs:
        f = lambda t: t[b:b + 1, d:d + 1].float().cpu().numpy()  # noqa: E731
        yr, hr = OC.scan(f(inp.u), f(inp.delta), inp.A[d:d + 1].cpu().numpy(), inp.B[b:b + 1].float().cpu().numpy(),
                         inp.C[b:b + 1].float().cpu().numpy(), inp.D[d:d + 1].cpu().numpy(), f(inp.z),
                         inp.delta_bias[d:d + 1].cpu().numpy(), softplus=True, z_mode=2, disc=0)
        yg = y[b, d].float().cpu().numpy()
        hg = hT[b, d].cpu().numpy()
        ey = max(ey, float(np.linalg.norm(yg - yr[0, 0]) / np.linalg.norm(yr[0, 0])))
        eh = max(eh, float(np.linalg.norm(hg - hr[0, 0]) / np.linalg.norm(hr[0, 0])))
    return [ey, eh]


def config5_sharded(args, dev, world, rank, per_rank_gbs, weak_mlstm):
    """The long-context workloads as ONE global job split over the ranks by
    batch rows (no collective on the data path): the selective scan batch 8 x
    32768 x 4096 (dstate 16) and the mLSTM batch 8 x 8 heads x 32768 x 512
    (per-head gates, chunk 128).  Rank r runs rows shard_range(8, world, r);
    after timing, NCCL all-gathers the output and final-state shards to every
    rank and rank 0 checks sampled rows of the gathered result against the C
    oracle, regenerating those rows' inputs (workloads.scan_rows / mlstm_rows
    draw each row from its own seed).  Strong scaling: value = the global
    workload's units / the slowest rank's time; efficiency = value / (world x
    the per-rank rate of the same kernel on the full workload, measured in this
    run)."""
    import numpy as np
    from hybrid_model_mamba_xlstm_b200 import dist as D
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import selective_scan_fn
    from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_interface import mlstm_chunkwise_fwd
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_rows, scan_rows
    from oracle import build as OC
    GB, L, DM, N = 8, 32768, 4096, 16
    a, b = D.shard_range(GB, world, rank)
    steps = max(3, min(args.steps, 5))
    out = {}
    # ---- selective scan
    inp = scan_rows(range(a, b), L, DM, N, torch.bfloat16, seed=11, device=dev)
    fn = lambda: selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z,  # noqa: E731
                                   delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
    ms = _time_cuda(fn, steps, 3, dev, world)
    gbytes = _scan_bytes(GB, L, DM, N)
    val = gbytes / ms / 1e6
    y, hT = fn()
    yall, hall = D.gather_rows(y, GB, world), D.gather_rows(hT, GB, world)
    del y, hT, inp
    err = [0.0, 0.0]
    if rank == 0:
        for bb, d in ((0, 0), (GB // 2, 2047), (GB - 1, DM - 1)):
            ri = scan_rows(range(bb, bb + 1), L, DM, N, torch.bfloat16, seed=11, device=dev)
            f = lambda t: t[:, d:d + 1].float().cpu().numpy()  # noqa: E731
            yr, hr = OC.scan(f(ri.u), f(ri.delta), ri.A[d:d + 1].cpu().numpy(), ri.B.float().cpu().numpy(),
                             ri.C.float().cpu().numpy(), ri.D[d:d + 1].cpu().numpy(), f(ri.z),
                             ri.delta_bias[d:d + 1].cpu().numpy(), softplus=True, z_mode=2, disc=0)
            e = lambda g, r: float(np.linalg.norm(g - r) / np.linalg.norm(r))  # noqa: E731
            err = [max(err[0], e(yall[bb, d].float().cpu().numpy(), yr[0, 0])),
                   max(err[1], e(hall[bb, d].cpu().numpy(), hr[0, 0]))]
            del ri
    del yall, hall
    torch.cuda.empty_cache()
    out["scan_b8_l32768_d4096_n16"] = {
        "metric": "selective-scan HBM GB/s, one global workload split over the ranks", "value": val,
        "unit": "GB/s", "ms": ms, "rows_per_rank": b - a, "scaling": "strong",
        "efficiency": val / (world * per_rank_gbs),
        "verification": {"max_rel_err_y_hT": err, "tolerance": 2e-2, "ok": bool(max(err) <= 2e-2),
                         "checked": "rank 0, gathered y and final state of 3 (row, channel) pairs over all "
                                    "32768 steps vs the C oracle"}}
    # ---- mLSTM (key-streaming tcgen05 kernel)
    H, D2 = 8, 512
    mi = mlstm_rows(range(a, b), H, L, D2, torch.bfloat16, seed=12, device=dev)
    fn = lambda: mlstm_chunkwise_fwd(mi.q, mi.k, mi.v, mi.log_i, mi.log_f, return_state=True)  # noqa: E731
    ms = _time_cuda(fn, steps, 2, dev, world)
    fl = GB * H * (L / 128) * (2 * 128 * 128 * D2 * 2 + 2 * 128 * D2 * D2 * 2)
    val = fl / ms / 1e9
    h, (C, n, m) = fn()
    hall, Call, nall, mall = (D.gather_rows(t, GB, world) for t in (h, C, n, m))
    del h, C, n, m, mi
    err = [0.0, 0.0]
    if rank == 0:
        pairs = [(0, 0), (GB - 1, H - 1)]
        qs, ks, vs, igs, fgs = [], [], [], [], []
        for bb, hh in pairs:
            ri = mlstm_rows(range(bb, bb + 1), H, L, D2, torch.bfloat16, seed=12, device=dev)
            qs.append(ri.q[0, hh]); ks.append(ri.k[0, hh]); vs.append(ri.v[0, hh])
            igs.append(torch.exp(ri.log_i[0, hh])); fgs.append(torch.exp(ri.log_f[0, hh]))
            del ri
        st = lambda ts: torch.stack(ts)[None].float().cpu().numpy()  # noqa: E731
        hr, Cr, nr = OC.mlstm(st(qs), st(ks), st(vs), st(igs), st(fgs))
        e = lambda g, r: float(np.linalg.norm(g - r) / np.linalg.norm(r))  # noqa: E731
        for i, (bb, hh) in enumerate(pairs):
            em = float(torch.exp(mall[bb, hh]))
            err = [max(err[0], e(hall[bb, hh].float().cpu().numpy(), hr[0, i])),
                   max(err[1], e(Call[bb, hh].cpu().numpy() * em, Cr[0, i]))]
    del hall, Call, nall, mall
    torch.cuda.empty_cache()
    weak = weak_mlstm["value"] / world if weak_mlstm else None
    out["mlstm_b8_h8_l32768_d512"] = {
        "metric": "mLSTM chunkwise TFLOP/s, one global workload split over the ranks", "value": val,
        "unit": "TFLOP/s", "ms": ms, "chunk": 128, "rows_per_rank": b - a, "scaling": "strong",
        "efficiency": (val / (world * weak)) if weak else None,
        "verification": {"max_rel_err_h_C": err, "tolerance": 2e-2, "ok": bool(max(err) <= 2e-2),
                         "checked": "rank 0, gathered h and final C of 2 (row, head) pairs over all 32768 "
                                    "steps vs the C oracle"}}
    D.barrier(world)
    return out


def attach_cpu_baselines(sec):
    """The reference's own CPU functions (from baseline/_ref; all host threads,
    fp32) timed beside the secondary workloads, each on a bounded sample
    scaled to the secondary's unit: tfla_forward_pytorch (tfla_interface.py:
    84-139) for the mLSTM workloads, selective_scan_pytorch with head-repeated
    A and dt for SSD, the sLSTM loop of sLSTMBlock.forward
    (slstm_block.py:117-127) and HybridLanguageModel.forward (hybrid_lm.py:
    145-209) for the prefill."""
    ref = ref_pkg()
    if ref is None:
        return
    threads = _cpu_threads()
    import warnings
    warnings.simplefilter("ignore")
    from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs, ssd_inputs

    def timed(fn):
        t0 = time.perf_counter()
        with torch.no_grad():
            fn()
        return time.perf_counter() - t0

    def put(key, value, unit, sample, secs):
        if key in sec:
            sec[key]["cpu_baseline"] = {"value": value, "unit": unit, "cores": threads, "kind": "reference",
                                        "sample": sample, "seconds": secs}

    # mLSTM: the exact 2 x 4 x 2048 x 256 workload in full; the larger ones as a 4096-step prefix of
    # one (batch, head) pair (the loop's cost is linear in steps and pairs), scaled to the workload
    for key, (b, h, L, d, Ls, scale, full) in {
            "mlstm_b2_h4_l2048_d256": (2, 4, 2048, 256, 2048, 1.0, (2, 4, 2048)),
            "mlstm_b8_h8_l8192_d256": (1, 1, 4096, 256, 4096, 8.0 * 8 * 2, (8, 8, 8192)),
            "mlstm_b8_h8_l32768_d512": (1, 1, 4096, 512, 4096, 8.0 * 64, (8, 8, 32768))}.items():
        if key not in sec:
            continue
        inp = mlstm_inputs(b, h, Ls, d, torch.float32, seed=0)
        ex = lambda t: t[..., None].expand(*t.shape, d)  # noqa: E731
        args = (inp.q, inp.k, inp.v, ex(torch.exp(inp.log_i)), ex(torch.exp(inp.log_f)))
        secs = timed(lambda: ref["tfla"].tfla_forward_pytorch(*args))
        fl = full[0] * full[1] * full[2] / 128 * (2 * 128 * 128 * d * 2 + 2 * 128 * d * d * 2)
        put(key, fl / (secs * scale) / 1e12, "TFLOP/s",
            f"tfla_forward_pytorch {b}x{h}x{Ls}x{d} fp32" + (f", scaled x{int(scale)}" if scale > 1 else ""), secs)

    # backward: the reference's rule — its forward loop re-run under autograd
    # (SelectiveScanFunction.backward, scan_interface.py:62-100; TFLAFunction.backward,
    # tfla_interface.py:52-81) — timed for .backward() alone on a sample, scaled to the workload
    def timed_bwd(fwd, leaves):
        leaves = [t.detach().clone().requires_grad_(True) for t in leaves]
        out = fwd(*leaves)
        out = out[0] if isinstance(out, tuple) else out
        g = torch.randn_like(out)
        t0 = time.perf_counter()
        out.backward(g)
        return time.perf_counter() - t0

    if "mlstm_bwd_b8_h4_l2048_d512_channel_gates" in sec:
        # one (batch, head) pair x 512 steps of the 350M mLSTM layer shape, per-channel gates; x 32 pairs x 4
        inp = mlstm_inputs(1, 1, 512, 512, torch.float32, seed=0)
        g = torch.Generator().manual_seed(1)
        li = 0.5 * torch.randn(1, 1, 512, 512, generator=g)
        lf = torch.nn.functional.logsigmoid(torch.randn(1, 1, 512, 512, generator=g) + 3.0)
        secs = timed_bwd(lambda q, k, v, a, f: ref["tfla"].tfla_forward_pytorch(q, k, v, torch.exp(a), torch.exp(f)),
                         [inp.q, inp.k, inp.v, li, lf])
        put("mlstm_bwd_b8_h4_l2048_d512_channel_gates", secs * 128 * 1e3, "ms",
            "autograd backward of tfla_forward_pytorch, 1x1x512x512 per-channel gates, fp32, scaled x128", secs)
    if "ssd_bwd_b8_h32_p64_n128_l4096" in sec:
        # one batch row, 4 of the 32 heads (256 channels, head-repeated A and dt), 1024 of 4096 steps; x 8 x 8 x 4
        si = ssd_inputs(1, 1024, 4, 64, 128, seed=0)
        xs = si.x.float().reshape(1, 1024, 256)
        dts = si.dt.repeat_interleave(64, dim=2)
        As = si.A.repeat_interleave(64)[:, None].expand(256, 128).contiguous()
        secs = timed_bwd(lambda x, dt, a, bm, cm: ref["scan"].selective_scan_pytorch(x, dt, a, bm, cm,
                                                                                     si.D.repeat_interleave(64)),
                         [xs, dts, As, si.B.float(), si.C.float()])
        put("ssd_bwd_b8_h32_p64_n128_l4096", secs * 256 * 1e3, "ms",
            "autograd backward of selective_scan_pytorch (head-repeated A, dt), 1 row x 4 heads x 1024 steps, fp32, "
            "scaled x256", secs)
    if "scan_bwd_b8_l2048_d2048_n16" in sec:
        # one batch row x 256 of 2048 channels x 2048 steps; x 8 rows x 8
        from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
        s2 = scan_inputs(1, 2048, 256, 16, torch.float32, seed=0)
        tr = lambda t: t.transpose(1, 2).contiguous()  # noqa: E731  (B, L, D) as the reference takes it
        secs = timed_bwd(lambda u, dt, a, bm, cm: ref["scan"].selective_scan_pytorch(u, dt, a, bm, cm, s2.D),
                         [tr(s2.u), tr(torch.nn.functional.softplus(s2.delta + s2.delta_bias[:, None])), s2.A,
                          tr(s2.B), tr(s2.C)])
        nbytes = sec["scan_bwd_b8_l2048_d2048_n16"].get("roofline", {}).get("algorithmic", {}).get("bytes")
        if nbytes:
            put("scan_bwd_b8_l2048_d2048_n16", nbytes / (secs * 64) / 1e9, "GB/s",
                "autograd backward of selective_scan_pytorch, 1 row x 256 channels x 2048 steps, fp32, scaled x64",
                secs)
    # SSD: one of the 8 batch rows in full (32 heads x 64 = 2048 channels, dstate 128, 4096 steps), x 8
    si = ssd_inputs(1, 4096, 32, 64, 128, seed=0)
    x = si.x.float().reshape(1, 4096, 2048)
    dt = si.dt.repeat_interleave(64, dim=2)
    A = si.A.repeat_interleave(64)[:, None].expand(2048, 128).contiguous()
    secs = timed(lambda: ref["scan"].selective_scan_pytorch(x, dt, A, si.B.float(), si.C.float(),
                                                            si.D.repeat_interleave(64)))
    fl = 8 * (4096 / 128) * 2 * 128 * 128 * 128 + 8 * 32 * (4096 / 128) * (2 * 128 * 128 * 64 + 4 * 128 * 128 * 64)
    put("ssd_b8_h32_p64_n128_l4096", fl / (secs * 8) / 1e12, "TFLOP/s",
        "selective_scan_pytorch with head-repeated A, dt: 1 of 8 batch rows, fp32, scaled x8", secs)
    # sLSTM: the reference block's step loop at batch 8, 4 heads x 256, 2048 steps (projections included)
    from hybrid_xmamba.layers import slstm_block as sb
    torch.manual_seed(0)
    blk = sb.sLSTMBlock(1024, hidden_dim=1024, num_heads=4).eval()
    xs = torch.randn(8, 2048, 1024)
    z = torch.zeros(8, 4, 256)
    secs = timed(lambda: blk(xs, cache={"h": z.clone(), "c": z.clone()}))
    put("slstm_b8_h4_hd256_l2048", secs * 1e6 / 2048, "us/step",
        "sLSTMBlock.forward (its step loop and projections), batch 8 x 2048, fp32", secs)
    # prefill: the reference HybridLanguageModel at the 350M architecture, batch 1 x 256 tokens
    from hybrid_xmamba.models import configuration_hybrid as cm, hybrid_lm as hl
    orig = sb.sLSTMBlock.forward

    def fwd_with_cache(self, x, cache=None):  # the reference crashes without a shaped cache (slstm_block.py:109-112)
        if cache is None:
            zz = torch.zeros(x.shape[0], self.num_heads, self.head_dim, dtype=x.dtype)
            cache = {"h": zz.clone(), "c": zz.clone()}
        return orig(self, x, cache=cache)
    sb.sLSTMBlock.forward = fwd_with_cache
    try:
        cfg = cm.HybridConfig(vocab_size=50304, dim=1024, num_layers=24, layer_pattern=["mamba", "mamba", "mlstm",
                              "slstm"], state_size=16, conv_size=4, expand_factor=2, head_dim=512, num_heads=4,
                              slstm_num_heads=4, dropout=0.0)
        torch.manual_seed(0)
        model = hl.HybridLanguageModel(cfg).eval()
        ids = torch.randint(0, 50304, (1, 256))
        secs = timed(lambda: model(ids))
        if "prefill" in sec:
            for kind in ("weak", "strong"):
                sec["prefill"][kind]["cpu_baseline"] = {
                    "value": 256 / secs, "unit": "tok/s", "cores": threads, "kind": "reference", "seconds": secs,
                    "sample": "HybridLanguageModel.forward, hybrid-350M architecture, batch 1 x 256 tokens, fp32"}
        del model
    finally:
        sb.sLSTMBlock.forward = orig


def e2e_scan(dev, args, world):
    """The headline metric through ``selective_scan_fn`` with host buffers:
    every step copies its inputs from pinned host memory and reads its output
    back.  Copies in and out run on their own streams with double-buffered
    device buffers, so step i's read-back overlaps step i + 1's upload (PCIe
    is full duplex); both stay inside the timed region."""
    from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import selective_scan_fn
    from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
    W = WORKLOAD
    host = scan_inputs(1, W["seqlen"], W["dim"], W["dstate"], torch.bfloat16, seed=7, device=dev, on_device=True)
    names = ["u", "delta", "z", "B", "C"]
    pinned = {k: getattr(host, k).cpu().pin_memory() for k in names}
    dbuf = [{k: torch.empty_like(getattr(host, k)) for k in names} for _ in range(2)]
    ybuf = [torch.empty_like(host.u) for _ in range(2)]
    y_host = torch.empty(pinned["u"].shape, dtype=torch.bfloat16).pin_memory()
    s_in, s_comp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())
    d2h = y_host.numel() * y_host.element_size()
    used = [None, None]  # per buffer: event after the last kernel / read-back that used it

    def step(i):
        j = i % 2
        ev_in = torch.cuda.Event()
        with torch.cuda.stream(s_in):
            if used[j] is not None:
                s_in.wait_event(used[j])  # buffer j's previous kernel and read-back are done
            for k in names:
                dbuf[j][k].copy_(pinned[k], non_blocking=True)
            ev_in.record(s_in)
        ev_comp = torch.cuda.Event()
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_in)
            y = selective_scan_fn(dbuf[j]["u"], dbuf[j]["delta"], host.A, dbuf[j]["B"], dbuf[j]["C"], host.D,
                                  z=dbuf[j]["z"], delta_bias=host.delta_bias, delta_softplus=True)
            ybuf[j].copy_(y)
            ev_comp.record(s_comp)
        ev_out = torch.cuda.Event()
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp)
            y_host.copy_(ybuf[j], non_blocking=True)
            ev_out.record(s_out)
        used[j] = ev_out
        return ev_out

    for i in range(max(1, args.warmup)):
        step(i)
    torch.cuda.synchronize(dev)
    used[0] = used[1] = None
    steps = max(1, min(args.steps, 5))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    e0.record(s_in)
    for st in (s_comp, s_out):
        st.wait_event(e0)
    for i in range(steps):
        last = step(i)
    s_out.wait_event(last)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    nbytes = scan_inputs_bytes(1, W)
    return {"value": world * nbytes * steps / (ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "sample": "1 batch row per rank per step, pinned host buffers, copies in / out on their own streams",
            "ms_per_step": ms / steps}


def scan_inputs_bytes(batch, W):
    L, dm, n, es = W["seqlen"], W["dim"], W["dstate"], 2
    return batch * L * dm * 4 * es + 2 * batch * L * n * es + (dm * n + 2 * dm) * 4 + batch * dm * n * 4


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-secondary", action="store_true", help="only the headline scan workload")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args)
    try:
        run_ours(args, world, rank, local)
    finally:
        from hybrid_model_mamba_xlstm_b200 import dist as D
        D.finalize(world)


if __name__ == "__main__":
    main()
