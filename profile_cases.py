"""Small, self-contained GPU workloads for profiling one kernel family at a time.

    python profile_cases.py <case> [sizes...] [--reps N]

Each case builds seeded synthetic inputs on ``cuda:0``, runs the public entry
point ``reps`` times (default 2: one warm-up launch, one to capture) and prints
one JSON line with the last launch's CUDA-event time.  The sizes keep the
device footprint to a few GB so that a profiler capture of one launch ends in
a minute or two.

cases (default sizes):
  scan         B L D             (8 4096 4096)   selective_scan_fn, bf16, dstate 16, softplus, y*silu(z)
  ssd          B L H P N         (8 4096 32 64 128)
  mlstm        B H L D chunk     (8 8 2048 256 128)  per-head gates
  mlstm_stream B H L D           (8 4 2048 512)   per-channel gates (key-streaming kernel)
  mlstm_bwd    B H L D           (8 4 2048 512)   chunkwise backward, per-channel gates, bf16 (TF32 chunk GEMMs)
  ssd_bwd      B L H P N         (8 4096 32 64 128)  SSD backward (exact per-head chunk form, TF32 chunk GEMMs)
  scan_bwd     B L D             (8 2048 2048)   selective-scan backward, bf16 inputs, fp32 gradients
  slstm        B L H HD          (8 256 4 256)    recurrent R
  conv         B D L             (8 4096 2048)    causal depthwise conv1d(4) + SiLU
  mamba_layer  B L               (8 2048)         one hybrid-350M Mamba block
  prefill      B L               (8 2048)         the hybrid-350M model forward
  prefill_graph B L PIECES       (8 2048 4)       the same prefill as a wavefront replayed from a CUDA graph
  decode       B P               (1 512)          hybrid-350M: prefill P tokens, then time one-token steps
                                                  (eager, and replayed from a CUDA graph)
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _time(fn, reps):
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    out = None
    for i in range(reps):
        if i == reps - 1:
            ev[0].record()
        out = fn()
        if i == reps - 1:
            ev[1].record()
    torch.cuda.synchronize()
    return ev[0].elapsed_time(ev[1]), out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("sizes", nargs="*", type=int)
    ap.add_argument("--reps", type=int, default=2)
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    s = a.sizes

    if a.case == "scan":
        from hybrid_model_mamba_xlstm_b200.kernels.selective_scan import selective_scan_fn
        from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
        B, L, D = (s + [8, 4096, 4096][len(s):])[:3]
        inp = scan_inputs(B, L, D, 16, torch.bfloat16, seed=0, device="cuda", on_device=True)
        fn = lambda: selective_scan_fn(inp.u, inp.delta, inp.A, inp.B, inp.C, inp.D, z=inp.z,  # noqa: E731
                                       delta_bias=inp.delta_bias, delta_softplus=True, return_last_state=True)
        extra = {"GB/s": None, "bytes": inp.bytes_moved()}
    elif a.case == "ssd":
        from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan
        from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
        B, L, H, P, N = (s + [8, 4096, 32, 64, 128][len(s):])[:5]
        inp = ssd_inputs(B, L, H, P, N, seed=0, device="cuda")
        fn = lambda: ssd_chunk_scan(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D)  # noqa: E731
        extra = {"flops": inp.flops(256)}
    elif a.case == "mlstm":
        from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_interface import mlstm_chunkwise_fwd
        from hybrid_model_mamba_xlstm_b200.workloads import mlstm_inputs
        B, H, L, D, c = (s + [8, 8, 2048, 256, 128][len(s):])[:5]
        inp = mlstm_inputs(B, H, L, D, torch.bfloat16, seed=0, device="cuda", on_device=True)
        fn = lambda: mlstm_chunkwise_fwd(inp.q, inp.k, inp.v, inp.log_i, inp.log_f, chunk=c)  # noqa: E731
        extra = {"flops": inp.flops(c)}
    elif a.case == "mlstm_stream":
        from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_interface import mlstm_chunkwise_fwd
        B, H, L, D = (s + [8, 4, 2048, 512][len(s):])[:4]
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        q = (torch.randn(B, H, L, D, generator=g, device=dev) / D ** 0.5).to(torch.bfloat16)
        k = torch.randn(B, H, L, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(B, H, L, D, generator=g, device=dev).to(torch.bfloat16)
        li = torch.randn(B, H, L, D, generator=g, device=dev) * 0.1
        lf = torch.nn.functional.logsigmoid(torch.randn(B, H, L, D, generator=g, device=dev) * 0.1)
        fn = lambda: mlstm_chunkwise_fwd(q, k, v, li, lf)  # noqa: E731
        extra = {}
    elif a.case == "slstm":
        from hybrid_model_mamba_xlstm_b200.kernels.slstm import slstm_scan
        B, L, H, HD = (s + [8, 256, 4, 256][len(s):])[:4]
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        gates = (torch.randn(B, L, H, 4, HD, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        R = (torch.randn(H, HD, 4 * HD, generator=g, device=dev) / HD ** 0.5).to(torch.bfloat16)
        w = torch.ones(HD, device=dev)
        fn = lambda: slstm_scan(gates, w, R=R)  # noqa: E731
        extra = {"steps": L}
    elif a.case == "conv":
        from hybrid_model_mamba_xlstm_b200.kernels.conv import causal_conv1d
        B, D, L = (s + [8, 4096, 2048][len(s):])[:3]  # batch, channels, seqlen: x is (B, L, D)
        g = torch.Generator(device=dev)
        g.manual_seed(0)
        x = torch.randn(B, L, D, generator=g, device=dev).to(torch.bfloat16)
        w = torch.randn(D, 4, generator=g, device=dev) * 0.5
        bias = torch.randn(D, generator=g, device=dev) * 0.1
        fn = lambda: causal_conv1d(x, w, bias, activation="silu")  # noqa: E731
        extra = {"bytes": 2 * x.numel() * 2}
    elif a.case in ("mamba_layer", "prefill"):
        from hybrid_model_mamba_xlstm_b200 import layers as Lyr
        B, L = (s + [8, 2048][len(s):])[:2]
        torch.manual_seed(0)
        if a.case == "mamba_layer":
            cfg = Lyr.hybrid_350m_config(num_layers=1, layer_pattern=["mamba"])
            blk = Lyr.HybridLanguageModel(cfg).to(dev).to(torch.bfloat16).eval().layers[0]
            x = torch.randn(B, L, cfg.dim, device=dev, dtype=torch.bfloat16)
            fn = lambda: blk(x)  # noqa: E731
        else:
            model = Lyr.HybridLanguageModel(Lyr.hybrid_350m_config()).to(dev).to(torch.bfloat16).eval()
            ids = torch.randint(0, model.config.vocab_size, (B, L), device=dev)
            fn = lambda: model(ids)  # noqa: E731
        extra = {"tokens": B * L}
    elif a.case == "layer":
        # one layer of the 350M model on a (batch, tokens) piece with its recurrent cache, as the
        # prefill wavefront runs it: layer 0 Mamba, 2 mLSTM, 3 sLSTM
        from hybrid_model_mamba_xlstm_b200 import layers as Lyr
        idx, B, L = (s + [2, 1, 256][len(s):])[:3]
        torch.manual_seed(0)
        model = Lyr.HybridLanguageModel(Lyr.hybrid_350m_config()).to(dev).to(torch.bfloat16).eval()
        blk, caches = model.layers[idx], model.init_caches()
        x = torch.randn(B, L, model.config.dim, device=dev, dtype=torch.bfloat16)
        fn = lambda: blk.forward_pending(x, None, cache=caches[idx])  # noqa: E731
        extra = {"tokens": B * L, "mixer": type(blk.mixer).__name__}
    elif a.case == "prefill_graph":
        from hybrid_model_mamba_xlstm_b200 import layers as Lyr
        B, L, pieces = (s + [8, 2048, 4][len(s):])[:3]
        torch.manual_seed(0)
        model = Lyr.HybridLanguageModel(Lyr.hybrid_350m_config()).to(dev).to(torch.bfloat16).eval()
        ids = torch.randint(0, model.config.vocab_size, (B, L), device=dev)
        with torch.no_grad():
            pg = Lyr.PrefillGraph(model, B, L, pieces=pieces, device=dev)
        fn = lambda: pg(ids)  # noqa: E731
        extra = {"tokens": B * L, "pieces": pieces}
    elif a.case == "mlstm_bwd":
        # chunkwise mLSTM backward, per-channel gates (mLSTMBlock), bf16 q / k / v
        from hybrid_model_mamba_xlstm_b200.kernels.tfla.tfla_bwd import mlstm_chunkwise_bwd
        B, H, L, D = (s + [8, 4, 2048, 512][len(s):])[:4]
        g = torch.Generator(device=dev).manual_seed(0)
        q, k, v, dh = (torch.randn(B, H, L, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(4))
        q.mul_(D ** -0.5)
        li = torch.randn(B, H, L, D, generator=g, device=dev).mul_(0.5)
        lf = torch.nn.functional.logsigmoid(torch.randn(B, H, L, D, generator=g, device=dev))
        fn = lambda: mlstm_chunkwise_bwd(q, k, v, li, lf, dh)  # noqa: E731
        extra = {"chunk": 128, "path": "tcgen05 chunk GEMMs"}
    elif a.case == "scan_bwd":
        # selective-scan backward (softplus(delta + bias), y * silu(z)), bf16 inputs, fp32 gradients
        from hybrid_model_mamba_xlstm_b200.kernels.selective_scan.scan_interface import selective_scan_bwd
        from hybrid_model_mamba_xlstm_b200.workloads import scan_inputs
        B, L, D = (s + [8, 2048, 2048][len(s):])[:3]
        inp = scan_inputs(B, L, D, 16, torch.bfloat16, seed=0, device="cuda", on_device=True)
        dout = torch.randn(B, D, L, device=dev).to(torch.bfloat16)
        t = lambda x: x.transpose(1, 2)  # noqa: E731
        fn = lambda: selective_scan_bwd(t(dout), t(inp.u), t(inp.delta), inp.A, t(inp.B), t(inp.C), inp.D,  # noqa: E731
                                        t(inp.z), z_mode="silu", delta_bias=inp.delta_bias, delta_softplus=True)
        extra = {"bytes": B * L * D * (4 * 2 + 3 * 4) + B * L * 16 * (2 * 2 + 2 * 4)}
    elif a.case == "ssd_bwd":
        # SSD backward (exact per-head chunk form, TF32 chunk GEMMs) for the bf16 forward's inputs
        from hybrid_model_mamba_xlstm_b200.kernels.ssd import ssd_chunk_scan_bwd
        from hybrid_model_mamba_xlstm_b200.workloads import ssd_inputs
        B, L, H, P, N = (s + [8, 4096, 32, 64, 128][len(s):])[:5]
        inp = ssd_inputs(B, L, H, P, N, seed=0, device="cuda", on_device=True)
        dy = torch.randn(B, L, H, P, device=dev).to(torch.bfloat16)
        fn = lambda: ssd_chunk_scan_bwd(inp.x, inp.dt, inp.A, inp.B, inp.C, inp.D, dy)  # noqa: E731
        extra = {}
    elif a.case == "decode":
        from hybrid_model_mamba_xlstm_b200 import layers as Lyr
        B, P = (s + [1, 512][len(s):])[:2]
        torch.manual_seed(0)
        model = Lyr.HybridLanguageModel(Lyr.hybrid_350m_config()).to(dev).to(torch.bfloat16).eval()
        ids = torch.randint(0, model.config.vocab_size, (B, P), device=dev)
        tok = torch.randint(0, model.config.vocab_size, (B, 1), device=dev)
        with torch.no_grad():
            caches = model.init_caches()
            model(ids, caches=caches)
            eager_ms, _ = _time(lambda: model(tok, caches=caches), max(3, a.reps))
            dec = Lyr.GraphDecoder(model, B, dev)
            dec.prefill(ids)
            dec.step(tok)
            graph_ms, _ = _time(lambda: dec.step(tok), max(3, a.reps))
        print(json.dumps({"case": "decode", "sizes": [B, P], "eager_ms_per_token": eager_ms,
                          "graph_ms_per_token": graph_ms, "tokens/s (graph)": B / graph_ms * 1e3}), flush=True)
        return
    else:
        raise SystemExit(f"unknown case {a.case!r}")

    with torch.no_grad():
        ms, _ = _time(fn, max(1, a.reps))
    out = {"case": a.case, "sizes": s, "ms": ms}
    if "bytes" in extra:
        out["GB/s"] = extra["bytes"] / ms / 1e6
    if "flops" in extra:
        out["TFLOP/s"] = extra["flops"] / ms / 1e9
    if "tokens" in extra:
        out["tokens/s"] = extra["tokens"] / ms * 1e3
    if "steps" in extra:
        out["us/step"] = ms * 1e3 / extra["steps"]
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
