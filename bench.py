#!/usr/bin/env python
"""Kokoro decoder fwd+bwd throughput (audio-seconds / second) on 1..8 B200.

One step = one training step of the full Kokoro-82M iSTFTNet decoder on one
batch of synthetic clips per GPU: harmonic source, forward, L1 loss, backward
(gradients for every decoder weight and for the asr / style inputs), gradient
all-reduce across ranks (N > 1), Adam update. Default workload = BASELINE
config 2: batch 16 x T=200 asr frames (5 s clips) per GPU (weak scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload c2|c0|c3|c3lora|c1] [--eager]
For N > 1 launch with torchrun (one rank per GPU, NCCL over NVLink). On the
decoder workloads the forward, loss and backward of a step are recorded once as
a CUDA graph and replayed (--eager launches every kernel from the host instead);
the all-reduce and the Adam update run outside the graph.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Kokoro decoder fwd+bwd audio-seconds/sec at 1/2/4/8 B200; % tensor/HBM roofline"
# ncu capture (gpu__time_duration, dram__bytes_read/write) of conv_fwd_tc_kernel<tf32x3> on the probe
# case B=16, Ci=Co=128, L=24001, k=7, d=3: 443.7 us, 395.0 MB read + 162.7 MB written
NCU_CONV_FWD_TC = {"dram_bytes": 395.0e6 + 162.7e6, "flops": 2.0 * 16 * 128 * 128 * 7 * 24001}
UNIT = "audio-s/s"
WORKLOADS = {
    # name: (B per GPU, T asr frames (c1: samples L), description)
    "c2": (16, 200, "Kokoro-82M decoder fwd+bwd, B=16 x T=200 (5 s clips) per GPU, BASELINE config 2"),
    "c0": (1, 32, "Kokoro-82M decoder fwd+bwd, B=1 x T=32 (0.8 s), BASELINE config 0"),
    "c3": (64, 400, "Kokoro-82M decoder fwd+bwd, B=64 x T=400 (10 s clips) per GPU, BASELINE config 3 shapes"),
    "c3lora": (64, 400, "Kokoro-82M decoder conv-weight LoRA step (rank 8, scale 2, base frozen), B=64 x T=400 "
                        "(10 s clips) per GPU, BASELINE config 3"),
    "c1": (8, 24000, "one generator AdaINResBlock1 (C=128, k=7, dilations 1,3,5, Snake, AdaIN style 128) "
                     "fwd+bwd, x [8,128,24000], BASELINE config 1"),
}
# The bench's math mode on the decoder workloads: TF32x3 for the forward contractions,
# BF16x3 for the input- and weight-gradient contractions (the decoder's gradients are
# sensitive to the forward's rounding, not the backward's); the whole gradient stays
# within the 3xTF32 bar at config 2 (tests/test_gpu_config2.py). Pure TF32x3 and BF16x3
# are measured beside it.
BENCH_MATH = "tf32x3f"
MATH_NOTES = {
    "tf32x3f": "TF32x3 (each fp32 operand split into tf32 hi + lo, three products, fp32 accumulation) for the "
               "forward convs; BF16x3 (bf16 hi + lo, three products, fp32 accumulation) for the input- and "
               "weight-gradient convs; elementwise, normalisation and spectral work in fp32",
    "tf32x3w": "TF32x3 (each fp32 operand split into tf32 hi + lo, three products, fp32 accumulation) for the "
               "forward and input-gradient convs; BF16x3 (bf16 hi + lo, three products, fp32 accumulation) for "
               "the weight-gradient convs; elementwise, normalisation and spectral work in fp32",
    "tf32x3": "TF32x3 for every conv; elementwise, normalisation and spectral work in fp32",
    "bf16x3": "BF16x3 for every conv; elementwise, normalisation and spectral work in fp32",
}
# BASELINE config 1 reports conv throughput, not audio
C1_METRIC = "AdaINResBlock1 [8,128,24000] k7 fwd+bwd conv TFLOP/s (fwd+dgrad+wgrad); Snake/AdaIN GB/s"


_JSON_FD = None   # the original stdout of a multi-rank run (file descriptor 1 then points at stderr)


def emit_json(line):
    """The bench line, alone on stdout."""
    s = json.dumps(line) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(s)
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, s.encode())


def audio_seconds(B, T):
    return B * 600 * T / 24000.0


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return dict(hbm_gbs=d["hbm_gbs"], bf16_tflops=d["bf16_tflops"],
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained", d["bf16_tflops"]), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
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
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def run_cpu_baseline(cfg, T, threads=None):
    """The oracle (a CPU restatement of the reference composition) on a bounded
    sample: one clip of the workload's length, forward + backward."""
    import numpy as np

    from brosoundml_b200 import synth
    from oracle import oracle as orc

    prev = orc.threads()
    if threads:
        orc.set_threads(threads)
    o = orc.Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 1, T, 101)
    tgt = synth.make_target(cfg, 1, T, 102)
    # warm the library and the page cache on a tiny case
    xs = synth.make_inputs(cfg, 1, 2, 1)
    o.run(params, xs["asr"], xs["F0"], xs["N"], xs["style"])
    t0 = time.perf_counter()
    r = o.run(params, x["asr"], x["F0"], x["N"], x["style"])
    _, da = synth.l1_grad(r["audio"], tgt)
    o.run(params, x["asr"], x["F0"], x["N"], x["style"], daudio=da)
    dt = time.perf_counter() - t0
    cores = orc.threads()
    orc.set_threads(prev)
    del np
    return dict(value=audio_seconds(1, T) / dt, unit=UNIT, cores=cores, kind="port",
                sample=f"1 clip x T={T} ({audio_seconds(1, T):.1f} audio-s): harmonic source, fwd, L1, bwd "
                       f"(all grads) in the C++ oracle (oracle/kokoro_oracle.cpp), {dt:.1f} s")


def setup_decoder(args, B, T, dev, rank, math):
    """Full decoder training step: forward, L1, backward (all grads), all-reduce, Adam."""
    import torch

    from brosoundml_b200 import config, dp, synth
    from brosoundml_b200.decoder import Decoder, adam_step, l1_loss

    cfg = config.kokoro_82m()
    dec = Decoder(cfg, dev.index, math=math)
    params = torch.tensor(synth.init_params(dec.table, dec.n_params, 0), device=dev)
    x = synth.make_inputs(cfg, B, T, 1 + rank)
    tgt = synth.make_target(cfg, B, T, 1000 + rank)
    host = {k: torch.from_numpy(v).pin_memory() for k, v in x.items()}
    host["target"] = torch.from_numpy(tgt).pin_memory()
    d = {k: v.to(dev) for k, v in host.items()}
    grads = torch.empty(dec.n_params, device=dev)
    m = torch.zeros(dec.n_params, device=dev)
    v = torch.zeros(dec.n_params, device=dev)
    audio = torch.empty((B, dec.audio_len(T)), device=dev)
    lossbuf = torch.empty(1, device=dev)
    dabuf = torch.empty_like(audio)
    d_asr = torch.empty((B, cfg["asr_dim"], T), device=dev)
    d_style = torch.empty((B, cfg["style_dim"]), device=dev)
    state = {"step": 0}

    def fwd_bwd(inp):
        dec.forward(params, inp["asr"], inp["F0"], inp["N"], inp["style"], audio=audio)
        l1_loss(audio, inp["target"], lossbuf, dabuf)
        dec.backward(dabuf, grads=grads, d_asr=d_asr, d_style=d_style)   # all weights, asr and style

    def finish():
        dp.average_gradients(grads)   # one NCCL all-reduce of the flat gradient (N > 1)
        state["step"] += 1
        adam_step(params, grads, m, v, 1e-5, state["step"])

    graph = None
    if args.graph:
        # forward + loss + backward recorded once (after an eager pass that plans the
        # workspace) and replayed; the all-reduce and Adam (whose step count is a
        # launch argument) stay outside the graph
        from brosoundml_b200.decoder import Graph
        fwd_bwd(d)
        torch.cuda.synchronize()
        graph = Graph(torch.cuda.current_stream())
        with graph:
            fwd_bwd(d)

    def step(inp):
        if graph is None:
            fwd_bwd(inp)
        else:
            if inp is not d:
                for k in d:
                    d[k].copy_(inp[k], non_blocking=True)
            graph.replay()
        finish()

    def eager_step(inp):
        fwd_bwd(inp)
        finish()

    return dict(host=host, dev=d, step=step, eager_step=eager_step, result=lossbuf, prof=dec, metric=METRIC,
                unit=UNIT, units_per_step=audio_seconds(B, T), graph=graph,
                config={"audio_s_per_step_per_gpu": audio_seconds(B, T), "cuda_graph": graph is not None,
                        "weights": "random init N(0,0.02), Snake alpha 1", "optimizer": "Adam lr 1e-5"})


def setup_convlora(args, B, T, dev, rank, math):
    """rank-8 LoRA (A ~ N(0, 0.01), B = 0, scale 16/8) on every
    Conv1d / ConvTranspose1d weight, base frozen: forward of the adapted decoder, L1,
    backward, dA/dB, all-reduce of the LoRA gradients (N > 1), Adam on A and B."""
    import torch

    from brosoundml_b200 import config, dp, synth
    from brosoundml_b200.decoder import Decoder, l1_loss
    from brosoundml_b200.lora import ConvLora

    cfg = config.kokoro_82m()
    dec = Decoder(cfg, dev.index, math=math)
    lora = ConvLora(dec, rank=8, scale=16.0 / 8.0, seed=1)
    params = torch.tensor(synth.init_params(dec.table, dec.n_params, 0), device=dev)
    x = synth.make_inputs(cfg, B, T, 1 + rank)
    tgt = synth.make_target(cfg, B, T, 1000 + rank)
    host = {k: torch.from_numpy(v).pin_memory() for k, v in x.items()}
    host["target"] = torch.from_numpy(tgt).pin_memory()
    d = {k: v.to(dev) for k, v in host.items()}
    audio = torch.empty((B, dec.audio_len(T)), device=dev)
    lossbuf = torch.empty(1, device=dev)
    dabuf = torch.empty_like(audio)
    g = lora.grads()

    def step(inp):
        lora.forward(params, inp["asr"], inp["F0"], inp["N"], inp["style"], audio=audio)
        l1_loss(audio, inp["target"], lossbuf, dabuf)
        lora.zero_grad()
        lora.backward(dabuf)
        dp.average_gradients(g)       # one NCCL all-reduce of the flat LoRA gradient (N > 1)
        lora.adam_step(1e-4)

    return dict(host=host, dev=d, step=step, result=lossbuf, prof=dec, metric=METRIC, unit=UNIT,
                units_per_step=audio_seconds(B, T),
                config={"audio_s_per_step_per_gpu": audio_seconds(B, T), "lora_params": lora.n_params,
                        "lora": "rank 8, scale 2, every conv/convT weight, base frozen",
                        "weights": "random init N(0,0.02), Snake alpha 1", "optimizer": "Adam lr 1e-4 on A, B"})


def block_flops(B, C, L, k):
    """Algorithmic conv FLOPs of one AdaINResBlock1 fwd+bwd (6 stride-1 C->C convs,
    forward + input gradient + weight gradient)."""
    return 3 * 6 * 2.0 * B * C * C * k * L


def setup_block(args, B, L, dev, rank, math):
    """one AdaINResBlock1 (C=128, k=7, dilations 1,3,5) fwd+bwd
    with every gradient (conv weights and biases, Snake alphas, AdaIN fc, dx, d_style)."""
    import numpy as np
    import torch

    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import Block

    spec = dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5])
    blk = Block(spec, dev.index, math=math)
    rng = np.random.default_rng(0)
    p = np.zeros(blk.n_params, np.float32)
    for e in blk.table:
        sl = slice(e["offset"], e["offset"] + e["numel"])
        p[sl] = 1.0 if e["name"].startswith("alpha") else rng.normal(0, 0.02, e["numel"])
    params = torch.tensor(p, device=dev)
    r = np.random.default_rng(1 + rank)
    host = {"x": torch.from_numpy(r.standard_normal((B, 128, L), dtype=np.float32)).pin_memory(),
            "style": torch.from_numpy(r.standard_normal((B, 128), dtype=np.float32)).pin_memory(),
            "dy": torch.from_numpy(r.standard_normal((B, 128, L), dtype=np.float32)).pin_memory()}
    d = {k: v.to(dev) for k, v in host.items()}
    y = torch.empty((B, 128, L), device=dev)
    grads = torch.empty(blk.n_params, device=dev)
    dx = torch.empty((B, 128, L), device=dev)
    d_style = torch.empty((B, 128), device=dev)
    L_ = _lib.lib()
    from brosoundml_b200.decoder import _ptr, _stream

    def step(inp):
        blk.forward(params, inp["x"], inp["style"], y=y)
        _lib.check(L_.bsml_block_backward(blk._h, _ptr(inp["dy"]), _ptr(grads), _ptr(dx), _ptr(d_style), None,
                                          _stream()))

    fl = block_flops(B, 128, L, 7)
    return dict(host=host, dev=d, step=step, result=d_style[0, :1], prof=blk, metric=C1_METRIC, unit="TFLOP/s",
                units_per_step=fl / 1e12,
                config={"conv_flops_per_step": fl, "weights": "N(0,0.02), Snake alpha 1",
                        "inputs": "x, style, upstream grad N(0,1)"})


def run_cpu_baseline_block(B, L):
    """The block oracle on the whole config-1 workload (B clips x L samples), timed once."""
    import numpy as np

    from oracle import oracle as orc

    spec = dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5])
    o = orc.BlockOracle(spec)
    rng = np.random.default_rng(0)
    p = rng.normal(0, 0.02, o.n_params).astype(np.float32)
    x = rng.standard_normal((B, 128, L), dtype=np.float32)
    s = rng.standard_normal((B, 128), dtype=np.float32)
    dy = rng.standard_normal((B, 128, L), dtype=np.float32)
    o.run(p, x[:1, :, :256], s[:1], dy=dy[:1, :, :256])
    t0 = time.perf_counter()
    o.run(p, x, s, dy=dy)
    dt = time.perf_counter() - t0
    return dict(value=block_flops(B, 128, L, 7) / dt / 1e12, unit="TFLOP/s", cores=orc.threads(), kind="port",
                sample=f"the whole workload ({B} clips x L={L}) block fwd+bwd (all grads) in the C++ oracle, "
                       f"{dt:.1f} s")


def reference_arm_block(args):
    """Config 1 on the host cores: the block oracle over the whole workload per step."""
    import numpy as np

    from oracle import oracle as orc

    B, L, desc = WORKLOADS["c1"]
    o = orc.BlockOracle(dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5]))
    rng = np.random.default_rng(0)
    p = rng.normal(0, 0.02, o.n_params).astype(np.float32)
    x = rng.standard_normal((B, 128, L), dtype=np.float32)
    s = rng.standard_normal((B, 128), dtype=np.float32)
    dy = rng.standard_normal((B, 128, L), dtype=np.float32)
    for _ in range(args.warmup):
        o.run(p, x, s, dy=dy)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        o.run(p, x, s, dy=dy)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = block_flops(B, 128, L, 7) / dt / 1e12
    sample = f"the whole workload ({B} clips x L={L}) block fwd+bwd (all grads) per step, oracle/kokoro_oracle.cpp"
    line = {
        "impl": "reference", "metric": C1_METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": desc, "sample": sample},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": orc.threads(), "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reference_arm(args):
    """The reference's own CPU path cannot be built here (all its arithmetic is in
    the absent brotensor library), so this arm times the oracle port of it on the
    host cores, as the CPU baseline."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "c1":
        reference_arm_block(args)
        return
    from brosoundml_b200 import config

    cfg = config.kokoro_82m()
    B, T, desc = WORKLOADS[args.workload]
    from oracle import oracle as orc
    import numpy as np
    from brosoundml_b200 import synth

    o = orc.Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    sample_T = T
    x = synth.make_inputs(cfg, 1, sample_T, 101)
    tgt = synth.make_target(cfg, 1, sample_T, 102)

    def step():
        r = o.run(params, x["asr"], x["F0"], x["N"], x["style"])
        _, da = synth.l1_grad(r["audio"], tgt)
        o.run(params, x["asr"], x["F0"], x["N"], x["style"], daudio=da)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = audio_seconds(1, sample_T) / dt
    del np
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": desc, "sample": f"1 clip x T={sample_T} per step on host cores: per-clip "
                                               f"throughput of the same clip length (the GPU arm runs {B} clips "
                                               f"per step and GPU)"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": orc.threads(), "kind": "port",
                         "sample": f"1 clip x T={sample_T} fwd+bwd per step, oracle/kokoro_oracle.cpp"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


SWEEP_B = (1, 4, 16, 64, 256)
SWEEP_T = (50, 200, 800, 1600)
SWEEP_MAX_BT = 64 * 400   # B*T of config 3, whose caches (~110 GB) are the largest that fit 180 GB


def sweep(args):
    """BASELINE config 4 on one GPU: full decoder fwd+bwd (CUDA graph) per (B, T),
    one JSON line each; shapes whose caches exceed one GPU's memory are listed as
    skipped with the reason."""
    import gc

    import torch

    from brosoundml_b200.decoder import Decoder

    torch.cuda.set_device(0)
    torch.cuda.set_stream(torch.cuda.Stream())
    args.graph = not args.eager
    dev = torch.device("cuda", 0)
    math = args.math or BENCH_MATH
    peaks = load_peaks()
    tensor_peak = peaks["bf16_tflops_sustained"]   # measured dense bf16, sustained
    for B in SWEEP_B:
        for T in SWEEP_T:
            cfgd = {"workload": "BASELINE config 4 sweep: Kokoro-82M decoder fwd+bwd", "global_batch": B,
                    "seq_len": T, "parallelism": "dp1", "cuda_graph": args.graph}
            if B * T > SWEEP_MAX_BT:
                print(json.dumps({"metric": METRIC, "value": None, "unit": UNIT, "n_gpus": 1, "config": cfgd,
                                  "skipped": f"B*T = {B * T} > {SWEEP_MAX_BT}: the forward caches exceed one "
                                             "GPU's 180 GB (shard the batch over GPUs)"}), flush=True)
                continue
            w = setup_decoder(args, B, T, dev, 0, math)
            d, step = w["dev"], w["step"]
            for _ in range(args.warmup):
                step(d)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                step(d)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            w["prof"].set_profiling(True)
            w["eager_step"](d)
            prof = w["prof"].read_profile()
            w["prof"].set_profiling(False)
            conv_ms = sum(v[0] for k, v in prof.items() if k.startswith(("conv", "wgrad")))
            conv_fl = sum(v[1] for k, v in prof.items() if k.startswith(("conv", "wgrad")))
            tf = conv_fl / (conv_ms / 1e3) / 1e12 if conv_ms > 0 else 0.0
            nb_ms = prof["norm_bwd"][0]
            nb_gbs = prof["norm_bwd"][1] / (nb_ms / 1e3) / 1e9 if nb_ms > 0 else 0.0
            line = {"metric": METRIC, "value": audio_seconds(B, T) / (ms / 1e3), "unit": UNIT, "n_gpus": 1,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                    "dtype": math, "data": "synthetic", "config": cfgd,
                    "roofline": {"conv_tflops": tf, "conv_frac": tf / tensor_peak,
                                 "norm_bwd_gbs": nb_gbs, "norm_bwd_frac": nb_gbs / peaks["hbm_gbs"],
                                 "conv_share": conv_ms / ms, "peak_source": peaks["source"]}}
            print(json.dumps(line), flush=True)
            del w, d, step
            gc.collect()
            torch.cuda.synchronize()


def probe(args):
    """One kernel workload on its own (for timing a single launch class or an isolated
    ncu capture); prints one JSON line, not the bench contract's.
      --probe conv   one convolution (forward, input gradient, weight gradient) through
                     the C-ABI atoms on synthetic channels-first data; the CUDA-event time
                     of each call includes the atoms' layout transposes and plane conversions
      --probe block  one AdaINResBlock1 (dilations 1, 3, 5) forward + backward through the
                     block entry points, with the engine's per-class CUDA-event profile"""
    import ctypes

    import torch

    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import MATH, Block

    B, C, L, k, d = args.B, args.C, args.L, args.k, args.d
    math = args.math or "tf32x3"
    lib = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(0)
    out = {}
    if args.probe == "conv":
        p = d * (k - 1) // 2
        _lib.check(lib.bsml_set_atom_math(MATH[math]))
        x = torch.randn((B, C, L), device="cuda", generator=g)
        dy = torch.randn((B, C, L), device="cuda", generator=g)
        W = torch.randn((C, C, k), device="cuda", generator=g) * 0.05
        bias = torch.zeros(C, device="cuda")
        y, dx, dW, db = torch.empty_like(x), torch.empty_like(x), torch.empty_like(W), torch.empty_like(bias)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        calls = {
            "fwd": lambda: lib.bsml_conv1d_forward(P(x), B, C, L, P(W), P(bias), C, k, 1, p, d, P(y), st),
            "dgrad": lambda: lib.bsml_conv1d_backward_input(P(dy), B, C, L, P(W), C, k, 1, p, d, P(dx), st),
            "wgrad": lambda: lib.bsml_conv1d_backward_weight(P(dy), P(x), B, C, L, C, k, 1, p, d, P(dW), P(db), st),
        }
        flops = 2.0 * B * C * C * k * L
        for name, fn in calls.items():
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            _lib.check(fn())
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.reps):
                _lib.check(fn())
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.reps
            out[name] = {"ms_incl_conversions": ms, "tflops_incl_conversions": flops / (ms / 1e3) / 1e12}
    else:
        blk = Block(dict(kind=2, style_dim=128, cin=C, cout=C, kernel=k, dil=[1, 3, 5]), 0, math=math)
        params = torch.randn(blk.n_params, device="cuda", generator=g) * 0.02
        for e in blk.table:
            if e["name"].startswith("alpha"):
                params[e["offset"]:e["offset"] + e["numel"]] = 1.0
        x = torch.randn((B, C, L), device="cuda", generator=g)
        style = torch.randn((B, 128), device="cuda", generator=g)
        dy = torch.randn((B, C, L), device="cuda", generator=g)
        y = torch.empty_like(x)
        grads = torch.empty(blk.n_params, device="cuda")

        def step():
            blk.forward(params, x, style, y=y)
            blk.backward(dy, grads=grads)

        step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            step()
        e1.record()
        torch.cuda.synchronize()
        blk.set_profiling(True)
        step()
        prof = blk.read_profile()
        blk.set_profiling(False)
        out["ms_per_step"] = e0.elapsed_time(e1) / args.reps
        for name, (ms, work, n) in prof.items():
            if n:
                key = "tflops" if name.startswith(("conv", "wgrad")) else "gbs"
                out[name] = {"ms": ms, "launches": n, key: work / (ms / 1e3) / (1e12 if key == "tflops" else 1e9)}
    out["device_error"] = int(lib.bsml_device_error())
    print(json.dumps({"probe": args.probe, "B": B, "C": C, "L": L, "k": k, "d": d, "math": math, **out}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--math", default=None, choices=["fp32", "tf32x3", "bf16", "bf16x3", "tf32x3w", "tf32x3f"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-alt-mode", action="store_true", help="skip the BF16x3 measurement beside TF32x3")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 4: one JSON line per (B, T) of the shape sweep that fits one GPU")
    ap.add_argument("--eager", action="store_true",
                    help="launch every kernel from the host instead of replaying forward + loss + backward as "
                         "one CUDA graph (decoder workloads)")
    ap.add_argument("--batch", type=int, default=None,
                    help="clips per GPU instead of the workload's (a smaller case for profiler captures; "
                         "the bench line's config then names the batch)")
    ap.add_argument("--probe", default=None, choices=["conv", "block"],
                    help="time one kernel workload on its own instead (see probe()); sizes below")
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--C", type=int, default=128)
    ap.add_argument("--L", type=int, default=24001)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--d", type=int, default=3)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.probe:
        probe(args)
        return

    if args.impl == "reference":
        reference_arm(args)
        return
    if args.sweep:
        sweep(args)
        return

    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from brosoundml_b200 import config
    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import Decoder

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        # rank 0's stdout carries only the JSON line: file descriptor 1 is pointed at
        # stderr, so NCCL's log (written to C stdout) lands there, and the JSON line
        # goes to a duplicate of the original stdout. Without a caller's NCCL_DEBUG the
        # log holds the communicator set-up lines (version, ranks, transports).
        global _JSON_FD
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    math = args.math or BENCH_MATH
    B, T, desc = WORKLOADS[args.workload]
    if args.batch:
        B = args.batch
        desc = f"{desc} [batch overridden: B={B} per GPU]"
    dev = torch.device("cuda", local)
    args.graph = not args.eager and args.workload in ("c0", "c2", "c3")
    if args.graph:
        torch.cuda.set_stream(torch.cuda.Stream())   # graph capture needs a non-default stream
    if args.workload == "c1":
        w = setup_block(args, B, T, dev, rank, math)
    elif args.workload == "c3lora":
        w = setup_convlora(args, B, T, dev, rank, math)
    else:
        w = setup_decoder(args, B, T, dev, rank, math)
    host, d, train_step, result = w["host"], w["dev"], w["step"], w["result"]
    prof_src = w["prof"]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x_ms):
        t = torch.tensor([x_ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        train_step(d)
    barrier()
    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
        time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = _lib.lib().bsml_launch_count()
    barrier()
    e0.record(st)
    for _ in range(args.steps):
        train_step(d)
    e1.record(st)
    barrier()
    launches = (_lib.lib().bsml_launch_count() - n0) // max(args.steps, 1)
    if w.get("graph") is not None:
        launches += w["graph"].kernels   # kernels a replay issues (not counted on the host)
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    clk = clocks.stop() if rank == 0 else None
    per_step, unit = w["units_per_step"], w["unit"]
    value = world * per_step / (ms / 1e3)

    # e2e: the public API with host buffers, H2D of the step's inputs and D2H of the loss every step
    e2e = None
    if not args.no_e2e:
        h2d = sum(t.numel() * 4 for t in host.values())
        loss_host = torch.empty(1).pin_memory()
        e2e_steps = max(1, args.steps)
        barrier()
        e0.record(st)
        for _ in range(e2e_steps):
            if w.get("graph") is not None:   # the graph reads fixed buffers: copy the step's inputs into them
                for k, t in host.items():
                    d[k].copy_(t, non_blocking=True)
                train_step(d)
            else:
                inp = {k: t.to(dev, non_blocking=True) for k, t in host.items()}
                train_step(inp)
            loss_host.copy_(result, non_blocking=True)
        e1.record(st)
        barrier()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
        e2e = {"value": world * per_step / (ms_e2e / 1e3), "unit": unit, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": 4, "ms_per_step": ms_e2e}

    # roofline: one profiled step (per-class CUDA events), after the timed region
    prof_src.set_profiling(True)
    w.get("eager_step", train_step)(d)   # the profile records per-class events: an eager step
    prof = prof_src.read_profile()
    prof_src.set_profiling(False)
    peaks = load_peaks()
    rl_all = {}
    for k, (pms, work, n) in prof.items():
        if pms <= 0:
            continue
        if k.startswith(("conv", "wgrad")):
            rl_all[k] = {"ms": pms, "launches": n, "tflops": work / (pms / 1e3) / 1e12, "share": pms / ms,
                         "flops_per_launch": work / max(n, 1)}
        else:
            gbs = work / (pms / 1e3) / 1e9
            rl_all[k] = {"ms": pms, "launches": n, "gbs": gbs, "share": pms / ms,
                         "frac_of_hbm_peak": gbs / load_peaks()["hbm_gbs"],
                         "bytes": ("algorithmic: AdaIN+Snake forward 8 B per element (read x, write y), backward "
                                   "12 B (read x and dy, write dx); the operand planes written for the next "
                                   "conv, the recomputed Snake operand and the backward's second read of x "
                                   "and dy are not counted. DRAM traffic per element in the ncu capture "
                                   "(profiles/kernels_other_than_tcgen05_bench_c2_B6_T200_tf32x3.md): forward "
                                   "12 B, backward 32-40 B over its two passes")}
    dom = max(rl_all, key=lambda k: rl_all[k]["ms"])
    # the measured dense bf16 figure is the tensor roofline (sustained: these kernels run
    # inside a long step); TF32 operands run at half that rate on the same pipe
    bf16_peak = peaks["bf16_tflops_sustained"]
    if dom.startswith(("conv", "wgrad")):
        ach = rl_all[dom]["tflops"]
        traffic = None
        note = (f"dominant kernel class '{dom}'; achieved = useful conv FLOPs / CUDA-event time; peak = "
                f"{peaks['source']} dense bf16 (sustained)")
        extra = {}
        if dom.endswith("_simt"):
            note += "; this class runs on fp32 CUDA cores"
        elif math == "bf16x3" or (math in ("tf32x3w", "tf32x3f") and dom.startswith("wgrad")):
            extra = {"tensor_pipe_frac_issued": 3.0 * ach / bf16_peak}
            note += (f"; BF16x3 issues 3 bf16 products per useful one: {3 * ach / bf16_peak:.0%} of the bf16 rate "
                     "is issued")
        elif math in ("tf32x3", "tf32x3w", "tf32x3f"):
            tf32_peak = bf16_peak / 2.0
            extra = {"tf32_peak": tf32_peak, "frac_of_tf32_peak": ach / tf32_peak,
                     "tensor_pipe_frac_issued": 3.0 * ach / tf32_peak}
            note += (f"; TF32x3 (fp32-grade) runs tf32 operands, whose dense rate is half of bf16, and issues "
                     f"3 tensor products per useful one: {3 * ach / tf32_peak:.0%} of the tf32 rate is issued")
            if math == "tf32x3f" and dom == "conv_tc":
                note += ("; under tf32x3f this class also holds the input-gradient convs, which run BF16x3 (a bf16 "
                         "product at twice the tf32 rate), so the issued fraction above overstates the tf32 pipe "
                         "time")
            if dom == "conv_tc":
                # DRAM bytes per FLOP of conv_fwd_tc_kernel from one ncu capture of the probe case
                # (python bench.py --probe conv --B 16 --C 128 --L 24001 --k 7 --d 3 --math tf32x3),
                # scaled to this class's average launch by its FLOPs
                traffic = NCU_CONV_FWD_TC["dram_bytes"] / NCU_CONV_FWD_TC["flops"] * rl_all[dom]["flops_per_launch"]
                note += "; traffic scaled from the ncu capture of the probe case by FLOPs"
        roofline = dict({"bound": "tensor", "achieved": ach, "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": ach / bf16_peak, "traffic": traffic, "note": note}, **extra)
    else:
        ach = rl_all[dom]["gbs"]
        roofline = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": ach / peaks["hbm_gbs"], "traffic": None,
                    "note": f"dominant class '{dom}'; peak of {peaks['source']} copy bandwidth"}

    # the other fp32-accumulating tensor-core modes, measured the same way in the same run:
    # TF32x3 throughout, and BF16x3 (bf16 hi + lo operands, three products)
    modes = None
    w_config, w_metric = w["config"], w["metric"]
    alt = {"tf32x3f": ("tf32x3", "bf16x3"), "tf32x3w": ("tf32x3", "bf16x3"), "tf32x3": ("bf16x3",)}.get(math, ())
    if args.workload in ("c2", "c0") and alt and not args.no_alt_mode:
        del w, host, d, train_step, result, prof_src
        import gc
        parity = {"tf32x3": "tests/test_gpu_config2.py runs this workload in TF32x3 against the float64 oracle "
                            "(the 3xTF32 bar, rel-L2 <= 1e-4)",
                  "bf16x3": "tests/test_gpu_config2.py runs this workload in BF16x3 against the float64 oracle "
                            "(BASELINE's BF16 bar, rel-L2 <= 2e-2)"}
        modes = {}
        for m2 in alt:
            gc.collect()
            torch.cuda.synchronize()
            w2 = setup_decoder(args, B, T, dev, rank, m2)
            for _ in range(args.warmup):
                w2["step"](w2["dev"])
            barrier()
            e0.record(st)
            for _ in range(args.steps):
                w2["step"](w2["dev"])
            e1.record(st)
            barrier()
            ms2 = max_over_ranks(e0.elapsed_time(e1)) / args.steps
            modes[m2] = {"value": world * w2["units_per_step"] / (ms2 / 1e3), "unit": UNIT, "ms_per_step": ms2,
                         "parity": parity[m2]}
            del w2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in ("c2", "c0"):
        cpu = run_cpu_baseline(config.kokoro_82m(), T)
        # one core, on a shorter clip so the sample stays bounded (per-clip throughput
        # grows slowly with length: the conv work is linear in T)
        one = run_cpu_baseline(config.kokoro_82m(), min(T, 32), threads=1)
        cpu["single_core"] = {"value": one["value"], "unit": UNIT, "cores": one["cores"], "sample": one["sample"]}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "c1":
        cpu = run_cpu_baseline_block(B, T)

    if rank == 0:
        line = {
            "metric": w_metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": math, "data": "synthetic",
            "dtype_note": MATH_NOTES.get(math, math),
            "config": dict({"workload": desc, "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world}",
                            "l2": "working set (GBs of cached activations) >> 126 MB L2; no flush needed"},
                           **w_config),
            "clocks": clk, "e2e": e2e, "gpu_launches": int(launches), "roofline": roofline,
            "roofline_by_class": rl_all, "cpu_baseline": cpu, "other_modes": modes,
        }
        emit_json(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    del np


if __name__ == "__main__":
    main()
