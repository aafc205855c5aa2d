"""Drive one convolution (forward, input gradient, weight gradient) through the C ABI
on synthetic channels-first data, e.g. for an isolated ncu capture or timing of the
tensor-core kernels:

  python -m brosoundml_b200.kernel_probe --B 16 --C 128 --L 24001 --k 7 --d 3 --math tf32x3

Prints one JSON line with the CUDA-event time of each call (these include the
layout transposes and operand-plane conversions of the atom entry points).

  python -m brosoundml_b200.kernel_probe --op block --B 16 --C 128 --L 24000 --k 7

runs one AdaINResBlock1 (dilations 1, 3, 5) forward + backward through the block
entry points instead, with the engine's per-class CUDA-event profile (the fused
AdaIN + Snake kernels' algorithmic bytes and time).
"""

from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import _lib

MATH = {"fp32": 0, "tf32x3": 1, "bf16": 2, "bf16x3": 3}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--C", type=int, default=128)
    ap.add_argument("--L", type=int, default=24001)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--d", type=int, default=3)
    ap.add_argument("--math", default="tf32x3", choices=sorted(MATH))
    ap.add_argument("--reps", type=int, default=1)
    ap.add_argument("--op", default="conv", choices=["conv", "block"])
    args = ap.parse_args()
    if args.op == "block":
        return block(args)
    B, C, L, k, d = args.B, args.C, args.L, args.k, args.d
    p = d * (k - 1) // 2
    lib = _lib.lib()
    _lib.check(lib.bsml_set_atom_math(MATH[args.math]))
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn((B, C, L), device="cuda", generator=g)
    dy = torch.randn((B, C, L), device="cuda", generator=g)
    W = torch.randn((C, C, k), device="cuda", generator=g) * 0.05
    bias = torch.zeros(C, device="cuda")
    y = torch.empty_like(x)
    dx = torch.empty_like(x)
    dW = torch.empty_like(W)
    db = torch.empty_like(bias)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = {}
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
    out["device_error"] = int(lib.bsml_device_error())
    print(json.dumps({"B": B, "C": C, "L": L, "k": k, "d": d, "math": args.math, **out}))


def block(args):
    from .decoder import Block

    B, C, L, k = args.B, args.C, args.L, args.k
    blk = Block(dict(kind=2, style_dim=128, cin=C, cout=C, kernel=k, dil=[1, 3, 5]), 0, math=args.math)
    g = torch.Generator(device="cuda").manual_seed(0)
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
    out = {"ms_per_step": e0.elapsed_time(e1) / args.reps}
    for name, (ms, work, n) in prof.items():
        if n:
            key = "tflops" if name.startswith(("conv", "wgrad")) else "gbs"
            out[name] = {"ms": ms, "launches": n, key: work / (ms / 1e3) / (1e12 if key == "tflops" else 1e9)}
    out["device_error"] = int(_lib.lib().bsml_device_error())
    print(json.dumps({"op": "block", "B": B, "C": C, "L": L, "k": k, "math": args.math, **out}))


if __name__ == "__main__":
    main()
