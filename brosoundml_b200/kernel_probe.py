"""Drive one convolution (forward, input gradient, weight gradient) through the C ABI
on synthetic channels-first data, e.g. for an isolated ncu capture or timing of the
tensor-core kernels:

  python -m brosoundml_b200.kernel_probe --B 16 --C 128 --L 24001 --k 7 --d 3 --math tf32x3

Prints one JSON line with the CUDA-event time of each call (these include the
layout transposes and operand-plane conversions of the atom entry points).
"""

from __future__ import annotations

import argparse
import ctypes
import json

import torch

from . import _lib

MATH = {"fp32": 0, "tf32x3": 1, "bf16": 2}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--C", type=int, default=128)
    ap.add_argument("--L", type=int, default=24001)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--d", type=int, default=3)
    ap.add_argument("--math", default="tf32x3", choices=sorted(MATH))
    ap.add_argument("--reps", type=int, default=1)
    args = ap.parse_args()
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


if __name__ == "__main__":
    main()
