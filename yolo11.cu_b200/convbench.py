"""Time one convolution shape through the kernel ABI (yk_conv), for tuning and profiling.

    python yolo11.cu_b200/convbench.py B,H,W,Cin,Cout,k,s [--algo A --tile T --msub M]
                                       [--iters N] [--res] [--dw] [--act 0|1]

Allocates NHWC fp16 input / output (and residual) with torch on cuda:0, runs the conv
`--warmup` times, then times `--iters` launches with CUDA events (inputs larger than L2 for
the shapes of interest; otherwise the number is an L2-resident figure) and prints one JSON
line: microseconds per launch, TFLOP/s (2*M*N*K) and GB/s of algorithmic traffic (input,
weights, output, residual once each).  algo/tile/msub are YkConv's fields (0 = heuristic).
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import sys

PKG = os.path.dirname(os.path.abspath(__file__))


def _runtime():
    if "yolo11_cu_b200" not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            "yolo11_cu_b200", os.path.join(PKG, "__init__.py"), submodule_search_locations=[PKG])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["yolo11_cu_b200"] = mod
        spec.loader.exec_module(mod)
    from yolo11_cu_b200 import runtime
    return runtime


def main(argv=None):
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("shape", help="B,H,W,Cin,Cout,k,s")
    ap.add_argument("--algo", type=int, default=0)
    ap.add_argument("--tile", type=int, default=0)
    ap.add_argument("--msub", type=int, default=0)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--res", action="store_true", help="fused residual add")
    ap.add_argument("--dw", action="store_true", help="depthwise (groups = Cin = Cout)")
    ap.add_argument("--act", type=int, default=1, help="1 SiLU (default), 0 identity")
    a = ap.parse_args(argv)
    B, H, W, Cin, Cout, k, s = (int(v) for v in a.shape.split(","))
    rt = _runtime()
    lib = rt.load()
    dev = torch.device("cuda:0")
    p = k // 2
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    g = torch.Generator().manual_seed(0)
    groups = Cin if a.dw else 1
    x = torch.randn(B, H, W, Cin, generator=g).half().to(dev)
    w = (torch.randn(Cout, k, k, Cin // groups, generator=g) / (Cin // groups * k * k) ** 0.5).half().to(dev)
    b = (torch.randn(Cout, generator=g) * 0.1).float().to(dev)
    y = torch.empty(B, Ho, Wo, Cout, dtype=torch.half, device=dev)
    r = torch.randn(B, Ho, Wo, Cout, generator=g).half().to(dev) if a.res else None
    prm = rt.YkConv(w.data_ptr(), b.data_ptr(), k, s, p, groups, a.act, Cin, Cout, a.tile, a.msub,
                    a.algo)
    xv, yv = rt.tview(x), rt.tview(y)
    rv = rt.tview(r) if r is not None else None
    st = torch.cuda.current_stream()

    def launch():
        rc = lib.yk_conv(C.byref(xv), C.byref(yv), C.byref(rv) if rv is not None else None,
                         C.byref(prm), st.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"yk_conv {rc}: {lib.yk_last_cuda_error().decode()}")

    for _ in range(a.warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.iters):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    if lib.yk_fetch_device_error():
        raise RuntimeError("device error word set")
    us = e0.elapsed_time(e1) * 1000 / a.iters
    M = B * Ho * Wo
    flops = 2.0 * M * Cout * k * k * (Cin // groups)
    nbytes = 2.0 * (B * H * W * Cin + w.numel() + M * Cout * (2 if a.res else 1))
    print(json.dumps({"shape": a.shape, "algo": a.algo, "tile": a.tile, "msub": a.msub,
                      "res": a.res, "us": round(us, 2), "tflops": round(flops / us / 1e6, 1),
                      "gbs": round(nbytes / us / 1e3, 1)}), flush=True)


if __name__ == "__main__":
    main()
