"""Time decode + NMS through the kernel ABI (yk_decode / yk_nms) on seeded synthetic heads,
for tuning and profiling the post-processing.

    python yolo11.cu_b200/postbench.py [--cluster 0|1|2|4|8 ...] [--lib path/to/libyolob200.so]

Heads of one 640 image (8400 anchors, 80 class channels): box logits N(0, 1); class logits
N(0, 1) + bias on the first k classes and -20 on the rest, for the (bias, k) cases below;
conf 0.25, IoU 0.7, max 300.  yk_decode runs once, then yk_nms three times untimed and 50
times back to back between CUDA events on the stream (the figure includes each launch's
overhead).  --cluster forces the NMS cluster size (yk_test_nms_cluster; 0 = the library's
rule).  With a library built with -DYK_NMS_PROF, the phase times of image 0 (%globaltimer
at the phase boundaries of the last launch) are printed too.  One JSON line per case and
cluster size.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CASES = [(-2.9, 1), (-3.5, 4), (-2.9, 4), (-4.0, 80), (-3.0, 80)]   # (class bias, classes)
PHASES = ["gather", "sort", "segments", "mask_offsets", "masks", "suppression", "output"]


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
    ap.add_argument("--cluster", type=int, nargs="*", default=[0])
    ap.add_argument("--lib", default=None)
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args(argv)
    rt = _runtime()
    lib = rt.load(a.lib) if a.lib else rt.load()
    prof = getattr(lib, "yk_nms_prof", None)
    cuda = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    S, B, NC = 640, 1, 80
    sizes = [(S // 8, 8), (S // 16, 16), (S // 32, 32)]
    A = sum(n * n for n, _ in sizes)
    for bias, k in CASES:
        g = torch.Generator().manual_seed(0)
        box = [torch.randn(B, n, n, 64, generator=g).half().to(cuda) for n, _ in sizes]
        cls = []
        for n, _ in sizes:
            c = torch.full((B, n, n, NC), -20.0)
            c[..., :k] = torch.randn(B, n, n, k, generator=g) + bias
            cls.append(c.half().to(cuda))
        lv = (rt.YkLevel * 3)()
        for i, ((n, s), b, c) in enumerate(zip(sizes, box, cls)):
            lv[i].box, lv[i].cls, lv[i].stride = rt.tview(b), rt.tview(c), s
        wsb = lib.yk_post_workspace_bytes(B, A)
        ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
        od = torch.zeros(B, 300, 6, device=cuda)
        oi = torch.zeros(B, 300, dtype=torch.int32, device=cuda)
        oc = torch.zeros(B, dtype=torch.int32, device=cuda)
        rc = torch.zeros(B, dtype=torch.int32, device=cuda)
        post = rt.YkPost(ws.data_ptr(), wsb, od.data_ptr(), oi.data_ptr(), oc.data_ptr(),
                         rc.data_ptr())
        assert lib.yk_decode(lv, 3, B, NC, 0.25, C.byref(post), st) == 0
        for cs in a.cluster:
            assert lib.yk_test_nms_cluster(cs) == 0
            for _ in range(3):
                assert lib.yk_nms(B, A, 0.7, 300, C.byref(post), st) == 0
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                lib.yk_nms(B, A, 0.7, 300, C.byref(post), st)
            e1.record()
            torch.cuda.synchronize()
            line = {"classes": k, "bias": bias, "cluster": cs, "candidates": int(rc.item()),
                    "kept": int(oc.item()), "nms_us": round(e0.elapsed_time(e1) / a.iters * 1e3, 1)}
            if prof is not None:
                buf = (C.c_ulonglong * 8)()
                if prof(buf) == 0:
                    t = list(buf)
                    line["phases_us"] = {PHASES[i]: round((t[i + 1] - t[i]) / 1e3, 2)
                                         for i in range(7)}
            print(json.dumps(line), flush=True)
        lib.yk_test_nms_cluster(0)


if __name__ == "__main__":
    main()
