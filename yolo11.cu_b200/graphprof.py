"""Replay one engine's pipeline graph with the CUDA profiler window around the replays only,
so an `ncu --profile-from-start off` launch list holds just the graph's kernels.

    python yolo11.cu_b200/graphprof.py MODEL BATCH [--imgsz S] [--frame HxW] [--reps N]
    ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none \\
        --csv --log-file out.csv python yolo11.cu_b200/graphprof.py yolo11m 32

The model directory is models/<name>[-S] (exported on first use), tiles come from its
batch-B tuning cache, the frames are seeded synthetic frames resident on the device (bound
with yolo_bind_frames), and the graph is the one yolo_run_frames replays.  Prints the
calibrated graph time and the graph's kernel count.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("model")
    ap.add_argument("batch", type=int)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--frame", default="720x1280")
    ap.add_argument("--reps", type=int, default=2)
    a = ap.parse_args(argv)
    if "yolo11_cu_b200" not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            "yolo11_cu_b200", os.path.join(PKG, "__init__.py"), submodule_search_locations=[PKG])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["yolo11_cu_b200"] = mod
        spec.loader.exec_module(mod)
    import numpy as np
    import torch
    from yolo11_cu_b200 import export, frames, runtime as rt
    h, w = (int(v) for v in a.frame.split("x"))
    d = export.ensure_model_dir(a.model, os.path.join(ROOT, "models"), a.imgsz, (h, w))
    os.environ["YOLO_TUNE_CACHE"] = os.path.join(d, f"tune_b{a.batch}.txt")
    eng = rt.Engine(d, a.batch, device=0)
    dev = torch.from_numpy(np.stack([frames.synthetic_bgr(h, w, seed=i) for i in range(a.batch)])).cuda()
    torch.cuda.synchronize()
    eng.bind_frames(0, dev.data_ptr(), h, w, a.batch, False)
    ms = eng.frames_exec_ms(0, a.batch)
    for _ in range(3):
        eng.run_frames(0, a.batch)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(a.reps):
        eng.run_frames(0, a.batch)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"{a.model} batch {a.batch}: graph {ms:.3f} ms, "
          f"{eng.lib.yolo_graph_kernels(eng.h, 0, a.batch)} kernels per replay", flush=True)
    eng.close()


if __name__ == "__main__":
    main()
