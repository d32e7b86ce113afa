"""Throughput and latency of the gRPC batching server (serve.py) under concurrent clients.

    python yolo11.cu_b200/servebench.py [--model yolo11n] [--clients 64] [--seconds 10]
                                        [--max-batch 32] [--target-ms 50] [--procs 8]
                                        [--decode gpu|cpu] [--decoders 8]

Starts the server in this process on 127.0.0.1 (two engine handles of the model, exported
from the seeded random-init weights if missing) and drives it from `--procs` client
processes with `--clients` concurrent streams in total, each sending seeded synthetic
640x480 JPEG frames (quality 90) back to back for `--seconds` after a warm-up.  Prints one
JSON line: images/s, latency p50 / p99 (ms, client side), mean batch, requests.  The
reference publishes 1,123 img/s at p50 55 ms with 64 clients on an RTX 3060 Ti
(README.md:141-143); its images are COCO photos, seeded frames of the same size stand in.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import socket
import sys
import threading
import time

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)


def _load_serve():
    import importlib.util
    spec = importlib.util.spec_from_file_location("yolo_serve_bench", os.path.join(PKG, "serve.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _frames(n, seed0):
    import cv2
    sys.path.insert(0, PKG)
    import frames
    return [cv2.imencode(".jpg", frames.synthetic_bgr(480, 640, seed=seed0 + i),
                         [cv2.IMWRITE_JPEG_QUALITY, 90])[1].tobytes() for i in range(n)]


def _client_proc(port, streams, warm_s, run_s, model, seed, q):
    import grpc
    serve = _load_serve()
    Req, _ = serve.yolo_proto()
    imgs = _frames(8, seed)
    t_start = time.monotonic() + warm_s
    t_end = t_start + run_s
    lat, batches = [], []
    lock = threading.Lock()

    def stream(k):
        with grpc.insecure_channel(f"127.0.0.1:{port}") as ch:
            detect = serve.detect_stub(ch)
            i = k
            while True:
                t0 = time.monotonic()
                if t0 >= t_end:
                    return
                r = detect(Req(image=imgs[i % len(imgs)], model=model), timeout=60)
                t1 = time.monotonic()
                i += 1
                if t0 >= t_start and t1 <= t_end:
                    with lock:
                        lat.append((t1 - t0) * 1e3)
                        batches.append(r.batch)

    ths = [threading.Thread(target=stream, args=(k,)) for k in range(streams)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    q.put((lat, batches))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="yolo11n")
    ap.add_argument("--clients", type=int, default=64)
    ap.add_argument("--procs", type=int, default=8)
    ap.add_argument("--seconds", type=float, default=10.0)
    ap.add_argument("--warmup", type=float, default=3.0)
    ap.add_argument("--max-batch", type=int, default=32)
    ap.add_argument("--target-ms", type=float, default=50.0)
    ap.add_argument("--decode", choices=("gpu", "cpu"), default="gpu")
    ap.add_argument("--decoders", type=int, default=8)
    a = ap.parse_args(argv)
    serve = _load_serve()
    rt = serve._runtime()
    from yolo11_cu_b200 import export
    d = export.ensure_model_dir(a.model, os.path.join(ROOT, "models"), 640)
    engines = [rt.Engine(d, a.max_batch, device=0) for _ in range(2)]
    for e in engines:
        e.exec_ms(a.max_batch)          # graphs captured and timed before traffic
    batcher = serve.Batcher([(a.model, engines, a.max_batch)], a.target_ms, decode=a.decode,
                            decoders=a.decoders)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = serve.make_server(batcher, f"127.0.0.1:{port}", workers=max(64, 2 * a.clients))
    server.start()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = []
    per = [a.clients // a.procs + (1 if i < a.clients % a.procs else 0) for i in range(a.procs)]
    for i, n in enumerate(per):
        if n:
            p = ctx.Process(target=_client_proc,
                            args=(port, n, a.warmup, a.seconds, a.model, 100 * i, q))
            p.start()
            procs.append(p)
    lat, bat = [], []
    for _ in procs:
        l, b = q.get(timeout=a.warmup + a.seconds + 120)
        lat += l
        bat += b
    for p in procs:
        p.join(30)
    server.stop(0)
    batcher.close()
    import numpy as np
    lat = np.array(lat)
    print(json.dumps({
        "metric": "images/s through yolo.Yolo/Detect", "model": a.model, "clients": a.clients,
        "client_procs": len(procs), "max_batch": a.max_batch, "target_ms": a.target_ms,
        "decode": a.decode, "decoders": a.decoders,
        "images_per_s": round(len(lat) / a.seconds, 1),
        "p50_ms": round(float(np.percentile(lat, 50)), 2) if len(lat) else None,
        "p99_ms": round(float(np.percentile(lat, 99)), 2) if len(lat) else None,
        "mean_batch": round(float(np.mean(bat)), 2) if bat else None,
        "requests": int(len(lat)), "frame": "640x480 JPEG q90, seeded synthetic"}), flush=True)


if __name__ == "__main__":
    main()
