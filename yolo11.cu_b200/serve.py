"""yoloserve: the gRPC batch-labeling server over the engine's C ABI.

    python yolo11.cu_b200/serve.py [--dir models/yolo11n[:maxB]]... [--addr 0.0.0.0:50051]
                                   [--max-batch 16] [--target-ms 50] [--device 0]

The reference server (server/serve.cpp) is C++ on grpc++; this image has neither grpc++ nor
protoc, so the server is written against grpcio, with the message and service types of
proto/yolo.proto built at run time from their descriptors (`yolo_proto()`): same package,
service, method, field names and numbers, so the reference's clients talk to it unchanged.

Behaviour (server/serve.cpp):
  * `Yolo.Detect(DetectRequest) -> DetectResponse`, one image per call, routed by
    `DetectRequest.model` (model directory basename; empty = the first --dir); an unknown
    model or an undecodable image answers INVALID_ARGUMENT (serve.cpp:309-331).
  * deadline-aware dynamic batching (serve.cpp:163-191): each model has its own queue; the
    batcher fires the most urgent queue as soon as it is full (its max batch) or its oldest
    request's slack, target - waited - exec_ms(max batch) - decode EMA - 1 ms safety, runs
    out; otherwise it waits for more work (at most 200 us at a time).
  * two-stage pipeline (serve.cpp:264-302): the next batch is decoded and preprocessed while
    the GPU runs the current one.  Here each model holds two engine handles used in turn, so
    batch k+1's decode and letterbox go into one handle's slots while batch k's graph runs
    on the other's; the results of batch k are read before that handle is refilled.
  * decode: JPEG by nvJPEG through `yolo_preprocess_jpeg` one image after another (the
    handle has one nvJPEG state), other formats (PNG, ...) on the CPU (cv2; the reference
    uses stb_image); or (--decode cpu) every image of a batch on a pool of CPU threads
    (OpenCV; the reference's decoder pool runs nvJPEG's CPU Huffman stage on 8 threads,
    serve.cpp:104-146), then uploaded and preprocessed on the GPU.
  * responses: boxes (detect / segment), rotated boxes (obb), top-5 classes (classify),
    segment masks as row-major 0/1 run lengths starting with a 0-run plus the letterbox
    geometry (serve.cpp:193-259); queue_ms, infer_ms, batch as the reference fills them.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import threading
import time
from collections import deque
from concurrent import futures

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
TASKS = {0: "detect", 1: "obb", 2: "classify", 3: "segment"}


# ---------------- proto/yolo.proto, built from descriptors ----------------
_PROTO = None


def yolo_proto():
    """(DetectRequest, DetectResponse) message classes of package `yolo` (proto/yolo.proto)."""
    global _PROTO
    if _PROTO is not None:
        return _PROTO
    from google.protobuf import descriptor_pb2, descriptor_pool, message_factory
    F = descriptor_pb2.FieldDescriptorProto
    fd = descriptor_pb2.FileDescriptorProto(name="yolo.proto", package="yolo", syntax="proto3")

    def msg(name, fields):
        m = fd.message_type.add(name=name)
        for fname, num, ftype, label, tname in fields:
            f = m.field.add(name=fname, number=num, type=ftype, label=label)
            if tname:
                f.type_name = tname

    opt, rep = F.LABEL_OPTIONAL, F.LABEL_REPEATED
    msg("DetectRequest", [("image", 1, F.TYPE_BYTES, opt, None),
                          ("model", 2, F.TYPE_STRING, opt, None)])
    msg("Box", [("x1", 1, F.TYPE_FLOAT, opt, None), ("y1", 2, F.TYPE_FLOAT, opt, None),
                ("x2", 3, F.TYPE_FLOAT, opt, None), ("y2", 4, F.TYPE_FLOAT, opt, None),
                ("score", 5, F.TYPE_FLOAT, opt, None), ("cls", 6, F.TYPE_INT32, opt, None)])
    msg("RBox", [("cx", 1, F.TYPE_FLOAT, opt, None), ("cy", 2, F.TYPE_FLOAT, opt, None),
                 ("w", 3, F.TYPE_FLOAT, opt, None), ("h", 4, F.TYPE_FLOAT, opt, None),
                 ("angle", 5, F.TYPE_FLOAT, opt, None), ("score", 6, F.TYPE_FLOAT, opt, None),
                 ("cls", 7, F.TYPE_INT32, opt, None)])
    msg("ClassProb", [("id", 1, F.TYPE_INT32, opt, None), ("prob", 2, F.TYPE_FLOAT, opt, None)])
    msg("Mask", [("rle", 1, F.TYPE_UINT32, rep, None)])
    msg("DetectResponse", [
        ("boxes", 1, F.TYPE_MESSAGE, rep, ".yolo.Box"),
        ("queue_ms", 2, F.TYPE_FLOAT, opt, None), ("infer_ms", 3, F.TYPE_FLOAT, opt, None),
        ("batch", 4, F.TYPE_INT32, opt, None), ("task", 5, F.TYPE_STRING, opt, None),
        ("rboxes", 6, F.TYPE_MESSAGE, rep, ".yolo.RBox"),
        ("classes", 7, F.TYPE_MESSAGE, rep, ".yolo.ClassProb"),
        ("masks", 8, F.TYPE_MESSAGE, rep, ".yolo.Mask"),
        ("mask_h", 9, F.TYPE_UINT32, opt, None), ("mask_w", 10, F.TYPE_UINT32, opt, None),
        ("lb_scale", 11, F.TYPE_FLOAT, opt, None), ("lb_top", 12, F.TYPE_INT32, opt, None),
        ("lb_left", 13, F.TYPE_INT32, opt, None)])
    svc = fd.service.add(name="Yolo")
    svc.method.add(name="Detect", input_type=".yolo.DetectRequest",
                   output_type=".yolo.DetectResponse")
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    get = message_factory.GetMessageClass
    _PROTO = (get(pool.FindMessageTypeByName("yolo.DetectRequest")),
              get(pool.FindMessageTypeByName("yolo.DetectResponse")))
    return _PROTO


METHOD = "/yolo.Yolo/Detect"


def rle_encode(mask: np.ndarray) -> list[int]:
    """Row-major 0/1 run lengths starting with a 0-run (serve.cpp:193-203)."""
    m = (np.ascontiguousarray(mask).reshape(-1) != 0).astype(np.int8)
    if m.size == 0:
        return [0]
    cuts = np.flatnonzero(np.diff(m)) + 1
    runs = np.diff(np.concatenate(([0], cuts, [m.size]))).tolist()
    return ([0] + runs) if m[0] else runs


# ---------------- batcher ----------------
class _Req:
    __slots__ = ("model", "data", "arrival", "resp", "ok", "done")

    def __init__(self, model, data, resp):
        self.model, self.data, self.resp = model, data, resp
        self.arrival = time.monotonic()
        self.ok = False
        self.done = threading.Event()


class _Model:
    def __init__(self, name, engines, max_batch):
        self.name = name
        self.engines = engines            # two handles, used in turn
        self.turn = 0
        self.max_batch = max_batch
        self.task = engines[0].task()
        self.task_name = TASKS.get(self.task, "detect")
        self.mask_hw = engines[0].mask_dim() if self.task == 3 else (0, 0)
        self.q: deque[_Req] = deque()


class Batcher:
    """Per-model queues, the deadline-slack firing rule and the two-stage worker.

    `models`: list of (name, [engine, engine], max_batch); an engine is anything with the
    runtime.Engine methods the worker calls (task, mask_dim, exec_ms, preprocess_jpeg,
    preprocess_host, preprocess_host_batch, run_async, sync, get, get_obb, get_cls,
    get_mask, slot_geom)."""

    def __init__(self, models, target_ms=50.0, safety_ms=1.0, response_cls=None,
                 decode="gpu", decoders=8):
        self.models = [_Model(n, e, b) for n, e, b in models]
        # decode="gpu": JPEG by nvJPEG on the handle, one image after another; "cpu": every
        # image of a batch decoded by OpenCV on a pool of `decoders` threads (the reference's
        # decoder pool, serve.cpp:104-146), then uploaded and preprocessed on the GPU
        self.decode = decode
        self.pool = futures.ThreadPoolExecutor(max_workers=decoders) if decode == "cpu" else None
        self.names = {m.name: i for i, m in enumerate(self.models)}
        self.target_ms, self.safety_ms = target_ms, safety_ms
        self.decode_ema_ms = 2.0
        self.cv = threading.Condition()
        self.response_cls = response_cls or yolo_proto()[1]
        self.served = 0
        self._stop = False
        self._thread = threading.Thread(target=self._worker, name="yolo-batcher", daemon=True)
        self._thread.start()

    # -- request side --
    def submit(self, model: str, data: bytes, timeout: float | None = None):
        """Queue one image; returns (ok, DetectResponse) once its batch has run.  Raises
        KeyError for an unknown model name (empty = the first model)."""
        mi = self.names[model] if model else 0
        r = _Req(mi, data, self.response_cls())
        with self.cv:
            self.models[mi].q.append(r)
            self.cv.notify_all()
        if not r.done.wait(timeout):
            raise TimeoutError("request not served in time")
        return r.ok, r.resp

    def close(self):
        with self.cv:
            self._stop = True
            self.cv.notify_all()
        self._thread.join(timeout=5)
        if self.pool is not None:
            self.pool.shutdown(wait=False)

    # -- the firing rule (serve.cpp:163-191) --
    def slack_ms(self, m: _Model, now: float) -> float:
        waited = (now - m.q[0].arrival) * 1e3
        return (self.target_ms - waited - m.engines[0].exec_ms(m.max_batch) -
                self.decode_ema_ms - self.safety_ms)

    def pick(self, now: float):
        """(model index, fire) of the most urgent non-empty queue, or (-1, False)."""
        pick, fire, best = -1, False, 1e30
        for i, m in enumerate(self.models):
            if not m.q:
                continue
            slack = self.slack_ms(m, now)
            ready = len(m.q) >= m.max_batch or slack <= 0
            if (ready and not fire) or (ready == fire and slack < best):
                pick, best, fire = i, slack, fire or ready
        return pick, fire, best

    def _collect(self):
        with self.cv:
            while True:
                if self._stop:
                    return -1, []
                pick, fire, best = self.pick(time.monotonic())
                if pick >= 0 and fire:
                    break
                wait = 0.2 if pick < 0 else min(max(best, 0.0) * 1e-3, 200e-6)
                self.cv.wait(timeout=wait)
            m = self.models[pick]
            B = min(len(m.q), m.max_batch)
            return pick, [m.q.popleft() for _ in range(B)]

    # -- the two-stage worker (serve.cpp:264-302) --
    @staticmethod
    def _cpu_decode(data: bytes):
        try:
            import cv2
            return cv2.imdecode(np.frombuffer(data, np.uint8), cv2.IMREAD_COLOR)
        except Exception:
            return None

    def _load_batch(self, m: _Model, eng, batch) -> list[bool]:
        """Decode and preprocess the batch's images into slots 0..B-1 of `eng`."""
        ok = [False] * len(batch)
        if self.decode == "cpu":
            imgs = list(self.pool.map(lambda r: self._cpu_decode(r.data), batch))
            good = [(i, im) for i, im in enumerate(imgs) if im is not None]
            if good:
                eng.preprocess_host_batch([im for _, im in good], [i for i, _ in good])
            for i, _ in good:
                ok[i] = True
            return ok
        for i, r in enumerate(batch):
            data = r.data
            try:
                if len(data) > 3 and data[0] == 0xFF and data[1] == 0xD8:
                    ok[i] = eng.preprocess_jpeg(data, i) == 0
                else:
                    img = self._cpu_decode(data)
                    if img is not None:
                        eng.preprocess_host(img, i)
                        ok[i] = True
            except Exception:
                ok[i] = False
        return ok

    def _respond(self, m: _Model, eng, batch, ok, t_launch):
        eng.sync()
        infer_ms = (time.monotonic() - t_launch) * 1e3
        for i, r in enumerate(batch):
            resp = r.resp
            resp.task = m.task_name
            if ok[i]:
                if m.task == 2:
                    ids, probs = eng.get_cls(i, 5)
                    for c, p in zip(ids, probs):
                        resp.classes.add(id=int(c), prob=float(p))
                elif m.task == 1:
                    for cx, cy, w, h, a, s, c in eng.get_obb(i):
                        resp.rboxes.add(cx=cx, cy=cy, w=w, h=h, angle=a, score=s, cls=int(c))
                else:
                    dets = eng.get(i)
                    for x1, y1, x2, y2, s, c in dets:
                        resp.boxes.add(x1=x1, y1=y1, x2=x2, y2=y2, score=s, cls=int(c))
                    if m.task == 3:
                        resp.mask_h, resp.mask_w = m.mask_hw
                        sc, top, left = eng.slot_geom(i)
                        resp.lb_scale, resp.lb_top, resp.lb_left = sc, top, left
                        for j in range(len(dets)):
                            mk = eng.get_mask(i, j)
                            mm = resp.masks.add()
                            if mk is not None:
                                mm.rle.extend(rle_encode(mk))
            resp.queue_ms = (t_launch - r.arrival) * 1e3
            resp.infer_ms = infer_ms
            resp.batch = len(batch)
            r.ok = bool(ok[i])
            r.done.set()
        self.served += len(batch)

    def _worker(self):
        prev = None   # (model, engine, batch, ok, t_launch) on the GPU
        while True:
            mi, batch = self._collect()
            if mi < 0:
                break
            m = self.models[mi]
            eng = m.engines[m.turn]
            m.turn ^= 1
            t0 = time.monotonic()
            try:   # into the idle handle while prev's graph runs
                ok = self._load_batch(m, eng, batch)
            except Exception:
                ok = [False] * len(batch)
            self.decode_ema_ms = 0.9 * self.decode_ema_ms + 0.1 * (time.monotonic() - t0) * 1e3
            if prev is not None:
                self._respond(*prev)
                prev = None
            t_launch = time.monotonic()
            eng.run_async(len(batch))
            prev = (m, eng, batch, ok, t_launch)
            # nothing else queued: finish now instead of waiting for more traffic
            with self.cv:
                idle = all(not mm.q for mm in self.models)
            if idle:
                self._respond(*prev)
                prev = None
        if prev is not None:
            self._respond(*prev)


# ---------------- gRPC service ----------------
def make_server(batcher: Batcher, addr: str, workers: int = 64):
    """A grpc.Server serving yolo.Yolo/Detect on `addr` (not started)."""
    import grpc
    req_cls, resp_cls = yolo_proto()

    def detect(request, context):
        try:
            ok, resp = batcher.submit(request.model, request.image)
        except KeyError:
            context.abort(grpc.StatusCode.INVALID_ARGUMENT, "unknown model: " + request.model)
        if not ok:
            context.abort(grpc.StatusCode.INVALID_ARGUMENT, "image decode failed")
        return resp

    handler = grpc.method_handlers_generic_handler("yolo.Yolo", {
        "Detect": grpc.unary_unary_rpc_method_handler(
            detect, request_deserializer=req_cls.FromString,
            response_serializer=resp_cls.SerializeToString)})
    server = grpc.server(futures.ThreadPoolExecutor(max_workers=workers),
                         options=[("grpc.max_receive_message_length", 64 << 20)])
    server.add_generic_rpc_handlers((handler,))
    if server.add_insecure_port(addr) == 0:
        raise RuntimeError("cannot listen on " + addr)
    return server


def detect_stub(channel):
    """Client call for yolo.Yolo/Detect on a grpc channel (what a generated stub does)."""
    req_cls, resp_cls = yolo_proto()
    return channel.unary_unary(METHOD, request_serializer=req_cls.SerializeToString,
                               response_deserializer=resp_cls.FromString)


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
    ap = argparse.ArgumentParser(description="gRPC batch-labeling server (yolo.Yolo/Detect)")
    ap.add_argument("--dir", action="append", default=[],
                    help="model directory, optionally :maxB (repeat for several models)")
    ap.add_argument("--addr", default="0.0.0.0:50051")
    ap.add_argument("--max-batch", type=int, default=16)
    ap.add_argument("--target-ms", type=float, default=50.0)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--decode", choices=("gpu", "cpu"), default="gpu",
                    help="JPEG decode: nvJPEG per image on the handle, or a CPU thread pool")
    ap.add_argument("--decoders", type=int, default=8)
    a = ap.parse_args(argv)
    rt = _runtime()
    specs = []
    for spec in a.dir or ["models/yolo11n"]:
        maxb = a.max_batch
        head, sep, tail = spec.rpartition(":")
        if sep and "/" not in tail and tail.isdigit():
            spec, maxb = head, int(tail)
        name = os.path.basename(os.path.normpath(spec))
        engines = [rt.Engine(spec, maxb, device=a.device) for _ in range(2)]
        print(f"model '{name}': task={TASKS.get(engines[0].task(), 'detect')} max-batch={maxb}",
              flush=True)
        specs.append((name, engines, maxb))
    batcher = Batcher(specs, a.target_ms, decode=a.decode, decoders=a.decoders)
    server = make_server(batcher, a.addr)
    server.start()
    print(f"yoloserve listening on {a.addr} ({len(specs)} models, target={a.target_ms:.0f} ms)",
          flush=True)
    server.wait_for_termination()


if __name__ == "__main__":
    main()
