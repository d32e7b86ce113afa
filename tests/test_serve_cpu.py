"""The gRPC batching server (yolo11.cu_b200/serve.py) on the CPU: the run-time proto
descriptors against the reference's proto/yolo.proto (fixture tests/golden/
yolo_proto_fields.json), the mask run-length code, and the batcher / service with fake
engines (firing on a full queue or on spent slack, routing by model name, decode failures,
the two-stage handle alternation) through a real gRPC server on 127.0.0.1."""
import json
import os
import socket
import threading
import time

import numpy as np
import pytest

from conftest import GOLDEN, PKG_DIR

import importlib.util

_spec = importlib.util.spec_from_file_location("yolo_serve", os.path.join(PKG_DIR, "serve.py"))
serve = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(serve)


def _type_name(f):
    from google.protobuf.descriptor import FieldDescriptor as FD
    names = {FD.TYPE_FLOAT: "float", FD.TYPE_INT32: "int32", FD.TYPE_UINT32: "uint32",
             FD.TYPE_BYTES: "bytes", FD.TYPE_STRING: "string"}
    return f.message_type.name if f.type == FD.TYPE_MESSAGE else names[f.type]


def _repeated(f):
    return f.is_repeated if hasattr(type(f), "is_repeated") else f.label == f.LABEL_REPEATED


def test_proto_matches_reference():
    """Every message and field of the reference's yolo.proto, with its number, type and
    cardinality, exists in the run-time descriptors, and nothing else does."""
    with open(os.path.join(GOLDEN, "yolo_proto_fields.json")) as f:
        spec = json.load(f)
    req, resp = serve.yolo_proto()
    fd = req.DESCRIPTOR.file
    assert fd.package == spec["package"] == "yolo"
    assert set(fd.message_types_by_name) == set(spec["messages"])
    for name, fields in spec["messages"].items():
        d = fd.message_types_by_name[name]
        got = sorted((f.name, f.number, _type_name(f), _repeated(f)) for f in d.fields)
        want = sorted((f["name"], f["number"], f["type"], f["repeated"]) for f in fields)
        assert got == want, name
    svc = fd.services_by_name["Yolo"]
    assert [(m.name, m.input_type.name, m.output_type.name) for m in svc.methods] == \
        [(m["name"], m["input"], m["output"]) for m in spec["services"]["Yolo"]]
    assert serve.METHOD == "/yolo.Yolo/Detect"


def _rle_decode(runs, n):
    out, v = [], 0
    for r in runs:
        out += [v] * r
        v ^= 1
    assert len(out) == n
    return np.array(out, np.uint8)


@pytest.mark.parametrize("seed", range(6))
def test_rle_round_trip(seed):
    rng = np.random.default_rng(seed)
    h, w = rng.integers(1, 40, 2)
    m = (rng.random((h, w)) < rng.random()).astype(np.uint8)
    if seed == 0:
        m[:] = 1
    if seed == 1:
        m[:] = 0
    runs = serve.rle_encode(m)
    assert all(r >= 0 for r in runs) and all(r > 0 for r in runs[1:])
    assert np.array_equal(_rle_decode(runs, m.size), m.reshape(-1))


def _jpeg_like(tag: int) -> bytes:
    return bytes([0xFF, 0xD8]) + tag.to_bytes(4, "little") + b"\x00" * 10


class FakeEngine:
    """Slots hold the identity of the image preprocessed into them; run_async copies the
    slots to the results, get returns one box whose score encodes the identity.  Records
    whether a handle's slots were overwritten before its results had been read."""

    def __init__(self, task=0, exec_ms=1.0, max_batch=8):
        self._task, self._exec = task, exec_ms
        self.slots = [None] * max_batch
        self.results = None
        self.unread = False
        self.clobbered = 0
        self.runs = []

    def task(self):
        return self._task

    def mask_dim(self):
        return (4, 6)

    def exec_ms(self, B):
        return self._exec

    def _put(self, slot, ident):
        if self.unread:
            self.clobbered += 1
        self.slots[slot] = ident

    def preprocess_jpeg(self, data, slot):
        self._put(slot, int.from_bytes(data[2:6], "little"))
        return 0

    def preprocess_host(self, bgr, slot):
        self._put(slot, 1_000_000 + int(bgr.sum()) % 1000)

    def preprocess_host_batch(self, bgrs, slots):
        for b, s in zip(bgrs, slots):
            self.preprocess_host(b, s)

    def run_async(self, B):
        time.sleep(0.002)
        self.results = list(self.slots[:B])
        self.unread = True
        self.runs.append(B)

    def sync(self):
        pass

    def get(self, slot):
        self.unread = False
        return [(0.0, 0.0, 1.0, 1.0, float(self.results[slot]), 7)]

    def get_obb(self, slot):
        self.unread = False
        return [(1.0, 2.0, 3.0, 4.0, 0.5, float(self.results[slot]), 2)]

    def get_cls(self, slot, k):
        self.unread = False
        return [self.results[slot] % 1000, 1], [0.75, 0.25]

    def slot_geom(self, slot):
        return (0.5, 3, 4)

    def get_mask(self, slot, det):
        m = np.zeros((4, 6), np.uint8)
        m[1:3, 2:5] = 1
        return m


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_batcher_fires_on_full_queue():
    eng = [FakeEngine(), FakeEngine()]
    b = serve.Batcher([("m", eng, 4)], target_ms=1e6)
    out = {}
    ths = [threading.Thread(target=lambda i=i: out.__setitem__(i, b.submit("", _jpeg_like(i))))
           for i in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(10)
    b.close()
    assert all(out[i][0] for i in range(4))
    assert [out[i][1].batch for i in range(4)] == [4] * 4
    assert sorted(out[i][1].boxes[0].score for i in range(4)) == [0, 1, 2, 3]


def test_batcher_fires_on_slack():
    """One request, a far from full queue: it leaves once its slack (target - waited -
    exec(max batch) - decode EMA - 1 ms) is spent, not later."""
    eng = [FakeEngine(exec_ms=2.0), FakeEngine(exec_ms=2.0)]
    b = serve.Batcher([("m", eng, 64)], target_ms=30.0)
    t0 = time.monotonic()
    ok, resp = b.submit("", _jpeg_like(5), timeout=10)
    dt = (time.monotonic() - t0) * 1e3
    b.close()
    assert ok and resp.batch == 1 and resp.boxes[0].score == 5
    assert 20.0 <= resp.queue_ms <= 150.0, resp.queue_ms   # slack 30 - 2 - 2 - 1 = 25 ms
    assert dt < 1000


def test_routing_tasks_and_failures():
    det = [FakeEngine(0), FakeEngine(0)]
    seg = [FakeEngine(3), FakeEngine(3)]
    obb = [FakeEngine(1), FakeEngine(1)]
    cls = [FakeEngine(2), FakeEngine(2)]
    b = serve.Batcher([("det", det, 2), ("seg", seg, 2), ("obb", obb, 2), ("cls", cls, 2)],
                      target_ms=5.0)
    ok, r = b.submit("", _jpeg_like(11), timeout=10)
    assert ok and r.task == "detect" and r.boxes[0].score == 11
    ok, r = b.submit("seg", _jpeg_like(12), timeout=10)
    assert ok and r.task == "segment" and (r.mask_h, r.mask_w) == (4, 6)
    assert (r.lb_scale, r.lb_top, r.lb_left) == (0.5, 3, 4)
    m = np.zeros((4, 6), np.uint8)
    m[1:3, 2:5] = 1
    assert np.array_equal(_rle_decode(list(r.masks[0].rle), 24), m.reshape(-1))
    ok, r = b.submit("obb", _jpeg_like(13), timeout=10)
    assert ok and r.task == "obb" and r.rboxes[0].score == 13 and not r.boxes
    ok, r = b.submit("cls", _jpeg_like(14), timeout=10)
    assert ok and r.task == "classify" and [c.id for c in r.classes] == [14, 1]
    with pytest.raises(KeyError):
        b.submit("nope", _jpeg_like(1))
    ok, r = b.submit("det", b"not an image", timeout=10)
    assert not ok
    import cv2
    img = np.full((5, 7, 3), 3, np.uint8)
    png = cv2.imencode(".png", img)[1].tobytes()
    ok, r = b.submit("det", png, timeout=10)
    assert ok and r.boxes[0].score == 1_000_000 + int(img.sum()) % 1000
    b.close()


def test_two_stage_alternation_many_clients():
    """Many concurrent clients: every response carries its own image's result (a handle's
    results are read before the handle is refilled) and both handles are used."""
    eng = [FakeEngine(exec_ms=0.5), FakeEngine(exec_ms=0.5)]
    b = serve.Batcher([("m", eng, 8)], target_ms=4.0)
    res = {}

    def client(c):
        for k in range(12):
            ident = c * 100 + k
            ok, r = b.submit("", _jpeg_like(ident), timeout=20)
            res[ident] = (ok, r.boxes[0].score, r.batch)

    ths = [threading.Thread(target=client, args=(c,)) for c in range(10)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(60)
    b.close()
    assert len(res) == 120
    assert all(ok and score == ident for ident, (ok, score, _) in res.items())
    assert eng[0].runs and eng[1].runs
    assert eng[0].clobbered == 0 and eng[1].clobbered == 0
    assert max(bt for _, _, bt in res.values()) > 1


def test_grpc_end_to_end():
    import grpc
    eng = [FakeEngine(), FakeEngine()]
    b = serve.Batcher([("yolo11n", eng, 4)], target_ms=5.0)
    port = _free_port()
    server = serve.make_server(b, f"127.0.0.1:{port}", workers=8)
    server.start()
    try:
        Req, _ = serve.yolo_proto()
        with grpc.insecure_channel(f"127.0.0.1:{port}") as ch:
            detect = serve.detect_stub(ch)
            r = detect(Req(image=_jpeg_like(42)), timeout=10)
            assert r.task == "detect" and r.boxes[0].score == 42 and r.batch == 1
            r = detect(Req(image=_jpeg_like(43), model="yolo11n"), timeout=10)
            assert r.boxes[0].score == 43
            with pytest.raises(grpc.RpcError) as e:
                detect(Req(image=_jpeg_like(1), model="other"), timeout=10)
            assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
            assert "unknown model" in e.value.details()
            with pytest.raises(grpc.RpcError) as e:
                detect(Req(image=b"garbage"), timeout=10)
            assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
            assert "decode" in e.value.details()
    finally:
        server.stop(0)
        b.close()


def test_cpu_decode_pool():
    """decode="cpu": a batch's images decoded on the thread pool (PNG and BMP alike), an
    undecodable one fails alone while the rest of its batch is served."""
    import cv2
    eng = [FakeEngine(), FakeEngine()]
    b = serve.Batcher([("m", eng, 4)], target_ms=1e6, decode="cpu", decoders=3)
    imgs = [np.full((6, 9, 3), 10 + i, np.uint8) for i in range(3)]
    blobs = [cv2.imencode(".png", imgs[0])[1].tobytes(), cv2.imencode(".png", imgs[1])[1].tobytes(),
             cv2.imencode(".bmp", imgs[2])[1].tobytes(), b"\xff\xd8 broken"]
    out = {}
    ths = [threading.Thread(target=lambda i=i: out.__setitem__(i, b.submit("", blobs[i], timeout=10)))
           for i in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(20)
    b.close()
    for i in range(3):
        ok, r = out[i]
        assert ok and r.batch == 4 and r.boxes[0].score == 1_000_000 + int(imgs[i].sum()) % 1000
    assert out[3][0] is False
