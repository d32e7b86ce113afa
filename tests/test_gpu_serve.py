"""The gRPC batching server on the GPU: real engines behind yolo.Yolo/Detect on 127.0.0.1,
several concurrent clients sending JPEG and PNG images to a detect and a segment model, with
JPEG decoded by nvJPEG on the handle or on the CPU decoder pool.  Every response must equal what the engine returns for that image alone
(same handle options, heuristic tiles, so batch composition cannot change a result): boxes
bit for bit, segment masks as decoded run lengths, letterbox geometry."""
import importlib.util
import os
import socket
import threading

import numpy as np
import pytest

from conftest import MODELS, PKG_DIR

pytestmark = pytest.mark.gpu

_spec = importlib.util.spec_from_file_location("yolo_serve_gpu", os.path.join(PKG_DIR, "serve.py"))
serve = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(serve)


def _rle_decode(runs, n):
    out = np.zeros(n, np.uint8)
    pos, v = 0, 0
    for r in runs:
        out[pos:pos + r] = v
        pos += r
        v ^= 1
    assert pos == n
    return out


def _images():
    import cv2
    from yolo11_cu_b200 import frames
    out = []
    for i, (h, w) in enumerate([(720, 1280), (1080, 810), (480, 640), (333, 517), (640, 640),
                                (1080, 1920)]):
        bgr = frames.synthetic_bgr(h, w, seed=40 + i)
        out.append(cv2.imencode(".jpg", bgr, [cv2.IMWRITE_JPEG_QUALITY, 92])[1].tobytes())
    out.append(cv2.imencode(".png", frames.synthetic_bgr(400, 600, seed=60))[1].tobytes())
    return out


def _direct(eng, data, decode):
    """The engine alone on one image: (boxes, masks, geometry)."""
    import cv2
    if decode == "gpu" and data[:2] == b"\xff\xd8":
        assert eng.preprocess_jpeg(data, 0) == 0
    else:
        eng.preprocess_host(cv2.imdecode(np.frombuffer(data, np.uint8), cv2.IMREAD_COLOR), 0)
    eng.run(1)
    dets = eng.get(0)
    masks = [eng.get_mask(0, j) for j in range(len(dets))] if eng.task() == 3 else []
    return dets, masks, eng.slot_geom(0)


@pytest.mark.parametrize("decode", ["gpu", "cpu"])
def test_serve_matches_engine(lib, cuda, pkg, decode):
    import grpc
    from yolo11_cu_b200 import export, runtime as rt
    det_dir = export.ensure_model_dir("yolo11n", MODELS, 640)
    seg_dir = export.ensure_model_dir("yolo11n-seg", MODELS, 640)
    mk = lambda d, b: rt.Engine(d, b, device=0, autotune=False)
    batcher = serve.Batcher([("yolo11n", [mk(det_dir, 4), mk(det_dir, 4)], 4),
                             ("yolo11n-seg", [mk(seg_dir, 2), mk(seg_dir, 2)], 2)],
                            target_ms=20.0, decode=decode, decoders=4)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    server = serve.make_server(batcher, f"127.0.0.1:{port}", workers=16)
    server.start()
    imgs = _images()
    jobs = [(m, i) for m in ("", "yolo11n-seg") for i in range(len(imgs))] * 2
    got = {}
    try:
        Req, _ = serve.yolo_proto()

        def client(c):
            with grpc.insecure_channel(f"127.0.0.1:{port}") as ch:
                detect = serve.detect_stub(ch)
                for k in range(c, len(jobs), 4):
                    m, i = jobs[k]
                    got[k] = detect(Req(image=imgs[i], model=m), timeout=60)

        ths = [threading.Thread(target=client, args=(c,)) for c in range(4)]
        for t in ths:
            t.start()
        for t in ths:
            t.join(120)
    finally:
        server.stop(0)
        batcher.close()
    assert len(got) == len(jobs)
    ref_det, ref_seg = mk(det_dir, 4), mk(seg_dir, 2)
    want = {(m, i): _direct(ref_seg if m else ref_det, imgs[i], decode)
            for m in ("", "yolo11n-seg") for i in range(len(imgs))}
    assert max(r.batch for r in got.values()) >= 1
    for k, r in got.items():
        m, i = jobs[k]
        dets, masks, geom = want[(m, i)]
        assert r.task == ("segment" if m else "detect")
        boxes = [(b.x1, b.y1, b.x2, b.y2, b.score, b.cls) for b in r.boxes]
        assert boxes == [tuple(np.float32(v).item() if j < 5 else v for j, v in enumerate(d))
                         for d in dets], (k, m, i)
        if m:
            ph, pw = ref_seg.mask_dim()
            assert (r.mask_h, r.mask_w) == (ph, pw)
            assert (np.float32(r.lb_scale), r.lb_top, r.lb_left) == \
                (np.float32(geom[0]), geom[1], geom[2])
            assert len(r.masks) == len(masks)
            for mm, ref in zip(r.masks, masks):
                assert np.array_equal(_rle_decode(list(mm.rle), ph * pw), ref.reshape(-1))
    assert sum(len(r.boxes) for r in got.values()) > 0
