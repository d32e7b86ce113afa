"""JPEG front end (yolo_preprocess_jpeg): nvJPEG decode on the GPU, then the task's own
preprocessing into the slot.  Compared with the same preprocessing (C oracle) of the frame
as libjpeg (cv2.imdecode) decodes it.  The two decoders' IDCT and chroma upsampling differ
(about 22 levels at the 99.9th percentile on the synthetic frame's hard rectangle edges), so
the gate is the mean (|diff| < 1.5/255, which a wrong channel order or a misplaced frame
fails by far) with a loose tail bound (99.9th percentile <= 0.15); geometry must be
identical."""
import os

import numpy as np
import pytest
import torch

from conftest import MODELS

import graph_ref

pytestmark = pytest.mark.gpu


def _jpeg(h, w, seed):
    import cv2
    from yolo11_cu_b200 import frames
    bgr = frames.synthetic_bgr(h, w, seed=seed)
    ok, enc = cv2.imencode(".jpg", bgr, [cv2.IMWRITE_JPEG_QUALITY, 95])
    assert ok
    data = enc.tobytes()
    return data, cv2.imdecode(np.frombuffer(data, np.uint8), cv2.IMREAD_COLOR)


def _close(got, ref):
    d = np.abs(got.astype(np.float32) - ref.astype(np.float32))
    assert d.mean() < 1.5 / 255, d.mean()
    assert np.quantile(d, 0.999) <= 0.15, np.quantile(d, 0.999)


def test_jpeg_letterbox_detect(lib, cuda, pkg):
    from yolo11_cu_b200 import export, runtime as rt
    d = export.ensure_model_dir("yolo11n", MODELS, 640)
    data, dec = _jpeg(1080, 810, 0)
    eng = rt.Engine(d, 2)
    assert eng.preprocess_jpeg(data, 1) == 0
    got = eng.read(0, 2)[1]
    _close(got, graph_ref.letterbox(dec, 640))
    scale, top, left = eng.slot_geom(1)
    dev = torch.from_numpy(dec).to(cuda)
    torch.cuda.synchronize()
    eng.preprocess(dev.data_ptr(), dec.shape[0], dec.shape[1], 0)
    assert eng.slot_geom(0) == (scale, top, left)
    eng.run(2)
    eng._check()
    n0, n1 = len(eng.get(0)), len(eng.get(1))
    assert n1 > 0 and abs(n0 - n1) <= max(3, 0.3 * n0)
    assert eng.preprocess_jpeg(b"\x89PNG not a jpeg", 0) == -1
    assert b"not a JPEG" in lib.yolo_last_error()


def test_jpeg_classify(lib, cuda, pkg):
    from yolo11_cu_b200 import export, runtime as rt
    d = export.ensure_model_dir("yolo11n-cls", MODELS, 224)
    data, dec = _jpeg(480, 640, 3)
    eng = rt.Engine(d, 1)
    assert eng.preprocess_jpeg(data, 0) == 0
    ref, _ = graph_ref.preprocess_cls(dec, 224)
    _close(eng.read(0, 1)[0], ref)
    eng.run(1)
    eng._check()
    ids, probs = eng.get_cls(0, 5)
    assert len(ids) == 5 and probs[0] > 0
