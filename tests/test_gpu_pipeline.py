"""The one-graph pipeline (yolo_bind_frames / yolo_run_frames): H2D + batched letterbox + net +
decode + NMS + D2H replayed as one CUDA graph, the reference CLI's `pipeline` graph
(engine/engine.cu:1992-2004) behind the engine API.  It must give the same bits as the
reference-shaped path (yolo_preprocess per slot, then yolo_run), from host or device frames.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from conftest import MODELS

pytestmark = pytest.mark.gpu


def _model(name, S=640):
    from yolo11_cu_b200 import export
    return export.ensure_model_dir(name, MODELS, S)


@pytest.mark.parametrize("name,B,hw", [("yolo11n", 3, (720, 1280)), ("yolo11n-seg", 2, (1080, 810))])
def test_pipeline_matches_per_slot_path(lib, cuda, pkg, name, B, hw):
    from yolo11_cu_b200 import frames, runtime as rt
    d = _model(name)
    bgr = np.stack([frames.synthetic_bgr(*hw, seed=40 + i) for i in range(B)])
    host = torch.from_numpy(bgr).pin_memory()
    dev = host.to(cuda)
    torch.cuda.synchronize()
    eng = rt.Engine(d, B, autotune=False)
    fb = hw[0] * hw[1] * 3
    for s in range(B):
        eng.preprocess(dev.data_ptr() + s * fb, hw[0], hw[1], s)
    eng.run(B)
    eng._check()
    want = [eng.get(s) for s in range(B)]
    want_in = eng.read(0, B)
    want_masks = [eng.get_mask(0, i) for i in range(min(5, len(want[0])))] if name.endswith("seg") else []
    assert len(want[0]) > 0
    for id_, buf, is_host in ((0, host, True), (1, dev, False)):
        eng.write(0, np.zeros_like(want_in))            # the graph must refill the input
        eng.bind_frames(id_, buf.data_ptr(), hw[0], hw[1], B, is_host)
        eng.run_frames(id_, B)
        assert np.array_equal(eng.read(0, B).view(np.uint16), want_in.view(np.uint16))
        assert [eng.get(s) for s in range(B)] == want
        assert eng.get_batch(B) == want
        assert [eng.slot_geom(s) for s in range(B)] == [eng.slot_geom(0)] * B
        for i, m in enumerate(want_masks):
            assert np.array_equal(eng.get_mask(0, i), m)
        assert eng.frames_exec_ms(id_, B) > 0
    # a smaller batch of the same binding has its own graph
    eng.run_frames(1, 1)
    assert eng.get(0) == want[0]
    eng.close()


def test_pipeline_rejects_bad_bindings(lib, cuda, pkg):
    from yolo11_cu_b200 import runtime as rt
    d = _model("yolo11n")
    eng = rt.Engine(d, 2, autotune=False)
    pageable = np.zeros((2, 64, 64, 3), np.uint8)
    with pytest.raises(RuntimeError, match="page-locked"):
        eng.bind_frames(0, pageable.ctypes.data, 64, 64, 2, True)
    dev = torch.zeros(2, 64, 64, 3, dtype=torch.uint8, device=cuda)
    with pytest.raises(RuntimeError, match="device memory"):
        eng.bind_frames(0, pageable.ctypes.data, 64, 64, 2, False)
    with pytest.raises(RuntimeError, match="bad arguments"):
        eng.bind_frames(0, dev.data_ptr(), 64, 64, 3, False)     # more frames than slots
    with pytest.raises(RuntimeError, match="bad arguments"):
        eng.bind_frames(4, dev.data_ptr(), 64, 64, 1, False)
    with pytest.raises(RuntimeError, match="bad binding"):
        eng.run_frames(2, 1)                                      # never bound
    eng.bind_frames(2, dev.data_ptr(), 64, 64, 1, False)
    with pytest.raises(RuntimeError, match="bad binding"):
        eng.run_frames(2, 2)                                      # past the bound count
    eng.run_frames(2, 1)
    eng.close()


def test_two_bindings_in_flight(lib, cuda, pkg):
    """Two bound frame arrays launched back to back without a sync in between: each
    binding's results stay in its own pinned block (yolo_get_frames), equal to running each
    alone, and yolo_get reads the most recently launched run."""
    from yolo11_cu_b200 import frames, runtime as rt
    d = _model("yolo11n")
    hw, B = (720, 1280), 3
    a = torch.from_numpy(np.stack([frames.synthetic_bgr(*hw, seed=60 + i) for i in range(B)])).to(cuda)
    b = torch.from_numpy(np.stack([frames.synthetic_bgr(*hw, seed=70 + i) for i in range(B)])).to(cuda)
    torch.cuda.synchronize()
    eng = rt.Engine(d, B, autotune=False)
    eng.bind_frames(0, a.data_ptr(), hw[0], hw[1], B, False)
    eng.bind_frames(1, b.data_ptr(), hw[0], hw[1], B, False)
    eng.run_frames(0, B)
    want_a = eng.get_batch(B)
    eng.run_frames(1, B)
    want_b = eng.get_batch(B)
    assert want_a != want_b and len(want_a[0]) > 0
    eng.run_frames_async(0, B)
    eng.run_frames_async(1, B)
    eng.sync()
    assert eng.get_frames(0, B) == want_a
    assert eng.get_frames(1, B) == want_b
    assert eng.get_batch(B) == want_b            # the most recent launch
    eng.close()
