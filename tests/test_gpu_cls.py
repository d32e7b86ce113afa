"""Classification (task "classify") on the GPU through the C ABI.

* yk_gap / yk_softmax against torch fp32 (tolerance 1e-3 of the largest value: fp16 in and
  out, fp32 sums);
* yk_preprocess_cls bit for bit against the C oracle (oracle/postproc_ref.c, a restatement
  of the reference's k_preprocess_cls + clsGeom) on frames that downscale, upscale, and hit
  odd crop offsets;
* the whole model (yolo11n-cls at 224, the reference's yolo11n-cls topology with seeded
  weights): per-op isolation against the oracle interpreter, and end to end through
  yolo_preprocess_cls / yolo_run / yolo_get_cls against the oracle forward of the same input,
  with every batch slot agreeing.  The per-op comparison against the reference's own
  exporter outputs runs in test_gpu_model.py (golden case yolo11n-cls-224).
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from conftest import MODELS

import graph_ref

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def _vw(rt, t, coff=0, Cv=None):
    return rt.tview(t, coff, Cv)


@pytest.mark.parametrize("B,H,W,C_", [(1, 7, 7, 1280), (4, 7, 7, 256), (2, 3, 5, 64), (3, 1, 1, 8)])
def test_gap(lib, cuda, B, H, W, C_):
    from yolo11_cu_b200 import runtime as rt
    x = torch.randn(B, H, W, C_ + 8, device=cuda).half()
    y = torch.full((B, 1, 1, C_ + 16), 7.0, device=cuda).half()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_gap(C.byref(_vw(rt, x, 8, C_)), C.byref(_vw(rt, y, 8, C_)), st) == 0
    torch.cuda.synchronize()
    ref = x[..., 8:].float().mean(dim=(1, 2))
    got = y[:, 0, 0, 8:8 + C_].float()
    assert (got - ref).abs().max().item() <= 1e-3 * (ref.abs().max().item() + 1e-6) + 1e-3
    assert torch.all(y[..., :8] == 7.0) and torch.all(y[..., 8 + C_:] == 7.0)


@pytest.mark.parametrize("B,C_", [(1, 1000), (5, 1000), (2, 37), (1, 1)])
def test_softmax(lib, cuda, B, C_):
    from yolo11_cu_b200 import runtime as rt
    x = (torch.randn(B, 1, 1, C_, device=cuda) * 4).half()
    y = torch.empty_like(x)
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_softmax(C.byref(_vw(rt, x)), C.byref(_vw(rt, y)), st) == 0
    torch.cuda.synchronize()
    ref = torch.softmax(x.float(), dim=-1)
    assert (y.float() - ref).abs().max().item() <= 1e-3 * ref.max().item()
    assert abs(y.float().sum(-1) - 1).max().item() < 1e-2


@pytest.mark.parametrize("sh,sw,S", [(1080, 810, 224), (480, 640, 224), (100, 300, 224),
                                     (224, 224, 224), (333, 517, 96), (31, 19, 64)])
def test_preprocess_cls_bitexact(lib, cuda, sh, sw, S):
    from yolo11_cu_b200 import frames, runtime as rt
    bgr = frames.synthetic_bgr(sh, sw, seed=sh + sw)
    dev = torch.from_numpy(bgr).to(cuda)
    y = torch.zeros(2, S, S, 3, dtype=torch.half, device=cuda)
    geom = (C.c_int * 4)()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_preprocess_cls(C.c_void_p(dev.data_ptr()), sh, sw, C.byref(_vw(rt, y)), 1,
                                 geom, st) == 0
    torch.cuda.synchronize()
    ref, rgeom = graph_ref.preprocess_cls(bgr, S)
    assert tuple(geom) == rgeom
    got = y[1].cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    assert torch.all(y[0] == 0)                  # other slots untouched


def _cls_dir():
    from yolo11_cu_b200 import export
    return export.ensure_model_dir("yolo11n-cls", MODELS, 224)


def test_cls_per_op_vs_oracle(lib, cuda, pkg):
    from yolo11_cu_b200 import runtime as rt
    d = _cls_dir()
    g = graph_ref.Graph(d)
    assert g.task == "classify" and g.nc == 1000
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    _, outs = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=True)
    eng = rt.Engine(d, 2, autotune=True, fuse=False)
    assert eng.task() == 2
    eng.write(0, np.stack([x, x]))
    for k in range(eng.num_ops()):
        assert eng.run_op(k, 2) == 0
        t = g.out_tensor(k)
        got = eng.read(t, 2).astype(np.float32)
        for b in range(2):
            rel = np.abs(got[b] - outs[k]).max() / (np.abs(outs[k]).max() + 1e-6)
            assert rel <= TOL, (k, g.ops[k][0], rel)
        eng.write(t, np.repeat(outs[k][None].astype(np.float16), 2, 0))


@pytest.mark.parametrize("B", [1, 4])
def test_cls_end_to_end(lib, cuda, pkg, B):
    from yolo11_cu_b200 import frames, runtime as rt
    d = _cls_dir()
    g = graph_ref.Graph(d)
    bgr = frames.synthetic_bgr(1080, 810, seed=0)
    dev = torch.from_numpy(bgr).to(cuda)
    torch.cuda.synchronize()
    eng = rt.Engine(d, B)
    for s in range(B):
        eng.preprocess_cls(dev.data_ptr(), 1080, 810, s)
    eng.run(B)
    eng._check()
    # the engine's input is the oracle's preprocessing, bit for bit
    xin, _ = graph_ref.preprocess_cls(bgr, g.S)
    got_in = eng.read(0, B)
    for s in range(B):
        assert np.array_equal(got_in[s].view(np.uint16), xin.view(np.uint16))
    # fp32 oracle forward of the same input
    bufs, _ = graph_ref.run_graph(g, xin.astype(np.float32), round_fp16=False)
    probs = graph_ref.tensor_hwc(g, bufs, g.out_tensor(len(g.ops) - 1)).reshape(-1)
    order = np.argsort(-probs, kind="stable")
    ids0, p0 = eng.get_cls(0, 5)
    assert len(ids0) == 5
    assert ids0[0] == order[0]
    # |dp| < 5e-3 per listed class (fp16 engine vs fp32 oracle)
    for i, p in zip(ids0, p0):
        assert abs(p - probs[i]) < 5e-3, (i, p, probs[i])
    assert p0 == sorted(p0, reverse=True)
    for s in range(1, B):                        # batch self-consistency
        assert eng.get_cls(s, 5) == (ids0, p0)
    assert eng.get(0) == []                      # no detections on a classify handle
    k = eng.get_cls(0, 2000)[0]
    assert len(k) == 1000                        # k clamps to nc
