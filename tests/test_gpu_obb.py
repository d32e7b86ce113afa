"""Oriented boxes (task "obb") on the GPU through the C ABI.

* yk_decode_obb + yk_nms_obb bit for bit against the C oracle (oracle/postproc_ref.c, a
  restatement of the reference's k_decode_obb / probiou / k_nms_obb) on seeded head tensors:
  candidate counts, survivor records and their order; with few and with many (> 4096)
  candidates, and with tied scores;
* the whole model (yolo11n-obb at 1024, the reference's yolo11-obb topology with seeded
  weights): per-op isolation against the oracle interpreter, and end to end through
  yolo_preprocess / yolo_run / yolo_get_obb against the oracle's decode + NMS of the
  engine's own head tensors, every batch slot agreeing.  Per-op parity against the
  reference's own exporter outputs is the golden case yolo11n-obb-128 (test_gpu_model.py).
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


def _levels(rt, heads):
    arr = (rt.YkLevel * len(heads))()
    for i, (b, c, a, st) in enumerate(heads):
        arr[i].box = rt.tview(b)
        arr[i].cls = rt.tview(c)
        arr[i].coef = rt.tview(a)
        arr[i].stride = st
    return arr


def _run_post(lib, rt, heads, B, nc, conf, iou, max_out=300):
    A = sum(b.shape[1] * b.shape[2] for b, _, _, _ in heads)
    ws = torch.zeros(lib.yk_obb_workspace_bytes(B, A), dtype=torch.uint8, device="cuda")
    out = torch.zeros(B, max_out, 7, device="cuda")
    cnt = torch.zeros(B, dtype=torch.int32, device="cuda")
    raw = torch.zeros(B, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    lv = _levels(rt, heads)
    assert lib.yk_decode_obb(lv, len(heads), B, nc, conf, C.c_void_p(ws.data_ptr()), st) == 0
    assert lib.yk_nms_obb(B, A, iou, max_out, C.c_void_p(ws.data_ptr()),
                          C.c_void_p(out.data_ptr()), C.c_void_p(cnt.data_ptr()),
                          C.c_void_p(raw.data_ptr()), st) == 0
    torch.cuda.synchronize()
    assert lib.yk_fetch_device_error() == 0
    return out.cpu().numpy(), cnt.cpu().numpy(), raw.cpu().numpy()


def _check_vs_oracle(heads, out, cnt, raw, B, nc, conf, iou, max_out=300):
    for b in range(B):
        lv = [(h[b].cpu().numpy(), c[b].cpu().numpy(), a[b].cpu().numpy(), st) for h, c, a, st in heads]
        recs = graph_ref.decode_obb(lv, nc, conf)
        keep = graph_ref.nms_obb(recs, iou, max_out)
        assert raw[b] == len(recs)
        assert cnt[b] == len(keep)
        got = out[b, :cnt[b]]
        assert np.array_equal(got.view(np.uint32), keep[:, :7].view(np.uint32)), b


@pytest.mark.parametrize("S,bias,B,quant", [(256, -1.0, 2, False), (640, 1.0, 1, False),
                                            (256, 0.0, 2, True)])
def test_decode_nms_obb_bitexact(lib, cuda, S, bias, B, quant):
    """quant: coarse logits so many scores tie (order then falls back to anchor index)."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(S + B)
    nc = 15
    heads = []
    for st in (8, 16, 32):
        H = S // st
        box = torch.randn(B, H, H, 64, generator=g) * 2
        cls = torch.randn(B, H, H, 16, generator=g) * 2 + bias
        cls[..., nc:] = 0
        if quant:
            cls = torch.round(cls * 2) / 2
        ang = torch.randn(B, H, H, 8, generator=g) * 2
        heads.append((box.half().to(cuda), cls.half().to(cuda), ang.half().to(cuda), st))
    out, cnt, raw = _run_post(lib, rt, heads, B, nc, 0.25, 0.45)
    if S == 640:
        assert raw[0] > 4096                 # past one 1024-thread pass and past 4096
    _check_vs_oracle(heads, out, cnt, raw, B, nc, 0.25, 0.45)


def _obb_dir():
    from yolo11_cu_b200 import export
    return export.ensure_model_dir("yolo11n-obb", MODELS, 1024)


def test_obb_per_op_vs_oracle(lib, cuda, pkg):
    from yolo11_cu_b200 import runtime as rt
    d = _obb_dir()
    g = graph_ref.Graph(d)
    assert g.task == "obb" and g.nc == 15
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    _, outs = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=True)
    eng = rt.Engine(d, 1, autotune=True, fuse=False)
    assert eng.task() == 1
    eng.write(0, x)
    for k in range(eng.num_ops()):
        r = eng.run_op(k, 1)
        if r == 1:
            continue
        t = g.out_tensor(k)
        got = eng.read(t, 1)[0].astype(np.float32)
        rel = np.abs(got - outs[k]).max() / (np.abs(outs[k]).max() + 1e-6)
        assert rel <= TOL, (k, g.ops[k][0], rel)
        eng.write(t, outs[k][None].astype(np.float16))


def test_obb_end_to_end(lib, cuda, pkg):
    from yolo11_cu_b200 import frames, runtime as rt
    d = _obb_dir()
    g = graph_ref.Graph(d)
    B = 2
    eng = rt.Engine(d, B)
    bgr = frames.synthetic_bgr(1080, 810, seed=0)
    dev = torch.from_numpy(bgr).to(cuda)
    torch.cuda.synchronize()
    for s in range(B):
        eng.preprocess(dev.data_ptr(), 1080, 810, s)
    eng.run(B)
    eng._check()
    scale, top, left = eng.slot_geom(0)
    heads = [(eng.read(b_, B), eng.read(c_, B), eng.read(a_, B), st) for b_, c_, a_, st in g.levels()]
    dets0 = eng.get_obb(0)
    assert len(dets0) > 0 and eng.get(0) == []
    for s in range(B):
        recs = graph_ref.decode_obb([(b[s], c[s], a[s], st) for b, c, a, st in heads], g.nc, 0.25)
        keep = graph_ref.nms_obb(recs, 0.45, 300)
        assert eng.raw_count(s) == len(recs)
        dets = eng.get_obb(s)
        assert len(dets) == len(keep)
        got = np.array(dets, np.float32).reshape(-1, 7)
        # mapped back as the reference: (cx - left) / scale, w / scale, angle unchanged
        xb = (keep[:, 0] - np.float32(left)) / np.float32(scale)
        wb = keep[:, 2] / np.float32(scale)
        assert np.array_equal(got[:, 0], xb.astype(np.float32))
        assert np.array_equal(got[:, 2], wb.astype(np.float32))
        assert np.array_equal(got[:, 4].view(np.uint32), keep[:, 6].view(np.uint32))
        assert np.array_equal(got[:, 5].view(np.uint32), keep[:, 4].view(np.uint32))
        assert np.array_equal(got[:, 6], keep[:, 5])
        assert dets == dets0                      # batch self-consistency
