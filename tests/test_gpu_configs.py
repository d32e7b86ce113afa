"""Parity of the configurations the benchmark measures (the five BASELINE configs' shapes).

* yolo11m 640 (bench workload): per op at full size against the oracle interpreter with the
  reference's resync protocol, using the tile / algorithm choices the batch-32 bench engine
  tunes; then the benched engine itself — batch 32, the same tile cache, the one-graph
  pipeline over 32 synthetic 1280x720 frames — against the fp32 oracle forward of three
  slots (head tensors) and the C oracle's decode + NMS of the engine's own logits (bit-exact).
* yolo11x 1024: per op at full size against the oracle interpreter.
* yolo11n-seg 640 at batch 64: per-instance mask IoU of two slots against the fp32 forward
  (the reference's test/compare_seg.py criterion, IoU >= 0.995).
"""
import os

import numpy as np
import pytest
import torch

from conftest import MODELS

import graph_ref

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def _rel(got, ref):
    return float(np.abs(got.astype(np.float32) - ref).max() / (np.abs(ref).max() + 1e-6))


def _per_op(eng, g, outs, B):
    worst = (0.0, -1)
    for k in range(eng.num_ops()):
        if eng.run_op(k, B) == 1:
            continue
        t = g.out_tensor(k)
        got = eng.read(t, B)
        for b in range(B):
            rel = _rel(got[b], outs[k])
            assert rel <= TOL, (k, g.ops[k][0], rel)
            worst = max(worst, (rel, k))
        eng.write(t, np.repeat(outs[k][None].astype(np.float16), B, 0))
    return worst


def _engine(rt, d, B, **kw):
    """The bench's engine: tiles from (or tuned into) the model directory's batch-B cache."""
    os.environ["YOLO_TUNE_CACHE"] = os.path.join(d, f"tune_b{B}.txt")
    try:
        return rt.Engine(d, B, **kw)
    finally:
        del os.environ["YOLO_TUNE_CACHE"]


def test_yolo11m_per_op_bench_tiles(lib, cuda, pkg, capsys):
    from yolo11_cu_b200 import export, runtime as rt
    d = export.ensure_model_dir("yolo11m", MODELS, 640, (720, 1280))
    g = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    _, outs = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=True)
    eng = _engine(rt, d, 32, fuse=False)       # the batch-32 choices, run on 2 images
    eng.write(0, np.stack([x, x]))
    worst = _per_op(eng, g, outs, 2)
    eng.close()
    with capsys.disabled():
        print(f"\nyolo11m 640 per-op worst rel {worst[0]:.4f} (op {worst[1]})")


def test_yolo11x_1024_per_op(lib, cuda, pkg, capsys):
    from yolo11_cu_b200 import export, runtime as rt
    d = export.ensure_model_dir("yolo11x", MODELS, 1024, (1080, 1920))
    g = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    _, outs = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=True)
    eng = rt.Engine(d, 1, fuse=False)
    eng.write(0, x)
    worst = _per_op(eng, g, outs, 1)
    eng.close()
    with capsys.disabled():
        print(f"\nyolo11x 1024 per-op worst rel {worst[0]:.4f} (op {worst[1]})")


def _frames_on_device(n, hw, cuda, seed0=0):
    from yolo11_cu_b200 import frames
    bgr = np.stack([frames.synthetic_bgr(*hw, seed=seed0 + i) for i in range(n)])
    dev = torch.from_numpy(bgr).to(cuda)
    torch.cuda.synchronize()
    return bgr, dev


def test_yolo11m_bench_graph_b32(lib, cuda, pkg, capsys):
    """The exact engine the bench times: fused, autotuned at batch 32, one graph per step."""
    from yolo11_cu_b200 import export, runtime as rt
    hw, B = (720, 1280), 32
    d = export.ensure_model_dir("yolo11m", MODELS, 640, hw)
    g = graph_ref.Graph(d)
    bgr, dev = _frames_on_device(B, hw, cuda)
    eng = _engine(rt, d, B)
    eng.bind_frames(0, dev.data_ptr(), hw[0], hw[1], B, False)
    eng.run_frames(0, B)
    xs = eng.read(0, B)
    levels = g.levels()
    heads = [(eng.read(b_, B), eng.read(c_, B), st) for b_, c_, _, st in levels]
    rels = []
    for s in (0, 13, 31):
        assert np.array_equal(xs[s].view(np.uint16), graph_ref.letterbox(bgr[s], g.S).view(np.uint16))
        bufs, _ = graph_ref.run_graph(g, xs[s].astype(np.float32), round_fp16=False)
        for (b_, c_, _, _), (hb, hc, _) in zip(levels, heads):
            for t, got in ((b_, hb[s]), (c_, hc[s])):
                rel = _rel(got, graph_ref.tensor_hwc(g, bufs, t))
                rels.append(rel)
                assert rel <= TOL, (s, t, rel)
        recs = graph_ref.decode([(hb[s], hc[s], st) for hb, hc, st in heads], g.nc, 0.25)
        keep = graph_ref.nms(recs, 0.45, 300)
        dets = eng.get(s)
        assert eng.raw_count(s) == len(recs) and len(dets) == len(keep) > 0
        scale, top, left = eng.slot_geom(s)
        assert np.array_equal(np.float32([d_[4] for d_ in dets]).view(np.uint32),
                              keep[:, 4].view(np.uint32))
        assert [d_[5] for d_ in dets] == [int(c) for c in keep[:, 5]]
        x1 = (keep[:, 0] - np.float32(left)) / np.float32(scale)
        assert np.array_equal(np.float32([d_[0] for d_ in dets]), x1.astype(np.float32))
    eng.close()
    with capsys.disabled():
        print(f"\nyolo11m b32 bench graph: head tensors vs fp32 forward, worst rel {max(rels):.4f}")


def mask_ious(eng, slot, g, x, iou_nms=0.45, first=40):
    """Per-instance IoU of the engine's masks of `slot` against the fp32 oracle forward of
    its input x: each fp32 survivor (first `first`) is matched to the engine's same-class box
    of highest IoU (> 0.9) and the two masks compared (test/compare_seg.py:68-101)."""
    bufs, _ = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=False)
    levels = g.levels()
    heads = [(graph_ref.tensor_hwc(g, bufs, b_).astype(np.float16),
              graph_ref.tensor_hwc(g, bufs, c_).astype(np.float16), st) for b_, c_, _, st in levels]
    coefs = [graph_ref.tensor_hwc(g, bufs, cf).astype(np.float16) for _, _, cf, _ in levels]
    proto = graph_ref.tensor_hwc(g, bufs, g.proto()).astype(np.float16)
    keep = graph_ref.nms(graph_ref.decode(heads, g.nc), iou_nms, 300)
    Ws = [h[0].shape[1] for h in heads]
    bases = np.cumsum([0] + [w * w for w in Ws])
    scale, top, left = eng.slot_geom(slot)
    dets = np.array(eng.get(slot), np.float32).reshape(-1, 6)
    dets[:, [0, 2]] = dets[:, [0, 2]] * scale + left        # back to letterbox pixels
    dets[:, [1, 3]] = dets[:, [1, 3]] * scale + top
    ious = []
    for k in keep[:first]:
        same = np.nonzero(dets[:, 5] == k[5])[0]
        if len(same) == 0:
            continue
        s_ = dets[same]
        ix1 = np.maximum(s_[:, 0], k[0]); iy1 = np.maximum(s_[:, 1], k[1])
        ix2 = np.minimum(s_[:, 2], k[2]); iy2 = np.minimum(s_[:, 3], k[3])
        inter = np.clip(ix2 - ix1, 0, None) * np.clip(iy2 - iy1, 0, None)
        ua = (s_[:, 2] - s_[:, 0]) * (s_[:, 3] - s_[:, 1]) + (k[2] - k[0]) * (k[3] - k[1]) - inter
        j = int(np.argmax(inter / ua))
        if (inter / ua)[j] <= 0.9:
            continue
        a = int(k[6])
        li = int(np.searchsorted(bases, a, side="right") - 1)
        y, xx = divmod(a - bases[li], Ws[li])
        ref = graph_ref.mask(coefs[li][y, xx], proto, k, g.S).astype(bool)
        got = eng.get_mask(slot, int(same[j])).astype(bool)
        union = (ref | got).sum()
        ious.append(1.0 if union == 0 else (ref & got).sum() / union)
    return np.array(ious), min(first, len(keep))


def test_yolo11n_seg_b64_masks(lib, cuda, pkg, capsys):
    from yolo11_cu_b200 import export, runtime as rt
    hw, B = (1080, 810), 64
    d = export.ensure_model_dir("yolo11n-seg", MODELS, 640)
    g = graph_ref.Graph(d)
    _, dev = _frames_on_device(B, hw, cuda)
    eng = _engine(rt, d, B)
    eng.bind_frames(0, dev.data_ptr(), hw[0], hw[1], B, False)
    eng.run_frames(0, B)
    xs = eng.read(0, B)
    for s in (0, 63):
        ious, n = mask_ious(eng, s, g, xs[s])
        with capsys.disabled():
            print(f"\nyolo11n-seg b64 slot {s}: {len(ious)} of {n} matched, median "
                  f"{np.median(ious):.4f}, min {ious.min():.4f}, >= 0.995: {(ious >= 0.995).mean():.2f}")
        assert len(ious) >= 0.8 * n and n > 0
        assert np.median(ious) >= 0.995
        assert (ious >= 0.995).mean() >= 0.8
    eng.close()
