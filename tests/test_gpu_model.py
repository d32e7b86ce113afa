"""Whole-graph parity on the GPU through the yolo.h ABI.

1. Per-op isolation against the REFERENCE's own per-op outputs (golden fixtures made by the
   reference exporter, export/export.py:446-526 + 660): every op of the unfused graph runs on
   the GPU, its output is compared (max|gpu-ref|/max|ref| <= 1.5 %), then overwritten with the
   reference value so the next op sees exact inputs — the reference's dump + compare.py
   protocol (engine/engine.cu:1843-1888, test/compare.py:21-25; gate tightened 3 % -> 1.5 %).
2. The same at full size (yolo11n / yolov8n / yolo11n-seg at 640) against the oracle
   interpreter.
3. End to end (fused graph + CUDA graph + yolo_preprocess): survivors must equal the C
   oracle's decode + NMS of the engine's own head tensors bit for bit, and every batch slot
   given the same frame must agree (reference --batch self-consistency check).
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, MODELS, golden_cases, split_case

import graph_ref

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def _per_op(eng, g, refs_of, B=1):
    worst = (0.0, -1)
    for k in range(eng.num_ops()):
        r = eng.run_op(k, B)
        if r == 1:
            continue
        t = g.out_tensor(k)
        got = eng.read(t, B).astype(np.float32)
        ref = refs_of(k)
        for b in range(B):
            rel = np.abs(got[b] - ref).max() / (np.abs(ref).max() + 1e-6)
            assert rel <= TOL, (k, g.ops[k][0], rel)
            worst = max(worst, (rel, k))
        eng.write(t, np.repeat(ref[None].astype(np.float16), B, 0))
    return worst


@pytest.mark.parametrize("case", golden_cases())
def test_per_op_vs_reference_golden(lib, cuda, golden_dirs, case):
    from yolo11_cu_b200 import runtime as rt
    d = golden_dirs[case]
    g = graph_ref.Graph(d)
    refs = np.load(os.path.join(GOLDEN, case, "refs.npz"))
    x = np.fromfile(os.path.join(GOLDEN, case, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    eng = rt.Engine(d, 2, autotune=False, fuse=False)
    eng.write(0, np.stack([x, x]))
    worst = _per_op(eng, g, lambda k: refs[f"op{k:03d}"].astype(np.float32), B=2)
    print(case, "worst rel", worst)


def _model_dir(name, S=640):
    from yolo11_cu_b200 import export
    return export.ensure_model_dir(name, MODELS, S)


@pytest.mark.parametrize("name", ["yolo11n", "yolov8n", "yolo11n-seg"])
def test_per_op_vs_oracle_full_size(lib, cuda, name):
    from yolo11_cu_b200 import runtime as rt
    d = _model_dir(name)
    g = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    _, outs = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=True)
    eng = rt.Engine(d, 1, autotune=True, fuse=False)
    eng.write(0, x)
    worst = _per_op(eng, g, lambda k: outs[k])
    print(name, "worst rel", worst)


@pytest.mark.parametrize("name,B", [("yolo11n", 4), ("yolo11n-seg", 2), ("yolov8n", 1)])
def test_end_to_end_bitexact_post(lib, cuda, pkg, name, B):
    from yolo11_cu_b200 import frames, runtime as rt
    d = _model_dir(name)
    g = graph_ref.Graph(d)
    eng = rt.Engine(d, B, iou=0.7)
    bgr = frames.synthetic_bgr(1080, 810, seed=0)
    dev = torch.from_numpy(bgr).to(cuda)
    torch.cuda.synchronize()
    for s in range(B):
        eng.preprocess(dev.data_ptr(), 1080, 810, s)
    eng.run(B)
    eng._check()
    # the letterbox the engine produced is the oracle's, bit for bit
    lb = eng.read(0, B)
    ref_lb = graph_ref.letterbox(bgr, g.S)
    assert np.array_equal(lb[0].view(np.uint16), ref_lb.view(np.uint16))
    levels = g.levels()
    heads = [(eng.read(b_, B), eng.read(c_, B), st) for b_, c_, _, st in levels]
    scale, top, left = eng.slot_geom(0)
    dets0 = eng.get(0)
    assert len(dets0) > 0
    for s in range(B):
        recs = graph_ref.decode([(b[s], c[s], st) for b, c, st in heads], g.nc, 0.25)
        keep = graph_ref.nms(recs, 0.7, 300)
        assert eng.raw_count(s) == len(recs)
        dets = eng.get(s)
        assert len(dets) == len(keep)
        got = np.array([[d_[4], d_[5]] for d_ in dets], np.float32).reshape(-1, 2)
        assert np.array_equal(got[:, 0].view(np.uint32), keep[:, 4].view(np.uint32))
        assert np.array_equal(got[:, 1], keep[:, 5])
        # boxes mapped back to original coordinates exactly as the reference (x-left)/scale
        xb = (keep[:, 0] - np.float32(left)) / np.float32(scale)
        assert np.array_equal(np.float32([d_[0] for d_ in dets]), xb.astype(np.float32))
        assert dets == dets0                      # batch self-consistency
    if g.task == "segment":
        ph, pw = eng.mask_dim()
        assert (ph, pw) == (g.S // 4, g.S // 4)
        proto = eng.read(g.proto(), 1)[0]
        Ws = [eng.tensor_view(b_)[2] for b_, _, _, _ in levels]
        bases = np.cumsum([0] + [w * w for w in Ws])
        coefs = [eng.read(cf, 1)[0] for _, _, cf, _ in levels]
        recs = graph_ref.decode([(b[0], c[0], st) for b, c, st in heads], g.nc, 0.25)
        keep = graph_ref.nms(recs, 0.7, 300)
        for i in range(min(len(keep), 40)):
            a = int(keep[i, 6])
            li = int(np.searchsorted(bases, a, side="right") - 1)
            y, x = divmod(a - bases[li], Ws[li])
            ref = graph_ref.mask(coefs[li][y, x], proto, keep[i], g.S)
            assert np.array_equal(eng.get_mask(0, i), ref), i


def test_detections_close_to_fp32_forward(lib, cuda):
    """Compounded-path fidelity: fused fp16 engine vs the fp32 oracle forward on the same
    input; most fp32 survivors must have a same-class engine box with IoU > 0.8."""
    from yolo11_cu_b200 import runtime as rt
    d = _model_dir("yolo11n")
    g = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    bufs, _ = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=False)
    heads = [(graph_ref.tensor_hwc(g, bufs, b_).astype(np.float16),
              graph_ref.tensor_hwc(g, bufs, c_).astype(np.float16), st) for b_, c_, _, st in g.levels()]
    keep = graph_ref.nms(graph_ref.decode(heads, g.nc), 0.45, 300)
    eng = rt.Engine(d, 1)
    eng.write(0, x)
    eng.run(1)
    dets = np.array(eng.get(0), np.float32)   # slot geometry untouched: scale 1, no offset
    assert abs(len(dets) - len(keep)) <= max(3, 0.1 * len(keep))
    hit = 0
    for k in keep:
        same = dets[dets[:, 5] == k[5]]
        if len(same) == 0:
            continue
        ix1 = np.maximum(same[:, 0], k[0]); iy1 = np.maximum(same[:, 1], k[1])
        ix2 = np.minimum(same[:, 2], k[2]); iy2 = np.minimum(same[:, 3], k[3])
        inter = np.clip(ix2 - ix1, 0, None) * np.clip(iy2 - iy1, 0, None)
        ua = (same[:, 2] - same[:, 0]) * (same[:, 3] - same[:, 1]) + (k[2] - k[0]) * (k[3] - k[1]) - inter
        hit += (inter / ua).max() > 0.8
    assert hit >= 0.9 * len(keep)


def test_multistream_graph_matches(lib, cuda, pkg):
    """The forward captured over several streams (the op dependency DAG) must give the same
    bits as the single-stream graph: YK_STREAMS=force makes the engine keep it."""
    from yolo11_cu_b200 import frames, runtime as rt
    d = _model_dir("yolo11n")
    bgr = frames.synthetic_bgr(1080, 810, seed=0)
    dev = torch.from_numpy(bgr).to(cuda)
    torch.cuda.synchronize()
    res = {}
    for mode in ("force", None):
        if mode:
            os.environ["YK_STREAMS"] = mode
        try:
            eng = rt.Engine(d, 2, iou=0.7, autotune=False)   # same kernels in both runs
            for s in range(2):
                eng.preprocess(dev.data_ptr(), 1080, 810, s)
            eng.run(2)
            eng._check()
            res[mode] = ([eng.get(s) for s in range(2)],
                         [eng.read(t, 2) for t in (g_ for lv in graph_ref.Graph(d).levels() for g_ in lv[:2])])
            eng.close()
        finally:
            os.environ.pop("YK_STREAMS", None)
    dets_f, heads_f = res["force"]
    dets_s, heads_s = res[None]
    assert dets_f == dets_s and len(dets_f[0]) > 0
    for a, b in zip(heads_f, heads_s):
        assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_seg_masks_close_to_fp32_forward(lib, cuda, capsys):
    """Per-instance mask IoU of the fused fp16 engine against the fp32 oracle forward of the
    same input (yolo11n-seg 640): each fp32 survivor (first 40) is matched to the engine's
    same-class box of highest IoU (> 0.9) and the two 160x160 masks compared.  Measured on a
    B200: 30 of 30 matched, median 0.9992, minimum 0.991, 93 % at >= 0.995; the gate keeps
    margin for autotuned kernel choices: median >= 0.995 and >= 80 % of instances at >= 0.995."""
    from yolo11_cu_b200 import runtime as rt
    d = _model_dir("yolo11n-seg")
    g = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(d, "input.f16"), np.float16).reshape(g.S, g.S, 3)
    bufs, _ = graph_ref.run_graph(g, x.astype(np.float32), round_fp16=False)
    levels = g.levels()
    heads = [(graph_ref.tensor_hwc(g, bufs, b_).astype(np.float16),
              graph_ref.tensor_hwc(g, bufs, c_).astype(np.float16), st) for b_, c_, _, st in levels]
    coefs = [graph_ref.tensor_hwc(g, bufs, cf).astype(np.float16) for _, _, cf, _ in levels]
    proto = graph_ref.tensor_hwc(g, bufs, g.proto()).astype(np.float16)
    keep = graph_ref.nms(graph_ref.decode(heads, g.nc), 0.45, 300)
    Ws = [h[0].shape[1] for h in heads]
    bases = np.cumsum([0] + [w * w for w in Ws])
    eng = rt.Engine(d, 1)
    eng.write(0, x)
    eng.run(1)
    dets = np.array(eng.get(0), np.float32)
    ious = []
    for k in keep[:40]:
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
        got = eng.get_mask(0, int(same[j])).astype(bool)
        union = (ref | got).sum()
        ious.append(1.0 if union == 0 else (ref & got).sum() / union)
    ious = np.array(ious)
    with capsys.disabled():
        print(f"\nseg mask IoU vs fp32: {len(ious)} matched of {min(40, len(keep))}, "
              f"median {np.median(ious):.4f}, min {ious.min():.4f}, >= 0.995: {(ious >= 0.995).mean():.2f}")
    assert len(ious) >= 0.8 * min(40, len(keep))
    assert np.median(ious) >= 0.995
    assert (ious >= 0.995).mean() >= 0.8
