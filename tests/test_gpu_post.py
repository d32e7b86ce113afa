"""GPU pre/post-processing vs the C oracle (oracle/postproc_ref.c): bit-exact.

Given identical fp16 head tensors, the engine's decode + NMS must return the same survivors
(same anchor indices, same order, identical box / score bits) as the oracle's restatement of
the reference's k_decode / k_nms (engine/engine.cu:848-906, 1051-1123); letterbox and masks
must match byte for byte.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import graph_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hw,S", [((1080, 810), 640), ((720, 1280), 640), ((1080, 1920), 1024),
                                  ((37, 53), 64), ((640, 640), 640)])
def test_letterbox_bitexact(lib, cuda, pkg, hw, S):
    from yolo11_cu_b200 import frames, runtime as rt
    bgr = frames.synthetic_bgr(*hw, seed=3)
    d = torch.from_numpy(bgr).to(cuda)
    out = torch.zeros(2, S, S, 3, dtype=torch.half, device=cuda)
    sc, top, left = C.c_float(), C.c_int(), C.c_int()
    r = lib.yk_letterbox(C.c_void_p(d.data_ptr()), hw[0], hw[1], C.byref(rt.tview(out)), 1,
                         C.byref(sc), C.byref(top), C.byref(left),
                         torch.cuda.current_stream().cuda_stream)
    assert r == 0
    torch.cuda.synchronize()
    ref = graph_ref.letterbox(bgr, S)
    assert np.array_equal(out[1].cpu().numpy().view(np.uint16), ref.view(np.uint16))
    assert torch.all(out[0] == 0)


@pytest.mark.parametrize("hw,S,n,stride,off", [((720, 1280), 640, 5, 3, 0),
                                               ((1080, 1920), 1024, 3, 3, 0),
                                               ((1080, 810), 640, 2, 3, 0),
                                               ((333, 517), 640, 3, 3, 5),
                                               ((60, 100), 640, 2, 3, 0),
                                               ((720, 1280), 640, 2, 8, 0),
                                               ((1, 1), 64, 1, 3, 0), ((2, 3), 64, 2, 3, 9),
                                               ((5, 7), 640, 3, 3, 1)])
def test_letterbox_batch_bitexact(lib, cuda, pkg, hw, S, n, stride, off):
    """One launch over n equal-size frames into slots 1..n: every slot equals the oracle's
    letterbox of its own frame, the untouched slot stays zero.  stride 8 writes channels 0..2
    of an 8-channel buffer; off > 0 starts the frames off any 16-byte boundary with `off`
    bytes between them (rows then straddle the kernel's 16-byte staging words)."""
    from yolo11_cu_b200 import frames, runtime as rt
    bgrs = [frames.synthetic_bgr(*hw, seed=10 + i) for i in range(n)]
    fb = hw[0] * hw[1] * 3
    flat = np.zeros(off + n * (fb + off), np.uint8)
    for i, b in enumerate(bgrs):
        flat[off + i * (fb + off):off + i * (fb + off) + fb] = b.ravel()
    d = torch.from_numpy(flat).to(cuda)
    out = torch.zeros(n + 1, S, S, stride, dtype=torch.half, device=cuda)
    sc, top, left = C.c_float(), C.c_int(), C.c_int()
    v = rt.tview(out, 0, 3)
    r = lib.yk_letterbox_batch(C.c_void_p(d.data_ptr() + off), fb + off, n, hw[0], hw[1],
                               C.byref(v), 1, C.byref(sc), C.byref(top), C.byref(left),
                               torch.cuda.current_stream().cuda_stream)
    assert r == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in range(n):
        ref = graph_ref.letterbox(bgrs[i], S)
        assert np.array_equal(got[i + 1, :, :, :3].view(np.uint16), ref.view(np.uint16)), i
    assert not got[0].any()
    if stride > 3:
        assert not got[:, :, :, 3:].any()
    # geometry: the reference's host formula
    s_ = min(np.float32(S) / np.float32(hw[0]), np.float32(S) / np.float32(hw[1]))
    assert sc.value == np.float32(s_)
    # slot range past the view's batch is rejected without a launch
    assert lib.yk_letterbox_batch(C.c_void_p(d.data_ptr() + off), fb + off, n, hw[0], hw[1],
                                  C.byref(v), 2, None, None, None,
                                  torch.cuda.current_stream().cuda_stream) == -1


def _levels(S, B, g, cls_bias, box_scale=1.0, nc=80):
    sizes = [(S // 8, 8), (S // 16, 16), (S // 32, 32)]
    box = [(torch.randn(B, n, n, 64, generator=g) * box_scale).half() for n, _ in sizes]
    cls = [(torch.randn(B, n, n, nc, generator=g) + cls_bias).half() for n, _ in sizes]
    return sizes, box, cls


def _run_gpu_post(lib, rt, cuda, sizes, box, cls, B, iou, max_out, coef=None, proto=None, S=None,
                  nc=80):
    A = sum(n * n for n, _ in sizes)
    dev = [(b.to(cuda), c.to(cuda)) for b, c in zip(box, cls)]
    lv = (rt.YkLevel * 3)()
    keep = []
    for i, ((n, st), (b, c)) in enumerate(zip(sizes, dev)):
        lv[i].box = rt.tview(b)
        lv[i].cls = rt.tview(c)
        if coef is not None:
            cf = coef[i].to(cuda)
            keep.append(cf)
            lv[i].coef = rt.tview(cf)
        lv[i].stride = st
    wsb = lib.yk_post_workspace_bytes(B, A)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
    od = torch.zeros(B, max_out, 6, device=cuda)
    oi = torch.zeros(B, max_out, dtype=torch.int32, device=cuda)
    oc = torch.zeros(B, dtype=torch.int32, device=cuda)
    rc = torch.zeros(B, dtype=torch.int32, device=cuda)
    post = rt.YkPost(ws.data_ptr(), wsb, od.data_ptr(), oi.data_ptr(), oc.data_ptr(), rc.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_decode(lv, 3, B, nc, 0.25, C.byref(post), st) == 0
    assert lib.yk_nms(B, A, iou, max_out, C.byref(post), st) == 0
    masks = None
    if coef is not None:
        pr = proto.to(cuda)
        masks = torch.full((B, max_out, pr.shape[1], pr.shape[2]), 9, dtype=torch.uint8, device=cuda)
        assert lib.yk_masks(lv, 3, C.byref(rt.tview(pr)), S, S, max_out, C.byref(post),
                            C.c_void_p(masks.data_ptr()), st) == 0
    torch.cuda.synchronize()
    assert lib.yk_fetch_device_error() == 0
    return od.cpu().numpy(), oi.cpu().numpy(), oc.cpu().numpy(), rc.cpu().numpy(), \
        (masks.cpu().numpy() if masks is not None else None)


def _oracle(sizes, box, cls, img, iou, max_out, nc=80):
    lv = [(b[img].numpy(), c[img].numpy(), st) for (n, st), b, c in zip(sizes, box, cls)]
    recs = graph_ref.decode(lv, nc, 0.25)
    return recs, graph_ref.nms(recs, iou, max_out)


@pytest.mark.parametrize("S,B,cls_bias,iou,max_out", [
    (640, 2, -5.0, 0.45, 300),     # tens of candidates: rank sort
    (640, 2, -4.0, 0.45, 300),     # about a thousand candidates: radix sort in shared memory
    (640, 1, -4.0, 0.7, 300),
    (320, 3, -20.0, 0.45, 300),    # no candidates
    (320, 1, 6.0, 0.45, 300),      # every anchor is a candidate
    (640, 1, 6.0, 0.45, 50),       # max_out truncation
    (640, 1, 6.0, 0.7, 300),       # 8400 candidates: candidate arrays in the workspace
    (1024, 1, 6.0, 0.45, 300),     # 21504 candidates: candidate arrays in the workspace
])
def test_decode_nms_bitexact(lib, cuda, S, B, cls_bias, iou, max_out):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(S + B)
    sizes, box, cls = _levels(S, B, g, cls_bias)
    od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, B, iou, max_out)
    for img in range(B):
        recs, keep = _oracle(sizes, box, cls, img, iou, max_out)
        assert rc[img] == len(recs)
        assert oc[img] == len(keep)
        n = len(keep)
        assert np.array_equal(oi[img, :n], keep[:, 6].astype(np.int32))
        assert np.array_equal(od[img, :n].view(np.uint32), keep[:, :6].view(np.uint32))


@pytest.mark.parametrize("nc,bias,iou", [(1, -2.9, 0.7), (2, -2.3, 0.7), (4, -2.0, 0.45),
                                          (8, -1.2, 0.7), (3, -2.9, 0.3)])
def test_nms_few_classes_bitexact(lib, cuda, nc, bias, iou):
    """Few classes of tens to hundreds of candidates each: the greedy path (classes up to
    128) and the bit-mask path (129..512, masks in shared memory below 512 candidates and
    in the workspace above) must both give the oracle's survivors bit for bit."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(100 + nc)
    sizes, box, cls = _levels(640, 1, g, bias, nc=8)   # 8 channels (16-byte rows), nc used
    od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, 1, iou, 300, nc=nc)
    recs, keep = _oracle(sizes, box, cls, 0, iou, 300, nc=nc)
    assert rc[0] == len(recs) > 0
    assert oc[0] == len(keep)
    n = len(keep)
    assert np.array_equal(oi[0, :n], keep[:, 6].astype(np.int32))
    assert np.array_equal(od[0, :n].view(np.uint32), keep[:, :6].view(np.uint32))


@pytest.mark.parametrize("S,nc,bias", [(320, 600, 1.0), (640, 304, -1.0)])
def test_decode_nms_many_classes(lib, cuda, S, nc, bias):
    """More than 256 classes: the class order takes two radix digits."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(S + nc)
    sizes, box, cls = _levels(S, 1, g, bias, nc=nc)
    od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, 1, 0.45, 300, nc=nc)
    recs, keep = _oracle(sizes, box, cls, 0, 0.45, 300, nc=nc)
    assert rc[0] == len(recs) and oc[0] == len(keep)
    assert np.array_equal(oi[0, :oc[0]], keep[:, 6].astype(np.int32))
    assert np.array_equal(od[0, :oc[0]].view(np.uint32), keep[:, :6].view(np.uint32))


def test_decode_nms_one_class(lib, cuda):
    """Every candidate in one class: one long class segment and many kept boxes (the
    kept list spills past the shared-memory cache into the workspace)."""
    from yolo11_cu_b200 import runtime as rt
    S = 320
    g = torch.Generator().manual_seed(77)
    sizes, box, cls = _levels(S, 1, g, -12.0, box_scale=0.5)
    for c in cls:
        c[..., 5] = (torch.randn(c.shape[:-1], generator=g) + 2.0).half()
    od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, 1, 0.45, 300)
    recs, keep = _oracle(sizes, box, cls, 0, 0.45, 300)
    assert rc[0] == len(recs) > 1000
    assert oc[0] == len(keep) > 32
    assert np.array_equal(oi[0, :oc[0]], keep[:, 6].astype(np.int32))
    assert np.array_equal(od[0, :oc[0]].view(np.uint32), keep[:, :6].view(np.uint32))


def test_nms_ties_deterministic(lib, cuda):
    """Identical logits everywhere: every score ties; order must be by anchor index."""
    from yolo11_cu_b200 import runtime as rt
    S, B = 320, 2
    sizes = [(S // 8, 8), (S // 16, 16), (S // 32, 32)]
    box = [torch.zeros(B, n, n, 64).half() for n, _ in sizes]
    cls = [torch.full((B, n, n, 80), 1.0).half() for n, _ in sizes]
    od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, B, 0.45, 300)
    recs, keep = _oracle(sizes, box, cls, 0, 0.45, 300)
    assert oc[0] == oc[1] == len(keep)
    assert np.array_equal(oi[0, :oc[0]], keep[:, 6].astype(np.int32))
    assert np.array_equal(oi[0], oi[1])


def test_masks_bitexact(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    S, B = 320, 2
    g = torch.Generator().manual_seed(9)
    sizes, box, cls = _levels(S, B, g, -3.0)
    coef = [torch.randn(B, n, n, 32, generator=g).half() for n, _ in sizes]
    proto = torch.randn(B, S // 4, S // 4, 32, generator=g).half()
    od, oi, oc, rc, masks = _run_gpu_post(lib, rt, cuda, sizes, box, cls, B, 0.45, 300, coef, proto, S)
    Ws = [n for n, _ in sizes]
    bases = np.cumsum([0] + [n * n for n in Ws])
    for img in range(B):
        assert oc[img] > 0
        for d in range(oc[img]):
            a = oi[img, d]
            li = int(np.searchsorted(bases, a, side="right") - 1)
            y, x = divmod(a - bases[li], Ws[li])
            ref = graph_ref.mask(coef[li][img, y, x].numpy(), proto[img].numpy(), od[img, d], S)
            assert np.array_equal(masks[img, d], ref), (img, d)


@pytest.mark.parametrize("csize", [1, 2, 4, 8])
def test_nms_cluster_sizes_bitexact(lib, cuda, csize):
    """The NMS launch spreads an image over a cluster of 1-8 CTAs (redundant sort in each
    CTA with the candidates in shared memory, CTA 0 alone with them in the workspace; mask
    rows and classes shared out).  Every size must give the oracle's survivors bit for bit:
    one class with bit-mask rows in shared memory, few classes with rows in the workspace,
    80 classes, and 8400 candidates in the workspace, over batches of 1 and 3."""
    from yolo11_cu_b200 import runtime as rt
    cases = [(1, -2.9, 0.7, 1, 8), (4, -2.0, 0.45, 1, 8), (80, -4.0, 0.45, 3, 80),
             (80, -3.0, 0.7, 1, 80), (80, 6.0, 0.45, 1, 80)]
    assert lib.yk_test_nms_cluster(csize) == 0
    try:
        for nc, bias, iou, B, ch in cases:
            g = torch.Generator().manual_seed(500 + nc + B)
            sizes, box, cls = _levels(640, B, g, bias, nc=ch)
            od, oi, oc, rc, _ = _run_gpu_post(lib, rt, cuda, sizes, box, cls, B, iou, 300, nc=nc)
            for img in range(B):
                recs, keep = _oracle(sizes, box, cls, img, iou, 300, nc=nc)
                assert rc[img] == len(recs) > 0, (nc, bias, img)
                assert oc[img] == len(keep), (nc, bias, img)
                n = len(keep)
                assert np.array_equal(oi[img, :n], keep[:, 6].astype(np.int32)), (nc, bias, img)
                assert np.array_equal(od[img, :n].view(np.uint32), keep[:, :6].view(np.uint32))
    finally:
        lib.yk_test_nms_cluster(0)
    assert lib.yk_test_nms_cluster(3) == -1
