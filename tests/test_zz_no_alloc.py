"""The allocation-free decode + NMS entry point (yk_decode_nms_static).

It exists for callers that cannot call cudaMalloc (fixed device-memory budgets, plugins
whose host framework owns every allocation, loops that must never enter the allocator):
its scratch is a static device array inside the library.  Checked here through the C ABI
against the regular entry points (yk_decode + yk_nms with a caller-owned workspace), bit for
bit, on two calls in a row with different inputs — the static array keeps the previous
call's contents, which must not leak into the next result.  This file is collected last so
a failure here leaves every other test already run; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _heads(S, B, seed, cls_bias):
    g = torch.Generator().manual_seed(seed)
    sizes = [(S // 8, 8), (S // 16, 16), (S // 32, 32)]
    box = [torch.randn(B, n, n, 64, generator=g).half() for n, _ in sizes]
    cls = [(torch.randn(B, n, n, 80, generator=g) + cls_bias).half() for n, _ in sizes]
    return sizes, box, cls


def _levels(rt, sizes, box, cls, cuda):
    dev = [(b.to(cuda), c.to(cuda)) for b, c in zip(box, cls)]
    lv = (rt.YkLevel * 3)()
    for i, ((n, st), (b, c)) in enumerate(zip(sizes, dev)):
        lv[i].box = rt.tview(b)
        lv[i].cls = rt.tview(c)
        lv[i].stride = st
    return lv, dev


def _outs(B, max_out, cuda):
    return (torch.zeros(B, max_out, 6, device=cuda), torch.zeros(B, max_out, dtype=torch.int32, device=cuda),
            torch.zeros(B, dtype=torch.int32, device=cuda), torch.zeros(B, dtype=torch.int32, device=cuda))


def _regular(lib, rt, lv, A, B, iou, max_out, cuda, st):
    wsb = lib.yk_post_workspace_bytes(B, A)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
    od, oi, oc, rc = _outs(B, max_out, cuda)
    post = rt.YkPost(ws.data_ptr(), wsb, od.data_ptr(), oi.data_ptr(), oc.data_ptr(), rc.data_ptr())
    assert lib.yk_decode(lv, 3, B, 80, 0.25, C.byref(post), st) == 0
    assert lib.yk_nms(B, A, iou, max_out, C.byref(post), st) == 0
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in (od, oi, oc, rc)]


def _static(lib, lv, B, iou, max_out, cuda, st):
    od, oi, oc, rc = _outs(B, max_out, cuda)
    r = lib.yk_decode_nms_static(lv, 3, B, 80, 0.25, iou, max_out, C.c_void_p(od.data_ptr()),
                                 C.c_void_p(oi.data_ptr()), C.c_void_p(oc.data_ptr()),
                                 C.c_void_p(rc.data_ptr()), st)
    assert r == 0, lib.yk_last_cuda_error()
    torch.cuda.synchronize()
    assert lib.yk_fetch_device_error() == 0
    return [t.cpu().numpy() for t in (od, oi, oc, rc)]


def test_static_decode_nms_matches_regular_twice(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    st = torch.cuda.current_stream().cuda_stream
    # call 1: many candidates; call 2: a different, sparser input on the same static scratch
    for seed, bias, B in [(1, 2.0, 4), (2, -4.0, 3)]:
        sizes, box, cls = _heads(640, B, seed, bias)
        A = sum(n * n for n, _ in sizes)
        lv, keep = _levels(rt, sizes, box, cls, cuda)
        ref = _regular(lib, rt, lv, A, B, 0.45, 300, cuda, st)
        got = _static(lib, lv, B, 0.45, 300, cuda, st)
        assert ref[2].sum() > 0
        for r, g in zip(ref, got):
            assert np.array_equal(r.view(np.uint32) if r.dtype == np.float32 else r,
                                  g.view(np.uint32) if g.dtype == np.float32 else g)


def test_static_rejects_oversize(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    st = torch.cuda.current_stream().cuda_stream
    sizes, box, cls = _heads(640, 32, 3, -4.0)      # 32 x 8400 anchors > 8 MiB of scratch
    lv, keep = _levels(rt, sizes, box, cls, cuda)
    od, oi, oc, rc = _outs(32, 300, cuda)
    r = lib.yk_decode_nms_static(lv, 3, 32, 80, 0.25, 0.45, 300, C.c_void_p(od.data_ptr()),
                                 C.c_void_p(oi.data_ptr()), C.c_void_p(oc.data_ptr()),
                                 C.c_void_p(rc.data_ptr()), st)
    assert r != 0
    assert b"static" in lib.yk_last_cuda_error()
