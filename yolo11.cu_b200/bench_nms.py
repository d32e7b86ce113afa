"""NMS micro-benchmark: yk_decode once, then yk_nms timed over back-to-back calls (CUDA
events on the stream) on seeded synthetic heads of one 640 image (8400 anchors): box logits
N(0, 1), class logits N(0, 1) + bias on the first k classes and -20 on the rest; conf 0.25,
IoU 0.7, max_out 300.

    python yolo11.cu_b200/bench_nms.py [path/to/libyolob200.so]
"""
import ctypes as C
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import runtime as rt  # noqa: E402

CASES = [(-2.9, 1), (-2.0, 1), (-2.9, 4), (-4.0, 80), (-3.0, 80), (0.0, 80)]   # (bias, k)


def main():
    lib = rt.load(sys.argv[1] if len(sys.argv) > 1 else rt.LIB_PATH)
    cuda = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream
    S, B = 640, 1
    sizes = [(S // 8, 8), (S // 16, 16), (S // 32, 32)]
    A = sum(n * n for n, _ in sizes)
    for bias, k in CASES:
        g = torch.Generator().manual_seed(0)
        box = [torch.randn(B, n, n, 64, generator=g).half().to(cuda) for n, _ in sizes]
        cls = []
        for n, _ in sizes:
            c = torch.full((B, n, n, 80), -20.0)
            c[..., :k] = torch.randn(B, n, n, k, generator=g) + bias
            cls.append(c.half().to(cuda))
        lv = (rt.YkLevel * 3)()
        for i, ((n, s), b, c) in enumerate(zip(sizes, box, cls)):
            lv[i].box, lv[i].cls, lv[i].stride = rt.tview(b), rt.tview(c), s
        wsb = lib.yk_post_workspace_bytes(B, A)
        ws = torch.zeros(wsb, dtype=torch.uint8, device=cuda)
        od = torch.zeros(B, 300, 6, device=cuda)
        oi = torch.zeros(B, 300, dtype=torch.int32, device=cuda)
        oc = torch.zeros(B, dtype=torch.int32, device=cuda)
        rc = torch.zeros(B, dtype=torch.int32, device=cuda)
        post = rt.YkPost(ws.data_ptr(), wsb, od.data_ptr(), oi.data_ptr(), oc.data_ptr(), rc.data_ptr())
        assert lib.yk_decode(lv, 3, B, 80, 0.25, C.byref(post), st) == 0
        for _ in range(3):
            lib.yk_nms(B, A, 0.7, 300, C.byref(post), st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(50):
            lib.yk_nms(B, A, 0.7, 300, C.byref(post), st)
        e1.record()
        torch.cuda.synchronize()
        print(f"bias {bias} classes {k}: candidates {rc.item()} kept {oc.item()} "
              f"nms {e0.elapsed_time(e1) / 50 * 1000:.1f} us", flush=True)


if __name__ == "__main__":
    main()
