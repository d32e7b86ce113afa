"""Device-side failure path without a GPU fault: every mbarrier wait of the tensor-core
kernels is bounded; when one runs out the CTA sets the device error word, raises its abort
flag, every role unwinds and TMEM is freed, so the context stays usable.

The test shortens the wait budget to 1 ms and makes block 0 of a conv withhold its first
stage load (yk_test_inject: no expect-tx and no copy are issued for that stage, so no
transaction is mis-sized).  The MMA warp's wait on that stage runs out.  Checks: the launch
returns, yk_fetch_device_error reports a bounded-wait code, and a following normal launch
of the same conv is clean and correct.  No trap, no device assert, no endless loop.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu
WAIT_CODES = {0x101, 0x102, 0x103, 0x104}   # producer / MMA / epilogue / accumulator waits


def test_bounded_wait_gives_up_and_context_survives(lib, cuda, pkg):
    from yolo11_cu_b200 import runtime as rt
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(11)
    B, H, W, Cin, Cout = 2, 32, 32, 64, 64
    x = torch.randn(B, H, W, Cin, generator=g).half().to(cuda)
    w = (torch.randn(Cout, 1, 1, Cin, generator=g) / Cin ** 0.5).half().to(cuda)   # OHWI
    b = (torch.randn(Cout, generator=g) * 0.1).float().to(cuda)
    y = torch.zeros(B, H, W, Cout, dtype=torch.half, device=cuda)
    prm = rt.YkConv(w.data_ptr(), b.data_ptr(), 1, 1, 0, 1, 1, Cin, Cout, 64, 1, 1)
    xv, yv = rt.tview(x), rt.tview(y)
    st = torch.cuda.current_stream().cuda_stream
    ref = F.silu(F.conv2d(x.permute(0, 3, 1, 2).float(), w.permute(0, 3, 1, 2).float(), b))
    ref = ref.permute(0, 2, 3, 1)

    def conv():
        r = lib.yk_conv(C.byref(xv), C.byref(yv), None, C.byref(prm), st)
        torch.cuda.synchronize()
        return r

    assert conv() == 0 and lib.yk_fetch_device_error() == 0
    assert (y.float() - ref).abs().max() / ref.abs().max() < 1.5e-2
    y.zero_()
    try:
        assert lib.yk_test_inject(1, 1_000_000) == 0          # withhold one stage, 1 ms budget
        assert conv() == 0                                      # the kernel returns
        code = lib.yk_fetch_device_error()
        assert code in WAIT_CODES, hex(code)
        assert lib.yk_fetch_device_error() == 0                 # fetching clears the word
    finally:
        assert lib.yk_test_inject(0, 0) == 0
    # the context is intact: the same conv runs clean and correct, and so does torch
    y.zero_()
    assert conv() == 0 and lib.yk_fetch_device_error() == 0
    assert (y.float() - ref).abs().max() / ref.abs().max() < 1.5e-2
    assert torch.cuda.is_available() and float(torch.ones(4, device=cuda).sum()) == 4.0
