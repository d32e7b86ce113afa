"""GPU parity of the yk_* kernels (called through the C ABI) against plain torch fp32.

Tolerance (north_star: per-op deviation <= 1.5 % vs fp32): max|gpu - ref| / max|ref| < 1.5e-2
with fp16 inputs shared by both sides; the fp16 output rounding alone is ~5e-4.
"""
import ctypes as C

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
TOL = 1.5e-2


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / (b.abs().max() + 1e-6)).item()


def nhwc(t):
    return t.permute(0, 2, 3, 1)


def vw(rt, buf, coff, Cv):
    B, H, W, Ct = buf.shape
    return rt.view(buf.data_ptr(), B, H, W, Ct, coff, Cv)


def run_conv(lib, rt, x, w, b, k, s, p, act, groups=1, res=None, tile=0, msub=0, xc=(0, None),
             yc=(0, 0), algo=0):
    """x: NHWC fp16 buffer (view = channels xc[0]:xc[0]+Cin); output written into a fresh
    buffer with yc = (coff, extra channels) to exercise channel-slice stores."""
    B, H, W, _ = x.shape
    Cout = w.shape[0]
    Cin = w.shape[1] * groups
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    ybuf = torch.full((B, Ho, Wo, yc[0] + Cout + yc[1]), 7.0, dtype=torch.half, device=x.device)
    wt = w.permute(0, 2, 3, 1).contiguous().half()            # OHWI
    bt = b.float().contiguous()
    prm = rt.YkConv(wt.data_ptr(), bt.data_ptr(), k, s, p, groups, act, Cin, Cout, tile, msub,
                    algo)
    xv = vw(rt, x, xc[0], Cin)
    yv = vw(rt, ybuf, yc[0], Cout)
    rv = vw(rt, res, 0, Cout) if res is not None else None
    r = lib.yk_conv(C.byref(xv), C.byref(yv), C.byref(rv) if rv is not None else None,
                    C.byref(prm), torch.cuda.current_stream().cuda_stream)
    assert r == 0, (r, lib.yk_last_cuda_error())
    torch.cuda.synchronize()
    assert lib.yk_fetch_device_error() == 0
    xin = x[..., xc[0]:xc[0] + Cin].permute(0, 3, 1, 2).float()
    ref = F.conv2d(xin, wt.permute(0, 3, 1, 2).float(), bt, stride=s, padding=p, groups=groups)
    if act:
        ref = F.silu(ref)
    ref = nhwc(ref)
    if res is not None:
        ref = ref + res.float()
    out = ybuf[..., yc[0]:yc[0] + Cout]
    if yc[0]:
        assert torch.all(ybuf[..., :yc[0]] == 7.0)
    if yc[1]:
        assert torch.all(ybuf[..., yc[0] + Cout:] == 7.0)
    return out, ref


CONV_CASES = [
    # B, H, W, Cin, Cout, k, s, p
    (1, 20, 20, 64, 64, 1, 1, 0),
    (2, 40, 40, 32, 48, 3, 1, 1),
    (1, 33, 17, 8, 16, 3, 1, 1),       # thin channels, ragged M
    (1, 32, 32, 16, 8, 3, 1, 1),       # Cout 8 (padded N tile)
    (3, 40, 40, 64, 128, 3, 2, 1),     # stride 2
    (1, 20, 20, 256, 256, 1, 1, 0),
    (2, 10, 10, 512, 512, 3, 1, 1),    # deep K (4608)
    (1, 80, 80, 96, 200, 1, 1, 0),     # Cout not a tile multiple
    (1, 5, 7, 24, 40, 3, 2, 1),
    (1, 1, 1, 64, 80, 1, 1, 0),        # M = 1 (linear)
    (2, 12, 12, 96, 64, 3, 1, 1),      # im2col TMA, Cin not a multiple of 64
    (3, 13, 9, 64, 64, 3, 2, 1),       # im2col TMA, stride 2, odd sizes, tiles across images
    (2, 7, 7, 128, 32, 3, 1, 1),
    (2, 20, 20, 32, 64, 1, 1, 0),      # narrow-block TMA, 1x1
    (2, 21, 19, 16, 32, 3, 2, 1),      # narrow-block TMA im2col, stride 2
    (3, 16, 16, 32, 32, 3, 1, 1),
    (2, 32, 24, 8, 16, 3, 2, 1),       # 8-channel blocks (unswizzled TMA im2col)
    (1, 15, 15, 8, 64, 3, 1, 1),
]


@pytest.mark.parametrize("case", CONV_CASES)
@pytest.mark.parametrize("tile,msub", [(0, 0), (32, 4), (64, 1), (64, 2), (64, 4), (128, 1),
                                       (128, 2), (256, 1)])
def test_conv_tc(lib, cuda, case, tile, msub):
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout, k, s, p = case
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, k, k, generator=g) / (Cin * k * k) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), k, s, p, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8))
    assert rel(out, ref) < TOL


PATCH_CASES = [
    # B, H, W, Cin, Cout
    (1, 20, 20, 64, 64),
    (2, 40, 40, 128, 128),
    (1, 13, 29, 64, 96),       # ragged patch rows and columns, Cout not a tile multiple
    (2, 80, 80, 64, 64),
    (1, 9, 9, 256, 128),       # several 64-channel blocks
    (3, 7, 7, 512, 64),        # small images: one patch per image, 8 channel blocks
]


@pytest.mark.parametrize("case", PATCH_CASES + [(2, 40, 40, 32, 32), (1, 19, 23, 96, 64),
                                                (1, 33, 30, 32, 48)])
@pytest.mark.parametrize("tile,msub", [(32, 1), (32, 2), (64, 1), (64, 2), (128, 1), (128, 2),
                                       (256, 1)])
def test_conv_patch(lib, cuda, case, tile, msub):
    """3x3 stride-1 convs on halo patches (algo 2), channel-slice input and output views."""
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout = case
    if tile // 2 >= Cout or (tile == 32 and Cout > 64) or (Cin % 64 and tile > 64):
        pytest.skip("tile more than twice Cout, or no such configuration")
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) / (Cin * 9) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), 3, 1, 1, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8), algo=2)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("case", [c for c in CONV_CASES if c[3] >= 64])
@pytest.mark.parametrize("tile,msub", [(128, 1), (128, 2), (128, 4), (256, 2)])
def test_conv_transposed(lib, cuda, case, tile, msub):
    """Transposed tiles (algo 3): output channels on the MMA's M side, pixels on N."""
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout, k, s, p = case
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000 + 7)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, k, k, generator=g) / (Cin * k * k) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), k, s, p, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8), algo=3)
    assert rel(out, ref) < TOL


def test_conv_transposed_residual(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2, 30, 30, 128, generator=g).half().to(cuda)
    w = (torch.randn(192, 128, 3, 3, generator=g) / 34).to(cuda)
    b = (torch.randn(192, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 30, 30, 192, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, res=res, msub=2, algo=3)
    assert rel(out, ref) < TOL


PAIR_CASES = [c for c in CONV_CASES if c[3] >= 64] + [
    (2, 40, 40, 128, 512, 1, 1, 0),
    (1, 30, 30, 256, 384, 3, 2, 1),    # stride 2, Cout not a multiple of 256
    (3, 17, 13, 64, 256, 3, 1, 1),     # ragged pixel tiles across images
    (1, 9, 7, 512, 768, 1, 1, 0),      # fewer pixels than one pair tile
]


@pytest.mark.parametrize("case", PAIR_CASES)
def test_conv_pair(lib, cuda, case):
    """CTA pairs (algo 6): one M = 256 MMA over two SMs (cta_group::2)."""
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout, k, s, p = case
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000 + 17)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, k, k, generator=g) / (Cin * k * k) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), k, s, p, act=1, xc=(8, None),
                        yc=(8, 8), algo=6)
    assert rel(out, ref) < TOL


def test_conv_pair_residual(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(16)
    x = torch.randn(2, 30, 30, 256, generator=g).half().to(cuda)
    w = (torch.randn(256, 256, 1, 1, generator=g) / 16).to(cuda)
    b = (torch.randn(256, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 30, 30, 256, generator=g).half().to(cuda)
    for _ in range(2):   # repeated launches reuse the cached occupancy / attributes
        out, ref = run_conv(lib, rt, x, w, b, 1, 1, 0, act=1, res=res, algo=6)
        assert rel(out, ref) < TOL


@pytest.mark.parametrize("case", PATCH_CASES + [(2, 40, 40, 32, 32), (1, 19, 23, 96, 64),
                                                (1, 160, 160, 32, 32)])
@pytest.mark.parametrize("tile,msub", [(64, 1), (64, 2), (128, 1), (128, 2)])
def test_conv_patch_transposed(lib, cuda, case, tile, msub):
    """Halo patches with transposed tiles (algo 4): 64 (M = 64 MMA) or 128 output channels."""
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout = case
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000 + 11)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) / (Cin * 9) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), 3, 1, 1, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8), algo=4)
    assert rel(out, ref) < TOL


def test_conv_patch_transposed_residual(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(8)
    x = torch.randn(2, 30, 30, 64, generator=g).half().to(cuda)
    w = (torch.randn(64, 64, 3, 3, generator=g) / 24).to(cuda)
    b = (torch.randn(64, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 30, 30, 64, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, res=res, tile=64, msub=2, algo=4)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("case", PATCH_CASES + [(2, 40, 40, 32, 32), (1, 19, 23, 96, 64),
                                                (1, 160, 160, 32, 32), (1, 33, 30, 32, 48),
                                                (2, 64, 64, 48, 48), (1, 37, 29, 16, 32),
                                                (1, 21, 50, 80, 48), (2, 40, 33, 8, 16),
                                                (2, 40, 40, 128, 128), (4, 64, 64, 128, 128),
                                                (1, 20, 20, 64, 192)])
@pytest.mark.parametrize("tile,msub", [(32, 1), (32, 2), (64, 1)])
def test_conv_kx_folded(lib, cuda, case, tile, msub):
    """Halo patches with the horizontal taps folded into N (algo 5); Cin 48 / 16 / 80 take
    16-channel blocks, Cin 8 one zero-filled 16-channel block; filters of one or two
    channel blocks stay in shared memory, also with several output-channel tiles (each CTA
    keeps one: 128 -> 128 over 2 or 4 tiles, 64 -> 192 over 3 or 6, more tiles than SMs)."""
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin, Cout = case
    g = torch.Generator(device="cpu").manual_seed(hash(case) % 1000 + 13)
    x = torch.randn(B, H, W, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, 3, 3, generator=g) / (Cin * 9) ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), 3, 1, 1, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8), algo=5)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("C", [48, 16])
def test_conv_kx_folded_16ch_residual(lib, cuda, C):
    """16-channel blocks with a fused residual, as yolo11x's 48-channel bottlenecks."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(C)
    x = torch.randn(2, 45, 70, C, generator=g).half().to(cuda)
    w = (torch.randn(C, C, 3, 3, generator=g) / (C * 9) ** 0.5).to(cuda)
    b = (torch.randn(C, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 45, 70, C, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, res=res, tile=64, msub=1, algo=5)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("C", [64, 128])
def test_conv_kx_folded_residual(lib, cuda, C):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 30, 30, C, generator=g).half().to(cuda)
    w = (torch.randn(C, C, 3, 3, generator=g) / (C * 9) ** 0.5).to(cuda)
    b = (torch.randn(C, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 30, 30, C, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, res=res, tile=64, msub=1, algo=5)
    assert rel(out, ref) < TOL


def test_conv_patch_residual(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 30, 30, 128, generator=g).half().to(cuda)
    w = (torch.randn(128, 128, 3, 3, generator=g) / 34).to(cuda)
    b = (torch.randn(128, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 30, 30, 128, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, res=res, tile=128, msub=2, algo=2)
    assert rel(out, ref) < TOL


def test_conv_tc_residual_and_inplace(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 24, 24, 64, generator=g).half().to(cuda)
    w = (torch.randn(64, 64, 3, 3, generator=g) / 24).to(cuda)
    b = (torch.randn(64, generator=g) * 0.1).to(cuda)
    res = torch.randn(2, 24, 24, 64, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=0, res=res)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("cout,k,s,hw", [(16, 3, 2, (64, 48)), (64, 3, 2, (64, 48)),
                                         (96, 3, 2, (64, 48)), (16, 3, 1, (64, 48)),
                                         (16, 1, 1, (64, 48)), (32, 3, 2, (90, 122)),
                                         (48, 3, 2, (33, 17)), (80, 3, 2, (160, 160)),
                                         (64, 3, 2, (640, 640))])
def test_conv_first_layer(lib, cuda, cout, k, s, hw):
    """The 3-channel first conv: the warp-MMA stem kernel (k = 3, Cout <= 96) and the direct
    small-Cin kernel (other k)."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(4)
    x = torch.rand(2, hw[0], hw[1], 3, generator=g).half().to(cuda)
    w = (torch.randn(cout, 3, k, k, generator=g) / 5).to(cuda)
    b = (torch.randn(cout, generator=g) * 0.1).to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, k, s, k // 2, act=1)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("s", [1, 2])
def test_dwconv(lib, cuda, s):
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(5)
    C_ = 64
    x = torch.randn(2, 20, 20, C_, generator=g).half().to(cuda)
    w = (torch.randn(C_, 1, 3, 3, generator=g) / 3).to(cuda)
    b = (torch.randn(C_, generator=g) * 0.1).to(cuda)
    res = None
    if s == 1:
        res = torch.randn(2, 20, 20, C_, generator=g).half().to(cuda)
    out, ref = run_conv(lib, rt, x, w, b, 3, s, 1, act=1, groups=C_, res=res)
    assert rel(out, ref) < TOL


@pytest.mark.parametrize("B,H,W,C_,res", [(1, 13, 21, 96, False), (2, 80, 80, 256, False),
                                          (1, 17, 9, 512, True), (3, 8, 16, 64, True),
                                          (1, 1, 1, 8, False)])
def test_dwconv_tiles(lib, cuda, B, H, W, C_, res):
    """3x3 stride-1 depthwise on shared-memory tiles: partial channel tiles, ragged edges,
    channel-slice input / output views, residual."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(H * W + C_)
    x = torch.randn(B, H, W, C_ + 16, generator=g).half().to(cuda)
    w = (torch.randn(C_, 1, 3, 3, generator=g) / 3).to(cuda)
    b = (torch.randn(C_, generator=g) * 0.1).to(cuda)
    r = torch.randn(B, H, W, C_, generator=g).half().to(cuda) if res else None
    out, ref = run_conv(lib, rt, x, w, b, 3, 1, 1, act=1, groups=C_, res=r, xc=(8, None),
                        yc=(8, 8))
    assert rel(out, ref) < TOL


def _v(rt, t, coff=0, Cv=None):
    return rt.tview(t, coff, Cv)


@pytest.mark.parametrize("shape", [(2, 20, 20, 32), (3, 20, 20, 256), (1, 13, 17, 128),
                                   (1, 32, 32, 96), (1, 100, 100, 64), (32, 20, 20, 256),
                                   (148, 20, 80, 32)])
def test_maxpool_chain(lib, cuda, shape):
    """SPPF chain: shared-memory planes (small images; a fixed column per thread when a plane
    row has at most 256 16-byte chunks, else the flat walk) or the direct windows (large)."""
    from yolo11_cu_b200 import runtime as rt
    x = torch.randn(*shape, device=cuda).half()
    ys = [torch.empty_like(x) for _ in range(3)]
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_maxpool5x3(C.byref(_v(rt, x)), *[C.byref(_v(rt, y)) for y in ys], st) == 0
    y1 = torch.empty_like(x)
    assert lib.yk_maxpool5(C.byref(_v(rt, x)), C.byref(_v(rt, y1)), st) == 0
    torch.cuda.synchronize()
    t = x.permute(0, 3, 1, 2).float()
    refs = []
    for _ in range(3):
        t = F.max_pool2d(t, 5, 1, 2)
        refs.append(nhwc(t).half())
    assert torch.equal(y1, refs[0])
    for y, r in zip(ys, refs):
        assert torch.equal(y, r)


def test_upsample_ps2_copy_add(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(2, 8, 10, 48, device=cuda).half()
    up = torch.zeros(2, 16, 20, 64, device=cuda).half()
    assert lib.yk_upsample2(C.byref(_v(rt, x, 8, 32)), C.byref(_v(rt, up, 16, 32)), st) == 0
    ps = torch.zeros(2, 16, 20, 8, device=cuda).half()
    assert lib.yk_ps2(C.byref(_v(rt, x, 8, 32)), C.byref(_v(rt, ps)), st) == 0
    cp = torch.zeros(2, 8, 10, 24, device=cuda).half()
    assert lib.yk_copyc(C.byref(_v(rt, x, 0, 24)), C.byref(_v(rt, cp)), st) == 0
    cps = torch.zeros(2, 8, 10, 5, device=cuda).half()
    assert lib.yk_copyc(C.byref(_v(rt, x, 3, 5)), C.byref(_v(rt, cps)), st) == 0
    ad = torch.zeros(2, 8, 10, 16, device=cuda).half()
    assert lib.yk_add(C.byref(_v(rt, x, 0, 16)), C.byref(_v(rt, x, 16, 16)), C.byref(_v(rt, ad)), st) == 0
    torch.cuda.synchronize()
    xs = x[..., 8:40]
    assert torch.equal(up[..., 16:48], xs.repeat_interleave(2, 1).repeat_interleave(2, 2))
    assert torch.all(up[..., :16] == 0) and torch.all(up[..., 48:] == 0)
    ref = torch.zeros_like(ps)
    for di in range(2):
        for dj in range(2):
            q = 2 * di + dj
            ref[:, di::2, dj::2] = xs[..., q * 8:(q + 1) * 8]
    assert torch.equal(ps, ref)
    assert torch.equal(cp, x[..., :24]) and torch.equal(cps, x[..., 3:8])
    assert torch.equal(ad, (x[..., :16].float() + x[..., 16:32].float()).half())


@pytest.mark.parametrize("hw,heads", [((20, 20), 2), ((20, 20), 4), ((32, 32), 6), ((7, 7), 2)])
def test_attention(lib, cuda, hw, heads):
    from yolo11_cu_b200 import runtime as rt
    H, W = hw
    kd, hd = 32, 64
    qkv = torch.randn(3, H, W, heads * (2 * kd + hd) + 8, device=cuda).half()
    y = torch.zeros(3, H, W, heads * hd, device=cuda).half()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_attn(C.byref(_v(rt, qkv, 8, heads * (2 * kd + hd))), C.byref(_v(rt, y)), heads, kd, hd, st) == 0
    torch.cuda.synchronize()
    N = H * W
    t = qkv[..., 8:].float().reshape(3, N, heads, 2 * kd + hd).permute(0, 2, 3, 1)
    q, k, v = t.split([kd, kd, hd], dim=2)
    att = ((q.transpose(-2, -1) @ k) * kd ** -0.5).softmax(-1)
    ref = (v @ att.transpose(-2, -1)).reshape(3, heads * hd, N).permute(0, 2, 1).reshape(3, H, W, heads * hd)
    assert rel(y, ref) < TOL


def test_bad_arguments_rejected(lib, cuda):
    from yolo11_cu_b200 import runtime as rt
    st = torch.cuda.current_stream().cuda_stream
    x = torch.randn(1, 8, 8, 16, device=cuda).half()
    y = torch.zeros(1, 8, 8, 16, device=cuda).half()
    bad = rt.tview(x, 4, 16)       # coff + C > stride
    assert lib.yk_copyc(C.byref(bad), C.byref(rt.tview(y)), st) != 0
    assert lib.yk_attn(C.byref(rt.tview(x)), C.byref(rt.tview(y)), 1, 4, 8, st) != 0


@pytest.mark.parametrize("k,s,p", [(3, 2, 1), (3, 1, 1), (1, 1, 0)])
def test_im2col_thin(lib, cuda, k, s, p):
    from yolo11_cu_b200 import runtime as rt
    B, H, W, Cin = 2, 17, 12, 3
    x = torch.randn(B, H, W, Cin, device=cuda).half()
    Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    kp = (k * k * Cin + 7) // 8 * 8
    col = torch.full((B, Ho, Wo, kp), 5.0, device=cuda).half()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.yk_im2col(C.byref(rt.tview(x)), C.byref(rt.tview(col)), k, s, p, st) == 0
    torch.cuda.synchronize()
    xp = F.pad(x.permute(0, 3, 1, 2).float(), (p, p, p, p))
    ref = torch.zeros(B, Ho, Wo, kp, device=cuda)
    for ky in range(k):
        for kx in range(k):
            patch = xp[:, :, ky:ky + s * (Ho - 1) + 1:s, kx:kx + s * (Wo - 1) + 1:s]
            ref[..., (ky * k + kx) * Cin:(ky * k + kx + 1) * Cin] = patch.permute(0, 2, 3, 1)
    assert torch.equal(col.float(), ref)


@pytest.mark.parametrize("Cin,Cout,tile,msub", [(48, 64, 64, 2), (48, 64, 32, 4), (24, 40, 32, 1),
                                               (40, 96, 128, 1), (48, 256, 256, 1)])
def test_conv_1x1_padded_channel_block(lib, cuda, Cin, Cout, tile, msub):
    """1x1 convs whose Cin is no 8/16/32-channel block: one wider block whose channels past
    Cin the tensor maps zero-fill (48 -> 64, 24 -> 32, 40 -> three 16-channel blocks)."""
    from yolo11_cu_b200 import runtime as rt
    g = torch.Generator().manual_seed(Cin * 7 + Cout)
    x = torch.randn(2, 37, 41, Cin + 16, generator=g).half().to(cuda)
    w = (torch.randn(Cout, Cin, 1, 1, generator=g) / Cin ** 0.5)
    b = torch.randn(Cout, generator=g) * 0.1
    out, ref = run_conv(lib, rt, x, w.to(cuda), b.to(cuda), 1, 1, 0, act=1, tile=tile,
                        msub=msub, xc=(8, None), yc=(8, 8), algo=1)
    assert rel(out, ref) < TOL
