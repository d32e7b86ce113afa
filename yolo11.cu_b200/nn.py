"""Seeded random-init YOLOv8 / YOLO11 networks (detect and segment) as torch fp32 modules.

The engine consumes a model directory (``model.graph`` + ``weights.f16`` + ``bias.f32``),
not a checkpoint.  No ``.pt`` files and no ``ultralytics`` package exist on these machines,
so this module builds the networks from their published architecture (the yolo11 / yolov8
yaml layer lists, width/depth scaling, module definitions) with seeded random weights and
BatchNorm already folded into every convolution.

Module classes carry the attribute names the reference exporter walks
(``export/export.py:86-441``: ``Conv.conv/.act``, ``C2f.cv1/.cv2/.m/.c``, ``C3k.cv1..cv3``,
``Bottleneck.cv1/.cv2/.add``, ``SPPF.cv1/.cv2``, ``C2PSA.cv1/.cv2/.m/.c``,
``PSABlock.attn/.ffn``, ``Attention.qkv/.pe/.proj/.num_heads/.key_dim/.head_dim``,
``Detect.cv2/.cv3/.dfl/.stride/.nc``, ``Segment.cv4/.proto/.nm``, ``layer.f``) so the same
objects drive both this package's exporter and, in tests, the reference exporter itself.

Weight recipe (identical on every machine: numpy PCG64 only, no torch RNG):
  * every Conv+BN weight ~ N(0, gain2/fan_in) (Kaiming-normal; fan_in = Cin/g*k*k; gain2 = 2
    except where ``KAIMING_GAIN2`` keeps a deep random net's activations O(1));
  * every Conv+BN pair is folded: gamma~U(0.5,1.5), beta~N(0,0.1), mean~N(0,0.1),
    var~U(0.5,1.5), eps=1e-3, w' = w*gamma/sqrt(var+eps), b' = beta - mean*gamma/sqrt(var+eps);
  * the bare head convs (box/cls/mask-coef finals, no BN) get weight ~ N(0, 1/fan_in), bias 0
    for box/coef and the per-model constant ``CLS_BIAS`` for cls;
  * ConvTranspose2d (segment proto upsample) weight ~ N(0, 1/Cin), bias ~ N(0, 0.1);
  * the DFL conv is fixed to arange(16).
"""
from __future__ import annotations

import math
import re

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["build_model", "MODEL_SCALES", "Conv", "DWConv", "Concat", "Bottleneck", "C2f",
           "C3", "C3k", "C3k2", "SPPF", "Attention", "PSABlock", "C2PSA", "DFL", "Proto",
           "Detect", "Segment", "OBB", "Classify", "DetectionModel", "CLS_BIAS"]

# Constant bias of the final cls convs, per model: chosen once (frame 0 at 640) so that about
# 3 % of the 8400 anchors pass conf 0.25, i.e. NMS sees a few hundred candidates per image.
CLS_BIAS = {"yolo11n": -3.75, "yolo11s": -6.25, "yolo11m": -6.25, "yolo11l": -2.25,
            "yolo11x": -2.0, "yolov8n": -18.25, "yolov8s": -6.75, "yolov8m": -2.0,
            "yolo11n-seg": -1.64, "yolo11m-seg": -8.5, "yolov8n-seg": -16.75,
            "yolo11n-obb": -4.5}   # obb: frame 0 at 1024, ~4 % of 21504 anchors
CLS_BIAS_DEFAULT = -3.0
# Squared Kaiming gain of the Conv+BN weights, per model: 2 (He) unless the random net's
# activations then grow or shrink geometrically with depth; chosen once so the deepest layer's
# std on frame 0 stays O(1) (fp16 storage needs |x| far below 65504).
KAIMING_GAIN2 = {"yolo11l": 1.4, "yolo11x": 1.4, "yolov8n": 2.4, "yolov8n-seg": 2.2,
                 "yolo11n-obb": 1.75}

# (depth, width, max_channels) per published scale
MODEL_SCALES = {
    "yolo11": {"n": (0.50, 0.25, 1024), "s": (0.50, 0.50, 1024), "m": (0.50, 1.00, 512),
               "l": (1.00, 1.00, 512), "x": (1.00, 1.50, 512)},
    "yolov8": {"n": (0.33, 0.25, 1024), "s": (0.33, 0.50, 1024), "m": (0.67, 0.75, 768),
               "l": (1.00, 1.00, 512), "x": (1.00, 1.25, 512)},
}


def _ceil8(x: float) -> int:
    return int(math.ceil(x / 8) * 8)


class Conv(nn.Module):
    """Conv2d(k, s, p=k//2, groups) with BN folded into its bias, then SiLU (or identity)."""

    def __init__(self, c1, c2, k=1, s=1, p=None, g=1, act=True):
        super().__init__()
        self.conv = nn.Conv2d(c1, c2, k, s, k // 2 if p is None else p, groups=g, bias=True)
        self.act = nn.SiLU() if act is True else nn.Identity()

    def forward(self, x):
        return self.act(self.conv(x))


class DWConv(Conv):
    """Depthwise Conv (groups = gcd(c1, c2))."""

    def __init__(self, c1, c2, k=1, s=1, act=True):
        super().__init__(c1, c2, k, s, g=math.gcd(c1, c2), act=act)


class Concat(nn.Module):
    def __init__(self, d=1):
        super().__init__()
        self.d = d

    def forward(self, x):
        return torch.cat(x, self.d)


class Bottleneck(nn.Module):
    def __init__(self, c1, c2, shortcut=True, g=1, k=(3, 3), e=0.5):
        super().__init__()
        c_ = int(c2 * e)
        k1, k2 = (kk if isinstance(kk, int) else kk[0] for kk in k)   # square kernels
        self.cv1 = Conv(c1, c_, k1, 1)
        self.cv2 = Conv(c_, c2, k2, 1, g=g)
        self.add = shortcut and c1 == c2

    def forward(self, x):
        y = self.cv2(self.cv1(x))
        return x + y if self.add else y


class C2f(nn.Module):
    """cv1 -> split in two -> n blocks chained on the second half -> cv2(cat(all))."""

    def __init__(self, c1, c2, n=1, shortcut=False, g=1, e=0.5):
        super().__init__()
        self.c = int(c2 * e)
        self.cv1 = Conv(c1, 2 * self.c, 1, 1)
        self.cv2 = Conv((2 + n) * self.c, c2, 1)
        self.m = nn.ModuleList(Bottleneck(self.c, self.c, shortcut, g, k=((3, 3), (3, 3)), e=1.0)
                               for _ in range(n))

    def forward(self, x):
        y = list(self.cv1(x).chunk(2, 1))
        for m in self.m:
            y.append(m(y[-1]))
        return self.cv2(torch.cat(y, 1))


class C3(nn.Module):
    def __init__(self, c1, c2, n=1, shortcut=True, g=1, e=0.5):
        super().__init__()
        c_ = int(c2 * e)
        self.cv1 = Conv(c1, c_, 1, 1)
        self.cv2 = Conv(c1, c_, 1, 1)
        self.cv3 = Conv(2 * c_, c2, 1)
        self.m = nn.Sequential(*(Bottleneck(c_, c_, shortcut, g, k=((1, 1), (3, 3)), e=1.0)
                                 for _ in range(n)))

    def forward(self, x):
        return self.cv3(torch.cat((self.m(self.cv1(x)), self.cv2(x)), 1))


class C3k(C3):
    def __init__(self, c1, c2, n=1, shortcut=True, g=1, e=0.5, k=3):
        super().__init__(c1, c2, n, shortcut, g, e)
        c_ = int(c2 * e)
        self.m = nn.Sequential(*(Bottleneck(c_, c_, shortcut, g, k=(k, k), e=1.0)
                                 for _ in range(n)))


class C3k2(C2f):
    def __init__(self, c1, c2, n=1, c3k=False, e=0.5, g=1, shortcut=True):
        super().__init__(c1, c2, n, shortcut, g, e)
        self.m = nn.ModuleList(C3k(self.c, self.c, 2, shortcut, g) if c3k
                               else Bottleneck(self.c, self.c, shortcut, g) for _ in range(n))


class SPPF(nn.Module):
    def __init__(self, c1, c2, k=5):
        super().__init__()
        c_ = c1 // 2
        self.cv1 = Conv(c1, c_, 1, 1)
        self.cv2 = Conv(c_ * 4, c2, 1, 1)
        self.m = nn.MaxPool2d(kernel_size=k, stride=1, padding=k // 2)

    def forward(self, x):
        y = [self.cv1(x)]
        for _ in range(3):
            y.append(self.m(y[-1]))
        return self.cv2(torch.cat(y, 1))


class Attention(nn.Module):
    """Multi-head self-attention over the H*W tokens; qkv channels per head = [q kd, k kd, v hd]."""

    def __init__(self, dim, num_heads=8, attn_ratio=0.5):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.key_dim = int(self.head_dim * attn_ratio)
        self.scale = self.key_dim ** -0.5
        nh_kd = self.key_dim * num_heads
        self.qkv = Conv(dim, dim + nh_kd * 2, 1, act=False)
        self.proj = Conv(dim, dim, 1, act=False)
        self.pe = Conv(dim, dim, 3, 1, g=dim, act=False)

    def forward(self, x):
        B, C, H, W = x.shape
        N = H * W
        qkv = self.qkv(x)
        q, k, v = qkv.view(B, self.num_heads, self.key_dim * 2 + self.head_dim, N).split(
            [self.key_dim, self.key_dim, self.head_dim], dim=2)
        attn = ((q.transpose(-2, -1) @ k) * self.scale).softmax(dim=-1)
        x = (v @ attn.transpose(-2, -1)).view(B, C, H, W) + self.pe(v.reshape(B, C, H, W))
        return self.proj(x)


class PSABlock(nn.Module):
    def __init__(self, c, attn_ratio=0.5, num_heads=4, shortcut=True):
        super().__init__()
        self.attn = Attention(c, attn_ratio=attn_ratio, num_heads=num_heads)
        self.ffn = nn.Sequential(Conv(c, c * 2, 1), Conv(c * 2, c, 1, act=False))
        self.add = shortcut

    def forward(self, x):
        x = x + self.attn(x) if self.add else self.attn(x)
        return x + self.ffn(x) if self.add else self.ffn(x)


class C2PSA(nn.Module):
    def __init__(self, c1, c2, n=1, e=0.5):
        super().__init__()
        assert c1 == c2
        self.c = int(c1 * e)
        self.cv1 = Conv(c1, 2 * self.c, 1, 1)
        self.cv2 = Conv(2 * self.c, c1, 1)
        self.m = nn.Sequential(*(PSABlock(self.c, attn_ratio=0.5, num_heads=self.c // 64)
                                 for _ in range(n)))

    def forward(self, x):
        a, b = self.cv1(x).split((self.c, self.c), dim=1)
        return self.cv2(torch.cat((a, self.m(b)), 1))


class DFL(nn.Module):
    """Distribution focal loss integral: softmax over 16 bins -> expectation (weights arange)."""

    def __init__(self, c1=16):
        super().__init__()
        self.conv = nn.Conv2d(c1, 1, 1, bias=False).requires_grad_(False)
        self.conv.weight.data[:] = torch.arange(c1, dtype=torch.float32).view(1, c1, 1, 1)
        self.c1 = c1

    def forward(self, x):
        b, _, a = x.shape
        return self.conv(x.view(b, 4, self.c1, a).transpose(2, 1).softmax(1)).view(b, 4, a)


class Proto(nn.Module):
    def __init__(self, c1, c_=256, c2=32):
        super().__init__()
        self.cv1 = Conv(c1, c_, k=3)
        self.upsample = nn.ConvTranspose2d(c_, c_, 2, 2, 0, bias=True)
        self.cv2 = Conv(c_, c_, k=3)
        self.cv3 = Conv(c_, c2)

    def forward(self, x):
        return self.cv3(self.cv2(self.upsample(self.cv1(x))))


def _make_anchors(feats, strides, offset=0.5):
    pts, sts = [], []
    for f, s in zip(feats, strides):
        _, _, h, w = f.shape
        sy, sx = torch.meshgrid(torch.arange(h, dtype=torch.float32) + offset,
                                torch.arange(w, dtype=torch.float32) + offset, indexing="ij")
        pts.append(torch.stack((sx, sy), -1).view(-1, 2))
        sts.append(torch.full((h * w, 1), float(s)))
    return torch.cat(pts), torch.cat(sts)


class Detect(nn.Module):
    """Decoupled head: per level a box branch (64 = 4 sides x 16 DFL bins) and a cls branch."""

    def __init__(self, nc=80, ch=(), legacy=False):
        super().__init__()
        self.nc, self.nl, self.reg_max = nc, len(ch), 16
        self.no = nc + self.reg_max * 4
        self.stride = torch.tensor([8.0, 16.0, 32.0])
        c2, c3 = max(16, ch[0] // 4, self.reg_max * 4), max(ch[0], min(nc, 100))
        self.cv2 = nn.ModuleList(nn.Sequential(Conv(x, c2, 3), Conv(c2, c2, 3),
                                               nn.Conv2d(c2, 4 * self.reg_max, 1)) for x in ch)
        if legacy:
            self.cv3 = nn.ModuleList(nn.Sequential(Conv(x, c3, 3), Conv(c3, c3, 3),
                                                   nn.Conv2d(c3, nc, 1)) for x in ch)
        else:
            self.cv3 = nn.ModuleList(
                nn.Sequential(nn.Sequential(DWConv(x, x, 3), Conv(x, c3, 1)),
                              nn.Sequential(DWConv(c3, c3, 3), Conv(c3, c3, 1)),
                              nn.Conv2d(c3, nc, 1)) for x in ch)
        self.dfl = DFL(self.reg_max)

    def _levels(self, x):
        return [torch.cat((self.cv2[i](x[i]), self.cv3[i](x[i])), 1) for i in range(self.nl)]

    def _decode(self, x):
        """[B, 4+nc, A]: xywh boxes (letterbox px) and sigmoid class scores."""
        shape = x[0].shape
        x_cat = torch.cat([xi.view(shape[0], self.no, -1) for xi in x], 2)
        anchors, strides = (t.transpose(0, 1) for t in _make_anchors(x, self.stride))
        box, cls = x_cat.split((self.reg_max * 4, self.nc), 1)
        d = self.dfl(box)
        lt, rb = d.chunk(2, 1)
        x1y1, x2y2 = anchors.unsqueeze(0) - lt, anchors.unsqueeze(0) + rb
        dbox = torch.cat(((x1y1 + x2y2) / 2, x2y2 - x1y1), 1) * strides
        return torch.cat((dbox, cls.sigmoid()), 1)

    def forward(self, x):
        x = self._levels(x)
        return self._decode(x), x


class OBB(Detect):
    """Oriented-box head: Detect plus an angle branch (ne = 1 channel per anchor).

    theta = (sigmoid(angle logit) - 0.25) * pi; the DFL side distances (l, t, r, b) give the
    box size (l + r, t + b) along theta and the centre offset ((r - l) / 2, (b - t) / 2)
    rotated by theta from the anchor point; all times the level stride."""

    def __init__(self, nc=15, ne=1, ch=(), legacy=False):
        super().__init__(nc, ch, legacy)
        self.ne = ne
        c4 = max(ch[0] // 4, self.ne)
        self.cv4 = nn.ModuleList(nn.Sequential(Conv(x, c4, 3), Conv(c4, c4, 3),
                                               nn.Conv2d(c4, self.ne, 1)) for x in ch)

    def forward(self, x):
        bs = x[0].shape[0]
        ang = torch.cat([self.cv4[i](x[i]).view(bs, self.ne, -1) for i in range(self.nl)], 2)
        ang = (ang.sigmoid() - 0.25) * math.pi
        lv = self._levels(x)
        shape = lv[0].shape
        x_cat = torch.cat([xi.view(shape[0], self.no, -1) for xi in lv], 2)
        anchors, strides = (t.transpose(0, 1) for t in _make_anchors(lv, self.stride))
        box, cls = x_cat.split((self.reg_max * 4, self.nc), 1)
        lt, rb = self.dfl(box).chunk(2, 1)
        cos, sin = torch.cos(ang), torch.sin(ang)
        xf, yf = ((rb - lt) / 2).split(1, dim=1)
        xy = torch.cat([xf * cos - yf * sin, xf * sin + yf * cos], 1) + anchors.unsqueeze(0)
        dbox = torch.cat([xy, lt + rb], 1) * strides
        return torch.cat([dbox, cls.sigmoid(), ang], 1), (lv, ang)


class Segment(Detect):
    def __init__(self, nc=80, nm=32, npr=256, ch=(), legacy=False):
        super().__init__(nc, ch, legacy)
        self.nm, self.npr = nm, npr
        self.proto = Proto(ch[0], self.npr, self.nm)
        c4 = max(ch[0] // 4, self.nm)
        self.cv4 = nn.ModuleList(nn.Sequential(Conv(x, c4, 3), Conv(c4, c4, 3),
                                               nn.Conv2d(c4, self.nm, 1)) for x in ch)

    def forward(self, x):
        p = self.proto(x[0])
        bs = p.shape[0]
        mc = torch.cat([self.cv4[i](x[i]).view(bs, self.nm, -1) for i in range(self.nl)], 2)
        x = self._levels(x)
        return (torch.cat([self._decode(x), mc], 1), p), (x, mc, p)


class Classify(nn.Module):
    """Classification head: 1x1 Conv to 1280 (+SiLU), global average pool, Linear, softmax."""

    def __init__(self, c1, nc=1000):
        super().__init__()
        self.conv = Conv(c1, 1280, 1, 1)
        self.pool = nn.AdaptiveAvgPool2d(1)
        self.linear = nn.Linear(1280, nc)
        self.nc = nc

    def forward(self, x):
        x = self.linear(self.pool(self.conv(x)).flatten(1))
        return x.softmax(1), x       # (probs, logits), as the eval-mode head returns


# yaml layer lists: (from, repeats, module, args)
_YOLO11 = [
    (-1, 1, "Conv", [64, 3, 2]), (-1, 1, "Conv", [128, 3, 2]),
    (-1, 2, "C3k2", [256, False, 0.25]), (-1, 1, "Conv", [256, 3, 2]),
    (-1, 2, "C3k2", [512, False, 0.25]), (-1, 1, "Conv", [512, 3, 2]),
    (-1, 2, "C3k2", [512, True]), (-1, 1, "Conv", [1024, 3, 2]),
    (-1, 2, "C3k2", [1024, True]), (-1, 1, "SPPF", [1024, 5]), (-1, 2, "C2PSA", [1024]),
    (-1, 1, "Upsample", []), ([-1, 6], 1, "Concat", []), (-1, 2, "C3k2", [512, False]),
    (-1, 1, "Upsample", []), ([-1, 4], 1, "Concat", []), (-1, 2, "C3k2", [256, False]),
    (-1, 1, "Conv", [256, 3, 2]), ([-1, 13], 1, "Concat", []), (-1, 2, "C3k2", [512, False]),
    (-1, 1, "Conv", [512, 3, 2]), ([-1, 10], 1, "Concat", []), (-1, 2, "C3k2", [1024, True]),
]
_YOLOV8 = [
    (-1, 1, "Conv", [64, 3, 2]), (-1, 1, "Conv", [128, 3, 2]), (-1, 3, "C2f", [128, True]),
    (-1, 1, "Conv", [256, 3, 2]), (-1, 6, "C2f", [256, True]), (-1, 1, "Conv", [512, 3, 2]),
    (-1, 6, "C2f", [512, True]), (-1, 1, "Conv", [1024, 3, 2]), (-1, 3, "C2f", [1024, True]),
    (-1, 1, "SPPF", [1024, 5]),
    (-1, 1, "Upsample", []), ([-1, 6], 1, "Concat", []), (-1, 3, "C2f", [512]),
    (-1, 1, "Upsample", []), ([-1, 4], 1, "Concat", []), (-1, 3, "C2f", [256]),
    (-1, 1, "Conv", [256, 3, 2]), ([-1, 12], 1, "Concat", []), (-1, 3, "C2f", [512]),
    (-1, 1, "Conv", [512, 3, 2]), ([-1, 9], 1, "Concat", []), (-1, 3, "C2f", [1024]),
]


class DetectionModel(nn.Module):
    def __init__(self, name: str, nc: int = 80, imgsz: int = 640):
        super().__init__()
        m = re.fullmatch(r"(yolo11|yolov8)([nsmlx])(-seg|-cls|-obb)?", name)
        if not m:
            raise ValueError(f"unknown model name {name!r} (expected yolo11n, yolov8m-seg, ...)")
        family, scale = m.group(1), m.group(2)
        seg, cls, obb = m.group(3) == "-seg", m.group(3) == "-cls", m.group(3) == "-obb"
        depth, width, max_ch = MODEL_SCALES[family][scale]
        self.family, self.scale_name = family, scale
        self.task = "segment" if seg else "classify" if cls else "obb" if obb else "detect"
        if cls and nc == 80:
            nc = 1000      # ImageNet head
        if obb and nc == 80:
            nc = 15        # DOTA
        self.names = {i: f"class{i}" for i in range(nc)}
        self.args = {"imgsz": imgsz}
        layers, ch, save_ch = [], [3], []
        table = _YOLO11 if family == "yolo11" else _YOLOV8
        if cls:   # the backbone without SPPF (yolo11: its C2PSA directly after layer 8)
            table = table[:9] + ([(-1, 2, "C2PSA", [1024])] if family == "yolo11" else [])
        for i, (f, n, mod, args) in enumerate(table):
            n = max(round(n * depth), 1) if n > 1 else n
            c1 = ch[f] if isinstance(f, int) else None
            if mod == "Conv":
                c2 = _ceil8(min(args[0], max_ch) * width)
                layer = Conv(c1, c2, args[1], args[2])
            elif mod == "C3k2":
                c2 = _ceil8(min(args[0], max_ch) * width)
                c3k = bool(args[1]) or scale in "mlx"
                e = args[2] if len(args) > 2 else 0.5
                layer = C3k2(c1, c2, n, c3k, e)
            elif mod == "C2f":
                c2 = _ceil8(min(args[0], max_ch) * width)
                layer = C2f(c1, c2, n, bool(args[1]) if len(args) > 1 else False)
            elif mod == "SPPF":
                c2 = _ceil8(min(args[0], max_ch) * width)
                layer = SPPF(c1, c2, args[1])
            elif mod == "C2PSA":
                c2 = c1
                layer = C2PSA(c1, c2, n)
            elif mod == "Upsample":
                c2 = c1
                layer = nn.Upsample(None, 2, "nearest")
            elif mod == "Concat":
                c2 = sum(ch[j] for j in f)
                layer = Concat(1)
            else:
                raise AssertionError(mod)
            layer.f, layer.i = f, i
            layers.append(layer)
            if i == 0:
                ch = []
            ch.append(c2)
        if cls:
            head = Classify(ch[-1], nc)
            head.f, head.i = -1, len(layers)
            layers.append(head)
            self.model = nn.Sequential(*layers)
            self.stride = torch.tensor([32.0])
            return
        heads_from = [16, 19, 22] if family == "yolo11" else [15, 18, 21]
        hch = [ch[j] for j in heads_from]
        legacy = family == "yolov8"
        if seg:
            npr = _ceil8(min(256, max_ch) * width)
            head = Segment(nc, 32, npr, hch, legacy=legacy)
        elif obb:
            head = OBB(nc, 1, hch, legacy=legacy)
        else:
            head = Detect(nc, hch, legacy=legacy)
        head.f, head.i = heads_from, len(layers)
        layers.append(head)
        self.model = nn.Sequential(*layers)
        self.stride = head.stride

    def fuse(self):
        """BatchNorm is folded at construction; kept for interface compatibility."""
        return self

    def forward(self, x):
        y = []
        for m in self.model:
            if m.f != -1:
                x = y[m.f] if isinstance(m.f, int) else [x if j == -1 else y[j] for j in m.f]
            x = m(x)
            y.append(x)
        return x


def _init_weights(model: DetectionModel, seed: int, cls_bias: float, gain2: float):
    rng = np.random.Generator(np.random.PCG64(seed))
    head = model.model[-1]
    finals = {}
    for i in range(getattr(head, "nl", 0)):
        finals[id(head.cv2[i][-1])] = "box"
        finals[id(head.cv3[i][-1])] = "cls"
        if isinstance(head, (Segment, OBB)):
            finals[id(head.cv4[i][-1])] = "coef"

    def normal(shape, std):
        return rng.standard_normal(shape, dtype=np.float64).astype(np.float32) * np.float32(std)

    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, Conv):
                cv = mod.conv
                O, Ig, kh, kw = cv.weight.shape
                w = normal((O, Ig, kh, kw), math.sqrt(gain2 / (Ig * kh * kw)))
                gamma = rng.uniform(0.5, 1.5, O).astype(np.float32)
                beta = normal(O, 0.1)
                mean = normal(O, 0.1)
                var = rng.uniform(0.5, 1.5, O).astype(np.float32)
                sc = gamma / np.sqrt(var + np.float32(1e-3))
                cv.weight.copy_(torch.from_numpy(w * sc[:, None, None, None]))
                cv.bias.copy_(torch.from_numpy(beta - mean * sc))
            elif isinstance(mod, nn.Conv2d) and id(mod) in finals:
                O, Ig, kh, kw = mod.weight.shape
                mod.weight.copy_(torch.from_numpy(normal((O, Ig, kh, kw), 1.0 / math.sqrt(Ig))))
                b = np.full(O, cls_bias if finals[id(mod)] == "cls" else 0.0, np.float32)
                mod.bias.copy_(torch.from_numpy(b))
            elif isinstance(mod, nn.Linear):
                O, I = mod.weight.shape
                mod.weight.copy_(torch.from_numpy(normal((O, I), 4.0 / math.sqrt(I))))
                mod.bias.copy_(torch.from_numpy(normal(O, 0.1)))
            elif isinstance(mod, nn.ConvTranspose2d):
                Ci, Co, kh, kw = mod.weight.shape
                mod.weight.copy_(torch.from_numpy(normal((Ci, Co, kh, kw), 1.0 / math.sqrt(Ci))))
                mod.bias.copy_(torch.from_numpy(normal(Co, 0.1)))


def model_seed(name: str) -> int:
    """Stable per-model seed (independent of Python's salted str hash)."""
    return sum((i + 1) * ord(c) for i, c in enumerate(name)) % (2 ** 31)


def build_model(name: str, imgsz: int = 640, nc: int = 80, seed: int | None = None,
                cls_bias: float | None = None) -> DetectionModel:
    """Seeded random-init, BN-folded, eval-mode fp32 model (e.g. ``build_model('yolo11m')``)."""
    model = DetectionModel(name, nc=nc, imgsz=imgsz)
    cb = CLS_BIAS.get(name, CLS_BIAS_DEFAULT) if cls_bias is None else cls_bias
    _init_weights(model, model_seed(name) if seed is None else seed, cb,
                  KAIMING_GAIN2.get(name, 2.0))
    return model.float().eval().requires_grad_(False)
