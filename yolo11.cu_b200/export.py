"""Model-directory writer: torch YOLO module -> flat primitive-op graph + fp16 OHWI weights.

Writes the on-disk model format the engine loads (the reference's format, parsed by
``engine/engine.cu:88-141``):

    model.graph   ``YOLO11GRAPH 2`` / ``TASK`` header, ``B`` buffers, ``T`` channel views,
                  op lines
    weights.f16   every conv weight, fp16, OHWI = [Cout][kh][kw][Cin/g], in CONV-op order
    bias.f32      every conv bias, fp32, same order
    input.f16     letterboxed frame 0, NHWC fp16 (S x S x 3), RGB, /255
    bus_raw.u8 / bus_raw.txt   the raw BGR frame and its "h w" (CLI ``pipeline`` input)

Design: two passes.

1. Lowering (``_Lowering``) walks the layer list and turns every module into *declarations*
   (``Slab``: a buffer; ``Span``: a channel range of a slab) and *instructions* (``Instr``),
   all held as Python objects; nothing is numbered and no weight is packed yet.  Each
   composite module has one recipe below saying which slabs/spans it declares, in which
   order, and which instructions it issues.  Concats are zero-copy: a concat's slab is
   declared before the walk and every producer writes its span; a producer that feeds a
   second concat (or the input, or another concat) is copied in with COPYC.
2. Packing (``_Program.pack``) numbers slabs and spans in declaration order, lays weights
   and biases out in CONV-instruction order, and renders the text.  A conv's weights are
   zero-extended to the channel counts of the spans it reads and writes, which is how the
   head's class / angle branches get their multiple-of-8 widths (pad rows w = 0, b = 0).

The declaration and instruction order fixes every buffer, view and op index (and so the
``opNNN`` numbering of the parity fixtures); it is the reference exporter's
(``export/export.py:319-441``), which ``tests/test_oracle_golden.py`` checks byte for byte.
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn as nn

from . import nn as ynn

ACT_NONE, ACT_SILU = 0, 1


# ---------------- declarations and instructions ----------------
class Slab:
    """A buffer: H x W x C fp16 per image."""
    __slots__ = ("H", "W", "C", "id")

    def __init__(self, H, W, C):
        self.H, self.W, self.C, self.id = H, W, C, None


class Span:
    """Channels [c0, c0 + C) of a slab."""
    __slots__ = ("slab", "c0", "C", "id")

    def __init__(self, slab, c0, C):
        if c0 < 0 or c0 + C > slab.C:
            raise ValueError(f"span [{c0}, {c0 + C}) outside a {slab.C}-channel slab")
        self.slab, self.c0, self.C, self.id = slab, c0, C, None

    @property
    def H(self):
        return self.slab.H

    @property
    def W(self):
        return self.slab.W


class Instr:
    """One op line.  ``args`` mixes spans (rendered as their ids) and integers; a CONV also
    carries its weight [O, kh, kw, I] (float32), bias [O] and how to extend them."""
    __slots__ = ("kind", "args", "weight", "bias")

    def __init__(self, kind, *args, weight=None, bias=None):
        self.kind, self.args, self.weight, self.bias = kind, args, weight, bias


class _Program:
    def __init__(self):
        self.decls = []        # Slab / Span objects in declaration order
        self.instrs = []

    # declarations
    def slab(self, H, W, C):
        s = Slab(H, W, C)
        self.decls.append(s)
        return s

    def span(self, slab, c0, C):
        v = Span(slab, c0, C)
        self.decls.append(v)
        return v

    def new(self, H, W, C):
        """A slab of its own, wholly viewed."""
        return self.span(self.slab(H, W, C), 0, C)

    def issue(self, kind, *args, **kw):
        self.instrs.append(Instr(kind, *args, **kw))

    # packing
    def pack(self, task, nc, S):
        nslab = nspan = 0
        for d in self.decls:
            if isinstance(d, Slab):
                d.id, nslab = nslab, nslab + 1
            else:
                d.id, nspan = nspan, nspan + 1
        wblobs, bblobs, lines = [], [], []
        woff = boff = 0
        for ins in self.instrs:
            vals = [a.id if isinstance(a, Span) else int(a) for a in ins.args]
            if ins.kind == "CONV":
                w16 = np.ascontiguousarray(ins.weight, np.float16).ravel()
                b32 = np.ascontiguousarray(ins.bias, np.float32).ravel()
                vals += [woff, boff]
                woff += w16.size
                boff += b32.size
                wblobs.append(w16)
                bblobs.append(b32)
            lines.append(" ".join([ins.kind] + [str(v) for v in vals]))
        slabs = [d for d in self.decls if isinstance(d, Slab)]
        spans = [d for d in self.decls if isinstance(d, Span)]
        head = ["YOLO11GRAPH 2", f"TASK {task} {nc} {S}", f"{nslab} {nspan} {len(self.instrs)}"]
        head += [f"B {s.H} {s.W} {s.C}" for s in slabs]
        head += [f"T {v.slab.id} {v.c0} {v.C}" for v in spans]
        text = "\n".join(head + lines) + "\n"
        empty = np.zeros(0, np.float16)
        return (text, np.concatenate(wblobs) if wblobs else empty,
                np.concatenate(bblobs) if bblobs else np.zeros(0, np.float32))


# ---------------- weights ----------------
def _conv_parts(mod):
    """(nn.Conv2d, activation code) of a ynn.Conv or a bare nn.Conv2d."""
    if isinstance(mod, ynn.Conv):
        return mod.conv, ACT_SILU if isinstance(mod.act, nn.SiLU) else ACT_NONE
    return mod, ACT_NONE


def _extend(w, b, o_to, i_to):
    """Zero-extend OHWI weights to o_to output / i_to input channels, bias to o_to."""
    O, kh, kw, I = w.shape
    out = np.zeros((o_to, kh, kw, i_to), np.float32)
    out[:O, :, :, :I] = w
    bb = np.zeros(o_to, np.float32)
    bb[:O] = b
    return out, bb


# ---------------- lowering ----------------
def _round8(c):
    return (c + 7) // 8 * 8


class _Lowering:
    def __init__(self, model, S):
        self.p = _Program()
        self.model, self.S = model, S

    # -- primitive: one convolution from span `src` into `dst` (declared here if None) --
    def conv(self, src, mod, dst=None, width=None):
        cv, act = _conv_parts(mod)
        O, Ig, kh, kw = cv.weight.shape
        if kh != kw:
            raise ValueError("square kernels only")
        k, s, pd, groups = kh, cv.stride[0], cv.padding[0], cv.groups
        depthwise = groups > 1
        if depthwise and not (groups == O and Ig == 1):
            raise ValueError("grouped convs other than depthwise are not supported")
        if not depthwise and Ig > src.C:
            raise ValueError(f"conv wants {Ig} input channels, span has {src.C}")
        Ho, Wo = (src.H + 2 * pd - k) // s + 1, (src.W + 2 * pd - k) // s + 1
        if dst is None:
            dst = self.p.new(Ho, Wo, width or O)
        if (dst.H, dst.W) != (Ho, Wo) or dst.C < O:
            raise ValueError("conv output span has the wrong shape")
        w = cv.weight.detach().permute(0, 2, 3, 1).numpy()
        b = cv.bias.detach().numpy() if cv.bias is not None else np.zeros(O, np.float32)
        w, b = _extend(w, b, dst.C, 1 if depthwise else src.C)
        g_field = dst.C if depthwise else 1
        self.p.issue("CONV", src, dst, k, s, pd, g_field, act, src.C, dst.C, weight=w, bias=b)
        return dst

    def convs(self, src, mods, pad8=False):
        """A (nested) Sequential of convs, each into a span of its own."""
        if isinstance(mods, nn.Sequential):
            for m in mods:
                src = self.convs(src, m, pad8)
            return src
        O = _conv_parts(mods)[0].out_channels
        return self.conv(src, mods, width=_round8(O) if pad8 else None)

    def conv_transpose2(self, src, mod):
        """ConvTranspose2d(k=2, s=2) as a 1x1 CONV to 4C (quadrant q = 2*di + dj blocks of C
        channels) followed by PS2."""
        wt = mod.weight.detach()                   # [Cin, C, 2, 2]
        Cin, C = wt.shape[0], wt.shape[1]
        if tuple(wt.shape[2:]) != (2, 2) or mod.stride[0] != 2 or mod.padding[0] != 0 or Cin != src.C:
            raise ValueError("only ConvTranspose2d(k=2, s=2, p=0) is supported")
        quad = self.p.new(src.H, src.W, 4 * C)
        w = wt.permute(2, 3, 1, 0).reshape(4 * C, 1, 1, Cin).numpy()
        b = np.tile(mod.bias.detach().numpy(), 4)
        self.p.issue("CONV", src, quad, 1, 1, 0, 1, ACT_NONE, Cin, 4 * C, weight=w, bias=b)
        out = self.p.new(2 * src.H, 2 * src.W, C)
        self.p.issue("PS2", quad, out)
        return out

    # -- composite recipes --
    def bottleneck(self, src, m, dst):
        mid = self.conv(src, m.cv1)
        self.conv(mid, m.cv2, dst)
        if m.add:
            self.p.issue("ADD", dst, src, dst)

    def c3k(self, src, m, dst):
        h = m.cv1.conv.out_channels
        pair = self.p.slab(src.H, src.W, 2 * h)      # [ bottleneck chain | cv2 ]
        run = self.conv(src, m.cv1)
        blocks = list(m.m)
        for i, blk in enumerate(blocks):
            last = i == len(blocks) - 1
            tgt = self.p.span(pair, 0, h) if last else self.p.new(src.H, src.W, h)
            self.bottleneck(run, blk, tgt)
            run = tgt
        self.conv(src, m.cv2, self.p.span(pair, h, h))
        self.conv(self.p.span(pair, 0, 2 * h), m.cv3, dst)

    def c2f(self, src, m, dst):
        c, n = m.c, len(m.m)
        stack = self.p.slab(src.H, src.W, (2 + n) * c)   # [ cv1 (2c) | block 0 | block 1 ... ]
        self.conv(src, m.cv1, self.p.span(stack, 0, 2 * c))
        feed = self.p.span(stack, c, c)
        for i, blk in enumerate(m.m):
            tgt = self.p.span(stack, (2 + i) * c, c)
            (self.c3k if isinstance(blk, ynn.C3k) else self.bottleneck)(feed, blk, tgt)
            feed = tgt
        return self.conv(self.p.span(stack, 0, (2 + n) * c), m.cv2, dst)

    def sppf(self, src, m, dst):
        h = m.cv1.conv.out_channels
        pools = self.p.slab(src.H, src.W, 4 * h)         # [ cv1 | pool | pool^2 | pool^3 ]
        self.conv(src, m.cv1, self.p.span(pools, 0, h))
        for i in range(3):
            self.p.issue("MAXPOOL5", self.p.span(pools, i * h, h), self.p.span(pools, (i + 1) * h, h))
        return self.conv(self.p.span(pools, 0, 4 * h), m.cv2, dst)

    def psa_block(self, x, blk):
        """In place on span x: x += proj(attn(x) + pe(v)); x += ffn(x)."""
        at = blk.attn
        nh, kd, hd = at.num_heads, at.key_dim, at.head_dim
        if nh * hd != x.C:
            raise ValueError("attention heads do not tile the channels")
        qkv = self.conv(x, at.qkv)                       # per head [q kd | k kd | v hd]
        vslab = self.p.slab(x.H, x.W, x.C)
        for h in range(nh):
            self.p.issue("COPYC", self.p.span(qkv.slab, h * (2 * kd + hd) + 2 * kd, hd),
                         self.p.span(vslab, h * hd, hd))
        v = self.p.span(vslab, 0, x.C)
        att = self.p.new(x.H, x.W, x.C)
        self.p.issue("ATTN", qkv, att, nh, kd, hd)
        pe = self.conv(v, at.pe)
        self.p.issue("ADD", att, pe, att)
        proj = self.conv(att, at.proj)
        self.p.issue("ADD", x, proj, x)
        f = self.conv(self.conv(x, blk.ffn[0]), blk.ffn[1])
        self.p.issue("ADD", x, f, x)

    def c2psa(self, src, m, dst):
        c = m.c
        halves = self.p.slab(src.H, src.W, 2 * c)        # [ passthrough | attention path ]
        self.conv(src, m.cv1, self.p.span(halves, 0, 2 * c))
        path = self.p.span(halves, c, c)
        for blk in m.m:
            self.psa_block(path, blk)
        return self.conv(self.p.span(halves, 0, 2 * c), m.cv2, dst)

    # -- whole network --
    def run(self):
        net, S = self.model.model, self.S
        body = list(net)[:-1]
        x0 = self.p.new(S, S, 3)

        def srcs(i):
            f = body[i].f
            return [i - 1 if j == -1 else j for j in ([f] if isinstance(f, int) else f)]

        # output channels and side of every body layer
        chans, side = {-1: 3}, {-1: S}
        for i, m in enumerate(body):
            ins = srcs(i)
            hin = side[ins[0]]
            if isinstance(m, ynn.Conv):
                cv = m.conv
                chans[i] = cv.out_channels
                side[i] = (hin + 2 * cv.padding[0] - cv.kernel_size[0]) // cv.stride[0] + 1
            elif isinstance(m, (ynn.C2f, ynn.SPPF, ynn.C2PSA)):
                chans[i], side[i] = m.cv2.conv.out_channels, hin
            elif isinstance(m, nn.Upsample):
                chans[i], side[i] = chans[ins[0]], 2 * hin
            elif isinstance(m, ynn.Concat):
                chans[i], side[i] = sum(chans[j] for j in ins), hin
            else:
                raise ValueError(f"no lowering for {type(m).__name__} (layer {i})")

        # concat slabs, declared before the walk; each producer is routed into the first
        # concat that takes it, later consumers of it get a copy
        cat_slab, route, copy_in = {}, {}, {}
        for i, m in enumerate(body):
            if not isinstance(m, ynn.Concat):
                continue
            cat_slab[i] = self.p.slab(side[i], side[i], chans[i])
            c0 = 0
            for j in srcs(i):
                direct = j >= 0 and j not in route and not isinstance(body[j], ynn.Concat)
                if direct:
                    route[j] = (i, c0)
                else:
                    copy_in.setdefault(i, []).append((j, c0))
                c0 += chans[j]

        out = {-1: x0}
        for i, m in enumerate(body):
            src = out[srcs(i)[0]]
            dst = None
            if i in route:
                ci, c0 = route[i]
                dst = self.p.span(cat_slab[ci], c0, chans[i])
            if isinstance(m, ynn.Conv):
                y = self.conv(src, m, dst)
            elif isinstance(m, ynn.C2PSA):
                y = self.c2psa(src, m, dst)
            elif isinstance(m, ynn.SPPF):
                y = self.sppf(src, m, dst)
            elif isinstance(m, ynn.C2f):
                y = self.c2f(src, m, dst)
            elif isinstance(m, nn.Upsample):
                if float(m.scale_factor) != 2.0:
                    raise ValueError("only 2x upsampling is supported")
                y = dst if dst is not None else self.p.new(side[i], side[i], chans[i])
                self.p.issue("UPSAMPLE2", src, y)
            else:                                        # Concat
                for j, c0 in copy_in.get(i, []):
                    self.p.issue("COPYC", out[j], self.p.span(cat_slab[i], c0, chans[j]))
                y = self.p.span(cat_slab[i], 0, chans[i])
            out[i] = y
        self.head(net[-1], out, len(body))
        return self.p

    def head(self, det, out, nbody):
        if isinstance(det, ynn.Classify):
            # conv -> GAP -> linear (a 1x1 CONV on the [1, 1, C] pooled tensor) -> channel
            # softmax, each into a slab of its own (export/export.py:389-397)
            feat = self.conv(out[nbody - 1], det.conv)
            pooled = self.p.new(1, 1, feat.C)
            self.p.issue("GAP", feat, pooled)
            O, I = det.linear.weight.shape
            logits = self.p.new(1, 1, O)
            self.p.issue("CONV", pooled, logits, 1, 1, 0, 1, ACT_NONE, I, O,
                         weight=det.linear.weight.detach().numpy().reshape(O, 1, 1, I),
                         bias=det.linear.bias.detach().numpy())
            self.p.issue("SOFTMAX", logits, self.p.new(1, 1, O))
            return
        if not torch.allclose(det.dfl.conv.weight.view(-1), torch.arange(16, dtype=torch.float32)):
            raise ValueError("the DFL conv must be arange(16)")
        seg, obb = isinstance(det, ynn.Segment), isinstance(det, ynn.OBB)
        feats = [out[j] for j in det.f]
        proto = None
        if seg:
            if det.nm % 8:
                raise ValueError("mask coefficients must be a multiple of 8")
            pr = det.proto
            proto = self.conv(self.conv(self.conv_transpose2(self.conv(feats[0], pr.cv1),
                                                             pr.upsample), pr.cv2), pr.cv3)
        for i, (f, st) in enumerate(zip(feats, det.stride)):
            st = int(st)
            box = self.convs(f, det.cv2[i])
            cls = self.convs(f, det.cv3[i][:2], pad8=True)
            cls = self.conv(cls, det.cv3[i][2], width=_round8(det.nc))
            if obb:        # angle branch, the 1-channel final padded to 8
                ang = self.convs(f, det.cv4[i][:2])
                ang = self.conv(ang, det.cv4[i][2], width=_round8(det.ne))
                self.p.issue("DECODEOBB", box, cls, ang, st)
            elif seg:
                self.p.issue("DECODESEG", box, cls, self.convs(f, det.cv4[i]), st)
            else:
                self.p.issue("DECODE", box, cls, st)
        if seg:
            self.p.issue("MASKS", proto)


# ---------------- inputs and the directory ----------------
def letterbox(bgr: np.ndarray, S: int) -> np.ndarray:
    """cv2 INTER_LINEAR letterbox (pad 114) -> RGB float32 [S, S, 3] in [0, 1]."""
    import cv2
    h, w = bgr.shape[:2]
    r = min(S / h, S / w)
    nh, nw = round(h * r), round(w * r)
    im = cv2.resize(bgr, (nw, nh), interpolation=cv2.INTER_LINEAR)
    top, left = (S - nh) // 2, (S - nw) // 2
    out = np.full((S, S, 3), 114, np.uint8)
    out[top:top + nh, left:left + nw] = im
    return out[:, :, ::-1].astype(np.float32) / 255.0


def classify_input(bgr: np.ndarray, S: int) -> np.ndarray:
    """torchvision classify preprocessing (ultralytics classify_transforms): PIL bilinear
    (antialiased) resize of the shortest edge to S, center crop S x S, RGB /255 ->
    float32 [S, S, 3]."""
    from PIL import Image
    import torchvision.transforms as T
    rgb = np.ascontiguousarray(bgr[:, :, ::-1])
    t = T.Compose([T.Resize(S, interpolation=T.InterpolationMode.BILINEAR), T.CenterCrop(S),
                   T.ToTensor()])
    return t(Image.fromarray(rgb)).permute(1, 2, 0).numpy()


def lower(model: "ynn.DetectionModel", S: int) -> _Program:
    """The model's graph program at input size S (declarations + instructions, unnumbered)."""
    return _Lowering(model, S).run()


def export_model(name: str, out_dir: str, imgsz: int = 640, frame_hw=(1080, 810),
                 frame_seed: int = 0, model=None) -> None:
    """Write ``out_dir`` for the seeded model ``name`` at input size ``imgsz``."""
    from .frames import synthetic_bgr
    if imgsz % 32:
        raise ValueError("imgsz must be a multiple of 32")
    model = ynn.build_model(name, imgsz=imgsz) if model is None else model
    head = model.model[-1]
    task = ("segment" if isinstance(head, ynn.Segment) else
            "classify" if isinstance(head, ynn.Classify) else
            "obb" if isinstance(head, ynn.OBB) else "detect")
    nc = head.linear.out_features if task == "classify" else head.nc
    text, w16, b32 = lower(model, imgsz).pack(task, nc, imgsz)
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "model.graph"), "w") as f:
        f.write(text)
    w16.tofile(os.path.join(out_dir, "weights.f16"))
    b32.tofile(os.path.join(out_dir, "bias.f32"))
    bgr = synthetic_bgr(*frame_hw, seed=frame_seed)
    bgr.tofile(os.path.join(out_dir, "bus_raw.u8"))
    with open(os.path.join(out_dir, "bus_raw.txt"), "w") as f:
        f.write(f"{bgr.shape[0]} {bgr.shape[1]}")
    x = classify_input(bgr, imgsz) if task == "classify" else letterbox(bgr, imgsz)
    x.astype(np.float16).tofile(os.path.join(out_dir, "input.f16"))
    if task == "classify":
        with open(os.path.join(out_dir, "names.txt"), "w") as f:
            f.write("\n".join(model.names[i] for i in range(nc)) + "\n")


def ensure_model_dir(name: str, root: str, imgsz: int = 640, frame_hw=(1080, 810)) -> str:
    """Return ``root/<name>[-S]`` (S omitted at the model's default size: 640, 224 for
    classify, 1024 for obb), exporting it first if ``model.graph`` is missing."""
    default = 224 if name.endswith("-cls") else 1024 if name.endswith("-obb") else 640
    d = os.path.join(root, name if imgsz == default else f"{name}-{imgsz}")
    if not os.path.exists(os.path.join(d, "model.graph")):
        export_model(name, d, imgsz, frame_hw)
    return d
