"""Model-directory writer: torch YOLO module -> flat primitive-op graph + fp16 OHWI weights.

Produces the reference's on-disk model format, byte for byte the same as the reference
exporter (``export/export.py``) given the same modules:

    model.graph   text graph (``YOLO11GRAPH 2`` / ``TASK`` header, ``B`` buffers, ``T`` views,
                  op lines), parsed by the engine (reference parser ``engine/engine.cu:88-141``)
    weights.f16   every conv weight, fp16, OHWI = [Cout][kh][kw][Cin/g]
    bias.f32      every conv bias, fp32
    input.f16     letterboxed frame 0, NHWC fp16 (S x S x 3), RGB, /255
    bus_raw.u8 / bus_raw.txt   the raw BGR frame and its "h w" (CLI ``pipeline`` input)

Graph semantics (reference ``export/export.py:319-441``):
  * tensor 0 is the S x S x 3 input; every tensor is a (buffer, channel offset, C) view;
  * concats are zero-copy: the concat buffer is allocated up front and each producer writes
    its channel slice; a producer that feeds a second concat gets a COPYC;
  * composite modules decompose into CONV / ADD / MAXPOOL5 / UPSAMPLE2 / COPYC / ATTN / PS2;
  * the head emits DECODE (detect) or DECODESEG + a final MASKS op (segment);
  * cls-branch widths are zero-padded to multiples of 8 (pad rows w=0, b=0).

The emission order (which fixes every buffer, view and op index, and so the per-op
``opNNN`` numbering of the parity fixtures) follows the reference walker step for step.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn as nn

from . import nn as ynn

ACT_NONE, ACT_SILU = 0, 1


@dataclass
class GraphBuilder:
    bufs: list = field(default_factory=list)     # (H, W, Ctot)
    tens: list = field(default_factory=list)     # (buf, coff, C)
    ops: list = field(default_factory=list)      # tuples, first element = kind
    w16: list = field(default_factory=list)
    w32: list = field(default_factory=list)
    b32: list = field(default_factory=list)
    nw: int = 0
    nb: int = 0
    layer_out: dict = field(default_factory=dict)

    # ---- buffers and views ----
    def buffer(self, H, W, C):
        self.bufs.append((H, W, C))
        return len(self.bufs) - 1

    def view(self, b, coff, C):
        assert coff + C <= self.bufs[b][2]
        self.tens.append((b, coff, C))
        return len(self.tens) - 1

    def fresh(self, H, W, C):
        return self.view(self.buffer(H, W, C), 0, C)

    def hwc(self, t):
        b, _, C = self.tens[t]
        return self.bufs[b][0], self.bufs[b][1], C

    def _weights(self, w_ohwi, bias):
        self.w32.append(np.ascontiguousarray(w_ohwi, np.float32).ravel())
        w = np.ascontiguousarray(w_ohwi, np.float16).ravel()
        b = np.ascontiguousarray(bias, np.float32).ravel()
        offs = (self.nw, self.nb)
        self.w16.append(w)
        self.b32.append(b)
        self.nw += w.size
        self.nb += b.size
        return offs

    # ---- op emitters ----
    @staticmethod
    def _unwrap(mod):
        if isinstance(mod, ynn.Conv):
            return mod.conv, (ACT_SILU if isinstance(mod.act, nn.SiLU) else ACT_NONE)
        return mod, ACT_NONE

    def conv(self, x, mod, out=None, act=None):
        cv, a = self._unwrap(mod)
        a = a if act is None else act
        O, Ig, kh, kw = cv.weight.shape
        k, s, p, g = kh, cv.stride[0], cv.padding[0], cv.groups
        H, W, Cin = self.hwc(x)
        assert kh == kw and Ig * g == Cin and (g == 1 or (g == Cin and O == Cin))
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        if out is None:
            out = self.fresh(Ho, Wo, O)
        assert self.hwc(out) == (Ho, Wo, O)
        w = cv.weight.detach().permute(0, 2, 3, 1).contiguous().numpy()
        b = cv.bias.detach().numpy() if cv.bias is not None else np.zeros(O, np.float32)
        woff, boff = self._weights(w, b)
        self.ops.append(("CONV", x, out, k, s, p, g, a, Cin, O, woff, boff))
        return out

    def conv_pad8(self, x, mod, cpad=None, act=None):
        """Conv whose output (and dead input) channels are zero-padded to a multiple of 8."""
        cv, a = self._unwrap(mod)
        a = a if act is None else act
        O, Ig, kh, kw = cv.weight.shape
        cpad = (O + 7) // 8 * 8 if cpad is None else cpad
        H, W, Cin = self.hwc(x)
        dw = cv.groups > 1
        if O == cpad and Ig * cv.groups == Cin:
            return self.conv(x, mod, act=act)
        k, s, p = kh, cv.stride[0], cv.padding[0]
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        out = self.fresh(Ho, Wo, cpad)
        w = cv.weight.detach().permute(0, 2, 3, 1).contiguous().numpy()
        if not dw and Ig < Cin:
            w = np.concatenate([w, np.zeros((O, kh, kw, Cin - Ig), w.dtype)], 3)
        w = np.concatenate([w, np.zeros((cpad - O, kh, kw, w.shape[3]), w.dtype)], 0)
        b0 = cv.bias.detach().numpy() if cv.bias is not None else np.zeros(O, np.float32)
        b = np.concatenate([b0, np.zeros(cpad - O, np.float32)])
        woff, boff = self._weights(w, b)
        self.ops.append(("CONV", x, out, k, s, p, cpad if dw else 1, a, cpad if dw else Cin,
                         cpad, woff, boff))
        return out

    def op(self, *t):
        self.ops.append(tuple(t))
        return t[-1] if t[0] in ("MAXPOOL5", "UPSAMPLE2", "PS2", "COPYC") else None

    def convT2(self, x, mod, out=None):
        """ConvTranspose2d(k=2, s=2) = 1x1 CONV to 4C (quadrant q = 2*di+dj blocks) + PS2."""
        H, W, Cin = self.hwc(x)
        wt = mod.weight.detach()
        C = wt.shape[1]
        assert tuple(wt.shape) == (Cin, C, 2, 2) and mod.stride[0] == 2 and mod.padding[0] == 0
        w = wt.permute(2, 3, 1, 0).reshape(4 * C, 1, 1, Cin).numpy()
        b = np.tile(mod.bias.detach().numpy(), 4)
        woff, boff = self._weights(w, b)
        up4 = self.fresh(H, W, 4 * C)
        self.ops.append(("CONV", x, up4, 1, 1, 0, 1, ACT_NONE, Cin, 4 * C, woff, boff))
        if out is None:
            out = self.fresh(H * 2, W * 2, C)
        self.ops.append(("PS2", up4, out))
        return out

    # ---- serialisation ----
    def graph_text(self, task, nc, S):
        lines = ["YOLO11GRAPH 2", f"TASK {task} {nc} {S}",
                 f"{len(self.bufs)} {len(self.tens)} {len(self.ops)}"]
        lines += [f"B {H} {W} {C}" for (H, W, C) in self.bufs]
        lines += [f"T {b} {o} {C}" for (b, o, C) in self.tens]
        lines += [" ".join(str(v) for v in op) for op in self.ops]
        return "\n".join(lines) + "\n"


# ---------------- composite modules ----------------

def _bottleneck(g, x, m, out):
    t = g.conv(x, m.cv1)
    g.conv(t, m.cv2, out=out)
    if m.add:
        g.op("ADD", out, x, out)
    return out


def _c3k(g, x, m, out):
    H, W, _ = g.hwc(x)
    c_ = m.cv1.conv.out_channels
    cat = g.buffer(H, W, 2 * c_)
    blocks = list(m.m)
    cur = g.conv(x, m.cv1)
    for j, bo in enumerate(blocks):
        dst = g.view(cat, 0, c_) if j == len(blocks) - 1 else g.fresh(H, W, c_)
        cur = _bottleneck(g, cur, bo, dst)
    g.conv(x, m.cv2, out=g.view(cat, c_, c_))
    g.conv(g.view(cat, 0, 2 * c_), m.cv3, out=out)
    return out


def _c2f(g, x, m, out=None):
    H, W, _ = g.hwc(x)
    c, n = m.c, len(m.m)
    cat = g.buffer(H, W, (2 + n) * c)
    g.conv(x, m.cv1, out=g.view(cat, 0, 2 * c))
    prev = g.view(cat, c, c)
    for j, blk in enumerate(m.m):
        dst = g.view(cat, (2 + j) * c, c)
        (_c3k if isinstance(blk, ynn.C3k) else _bottleneck)(g, prev, blk, dst)
        prev = dst
    return g.conv(g.view(cat, 0, (2 + n) * c), m.cv2, out=out)


def _sppf(g, x, m, out=None):
    H, W, _ = g.hwc(x)
    c_ = m.cv1.conv.out_channels
    cat = g.buffer(H, W, 4 * c_)
    g.conv(x, m.cv1, out=g.view(cat, 0, c_))
    for j in range(3):
        g.op("MAXPOOL5", g.view(cat, j * c_, c_), g.view(cat, (j + 1) * c_, c_))
    return g.conv(g.view(cat, 0, 4 * c_), m.cv2, out=out)


def _psa(g, xio, blk):
    H, W, C = g.hwc(xio)
    at = blk.attn
    heads, kd, hd = at.num_heads, at.key_dim, at.head_dim
    assert heads * hd == C
    qkv = g.conv(xio, at.qkv)
    qb = g.tens[qkv][0]
    per = 2 * kd + hd
    vbuf = g.buffer(H, W, C)
    for h in range(heads):
        g.op("COPYC", g.view(qb, h * per + 2 * kd, hd), g.view(vbuf, h * hd, hd))
    vt = g.view(vbuf, 0, C)
    ao = g.fresh(H, W, C)
    g.ops.append(("ATTN", qkv, ao, heads, kd, hd))
    pe = g.conv(vt, at.pe)
    g.op("ADD", ao, pe, ao)
    pr = g.conv(ao, at.proj)
    g.op("ADD", xio, pr, xio)
    f1 = g.conv(xio, blk.ffn[0])
    f2 = g.conv(f1, blk.ffn[1])
    g.op("ADD", xio, f2, xio)


def _c2psa(g, x, m, out=None):
    H, W, _ = g.hwc(x)
    c = m.c
    cat = g.buffer(H, W, 2 * c)
    g.conv(x, m.cv1, out=g.view(cat, 0, 2 * c))
    b = g.view(cat, c, c)
    for blk in m.m:
        _psa(g, b, blk)
    return g.conv(g.view(cat, 0, 2 * c), m.cv2, out=out)


def _chain(g, x, mod, pad8=False):
    """Flatten (nested) Sequentials of convs into CONV ops."""
    if isinstance(mod, nn.Sequential):
        for sub in mod:
            x = _chain(g, x, sub, pad8)
        return x
    return g.conv_pad8(x, mod) if pad8 else g.conv(x, mod)


def build_graph(model: "ynn.DetectionModel", S: int) -> GraphBuilder:
    """Walk the model's layer list (following each layer's ``.f``) into a GraphBuilder."""
    net = model.model
    g = GraphBuilder()
    x0 = g.fresh(S, S, 3)
    nbody = len(net) - 1

    def sources(i):
        f = net[i].f
        return [i - 1 if j == -1 else j for j in ([f] if isinstance(f, int) else f)]

    # channel / spatial size of every body layer
    ch, hw = {-1: 3}, {-1: S}
    for i in range(nbody):
        m, src = net[i], sources(i)
        ih = hw[src[0]]
        if isinstance(m, ynn.Conv):
            cv = m.conv
            ch[i] = cv.out_channels
            hw[i] = (ih + 2 * cv.padding[0] - cv.kernel_size[0]) // cv.stride[0] + 1
        elif isinstance(m, (ynn.C2f, ynn.SPPF, ynn.C2PSA)):
            ch[i], hw[i] = m.cv2.conv.out_channels, ih
        elif isinstance(m, nn.Upsample):
            ch[i], hw[i] = ch[src[0]], ih * 2
        elif isinstance(m, ynn.Concat):
            ch[i], hw[i] = sum(ch[s] for s in src), ih
        else:
            raise RuntimeError(f"unsupported module {type(m).__name__} at layer {i}")

    # concat buffers first; each producer writes its slice of the first concat it feeds
    catbuf, feed, copies = {}, {}, {}
    for i in range(nbody):
        if not isinstance(net[i], ynn.Concat):
            continue
        catbuf[i] = g.buffer(hw[i], hw[i], ch[i])
        off = 0
        for s in sources(i):
            if s in feed or s < 0 or isinstance(net[s], ynn.Concat):
                copies.setdefault(i, []).append((s, off))
            else:
                feed[s] = (catbuf[i], off, ch[s])
            off += ch[s]

    outs = {-1: x0}
    for i in range(nbody):
        m, src = net[i], sources(i)
        xin = outs[src[0]]
        dst = g.view(*feed[i]) if i in feed else None
        if isinstance(m, ynn.Conv):
            y = g.conv(xin, m, out=dst)
        elif isinstance(m, ynn.C2PSA):
            y = _c2psa(g, xin, m, out=dst)
        elif isinstance(m, ynn.SPPF):
            y = _sppf(g, xin, m, out=dst)
        elif isinstance(m, ynn.C2f):
            y = _c2f(g, xin, m, out=dst)
        elif isinstance(m, nn.Upsample):
            assert float(m.scale_factor) == 2.0
            y = g.op("UPSAMPLE2", xin, dst if dst is not None else g.fresh(hw[i], hw[i], ch[i]))
        else:
            for s, off in copies.get(i, []):
                g.op("COPYC", outs[s], g.view(catbuf[i], off, ch[s]))
            y = g.view(catbuf[i], 0, ch[i])
        outs[i] = y
        g.layer_out[i] = y

    det = net[-1]
    if isinstance(det, ynn.Classify):
        # reference export/export.py:389-397: conv -> GAP -> linear (a 1x1 CONV on the
        # [1,1,1280] pooled tensor) -> channel SOFTMAX, each into a standalone buffer
        h = g.conv(outs[nbody - 1], det.conv)
        _, _, C = g.hwc(h)
        gp = g.fresh(1, 1, C)
        g.ops.append(("GAP", h, gp))
        O, I = det.linear.weight.shape
        logits = g.fresh(1, 1, O)
        woff, boff = g._weights(det.linear.weight.detach().numpy().reshape(O, 1, 1, I),
                                det.linear.bias.detach().numpy())
        g.ops.append(("CONV", gp, logits, 1, 1, 0, 1, ACT_NONE, I, O, woff, boff))
        probs = g.fresh(1, 1, O)
        g.ops.append(("SOFTMAX", logits, probs))
        g.layer_out[len(net) - 1] = probs
        g.det_ref, g.seg_ref, g.probs = [], None, probs
        return g
    assert torch.allclose(det.dfl.conv.weight.view(-1), torch.arange(16, dtype=torch.float32))
    seg = isinstance(det, ynn.Segment)
    obb = isinstance(det, ynn.OBB)
    feats = [outs[j] for j in det.f]
    strides = [int(s) for s in det.stride]
    g.det_ref, g.seg_ref = [], None
    if seg:
        assert det.nm % 8 == 0
        t = g.conv(feats[0], det.proto.cv1)
        t = g.convT2(t, det.proto.upsample)
        t = g.conv(t, det.proto.cv2)
        proto = g.conv(t, det.proto.cv3)
        g.seg_ref = {"proto": proto, "cv4": []}
    ncpad = (det.nc + 7) // 8 * 8
    for i, (f, st) in enumerate(zip(feats, strides)):
        b = _chain(g, f, det.cv2[i])
        c = _chain(g, f, det.cv3[i][:2], pad8=True)
        c = g.conv_pad8(c, det.cv3[i][2], ncpad)
        if obb:   # angle branch: 3x3, 3x3, then the 1-channel final zero-padded to 8
            a = _chain(g, f, det.cv4[i][:2])
            a = g.conv_pad8(a, det.cv4[i][2], (det.ne + 7) // 8 * 8)
            g.ops.append(("DECODEOBB", b, c, a, st))
            g.det_ref.append((b, c, a))
        elif seg:
            mc = _chain(g, f, det.cv4[i])
            g.ops.append(("DECODESEG", b, c, mc, st))
            g.seg_ref["cv4"].append(mc)
            g.det_ref.append((b, c, mc))
        else:
            g.ops.append(("DECODE", b, c, st))
            g.det_ref.append((b, c))
    if seg:
        g.ops.append(("MASKS", proto))
    return g


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


def export_model(name: str, out_dir: str, imgsz: int = 640, frame_hw=(1080, 810),
                 frame_seed: int = 0, model=None) -> GraphBuilder:
    """Write ``out_dir`` for the seeded model ``name`` at input size ``imgsz``."""
    from .frames import synthetic_bgr
    assert imgsz % 32 == 0
    model = ynn.build_model(name, imgsz=imgsz) if model is None else model
    g = build_graph(model, imgsz)
    os.makedirs(out_dir, exist_ok=True)
    head = model.model[-1]
    task = ("segment" if isinstance(head, ynn.Segment) else
            "classify" if isinstance(head, ynn.Classify) else
            "obb" if isinstance(head, ynn.OBB) else "detect")
    nc = head.linear.out_features if task == "classify" else head.nc
    with open(os.path.join(out_dir, "model.graph"), "w") as f:
        f.write(g.graph_text(task, nc, imgsz))
    np.concatenate(g.w16).tofile(os.path.join(out_dir, "weights.f16"))
    np.concatenate(g.b32).tofile(os.path.join(out_dir, "bias.f32"))
    bgr = synthetic_bgr(*frame_hw, seed=frame_seed)
    bgr.tofile(os.path.join(out_dir, "bus_raw.u8"))
    with open(os.path.join(out_dir, "bus_raw.txt"), "w") as f:
        f.write(f"{bgr.shape[0]} {bgr.shape[1]}")
    x = classify_input(bgr, imgsz) if task == "classify" else letterbox(bgr, imgsz)
    x.astype(np.float16).tofile(os.path.join(out_dir, "input.f16"))
    if task == "classify":
        with open(os.path.join(out_dir, "names.txt"), "w") as f:
            f.write("\n".join(model.names[i] for i in range(nc)) + "\n")
    return g


def ensure_model_dir(name: str, root: str, imgsz: int = 640, frame_hw=(1080, 810)) -> str:
    """Return ``root/<name>[-S]`` (S omitted at the model's default size: 640, 224 for
    classify, 1024 for obb), exporting it first if ``model.graph`` is missing."""
    default = 224 if name.endswith("-cls") else 1024 if name.endswith("-obb") else 640
    d = os.path.join(root, name if imgsz == default else f"{name}-{imgsz}")
    if not os.path.exists(os.path.join(d, "model.graph")):
        export_model(name, d, imgsz, frame_hw)
    return d

