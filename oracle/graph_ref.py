"""ORACLE / TEST INFRASTRUCTURE — torch fp32 interpreter of a model directory.

A CPU restatement of the reference's graph interpreter ``run_reference``
(``export/export.py:446-526``): every op of ``model.graph`` executed with torch fp32 on
[C, H, W] buffers, weights from ``weights.f16`` (fp16 values as fp32), biases from
``bias.f32``.  With ``round_fp16=True`` every op output is rounded through fp16 before it
is stored, exactly like the reference's per-op dump mode (``export/export.py:451-460``),
so op k's output is the reference's ``ref/opNNN.npy`` for op k.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use this module; it is
the checker, never the product.  Pinned against the reference's own exporter run on the same
weights (tests/golden/, tests/test_oracle_golden.py).

Also provides ``oracle_postproc`` (ctypes binding of postproc_ref.c) for decode / NMS /
masks / letterbox.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


class Graph:
    def __init__(self, model_dir: str):
        with open(os.path.join(model_dir, "model.graph")) as f:
            toks = f.read().split("\n")
        lines = [l.split() for l in toks if l.strip()]
        i = 0
        assert lines[0][0] == "YOLO11GRAPH"
        ver = int(lines[0][1])
        i = 1
        self.task, self.nc = "detect", 80
        if ver >= 2:
            _, self.task, nc, S = lines[1]
            self.nc = int(nc)
            i = 2
        nb, nt, no = map(int, lines[i])
        i += 1
        self.bufs = [tuple(map(int, l[1:4])) for l in lines[i:i + nb]]
        i += nb
        self.tens = [tuple(map(int, l[1:4])) for l in lines[i:i + nt]]
        i += nt
        self.ops = []
        for l in lines[i:i + no]:
            kind = l[0]
            self.ops.append((kind,) + tuple(int(v) for v in l[1:]))
        self.w16 = np.fromfile(os.path.join(model_dir, "weights.f16"), np.float16)
        self.b32 = np.fromfile(os.path.join(model_dir, "bias.f32"), np.float32)
        self.S = self.bufs[self.tens[0][0]][0]

    def out_tensor(self, k: int):
        op = self.ops[k]
        if op[0] in ("DECODE", "DECODESEG", "DECODEOBB", "MASKS"):
            return None
        return op[3] if op[0] == "ADD" else op[2]

    def levels(self):
        """[(box tensor, cls tensor, coef / angle tensor or None, stride)] in graph order."""
        out = []
        for op in self.ops:
            if op[0] == "DECODE":
                out.append((op[1], op[2], None, op[3]))
            elif op[0] in ("DECODESEG", "DECODEOBB"):   # third view: coefs / angle
                out.append((op[1], op[2], op[3], op[4]))
        return out

    def proto(self):
        for op in self.ops:
            if op[0] == "MASKS":
                return op[1]
        return None


def run_graph(g: Graph, x_hwc: np.ndarray, round_fp16: bool = True, inject=None,
              upto: int | None = None):
    """Run the graph on one image (x_hwc: [S, S, 3] float).  Returns (bufs, outs) where
    outs[k] is op k's output view as NHWC float32 (None for decode/masks ops).

    inject(k) -> array or None: if it returns an array, op k's output is replaced by it
    before later ops run (per-op isolation, like the reference's dump resync)."""
    torch.set_grad_enabled(False)
    bufs = [torch.zeros(C_, H, W) for (H, W, C_) in g.bufs]

    def rd(t):
        b, o, c = g.tens[t]
        return bufs[b][o:o + c]

    def wr(t, v):
        b, o, c = g.tens[t]
        v = torch.as_tensor(v, dtype=torch.float32)
        if round_fp16:
            v = v.half().float()
        bufs[b][o:o + c] = v

    wr(0, torch.from_numpy(np.asarray(x_hwc, np.float32).transpose(2, 0, 1).copy()))
    w32 = g.w16.astype(np.float32)
    outs = []
    for k, op in enumerate(g.ops):
        if upto is not None and k >= upto:
            break
        kind = op[0]
        if kind == "CONV":
            _, x, out, kk, s, p, gr, a, Cin, O, woff, boff = op
            Ig = Cin // gr
            w = torch.from_numpy(w32[woff:woff + O * kk * kk * Ig]).view(O, kk, kk, Ig).permute(0, 3, 1, 2)
            b = torch.from_numpy(g.b32[boff:boff + O].copy())
            y = F.conv2d(rd(x)[None], w.contiguous(), b, stride=s, padding=p, groups=gr)[0]
            if a == 1:
                y = F.silu(y)
            wr(out, y)
        elif kind == "ADD":
            _, a_, b_, out = op
            wr(out, rd(a_) + rd(b_))
        elif kind == "MAXPOOL5":
            _, x, out = op
            wr(out, F.max_pool2d(rd(x)[None], 5, 1, 2)[0])
        elif kind == "UPSAMPLE2":
            _, x, out = op
            wr(out, F.interpolate(rd(x)[None], scale_factor=2, mode="nearest")[0])
        elif kind == "PS2":
            _, x, out = op
            v = rd(x)
            Cq = v.shape[0] // 4
            H, W = v.shape[1:]
            y = torch.zeros(Cq, 2 * H, 2 * W)
            for di in range(2):
                for dj in range(2):
                    q = 2 * di + dj
                    y[:, di::2, dj::2] = v[q * Cq:(q + 1) * Cq]
            wr(out, y)
        elif kind == "COPYC":
            _, x, out = op
            wr(out, rd(x))
        elif kind == "ATTN":
            _, qkv, out, heads, kd, hd = op
            q = rd(qkv)
            H, W = q.shape[1:]
            N = H * W
            t = q.reshape(1, heads, 2 * kd + hd, N)
            q_, k_, v_ = t.split([kd, kd, hd], dim=2)
            att = ((q_.transpose(-2, -1) @ k_) * (kd ** -0.5)).softmax(dim=-1)
            wr(out, (v_ @ att.transpose(-2, -1)).reshape(heads * hd, H, W))
        elif kind == "GAP":             # export/export.py:501-502: mean over H, W
            _, x, out = op
            wr(out, rd(x).mean(dim=(1, 2), keepdim=True))
        elif kind == "SOFTMAX":         # export/export.py:503-504: channel softmax of [C,1,1]
            _, x, out = op
            wr(out, rd(x).softmax(dim=0))
        elif kind in ("DECODE", "DECODESEG", "DECODEOBB", "MASKS"):
            outs.append(None)
            continue
        else:
            raise RuntimeError(f"oracle: unsupported op {kind}")
        t = g.out_tensor(k)
        if inject is not None:
            v = inject(k)
            if v is not None:
                b, o, c = g.tens[t]
                bufs[b][o:o + c] = torch.from_numpy(np.asarray(v, np.float32).transpose(2, 0, 1).copy())
        outs.append(rd(t).permute(1, 2, 0).numpy().copy())
    return bufs, outs


def tensor_hwc(g: Graph, bufs, t: int) -> np.ndarray:
    b, o, c = g.tens[t]
    return bufs[b][o:o + c].permute(1, 2, 0).numpy().copy()


# ---------------- C post-processing oracle ----------------
_lib = None


def oracle_postproc():
    global _lib
    if _lib is None:
        so = os.path.join(HERE, "_build", "liboracle.so")
        src = os.path.join(HERE, "postproc_ref.c")
        if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
        lib = C.CDLL(so)
        lib.oref_decode_level.restype = C.c_int
        lib.oref_decode_level.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                          C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]
        lib.oref_nms.restype = C.c_int
        lib.oref_nms.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_void_p]
        lib.oref_mask.restype = None
        lib.oref_mask.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_void_p, C.c_float, C.c_float, C.c_void_p]
        lib.oref_letterbox.restype = None
        lib.oref_letterbox.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        lib.oref_letterbox_geom.restype = None
        lib.oref_letterbox_geom.argtypes = [C.c_int, C.c_int, C.c_int] + [C.c_void_p] * 5
        lib.oref_probiou.restype = C.c_float
        lib.oref_probiou.argtypes = [C.c_void_p, C.c_void_p]
        for n in ("oref_exp", "oref_sigmoid", "oref_sin", "oref_cos", "oref_log"):
            getattr(lib, n).restype = C.c_float
            getattr(lib, n).argtypes = [C.c_float]
        lib.oref_decode_obb_level.restype = C.c_int
        lib.oref_decode_obb_level.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                              C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]
        lib.oref_nms_obb.restype = C.c_int
        lib.oref_nms_obb.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_void_p]
        lib.oref_preprocess_cls.restype = None
        lib.oref_preprocess_cls.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                            C.c_void_p]
        lib.oref_quot_gt.restype = None
        lib.oref_quot_gt.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        lib.oref_div255_check.restype = C.c_long
        lib.oref_div255_check.argtypes = [C.c_uint, C.c_uint, C.c_uint]
        lib.oref_f2h.restype = C.c_uint16
        lib.oref_f2h.argtypes = [C.c_float]
        _lib = lib
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def preprocess_cls(bgr: np.ndarray, S: int):
    """Classify preprocessing (C oracle): ([S, S, 3] fp16 RGB, (rh, rw, top, left))."""
    lib = oracle_postproc()
    bgr = np.ascontiguousarray(bgr, np.uint8)
    out = np.zeros((S, S, 3), np.uint16)
    geom = np.zeros(4, np.int32)
    lib.oref_preprocess_cls(_p(bgr), bgr.shape[0], bgr.shape[1], S, _p(out), _p(geom))
    return out.view(np.float16), tuple(int(v) for v in geom)


def letterbox(bgr: np.ndarray, S: int) -> np.ndarray:
    """fp16 [S, S, 3] (reference k_preprocess formula)."""
    lib = oracle_postproc()
    bgr = np.ascontiguousarray(bgr, np.uint8)
    out = np.zeros((S, S, 3), np.uint16)
    lib.oref_letterbox(_p(bgr), bgr.shape[0], bgr.shape[1], S, _p(out))
    return out.view(np.float16)


def decode_obb(levels, nc: int, conf: float = 0.25):
    """levels: [(box fp16 [H,W,64], cls fp16 [H,W,>=nc], angle fp16 [H,W,>=1], stride)] of
    one image.  Returns [n, 8] float32 (cx cy w h score cls theta anchor), anchor order."""
    lib = oracle_postproc()
    recs, abase = [], 0
    for box, cls, ang, st in levels:
        box, cls, ang = (np.ascontiguousarray(t, np.float16) for t in (box, cls, ang))
        H, W = box.shape[:2]
        out = np.zeros((H * W, 8), np.float32)
        n = lib.oref_decode_obb_level(_p(box), box.shape[2], _p(cls), cls.shape[2], _p(ang),
                                      ang.shape[2], H, W, 0, nc, st, conf, abase, _p(out))
        recs.append(out[:n])
        abase += H * W
    return np.concatenate(recs) if recs else np.zeros((0, 8), np.float32)


def nms_obb(recs: np.ndarray, iou: float, max_out: int = 300) -> np.ndarray:
    lib = oracle_postproc()
    recs = np.ascontiguousarray(recs, np.float32)
    out = np.zeros((max(len(recs), 1), 8), np.float32)
    m = lib.oref_nms_obb(_p(recs), len(recs), iou, max_out, _p(out))
    return out[:m]


def decode(levels, nc: int, conf: float = 0.25):
    """levels: [(box fp16 [H,W,64], cls fp16 [H,W,>=nc], stride)] of one image.
    Returns [n, 7] float32 records (x1 y1 x2 y2 score cls anchor) in anchor order."""
    lib = oracle_postproc()
    recs, abase = [], 0
    for box, cls, st in levels:
        box = np.ascontiguousarray(box, np.float16)
        cls = np.ascontiguousarray(cls, np.float16)
        H, W = box.shape[:2]
        out = np.zeros((H * W, 7), np.float32)
        n = lib.oref_decode_level(_p(box), box.shape[2], _p(cls), cls.shape[2], H, W, 0, nc,
                                  st, conf, abase, _p(out))
        recs.append(out[:n])
        abase += H * W
    return np.concatenate(recs) if recs else np.zeros((0, 7), np.float32)


def nms(recs: np.ndarray, iou: float, max_out: int = 300) -> np.ndarray:
    lib = oracle_postproc()
    recs = np.ascontiguousarray(recs, np.float32)
    out = np.zeros((max(max_out, 1), 7), np.float32)
    n = lib.oref_nms(_p(recs), len(recs), iou, max_out, _p(out))
    return out[:n]


def mask(coef: np.ndarray, proto: np.ndarray, det, S: int) -> np.ndarray:
    """coef fp16 [nm]; proto fp16 [Ph, Pw, nm]; det x1 y1 x2 y2 (letterbox px)."""
    lib = oracle_postproc()
    coef = np.ascontiguousarray(coef, np.float16)
    proto = np.ascontiguousarray(proto, np.float16)
    Ph, Pw, nm = proto.shape
    d = np.ascontiguousarray(np.asarray(det[:4], np.float32))
    out = np.zeros((Ph, Pw), np.uint8)
    lib.oref_mask(_p(coef), nm, _p(proto), nm, Ph, Pw, 0, _p(d), np.float32(Pw) / np.float32(S),
                  np.float32(Ph) / np.float32(S), _p(out))
    return out
