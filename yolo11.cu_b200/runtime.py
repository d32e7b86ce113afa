"""ctypes binding of libyolob200.so: the yolo.h engine ABI and the yk.h kernel ABI.

The library is the product; this module only declares its C signatures so Python callers
(tests, bench) reach it exactly as a C caller would.  Importing it never falls back to
anything: if the library is missing, ``load()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libyolob200.so")
CLI_PATH = os.path.join(PKG, "bin", "yolocuda")


class YkView(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("batch", C.c_int), ("H", C.c_int), ("W", C.c_int),
                ("stride", C.c_int), ("coff", C.c_int), ("C", C.c_int)]


class YkConv(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("bias", C.c_void_p), ("k", C.c_int), ("s", C.c_int),
                ("p", C.c_int), ("groups", C.c_int), ("act", C.c_int), ("Cin", C.c_int),
                ("Cout", C.c_int), ("tile", C.c_int), ("msub", C.c_int),
                ("algo", C.c_int)]


class YkLevel(C.Structure):
    _fields_ = [("box", YkView), ("cls", YkView), ("coef", YkView), ("stride", C.c_int)]


class YkPost(C.Structure):
    _fields_ = [("ws", C.c_void_p), ("ws_bytes", C.c_size_t), ("outdets", C.c_void_p),
                ("outidx", C.c_void_p), ("outcnt", C.c_void_p), ("rawcnt", C.c_void_p)]


class YoloDet(C.Structure):
    _fields_ = [("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float),
                ("score", C.c_float), ("cls", C.c_int)]


class YoloObbDet(C.Structure):
    _fields_ = [("x", C.c_float), ("y", C.c_float), ("w", C.c_float), ("h", C.c_float),
                ("angle", C.c_float), ("score", C.c_float), ("cls", C.c_int)]


class YoloOptions(C.Structure):
    _fields_ = [("device", C.c_int), ("conf", C.c_float), ("iou", C.c_float),
                ("max_det", C.c_int), ("autotune", C.c_int), ("fuse", C.c_int)]


_P = C.POINTER
_SIGS = {
    # kernel ABI (include/yk.h)
    "yk_conv": (C.c_int, [_P(YkView), _P(YkView), _P(YkView), _P(YkConv), C.c_void_p]),
    "yk_im2col": (C.c_int, [_P(YkView), _P(YkView), C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "yk_maxpool5": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_maxpool5x3": (C.c_int, [_P(YkView)] * 4 + [C.c_void_p]),
    "yk_upsample2": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_ps2": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_copyc": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_add": (C.c_int, [_P(YkView), _P(YkView), _P(YkView), C.c_void_p]),
    "yk_attn": (C.c_int, [_P(YkView), _P(YkView), C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "yk_letterbox": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _P(YkView), C.c_int,
                               _P(C.c_float), _P(C.c_int), _P(C.c_int), C.c_void_p]),
    "yk_letterbox_batch": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int,
                                     _P(YkView), C.c_int, _P(C.c_float), _P(C.c_int),
                                     _P(C.c_int), C.c_void_p]),
    "yk_post_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "yk_obb_workspace_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "yk_decode_obb": (C.c_int, [_P(YkLevel), C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p,
                                C.c_void_p]),
    "yk_nms_obb": (C.c_int, [C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p, C.c_void_p,
                             C.c_void_p, C.c_void_p, C.c_void_p]),
    "yk_gap": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_softmax": (C.c_int, [_P(YkView), _P(YkView), C.c_void_p]),
    "yk_preprocess_cls": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _P(YkView), C.c_int,
                                    _P(C.c_int), C.c_void_p]),
    "yk_decode": (C.c_int, [_P(YkLevel), C.c_int, C.c_int, C.c_int, C.c_float, _P(YkPost),
                            C.c_void_p]),
    "yk_nms": (C.c_int, [C.c_int, C.c_int, C.c_float, C.c_int, _P(YkPost), C.c_void_p]),
    "yk_masks": (C.c_int, [_P(YkLevel), C.c_int, _P(YkView), C.c_int, C.c_int, C.c_int,
                           _P(YkPost), C.c_void_p, C.c_void_p]),
    "yk_decode_nms_static": (C.c_int, [_P(YkLevel), C.c_int, C.c_int, C.c_int, C.c_float,
                                       C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p]),
    "yk_fetch_device_error": (C.c_int, []),
    "yk_test_inject": (C.c_int, [C.c_int, C.c_ulonglong]),
    "yk_test_nms_cluster": (C.c_int, [C.c_int]),
    "yk_last_cuda_error": (C.c_char_p, []),
    "yk_launch_count": (C.c_longlong, []),
    # engine ABI (include/yolo.h)
    "yolo_create": (C.c_void_p, [C.c_char_p, C.c_int]),
    "yolo_task": (C.c_int, [C.c_void_p]),
    "yolo_exec_ms": (C.c_float, [C.c_void_p, C.c_int]),
    "yolo_stream": (C.c_void_p, [C.c_void_p]),
    "yolo_preprocess": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "yolo_run": (None, [C.c_void_p, C.c_int]),
    "yolo_run_async": (None, [C.c_void_p, C.c_int]),
    "yolo_sync": (None, [C.c_void_p]),
    "yolo_get": (C.c_int, [C.c_void_p, C.c_int, _P(YoloDet), C.c_int]),
    "yolo_preprocess_cls": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "yolo_preprocess_jpeg": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.c_int]),
    "yolo_get_cls": (C.c_int, [C.c_void_p, C.c_int, _P(C.c_int), _P(C.c_float), C.c_int]),
    "yolo_get_obb": (C.c_int, [C.c_void_p, C.c_int, _P(YoloObbDet), C.c_int]),
    "yolo_slot_geom": (None, [C.c_void_p, C.c_int, _P(C.c_float), _P(C.c_int), _P(C.c_int)]),
    "yolo_mask_dim": (None, [C.c_void_p, _P(C.c_int), _P(C.c_int)]),
    "yolo_get_mask": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "yolo_default_options": (None, [_P(YoloOptions)]),
    "yolo_create_ex": (C.c_void_p, [C.c_char_p, C.c_int, _P(YoloOptions)]),
    "yolo_destroy": (None, [C.c_void_p]),
    "yolo_last_error": (C.c_char_p, []),
    "yolo_raw_count": (C.c_int, [C.c_void_p, C.c_int]),
    "yolo_bind_frames": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                   C.c_int]),
    "yolo_run_frames_async": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "yolo_run_frames": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "yolo_frames_exec_ms": (C.c_float, [C.c_void_p, C.c_int, C.c_int]),
    "yolo_graph_kernels": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "yolo_conv_exec_ms": (C.c_float, [C.c_void_p, C.c_int, _P(C.c_int)]),
    "yolo_get_frames": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _P(YoloDet), C.c_int,
                                  _P(C.c_int)]),
    "yolo_get_batch": (C.c_int, [C.c_void_p, C.c_int, _P(YoloDet), C.c_int, _P(C.c_int)]),
    "yolo_run_op": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "yolo_num_ops": (C.c_int, [C.c_void_p]),
    "yolo_tensor_view": (C.c_int, [C.c_void_p, C.c_int, _P(C.c_void_p), _P(C.c_int),
                                   _P(C.c_int), _P(C.c_int), _P(C.c_int), _P(C.c_int)]),
    "yolo_read_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "yolo_write_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "yolo_profile": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _P(C.c_float), C.c_int]),
    "yolo_op_desc": (C.c_char_p, [C.c_void_p, C.c_int, _P(C.c_int)]),
    "yolo_op_shape": (C.c_int, [C.c_void_p, C.c_int, _P(C.c_int)]),
}

_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the engine library (raises OSError if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise OSError(f"{path} not built: run yolo11.cu_b200/build.py (or __graft_entry__.build())")
        lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args
        _lib = lib
    return _lib


def exported_symbols():
    return list(_SIGS)


def view(ptr, batch, H, W, stride, coff, Cv) -> YkView:
    return YkView(C.c_void_p(ptr), batch, H, W, stride, coff, Cv)


def tview(t, coff: int = 0, Cv: int | None = None) -> YkView:
    """YkView over a contiguous torch fp16 tensor [B, H, W, Ctot]."""
    B, H, W, Ct = t.shape
    return view(t.data_ptr(), B, H, W, Ct, coff, Ct - coff if Cv is None else Cv)


def np_contig(a):
    import numpy as np
    return np.ascontiguousarray(a)


class Engine:
    """Thin owner of a yolo_* handle (device = current CUDA device unless given)."""

    def __init__(self, model_dir: str, max_batch: int = 1, *, device: int = -1, conf=0.25,
                 iou=0.45, max_det=300, autotune=True, fuse=True):
        self.lib = load()
        o = YoloOptions()
        self.lib.yolo_default_options(C.byref(o))
        o.device, o.conf, o.iou, o.max_det = device, conf, iou, max_det
        o.autotune, o.fuse = int(autotune), int(fuse)
        self.max_det = max_det
        self.device = device
        self.h = self.lib.yolo_create_ex(model_dir.encode(), max_batch, C.byref(o))
        if not self.h:
            raise RuntimeError("yolo_create failed: " + self.lib.yolo_last_error().decode())
        self.max_batch = max_batch

    def close(self):
        if self.h:
            self.lib.yolo_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self):
        err = self.lib.yolo_last_error().decode()
        if err:
            raise RuntimeError(err)

    @property
    def stream(self) -> int:
        return self.lib.yolo_stream(self.h) or 0

    def preprocess(self, dev_bgr_ptr: int, h: int, w: int, slot: int):
        self.lib.yolo_preprocess(self.h, C.c_void_p(dev_bgr_ptr), h, w, slot)

    def preprocess_jpeg(self, data: bytes, slot: int) -> int:
        return self.lib.yolo_preprocess_jpeg(self.h, data, len(data), slot)

    def preprocess_cls(self, dev_bgr_ptr: int, h: int, w: int, slot: int):
        self.lib.yolo_preprocess_cls(self.h, C.c_void_p(dev_bgr_ptr), h, w, slot)

    def preprocess_host_batch(self, bgrs, slots):
        """preprocess_host for several frames: all uploads, then all preprocessing, one sync."""
        import torch
        dev = self.device if self.device >= 0 else torch.cuda.current_device()
        bufs = [torch.from_numpy(np_contig(b)).to(f"cuda:{dev}") for b in bgrs]
        cls = self.task() == 2
        for d, b, s in zip(bufs, bgrs, slots):
            h, w = b.shape[:2]
            if cls:
                self.preprocess_cls(d.data_ptr(), h, w, s)
            else:
                self.preprocess(d.data_ptr(), h, w, s)
        self.sync()
        self._check()

    def preprocess_host(self, bgr, slot: int):
        """Preprocess a host BGR u8 HWC frame (numpy) into `slot` with the task's own
        preprocessing: the frame goes to a device buffer of the handle's GPU first, which
        is held until the engine stream has consumed it."""
        import torch
        dev = self.device if self.device >= 0 else torch.cuda.current_device()
        d = torch.from_numpy(np_contig(bgr)).to(f"cuda:{dev}")
        h, w = bgr.shape[:2]
        if self.task() == 2:
            self.preprocess_cls(d.data_ptr(), h, w, slot)
        else:
            self.preprocess(d.data_ptr(), h, w, slot)
        self.sync()
        self._check()

    def task(self) -> int:
        return self.lib.yolo_task(self.h)

    def get_obb(self, slot: int, cap: int | None = None):
        cap = self.max_det if cap is None else cap
        arr = (YoloObbDet * cap)()
        n = self.lib.yolo_get_obb(self.h, slot, arr, cap)
        return [(d.x, d.y, d.w, d.h, d.angle, d.score, d.cls) for d in arr[:n]]

    def get_cls(self, slot: int, k: int = 5):
        ids, probs = (C.c_int * k)(), (C.c_float * k)()
        n = self.lib.yolo_get_cls(self.h, slot, ids, probs, k)
        return list(ids[:n]), list(probs[:n])

    def bind_frames(self, id: int, ptr: int, h: int, w: int, count: int, host: bool):
        if self.lib.yolo_bind_frames(self.h, id, C.c_void_p(ptr), h, w, count, int(host)) != 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())

    def run_frames_async(self, id: int, B: int):
        if self.lib.yolo_run_frames_async(self.h, id, B) != 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())

    def run_frames(self, id: int, B: int):
        if self.lib.yolo_run_frames(self.h, id, B) != 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())

    def frames_exec_ms(self, id: int, B: int) -> float:
        return self.lib.yolo_frames_exec_ms(self.h, id, B)

    def get_frames(self, id: int, B: int, cap: int | None = None):
        """Detections of slots 0..B-1 from binding id's most recent run (one C call)."""
        cap = self.max_det if cap is None else cap
        arr = (YoloDet * (cap * B))()
        cnt = (C.c_int * B)()
        if self.lib.yolo_get_frames(self.h, id, B, arr, cap, cnt) < 0:
            raise RuntimeError("yolo_get_frames failed")
        return [[(d.x1, d.y1, d.x2, d.y2, d.score, d.cls) for d in arr[s * cap:s * cap + cnt[s]]]
                for s in range(B)]

    def get_batch(self, B: int, cap: int | None = None):
        """Detections of slots 0..B-1 (one C call): list of per-slot lists."""
        cap = self.max_det if cap is None else cap
        arr = (YoloDet * (cap * B))()
        cnt = (C.c_int * B)()
        if self.lib.yolo_get_batch(self.h, B, arr, cap, cnt) < 0:
            raise RuntimeError("yolo_get_batch failed")
        return [[(d.x1, d.y1, d.x2, d.y2, d.score, d.cls) for d in arr[s * cap:s * cap + cnt[s]]]
                for s in range(B)]

    def run(self, B: int):
        self.lib.yolo_run(self.h, B)

    def run_async(self, B: int):
        self.lib.yolo_run_async(self.h, B)

    def sync(self):
        self.lib.yolo_sync(self.h)

    def exec_ms(self, B: int) -> float:
        return self.lib.yolo_exec_ms(self.h, B)

    def get(self, slot: int, cap: int | None = None):
        cap = self.max_det if cap is None else cap
        arr = (YoloDet * cap)()
        n = self.lib.yolo_get(self.h, slot, arr, cap)
        return [(d.x1, d.y1, d.x2, d.y2, d.score, d.cls) for d in arr[:n]]

    def raw_count(self, slot: int) -> int:
        return self.lib.yolo_raw_count(self.h, slot)

    def slot_geom(self, slot: int):
        s, t, l = C.c_float(), C.c_int(), C.c_int()
        self.lib.yolo_slot_geom(self.h, slot, C.byref(s), C.byref(t), C.byref(l))
        return s.value, t.value, l.value

    def mask_dim(self):
        ph, pw = C.c_int(), C.c_int()
        self.lib.yolo_mask_dim(self.h, C.byref(ph), C.byref(pw))
        return ph.value, pw.value

    def get_mask(self, slot: int, det: int):
        import numpy as np
        ph, pw = self.mask_dim()
        out = np.zeros((ph, pw), np.uint8)
        r = self.lib.yolo_get_mask(self.h, slot, det, out.ctypes.data_as(C.c_void_p))
        return out if r == 0 else None

    def num_ops(self) -> int:
        return self.lib.yolo_num_ops(self.h)

    def run_op(self, k: int, B: int) -> int:
        r = self.lib.yolo_run_op(self.h, k, B)
        if r < 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())
        return r

    def read(self, t: int, B: int = 1):
        """Graph tensor view t of images 0..B-1 as fp16 numpy [B, H, W, C]."""
        import numpy as np
        _, H, W, _, _, Cv = self.tensor_view(t)
        out = np.empty((B, H, W, Cv), np.float16)
        if self.lib.yolo_read_tensor(self.h, t, B, out.ctypes.data_as(C.c_void_p)) != 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())
        return out

    def write(self, t: int, arr):
        import numpy as np
        a = np.ascontiguousarray(arr, np.float16)
        if a.ndim == 3:
            a = a[None]
        if self.lib.yolo_write_tensor(self.h, t, a.shape[0], a.ctypes.data_as(C.c_void_p)) != 0:
            raise RuntimeError(self.lib.yolo_last_error().decode())

    def tensor_view(self, t: int):
        p = C.c_void_p()
        H, W, s, c, Cv = (C.c_int() for _ in range(5))
        if self.lib.yolo_tensor_view(self.h, t, C.byref(p), C.byref(H), C.byref(W), C.byref(s),
                                     C.byref(c), C.byref(Cv)) != 0:
            raise IndexError(t)
        return p.value, H.value, W.value, s.value, c.value, Cv.value
