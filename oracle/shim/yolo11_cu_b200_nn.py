"""Shim helper: imports the repository's module zoo (``yolo11.cu_b200/nn.py``) by path."""
import importlib.util
import os
import sys

_p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "yolo11.cu_b200", "nn.py")
_spec = importlib.util.spec_from_file_location("_yolo_b200_nn_impl", _p)
_mod = importlib.util.module_from_spec(_spec)
sys.modules["_yolo_b200_nn_impl"] = _mod
_spec.loader.exec_module(_mod)
globals().update({k: getattr(_mod, k) for k in dir(_mod) if not k.startswith("__")})
