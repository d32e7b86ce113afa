"""Test-only stand-in for the ``ultralytics`` package (ORACLE INFRASTRUCTURE, never shipped).

The reference exporter (``export/export.py``) and seg checker (``test/compare_seg.py``)
import ``ultralytics``, which is not installed here.  This shim exposes exactly the names
they touch and backs them with this repository's seeded random-init modules, so the
reference's own exporter, fp32 graph interpreter and level-1 decomposition assert run
unmodified on the same weights the engine is tested with.  The model is chosen by the
``.pt`` file stem (the file itself need not exist), e.g. ``YOLO('x/yolo11n.pt')``.
"""
import os
from pathlib import Path

__version__ = "0.0-shim"


class YOLO:
    def __init__(self, path):
        from yolo11_cu_b200_nn import build_model
        name = Path(str(path)).stem
        self.model = build_model(name, imgsz=int(os.environ.get("SHIM_IMGSZ", "640")))
        self.names = self.model.names
