"""Shim: ultralytics.nn.modules.head names backed by the repository's module zoo."""
from yolo11_cu_b200_nn import Classify, Detect, Segment  # noqa: F401


class OBB(Detect):      # never instantiated here; only used in isinstance checks
    pass

