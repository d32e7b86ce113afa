"""Shim: ultralytics.nn.modules.head names backed by the repository's module zoo."""
from yolo11_cu_b200_nn import OBB, Classify, Detect, Segment  # noqa: F401

