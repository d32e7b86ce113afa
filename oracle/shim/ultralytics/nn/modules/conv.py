"""Shim: ultralytics.nn.modules.conv names backed by the repository's module zoo."""
from yolo11_cu_b200_nn import Conv, DWConv, Concat  # noqa: F401
