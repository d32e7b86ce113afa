"""Shim: ultralytics.nn.modules.block names backed by the repository's module zoo."""
from yolo11_cu_b200_nn import (Bottleneck, C2f, C3, C3k, C3k2, SPPF, C2PSA, PSABlock,  # noqa: F401
                               Attention, DFL, Proto)
