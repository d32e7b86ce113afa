"""Seeded synthetic uint8 frames: smooth per-channel gradients plus 12 filled rectangles.

Frames stand in for the reference's bus.jpg / video inputs (no image datasets exist on these
machines).  Generation is pure numpy PCG64 integer arithmetic, so every machine produces the
same bytes.  ``synthetic_frame`` returns RGB; the engine ABI (``yolo_preprocess``) takes BGR,
so callers use ``to_bgr`` (or ``synthetic_bgr``) before upload.
"""
from __future__ import annotations

import numpy as np


def synthetic_frame(h: int, w: int, seed: int = 0) -> np.ndarray:
    """RGB uint8 [h, w, 3]."""
    rng = np.random.Generator(np.random.PCG64(seed))
    yy = np.arange(h, dtype=np.float64)[:, None] / max(h - 1, 1)
    xx = np.arange(w, dtype=np.float64)[None, :] / max(w - 1, 1)
    img = np.empty((h, w, 3), np.float64)
    for c in range(3):
        a, b, ph = rng.uniform(-1, 1), rng.uniform(-1, 1), rng.uniform(0, 2 * np.pi)
        fr = rng.uniform(0.5, 3.0)
        img[:, :, c] = 127.5 + 60 * (a * yy + b * xx) + 50 * np.sin(2 * np.pi * fr * (xx + yy) + ph)
    img = np.clip(np.rint(img), 0, 255).astype(np.uint8)
    for _ in range(12):
        rh, rw = int(rng.integers(h // 20, h // 3 + 1)), int(rng.integers(w // 20, w // 3 + 1))
        y0, x0 = int(rng.integers(0, h - rh + 1)), int(rng.integers(0, w - rw + 1))
        img[y0:y0 + rh, x0:x0 + rw] = rng.integers(0, 256, 3, dtype=np.uint8)
    return img


def to_bgr(rgb: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(rgb[..., ::-1])


def synthetic_bgr(h: int, w: int, seed: int = 0) -> np.ndarray:
    return to_bgr(synthetic_frame(h, w, seed))
