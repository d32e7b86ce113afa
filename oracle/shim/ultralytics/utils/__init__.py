"""Shim: ``ASSETS`` points at a folder whose ``bus.jpg`` holds the synthetic frame (PNG bytes)."""
import os
from pathlib import Path

ASSETS = Path(os.environ.get("SHIM_ASSETS", "/nonexistent"))
