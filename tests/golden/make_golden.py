"""Regenerate the golden fixtures under tests/golden/ from the REFERENCE's own exporter.

Runs the unmodified reference ``export/export.py`` (copied to a temp dir, never into this
repo) with the test-only ``ultralytics`` shim (oracle/shim) on this repository's seeded
random-init models, at small input sizes, and keeps:

    <model>-<S>/model.graph      the reference exporter's graph text
    <model>-<S>/digests.json     sha256 of weights.f16 / bias.f32 / input.f16 / bus_raw.u8
    <model>-<S>/input.f16        the reference's letterboxed input (cv2 INTER_LINEAR)
    <model>-<S>/refs.npz         per-op reference outputs opNNN (fp16: the reference rounds
                                 every op output through fp16 in this mode, so this is lossless)
    <model>-<S>/final.npy        the shim model's head output

Needs the reference checkout (build container only):
    python tests/golden/make_golden.py [--ref <reference checkout>]
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import json
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CASES = [("yolo11n", 64), ("yolov8n", 64), ("yolo11n-seg", 64), ("yolo11n", 160),
         ("yolo11n-cls", 224), ("yolo11n-obb", 128)]


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        h.update(f.read())
    return h.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("YOLO_REFERENCE_DIR"),
                    help="reference checkout (default: $YOLO_REFERENCE_DIR)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref <reference checkout> or set YOLO_REFERENCE_DIR")
    sys.path.insert(0, os.path.join(ROOT, "yolo11.cu_b200"))
    import cv2
    import frames  # noqa: E402  (the package's frame generator, imported by path)

    tmp = tempfile.mkdtemp(prefix="refexport_")
    try:
        os.makedirs(os.path.join(tmp, "export"))
        os.makedirs(os.path.join(tmp, "assets"))
        shutil.copy(os.path.join(args.ref, "export", "export.py"), os.path.join(tmp, "export"))
        png = os.path.join(tmp, "assets", "bus.png")
        cv2.imwrite(png, frames.synthetic_bgr(1080, 810, 0))
        os.replace(png, os.path.join(tmp, "assets", "bus.jpg"))    # PNG bytes; cv2 sniffs
        env = dict(os.environ, SHIM_ASSETS=os.path.join(tmp, "assets"),
                   PYTHONPATH=os.path.join(ROOT, "oracle", "shim"))
        for model, S in CASES:
            r = subprocess.run([sys.executable, os.path.join(tmp, "export", "export.py"), model,
                                str(S)], env=env, capture_output=True, text=True)
            if r.returncode:
                raise SystemExit(r.stdout + r.stderr)
            print(r.stdout.strip().splitlines()[-2])
            src = os.path.join(tmp, "build", model if S == 640 else f"{model}-{S}")
            dst = os.path.join(HERE, f"{model}-{S}")
            os.makedirs(dst, exist_ok=True)
            shutil.copy(os.path.join(src, "model.graph"), dst)
            shutil.copy(os.path.join(src, "input.f16"), dst)
            dig = {f: sha256(os.path.join(src, f))
                   for f in ("weights.f16", "bias.f32", "input.f16", "bus_raw.u8")}
            with open(os.path.join(dst, "digests.json"), "w") as f:
                json.dump(dig, f, indent=1, sort_keys=True)
            refs = {}
            for p in sorted(glob.glob(os.path.join(src, "ref", "op*.npy"))):
                a = np.load(p)
                h = a.astype(np.float16)
                assert np.array_equal(h.astype(np.float32), a), p   # fp16-rounded by the reference
                refs[os.path.basename(p)[:-4]] = h
            np.savez_compressed(os.path.join(dst, "refs.npz"), **refs)
            np.save(os.path.join(dst, "final.npy"), np.load(os.path.join(src, "ref", "final.npy")))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
