"""Pins the exporter and the oracle against the reference's own exporter output.

The golden fixtures (tests/golden/make_golden.py) were produced by running the reference's
unmodified export/export.py on the same seeded models.  Here:
  * this package's exporter must reproduce the reference's model.graph and weights / bias /
    input bytes exactly (sha256);
  * the oracle interpreter (oracle/graph_ref.py) must reproduce the reference interpreter's
    per-op outputs (export/export.py:446-526, fp16-rounded mode) on that graph.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_cases

import graph_ref


def _sha(p):
    with open(p, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


@pytest.mark.parametrize("case", golden_cases())
def test_exporter_matches_reference(case, golden_dirs):
    d, g = golden_dirs[case], os.path.join(GOLDEN, case)
    assert open(os.path.join(d, "model.graph")).read() == open(os.path.join(g, "model.graph")).read()
    dig = json.load(open(os.path.join(g, "digests.json")))
    for f, h in dig.items():
        assert _sha(os.path.join(d, f)) == h, f


@pytest.mark.parametrize("case", golden_cases())
def test_oracle_interpreter_matches_reference(case, golden_dirs):
    d, g = golden_dirs[case], os.path.join(GOLDEN, case)
    graph = graph_ref.Graph(d)
    x = np.fromfile(os.path.join(g, "input.f16"), np.float16).reshape(graph.S, graph.S, 3)
    refs = np.load(os.path.join(g, "refs.npz"))
    _, outs = graph_ref.run_graph(graph, x.astype(np.float32), round_fp16=True)
    n = 0
    for k, o in enumerate(outs):
        if o is None:
            continue
        r = refs[f"op{k:03d}"].astype(np.float32)
        assert o.shape == r.shape, k
        # same fp32 math up to summation order; values are fp16-rounded on both sides
        scale = np.abs(r).max() + 1e-6
        assert np.abs(o - r).max() / scale < 2e-3, (k, np.abs(o - r).max() / scale)
        n += 1
    assert n == len(refs.files)


def test_classify_preprocess_oracle_vs_torchvision(pkg):
    """The C classify preprocessing (geometry + antialiased triangle filter) against the
    torchvision path the reference exporter uses for input.f16: same resized size and crop,
    and within 2/255 per channel (PIL rounds its horizontal pass to uint8)."""
    from yolo11_cu_b200 import export, frames
    for sh, sw, S in [(1080, 810, 224), (480, 640, 224), (100, 300, 224), (333, 517, 96)]:
        bgr = frames.synthetic_bgr(sh, sw, seed=sh + sw)
        got, geom = graph_ref.preprocess_cls(bgr, S)
        ref = export.classify_input(bgr, S)
        short, long_ = min(sh, sw), max(sh, sw)
        assert min(geom[0], geom[1]) == S and max(geom[0], geom[1]) == S * long_ // short
        assert np.abs(got.astype(np.float32) - ref).max() <= 2.0 / 255 + 1e-6, (sh, sw)


def test_obb_decode_oracle_vs_reference_final():
    """The C OBB decode (DFL, angle, rotated centre) on the reference's own per-op head
    outputs against the reference exporter's decoded model output for the same input
    (final.npy): boxes within 0.1 px, angles within 3e-3 rad, scores within 1e-4 (fp16 head
    tensors on the oracle side)."""
    d = os.path.join(GOLDEN, "yolo11n-obb-128")
    refs = np.load(os.path.join(d, "refs.npz"))
    fin = np.load(os.path.join(d, "final.npy"))[0]
    body = [l.split() for l in open(os.path.join(d, "model.graph")).read().split("\n") if l.strip()]
    nb, nt, no = map(int, body[2])
    ops = body[3 + nb + nt:3 + nb + nt + no]
    writer = {}                       # tensor -> index of the op that wrote it (refs key)
    for k, op in enumerate(ops):
        if op[0] == "ADD":
            writer[int(op[3])] = k
        elif op[0] not in ("DECODE", "DECODEOBB", "DECODESEG", "MASKS"):
            writer[int(op[2])] = k
    levels = [(refs[f"op{writer[b]:03d}"], refs[f"op{writer[c]:03d}"], refs[f"op{writer[a]:03d}"], st)
              for b, c, a, st in (map(int, op[1:5]) for op in ops if op[0] == "DECODEOBB")]
    recs = graph_ref.decode_obb(levels, 15, 0.0)
    an = recs[:, 7].astype(int)
    assert len(recs) == fin.shape[1]
    assert np.abs(fin[:4, an].T - recs[:, :4]).max() < 0.1
    assert np.abs(fin[19, an] - recs[:, 6]).max() < 3e-3
    assert np.abs(fin[4:19, an].max(0) - recs[:, 4]).max() < 1e-4
