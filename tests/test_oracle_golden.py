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
