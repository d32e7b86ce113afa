"""CPU-only checks of the C ABI library: it loads, exports every function declared in
include/*.h, and rejects bad model directories on the host (host-side fault injection: the
loader checks everything before touching a GPU, so these run without one)."""
import ctypes as C
import os
import re
import shutil

import pytest

from conftest import ROOT, GOLDEN


def _declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    txt = re.sub(r"//.*", "", txt)
    return set(re.findall(r"\b((?:yolo|yk)_[a-z0-9_]+)\s*\(", txt))


def test_library_exports_every_declared_symbol(lib):
    from yolo11_cu_b200 import runtime
    names = _declared("yolo.h") | _declared("yk.h")
    assert len(names) > 30
    for n in names:
        assert hasattr(lib, n), n
    assert names <= set(runtime.exported_symbols())


def test_reference_abi_subset_present(lib):
    for n in ["yolo_create", "yolo_task", "yolo_exec_ms", "yolo_stream", "yolo_preprocess",
              "yolo_run", "yolo_run_async", "yolo_sync", "yolo_get", "yolo_slot_geom",
              "yolo_mask_dim", "yolo_get_mask"]:
        assert hasattr(lib, n)


def _bad_dir(tmp_path, golden_dirs, edit):
    d = tmp_path / "m"
    shutil.copytree(golden_dirs["yolo11n-64"], d)
    edit(d)
    return str(d)


@pytest.mark.parametrize("what", ["missing", "magic", "truncated", "task", "badop", "weights",
                                  "tensorref", "view"])
def test_loader_rejects_bad_model_dir(lib, golden_dirs, tmp_path, what):
    def edit(d):
        g = d / "model.graph"
        txt = g.read_text()
        if what == "missing":
            g.unlink()
        elif what == "magic":
            g.write_text(txt.replace("YOLO11GRAPH", "NOPE", 1))
        elif what == "truncated":
            g.write_text(txt[: len(txt) // 2])
        elif what == "task":
            g.write_text(txt.replace("TASK detect", "TASK classify", 1))
        elif what == "badop":
            g.write_text(txt.replace("\nMAXPOOL5", "\nFROBNICATE", 1))
        elif what == "weights":
            (d / "weights.f16").write_bytes((d / "weights.f16").read_bytes()[:1000])
        elif what == "tensorref":
            lines = txt.split("\n")
            i = next(k for k, l in enumerate(lines) if l.startswith("CONV"))
            parts = lines[i].split()
            parts[1] = "999999"
            lines[i] = " ".join(parts)
            g.write_text("\n".join(lines))
        elif what == "view":
            lines = txt.split("\n")
            i = next(k for k, l in enumerate(lines) if l.startswith("T "))
            lines[i] = "T 0 2 3"
            g.write_text("\n".join(lines))
    d = _bad_dir(tmp_path, golden_dirs, edit)
    h = lib.yolo_create(d.encode(), 1)
    assert not h
    assert lib.yolo_last_error().decode()


def test_null_handle_calls_are_safe(lib):
    assert lib.yolo_get(None, 0, None, 0) == 0
    assert lib.yolo_raw_count(None, 0) == -1
    assert lib.yolo_num_ops(None) == -1
    assert lib.yolo_get_mask(None, 0, 0, None) == -1
    assert lib.yolo_task(None) == 0
    lib.yolo_destroy(None)
