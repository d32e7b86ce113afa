"""Two handles on two GPUs, driven from two host threads in one process at once (the
per-GPU serving layout): every launcher's shared-memory attribute and cached device state
must be per device.  Skipped with fewer than two GPUs visible."""
import threading

import numpy as np
import pytest
import torch

from conftest import MODELS

pytestmark = pytest.mark.gpu


def test_two_devices_two_threads(lib, cuda, pkg):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from yolo11_cu_b200 import export, frames, runtime as rt
    d = export.ensure_model_dir("yolo11n", MODELS, 640)
    bgr = np.stack([frames.synthetic_bgr(720, 1280, seed=i) for i in range(4)])
    res, errs = {}, []

    def work(dev):
        try:
            torch.cuda.set_device(dev)
            buf = torch.from_numpy(bgr).to(f"cuda:{dev}")
            torch.cuda.synchronize(dev)
            eng = rt.Engine(d, 4, device=dev)
            eng.bind_frames(0, buf.data_ptr(), 720, 1280, 4, False)
            for _ in range(5):
                eng.run_frames(0, 4)
            res[dev] = eng.get_batch(4)
            eng.close()
        except Exception as e:          # reported by the main thread
            errs.append((dev, repr(e)))

    ts = [threading.Thread(target=work, args=(i,)) for i in (0, 1)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
    assert res[0] == res[1] and len(res[0][0]) > 0
