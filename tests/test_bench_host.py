"""Host-side pieces of bench.py that need no GPU: the stdout guard around
NCCL set-up and the packed per-step staging buffer."""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def test_stdout_guard_moves_native_writes_to_stderr():
    # NCCL prints from native code on descriptor 1; inside the guard that
    # must land on stderr, and stdout must work again after it
    code = (
        "import os, sys\n"
        f"sys.path.insert(0, {str(ROOT)!r})\n"
        "sys.argv = ['bench']\n"
        "import bench\n"
        "print('before', flush=True)\n"
        "with bench._stdout_to_stderr():\n"
        "    os.write(1, b'native\\n')\n"
        "    print('python', flush=True)\n"
        "print('after', flush=True)\n"
    )
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout == "before\nafter\n"
    assert "native\npython\n" in r.stderr


def test_staging_packs_each_put_into_its_own_slots(monkeypatch):
    import torch

    sys.path.insert(0, str(ROOT))
    import bench

    class _Event:
        def record(self):
            pass

        def synchronize(self):
            pass

    monkeypatch.setattr(torch.cuda, "Event", _Event)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    i32, i64 = torch.int32, torch.int64
    st = bench._Staging(torch, "cpu", {"tables": ((6, 4, 30), i32), "cow_src": (12, i32), "masks": (64, i64),
                                       "moves": ((50, 4), i32), "groups": (25, i32)})
    rng = np.random.default_rng(0)
    for _ in range(3):
        t = rng.integers(0, 1000, (6, 4, 30)).astype(np.int32)
        c = rng.integers(0, 9, 5).astype(np.int32)
        m = rng.integers(0, 2**62, 64).astype(np.int64)
        d = st.put({"tables": t, "cow_src": c, "masks": m})
        mv = rng.integers(0, 99, (17, 4)).astype(np.int32)
        g = np.arange(25, dtype=np.int32)
        d2 = st.put({"moves": mv, "groups": g})
        empty = st.put({"cow_src": np.zeros(0, np.int32)})
        assert empty["cow_src"].shape == (0,)
        # a later put leaves the slots of an earlier one as they were
        np.testing.assert_array_equal(d["tables"].numpy(), t)
        np.testing.assert_array_equal(d["cow_src"].numpy(), c)
        np.testing.assert_array_equal(d["masks"].numpy(), m)
        np.testing.assert_array_equal(d2["moves"].numpy(), mv)
        np.testing.assert_array_equal(d2["groups"].numpy(), g)
