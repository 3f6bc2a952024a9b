"""The guard regions of harness.Buffers (the out-of-place write check that
every GPU test's launches get through harness.run), exercised on CPU
buffers: writes planted just outside an output, far into a guard region and
into an input are each reported with the argument, the side and the first
offending byte; untouched buffers report nothing."""
import numpy as np
import pytest
import torch

from emmy_b200 import harness


class _Kern:
    """The part of a CompiledKernel that Buffers reads."""

    def __init__(self, args):
        self.info = {"args": args}


ARGS = [{"name": "x", "dtype": "f32", "shape": [1000]},
        {"name": "w", "dtype": "bf16", "shape": [7]},
        {"name": "y", "dtype": "f32", "shape": [1000], "output": True}]
G = 4096


def _bufs():
    ins = {"x": np.arange(1000, dtype=np.float32), "w": np.arange(7, dtype=np.uint16)}
    return harness.Buffers(_Kern(ARGS), ins, device="cpu", guard=G)


def test_untouched_buffers_report_nothing():
    b = _bufs()
    b.t["y"].copy_(b.t["x"] * 2)          # a full, in-place write of the output
    assert b.check_guards() == []
    assert np.array_equal(b.outputs()["y"], np.arange(1000, dtype=np.float32) * 2)


def test_data_keeps_values_and_alignment():
    b = _bufs()
    assert np.array_equal(b.t["x"].numpy(), np.arange(1000, dtype=np.float32))
    assert b.t["w"].dtype == torch.bfloat16 and b.t["w"].numel() == 7
    for name, t in b.t.items():
        assert t.data_ptr() - b._raw[name].data_ptr() == G      # G keeps 512-byte alignment


@pytest.mark.parametrize("where,offset", [("after", 0), ("after", G - 1), ("before", G - 1),
                                          ("before", 0)])
def test_write_outside_an_output_is_reported(where, offset):
    b = _bufs()
    raw = b._raw["y"]
    nb = 1000 * 4
    pos = G + nb + offset if where == "after" else offset
    raw[pos] = 0
    assert b.check_guards() == [("y", where, offset, 1)]


def test_write_into_an_input_is_reported():
    b = _bufs()
    b.t["x"].view(torch.uint8)[40:52] = 0x5A     # elements 10..12, every byte changed
    assert b.check_guards() == [("x", "input", 40, 12)]


def test_guard_must_keep_alignment():
    with pytest.raises(AssertionError):
        harness.Buffers(_Kern(ARGS), {"x": np.zeros(1000, np.float32),
                                      "w": np.zeros(7, np.uint16)}, device="cpu", guard=100)


def test_run_reads_the_guard_size_from_the_environment(monkeypatch):
    monkeypatch.setenv("EMMY_GUARD_BYTES", "8192")
    assert harness.guard_bytes() == 8192
    monkeypatch.setenv("EMMY_GUARD_BYTES", "")
    assert harness.guard_bytes() == 0


def test_the_suite_guards_its_launches():
    """tests/conftest.py turns the guards on for every harness.run of the
    session (unless the caller set EMMY_GUARD_BYTES itself)."""
    import os
    assert int(os.environ["EMMY_GUARD_BYTES"]) >= 4096
    assert harness.guard_bytes() == int(os.environ["EMMY_GUARD_BYTES"])
