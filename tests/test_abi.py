"""The C-ABI library loads without a GPU and exports exactly the entry points
include/emmy_b200.h declares; calls that need a GPU fail with an error code
(no crash, no fallback)."""
import ctypes
import re
import subprocess

from conftest import REPO

from emmy_b200 import native


def declared():
    h = (REPO / "include" / "emmy_b200.h").read_text()
    return re.findall(r"EMMY_API\s+[\w\s\*]+?\b(emmy_\w+)\s*\(", h)


def test_exports_match_header(native_lib):
    names = declared()
    assert names and sorted(names) == sorted(native.EXPORTS)
    for n in names:
        assert hasattr(native_lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIB_PATH)],
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (emmy_\w+)", out))
    assert exported == set(names)


def test_abi_version(native_lib):
    assert native_lib.emmy_abi_version() == 1


def test_bad_arguments_are_errors(native_lib):
    L = native_lib
    assert L.emmy_ptx_assemble(None, 0, None, None, 0, None) == -1
    assert b"bad argument" in L.emmy_last_error()
    assert L.emmy_tensormap_encode(None, 0, 0, 0, None, None, None, 0) == -1


def test_assemble_error_log(native_lib):
    import pytest
    with pytest.raises(native.EmmyError) as e:
        native.Image(".version 8.8\n.target sm_100a\n.address_size 64\n"
                     ".visible .entry x() { not_an_instruction; }\n")
    assert e.value.code == -3 and "not_an_instruction" in str(e.value)


def test_from_ptx_context_has_what_buffers_need():
    """A kernel given as PTX text under a meta entry carries everything the
    buffer setup of ``harness.run`` reads (arguments, scalars, outputs to
    zero before each launch)."""
    from emmy_b200 import harness, synth
    g, m = synth.full_sum(n=1 << 16, ctas=16).build()
    k = m["kernels"][0]
    ptx = harness.CompiledKernel(g, m).ptx
    pk = harness.CompiledKernel.from_ptx(ptx, k)
    assert pk.ctx.arg_order == k["arg_order"]
    assert pk.ctx.zero_outputs == list(k.get("zero_outputs", []))
    assert pk.ctx.zero_outputs                        # the split sum zeroes its output
