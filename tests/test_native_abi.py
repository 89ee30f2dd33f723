"""The C-ABI library loads without a GPU and exports every entry point the
public header declares (no compute calls)."""

import ctypes
import re
from pathlib import Path

from distributed_graph_flow_b200 import _native

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(dgfx_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"dgfx_sampler_sample", "dgfx_csr_build", "dgfx_spmm_csr", "dgfx_segment_sum"} <= names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_binding_covers_header():
    assert declared_functions() == set(_native.SIGNATURES)


def test_version_and_error_string_without_gpu():
    lib = _native.lib()
    assert lib.dgfx_version() >= 100
    assert isinstance(_native.last_error(), str)


def test_argument_errors_need_no_gpu():
    # Host-side validation runs before any CUDA call.
    lib = _native.lib()
    st = lib.dgfx_gather_rows(None, 0, 12, None, 1, None, None)
    assert st == _native.ERR_INVALID_ARGUMENT
    assert "multiple of 16" in _native.last_error()
    size = ctypes.c_size_t()
    assert lib.dgfx_csr_build_workspace_size(1000, 10, 10, 1, ctypes.byref(size)) == _native.OK
    assert size.value > 1000 * 24


def test_more_argument_errors_need_no_gpu():
    """Entry points added with the pipelined and captured paths validate
    their arguments on the host, before any CUDA call."""
    lib = _native.lib()
    assert lib.dgfx_graph_launch_with_inputs(None, None, None, 0, None, None, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert "dgfx_graph_launch_with_inputs" in _native.last_error()
    # A non-null exec with a copy whose pointers are missing is refused too.
    assert lib.dgfx_graph_launch_with_inputs(1, None, None, 8, None, None, 0, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.dgfx_publish_totals(None, None, None, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.dgfx_batch_mean(None, None, None, None, 1, 1, None, 7, 8, None, None) == _native.ERR_INVALID_ARGUMENT
    size = ctypes.c_size_t()
    assert lib.dgfx_segment_softmax_workspace_size(-1, 1, 1, 8, 0, 1, ctypes.byref(size)) == _native.ERR_INVALID_ARGUMENT
    assert lib.dgfx_segment_softmax_workspace_size(1000, 10, 8, 32, 1, 1, ctypes.byref(size)) == _native.OK
    assert size.value > 0
    assert lib.dgfx_spmm_workspace_size(100, 1000, 0, ctypes.byref(size)) == _native.ERR_INVALID_ARGUMENT
