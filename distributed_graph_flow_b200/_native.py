"""ctypes binding of the dgfx C ABI (include/dgfx.h).

This is the only place Python touches the native library. Failures raise:
INVALID_ARGUMENT / FAILED_PRECONDITION / NOT_FOUND become ``ValueError``
carrying the native message, like the reference's absl status caster
(dgf/src/util/status_caster.h:17-21, 83-88); everything else becomes
``RuntimeError``. There is no fallback: if libdgfx.so is missing the import
of the sampling or aggregation modules' native entry points fails loudly.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libdgfx.so"

OK = 0
ERR_INVALID_ARGUMENT = 3
ERR_NOT_FOUND = 5
ERR_FAILED_PRECONDITION = 9
ERR_INTERNAL = 13
ERR_CUDA = 100
ERR_WORKSPACE = 101
ERR_UNSUPPORTED = 102

F32 = 0
BF16 = 1

CALL_INDEX_DEVICE = (1 << 64) - 1  # DGFX_CALL_INDEX_DEVICE

MODE_RANDOM = 0
MODE_FIRST = 1
MODE_MOST_RECENT = 2

_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_p_i32 = ctypes.POINTER(ctypes.c_int32)
_p_i64 = ctypes.POINTER(ctypes.c_int64)


class CsrView(ctypes.Structure):
    """dgfx_csr_view: device view of one adjacency index."""

    _fields_ = [
        ("rowptr", _vp),
        ("col", _vp),
        ("ts", _vp),
        ("edge_pos", _vp),
        ("num_src", _i64),
        ("num_dst", _i64),
        ("num_edges", _i64),
    ]


class SampleOut(ctypes.Structure):
    """dgfx_sample_out: merged-batch output buffers (device pointers)."""

    _fields_ = [
        ("node_ids", _vp),
        ("node_offsets", _vp),
        ("edge_src", _vp),
        ("edge_dst", _vp),
        ("edge_offsets", _vp),
    ]


# Every symbol the header declares, with (restype, argtypes).
SIGNATURES = {
    "dgfx_last_error": (ctypes.c_char_p, []),
    "dgfx_version": (_int, []),
    "dgfx_csr_build_workspace_size": (_int, [_i64, _i64, _i64, _int, ctypes.POINTER(_sz)]),
    "dgfx_csr_build": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dgfx_sampler_create": (
        _int,
        [_i32, _p_i32, _p_i32, _p_i32, _i32, _p_i32, _p_i32, _p_i32, _p_i32, _i32, _i32, _p_i64, _i32,
         ctypes.POINTER(CsrView), ctypes.POINTER(CsrView), _i32, _i32, _u64, ctypes.POINTER(_vp)],
    ),
    "dgfx_sampler_destroy": (None, [_vp]),
    "dgfx_sampler_tree_size": (_int, [_vp, _p_i64]),
    "dgfx_sampler_workspace_size": (_int, [_vp, _i64, ctypes.POINTER(_sz)]),
    "dgfx_sampler_output_capacity": (_int, [_vp, _i64, _p_i64, _p_i64]),
    "dgfx_sampler_sample": (_int, [_vp, _vp, _vp, _vp, _i64, _u64, ctypes.POINTER(SampleOut), _vp, _sz, _vp]),
    "dgfx_sampler_sample_noalloc": (_int, [_vp, _vp, _vp, _vp, _i64, _u64, ctypes.POINTER(SampleOut), _vp]),
    "dgfx_sampler_sample_split": (_int, [_vp, _vp, _vp, _vp, _i64, _u64, ctypes.POINTER(SampleOut), _vp, _sz, _vp, _vp]),
    "dgfx_sampler_check": (_int, [_vp, _vp]),
    "dgfx_sampler_stats": (_int, [_vp, _vp, _p_i64]),
    "dgfx_gather_rows": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "dgfx_gather_rows_ranged": (_int, [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    "dgfx_spmm_workspace_size": (_int, [_i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "dgfx_spmm_csr": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _int, _i64, _i32, _vp, _sz, _vp]),
    "dgfx_segment_sum_workspace_size": (_int, [_i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "dgfx_segment_sum": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _int, _vp, _sz, _vp]),
    "dgfx_segment_softmax_workspace_size": (_int, [_i64, _i64, _i32, _i64, _int, _i32, ctypes.POINTER(_sz)]),
    "dgfx_segment_softmax": (_int, [_vp, _i32, _vp, _int, _i64, _vp, _i64, _i64, _i32, _vp, _int, _vp, _sz, _vp]),
    "dgfx_dense_concat_bf16": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i32, _vp, _vp]),
    "dgfx_dense_check": (_int, [_vp]),
    "dgfx_halo_partition_workspace_size": (_int, [_i64, _i32, ctypes.POINTER(_sz)]),
    "dgfx_halo_partition": (_int, [_vp, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dgfx_gather_rows_local": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp]),
    "dgfx_scatter_rows": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "dgfx_device_alloc": (_int, [_sz, ctypes.POINTER(_vp)]),
    "dgfx_device_free": (_int, [_vp]),
    "dgfx_ipc_get_handle": (_int, [_vp, _vp]),
    "dgfx_ipc_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "dgfx_ipc_close": (_int, [_vp]),
    "dgfx_gather_rows_p2p": (_int, [_vp, _i32, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    "dgfx_exchange_buffer_size": (_int, [_i32, _i64, _i64, ctypes.POINTER(_sz)]),
    "dgfx_exchange_partition": (_int, [_vp, _i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp]),
    "dgfx_exchange_serve": (_int, [_vp, _i32, _i32, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp]),
    "dgfx_exchange_scatter": (_int, [_vp, _i32, _i32, _i64, _i64, _vp, _vp, _vp]),
    "dgfx_exchange_barrier": (_int, [_vp, _i32, _i32, ctypes.c_uint32, _u64, _vp]),
    "dgfx_exchange_check": (_int, [_vp, _i32, _vp]),
    "dgfx_exchange_gather": (_int, [_vp, _vp, _i32, _i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _vp,
                                    _i64, _vp, _i64, _vp, ctypes.c_uint32, _u64, _vp]),
    "dgfx_edge_timestamps": (_int, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp]),
    "dgfx_random_walk_negatives_workspace_size": (_int, [_vp, _i64, _i32, _i32, _i32, ctypes.POINTER(_sz)]),
    "dgfx_random_walk_negatives": (_int, [_vp, _vp, _i64, _i32, _i32, _i32, _u64, _vp, _vp, _sz, _vp]),
    "dgfx_random_walk_negatives_check": (_int, [_vp, _vp]),
    "dgfx_id_index_table_bytes": (_int, [_i64, ctypes.POINTER(_sz)]),
    "dgfx_id_index_create": (_int, [_i32, _vp, _vp, _i64, _i64, _vp, _sz, _vp, ctypes.POINTER(_vp)]),
    "dgfx_id_index_destroy": (None, [_vp]),
    "dgfx_id_index_lookup": (_int, [_vp, _i32, _vp, _vp, _i64, _i64, _vp, ctypes.POINTER(_i64), _vp]),
    "dgfx_compact_pairs_workspace_size": (_int, [_i64, ctypes.POINTER(_sz)]),
    "dgfx_compact_pairs": (_int, [_vp, _vp, _i64, _vp, _vp, _vp, ctypes.POINTER(_i64), _vp, _sz, _vp]),
    "dgfx_timeseries_windows": (_int, [_vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "dgfx_gather_segments": (_int, [_vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp]),
    "dgfx_subgraph_union_workspace_size": (_int, [_i64, _i64, ctypes.POINTER(_sz)]),
    "dgfx_subgraph_union": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _i64, _i64, _vp, _vp,
                                   _vp, _vp, _vp, _vp, _sz, _vp]),
    "dgfx_merge_edgeset": (_int, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64, _i64, _i64, _vp, _vp, _vp]),
    "dgfx_sampler_set_kernel": (_int, [_vp, _i32]),
    "dgfx_csr_add_diagonal": (_int, [_vp, _vp, _i64, ctypes.c_float, _i32, _vp, _vp, _vp, _vp]),
    "dgfx_csr_row_ids": (_int, [_vp, _i64, _vp, _vp]),
    "dgfx_segment_counts": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "dgfx_gather_rows_scaled": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "dgfx_batch_csr": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "dgfx_batch_mean": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _int, _i64, _vp, _vp]),
    "dgfx_publish_totals": (_int, [_vp, _vp, _vp, _vp]),
    "dgfx_graph_launch_with_inputs": (_int, [_vp, _vp, _vp, _sz, _vp, _vp, _sz, _vp]),
    "dgfx_sampler_kernel_info": (_int, [_vp, _p_i32, _p_i32]),
    "dgfx_sampler_kernel_stats": (_int, [_vp, _vp, _p_i64]),
    "dgfx_synth_graph_workspace_size": (_int, [_i64, _i64, ctypes.POINTER(_sz)]),
    "dgfx_synth_graph": (_int, [_i64, _i64, ctypes.c_double, _i64, _u64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dgfx_synth_bipartite": (_int, [_i64, _i64, _i64, ctypes.c_double, _i64, _u64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "dgfx_synth_uniform_int": (_int, [_i64, _i64, _i64, _u64, ctypes.c_uint32, _vp, _vp]),
    "dgfx_synth_normal_features": (_int, [_i64, _i64, _i64, _u64, _int, _vp, _vp]),
    "dgfx_synth_normal_rows": (_int, [_vp, _i64, _i64, _u64, _int, _vp, _vp]),
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads libdgfx.so (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build the CUDA library first "
                "(python -m distributed_graph_flow_b200.build). There is no CPU fallback."
            )
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    msg = lib().dgfx_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raises the Python exception matching a dgfx status."""
    if status == OK:
        return
    msg = last_error()
    if status in (ERR_INVALID_ARGUMENT, ERR_FAILED_PRECONDITION, ERR_NOT_FOUND):
        raise ValueError(msg)
    raise RuntimeError(f"dgfx error {status}: {msg}")


def require_cuda():
    """Returns torch with a visible CUDA device, or raises (no CPU fallback)."""
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("dgfx kernels need a CUDA device (sm_100a); none is visible and there is no CPU fallback")
    return torch


def stream_handle(stream=None) -> int:
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)


def ptr(t) -> Optional[int]:
    """Device pointer of a torch tensor (None passes NULL)."""
    return None if t is None else int(t.data_ptr())


def elem_ptr(t, i: int) -> int:
    """Device pointer of element i of a 1-D tensor (negative i counts from the end)."""
    if i < 0:
        i += t.numel()
    return int(t.data_ptr()) + i * t.element_size()
