"""Sparse neighbour aggregation on B200 (torch tensors in and out).

The two forms the reference's GNN layers use:
  * ``segment_sum(data, segment_ids, num_segments, mean=...)`` —
    jax.ops.segment_sum as called in hetero_gnn.py:283-295 (mean divides by
    max(count, 1)); out-of-range ids are dropped.
  * ``csr_spmm(rowptr, col, x, val=None, normalize=...)`` — the
    ``SparseMatrix @ dense`` of homo_gnn_sparse_deferred.py:138-161 with rows
    = message targets and columns = message sources (message_passing.py:
    24-38); normalize=True is the row-normalised (mean) aggregation.
Both run in hand-written sm_100a kernels (csrc/aggregate.cu) and accumulate
in fp32; inputs/outputs are fp32 or bf16.
"""

from __future__ import annotations

import ctypes
from typing import Optional

from distributed_graph_flow_b200 import _native


def _dtype_code(t) -> int:
    torch = _native.require_cuda()
    if t == torch.float32:
        return _native.F32
    if t == torch.bfloat16:
        return _native.BF16
    raise ValueError(f"unsupported dtype {t}; expected float32 or bfloat16")


def csr_spmm(rowptr, col, x, val=None, normalize: bool = False, out=None, out_dtype=None, num_rows: Optional[int] = None,
             workspace=None, stream=None):
    """Y[r] = scale_r * sum_j val_j * X[col_j] over CSR row r.

    rowptr int64 [R+1], col int32 [nnz], val float32 [nnz] or None (ones),
    x [N, F] float32/bfloat16 (row-major, F a multiple of 8). normalize gives
    scale_r = 1 / max(deg_r, 1).
    """
    torch = _native.require_cuda()
    R = int(rowptr.numel()) - 1 if num_rows is None else int(num_rows)
    nnz = int(col.numel())
    F = int(x.shape[1])
    if out is None:
        out = torch.empty((R, F), dtype=out_dtype or x.dtype, device=x.device)
    if col.dtype != torch.int32 or rowptr.dtype != torch.int64:
        raise ValueError("rowptr must be int64 and col int32")
    if not x.is_contiguous() or not out.is_contiguous():
        raise ValueError("x and out must be contiguous")
    need = ctypes.c_size_t()
    _native.check(_native.lib().dgfx_spmm_workspace_size(R, nnz, F, ctypes.byref(need)))
    if workspace is None or workspace.numel() < need.value:
        workspace = torch.empty(need.value, dtype=torch.uint8, device=x.device)
    _native.check(
        _native.lib().dgfx_spmm_csr(
            _native.ptr(rowptr), _native.ptr(col), _native.ptr(val), R, int(x.shape[0]), nnz, _native.ptr(x),
            _dtype_code(x.dtype), _native.ptr(out), _dtype_code(out.dtype), F, int(bool(normalize)),
            _native.ptr(workspace), need.value, _native.stream_handle(stream),
        )
    )
    return out


def spmm_workspace(num_rows: int, nnz: int, feat: int, device):
    torch = _native.require_cuda()
    need = ctypes.c_size_t()
    _native.check(_native.lib().dgfx_spmm_workspace_size(num_rows, nnz, feat, ctypes.byref(need)))
    return torch.empty(need.value, dtype=torch.uint8, device=device)


def segment_sum(data, segment_ids, num_segments: int, mean: bool = False, indices_are_sorted: bool = False,
                out_dtype=None, stream=None):
    """jax.ops.segment_sum(data, segment_ids, num_segments) [/ max(count, 1)]."""
    torch = _native.require_cuda()
    n, F = int(data.shape[0]), int(data.shape[1])
    out = torch.empty((num_segments, F), dtype=out_dtype or data.dtype, device=data.device)
    ids = segment_ids.to(torch.int64).contiguous()
    need = ctypes.c_size_t()
    _native.check(_native.lib().dgfx_segment_sum_workspace_size(n, F, num_segments, ctypes.byref(need)))
    ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=data.device)
    _native.check(
        _native.lib().dgfx_segment_sum(
            _native.ptr(data.contiguous()), _dtype_code(data.dtype), _native.ptr(ids), n, F, int(num_segments),
            int(bool(mean)), int(bool(indices_are_sorted)), _native.ptr(out), _dtype_code(out.dtype),
            _native.ptr(ws), need.value, _native.stream_handle(stream),
        )
    )
    return out


def gather_rows(table, ids, stream=None):
    """out[i] = table[ids[i]] (rows of any dtype whose byte width is a
    multiple of 16; ids outside the table give zero rows)."""
    torch = _native.require_cuda()
    n = int(ids.numel())
    row_bytes = table.element_size() * (table.numel() // max(1, table.shape[0]))
    out = torch.empty((n,) + tuple(table.shape[1:]), dtype=table.dtype, device=table.device)
    _native.check(
        _native.lib().dgfx_gather_rows(
            _native.ptr(table), int(table.shape[0]), row_bytes, _native.ptr(ids.to(torch.int64).contiguous()), n,
            _native.ptr(out), _native.stream_handle(stream),
        )
    )
    return out
