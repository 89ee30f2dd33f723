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


def segment_softmax(logits, messages, segment_ids, num_segments: int, indices_are_sorted: bool = False,
                    out_dtype=None, stream=None):
    """Attention-weighted segment sum (hetero_graph_attention_network.py:
    242-263): softmax of ``logits`` [E, H] over the items of each segment
    (per head, max-subtracted, + 1e-9 in the denominator) weighting
    ``messages`` [E, H, D]; returns [num_segments, H, D]. One pass over the
    items (online softmax), fp32 accumulation."""
    torch = _native.require_cuda()
    if logits.dtype != torch.float32:
        raise ValueError("segment_softmax: logits must be float32")
    E, H = int(logits.shape[0]), int(logits.shape[1])
    if messages.dim() != 3 or int(messages.shape[0]) != E or int(messages.shape[1]) != H:
        raise ValueError("segment_softmax: messages must be [E, H, D] matching logits [E, H]")
    D = int(messages.shape[2])
    out = torch.empty((num_segments, H, D), dtype=out_dtype or messages.dtype, device=messages.device)
    ids = segment_ids.to(torch.int64).contiguous()
    need = ctypes.c_size_t()
    _native.check(_native.lib().dgfx_segment_softmax_workspace_size(
        E, num_segments, H, D, _dtype_code(messages.dtype), int(bool(indices_are_sorted)), ctypes.byref(need)))
    ws = torch.empty(max(1, need.value), dtype=torch.uint8, device=messages.device)
    _native.check(_native.lib().dgfx_segment_softmax(
        _native.ptr(logits.contiguous()), H, _native.ptr(messages.contiguous()), _dtype_code(messages.dtype), D,
        _native.ptr(ids), E, int(num_segments), int(bool(indices_are_sorted)), _native.ptr(out),
        _dtype_code(out.dtype), _native.ptr(ws), need.value, _native.stream_handle(stream)))
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


def dense_concat(x1, x2, weight, bias=None, relu: bool = True, out=None, stream=None):
    """act(concat[x1, x2] @ weight.T + bias) in bf16 on the tensor cores
    (tcgen05, fp32 accumulation): the Dense(+ReLU) update after aggregation
    (hetero_gnn.py:302-312). x1 [M, K1], x2 [M, K2] or None, weight [N, K1+K2]
    (torch Linear layout), bias fp32 [N] or None; K1, K2 and N multiples of 64.
    The concat is read from the two inputs, never materialised."""
    torch = _native.require_cuda()
    if x1.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or (x2 is not None and x2.dtype != torch.bfloat16):
        raise ValueError("dense_concat: x1, x2 and weight must be bfloat16")
    m, k1 = int(x1.shape[0]), int(x1.shape[1])
    k2 = 0 if x2 is None else int(x2.shape[1])
    if x2 is not None and int(x2.shape[0]) != m:
        raise ValueError("dense_concat: x1 and x2 must have the same number of rows")
    n = int(weight.shape[0])
    if int(weight.shape[1]) != k1 + k2:
        raise ValueError(f"dense_concat: weight is [{n}, {int(weight.shape[1])}], expected [N, {k1 + k2}]")
    for t in (x1, x2, weight):
        if t is not None and not t.is_contiguous():
            raise ValueError("dense_concat: inputs must be contiguous")
    if bias is not None and (bias.dtype != torch.float32 or int(bias.numel()) != n):
        raise ValueError("dense_concat: bias must be float32 [N]")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x1.device)
    _native.check(_native.lib().dgfx_dense_concat_bf16(
        _native.ptr(x1), k1, _native.ptr(x2), k2, m, _native.ptr(weight), _native.ptr(bias), n, int(bool(relu)),
        _native.ptr(out), _native.stream_handle(stream)))
    return out


def dense_check(stream=None):
    """Raises if a dense_concat launch hit a pipeline timeout since the last
    check (synchronises the stream)."""
    _native.check(_native.lib().dgfx_dense_check(_native.stream_handle(stream)))


def sage_mean_linear_relu(rowptr, col, x, weight, bias=None, agg=None, workspace=None, out=None, stream=None):
    """GraphSAGE-mean layer: agg = mean over in-neighbours (CSR rows = target
    nodes, col = source nodes) of x, then relu(concat[x, agg] @ weight.T +
    bias). x bf16 [N, F]; weight bf16 [N_out, 2F]. Two launches: the SpMM
    (HBM-bound gather, bf16 out) and the tensor-core dense layer."""
    torch = _native.require_cuda()
    n_rows = int(rowptr.numel()) - 1
    if agg is None:
        agg = torch.empty((n_rows, int(x.shape[1])), dtype=torch.bfloat16, device=x.device)
    csr_spmm(rowptr, col, x, normalize=True, out=agg, workspace=workspace, stream=stream)
    return dense_concat(x[:n_rows], agg, weight, bias, relu=True, out=out, stream=stream)


# ---------------------------------------------------------------------------
# Propagation matrices of the reference's sparse GNN layers, CSR transpose,
# segment-sum gradient, mean aggregation over a sampled batch.
# ---------------------------------------------------------------------------
def _symmetric_structure(src, dst, num_nodes: int, stream=None):
    """CSR (rowptr int64, col int32) of A + A^T for an edge list on one node
    set: every edge contributes (dst, src) and (src, dst); duplicates and
    self loops are kept (the sum of COO matrices keeps them too). Rows are
    sorted by column."""
    torch = _native.require_cuda()
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    s = src.to(torch.int64).contiguous()
    d = dst.to(torch.int64).contiguous()
    rows = torch.cat([d, s])
    cols = torch.cat([s, d])
    idx = ext.build_adjacency_index_device(rows, cols, None, num_nodes, num_nodes, False, False, stream=stream)
    return idx.rowptr, idx.col


def _add_diagonal(rowptr, col, num_nodes: int, diag: float, normalize: bool, stream=None):
    torch = _native.require_cuda()
    nnz = int(col.numel()) + num_nodes
    out_rowptr = torch.empty(num_nodes + 1, dtype=torch.int64, device=rowptr.device)
    out_col = torch.empty(max(nnz, 1), dtype=torch.int32, device=rowptr.device)[:nnz]
    out_val = torch.empty(max(nnz, 1), dtype=torch.float32, device=rowptr.device)[:nnz]
    _native.check(_native.lib().dgfx_csr_add_diagonal(
        _native.ptr(rowptr), _native.ptr(col), num_nodes, float(diag), int(bool(normalize)), _native.ptr(out_rowptr),
        _native.ptr(out_col), _native.ptr(out_val), _native.stream_handle(stream)))
    return out_rowptr, out_col, out_val


def gcn_matrix(src, dst, num_nodes: int, stream=None):
    """D^-1/2 (A + A^T + I) D^-1/2 as CSR (rowptr int64, col int32, val
    float32), D = row sums: the reference's GCN propagation matrix
    ``(adj + adj.transpose()).add_eye().normalize_symmetric()``
    (homo_gnn_sparse_deferred.py:293). Symmetric, so it is its own
    transpose."""
    rowptr, col = _symmetric_structure(src, dst, num_nodes, stream)
    return _add_diagonal(rowptr, col, num_nodes, 1.0, True, stream)


def gin_matrix(src, dst, num_nodes: int, epsilon: float = 0.0, stream=None):
    """A + A^T + (1 + epsilon) I as CSR (rowptr, col, val): the reference's
    GIN propagation matrix ``(adj + adj.transpose()).add_eye(1 +
    epsilon)`` (homo_gnn_sparse_deferred.py:526)."""
    rowptr, col = _symmetric_structure(src, dst, num_nodes, stream)
    return _add_diagonal(rowptr, col, num_nodes, 1.0 + float(epsilon), False, stream)


def csr_row_ids(rowptr, stream=None):
    """int64 row of every CSR entry."""
    torch = _native.require_cuda()
    R = int(rowptr.numel()) - 1
    nnz = int(rowptr[-1].item()) if R >= 0 else 0
    rows = torch.empty(max(nnz, 1), dtype=torch.int64, device=rowptr.device)[:nnz]
    _native.check(_native.lib().dgfx_csr_row_ids(_native.ptr(rowptr), R, _native.ptr(rows),
                                                 _native.stream_handle(stream)))
    return rows


def csr_transpose(rowptr, col, val, num_cols: int, stream=None):
    """Transpose of a CSR matrix [R, num_cols] -> [num_cols, R] (rowptr,
    col int32, val float32 or None); entries of a transposed row are in
    original row order."""
    torch = _native.require_cuda()
    from distributed_graph_flow_b200.sampling import _in_memory_sampler_ext as ext

    R = int(rowptr.numel()) - 1
    nnz = int(col.numel())
    rows = torch.empty(max(nnz, 1), dtype=torch.int64, device=rowptr.device)[:nnz]
    _native.check(_native.lib().dgfx_csr_row_ids(_native.ptr(rowptr), R, _native.ptr(rows),
                                                 _native.stream_handle(stream)))
    idx = ext.build_adjacency_index_device(rows, col.to(torch.int64), None, R, int(num_cols), True, val is not None,
                                           stream=stream)
    val_t = None
    if val is not None:
        val_t = torch.empty_like(val)
        val_t[idx.edge_pos] = val
    return idx.rowptr, idx.col, val_t


def segment_counts(segment_ids, num_segments: int, stream=None):
    torch = _native.require_cuda()
    ids = segment_ids.to(torch.int64).contiguous()
    cnt = torch.empty(max(1, num_segments), dtype=torch.int32, device=ids.device)[:num_segments]
    _native.check(_native.lib().dgfx_segment_counts(_native.ptr(ids), int(ids.numel()), int(num_segments),
                                                    _native.ptr(cnt), _native.stream_handle(stream)))
    return cnt


def gather_rows_scaled(src, segment_ids, num_segments: int, counts=None, stream=None):
    """out[i] = src[ids[i]] / max(counts[ids[i]], 1) (no division if counts is
    None); zero rows for ids outside [0, num_segments)."""
    torch = _native.require_cuda()
    ids = segment_ids.to(torch.int64).contiguous()
    src = src.contiguous()
    F = int(src.numel() // max(1, src.shape[0])) if src.dim() > 1 else 1
    out = torch.empty((int(ids.numel()),) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    _native.check(_native.lib().dgfx_gather_rows_scaled(
        _native.ptr(src), _dtype_code(src.dtype), _native.ptr(ids), int(ids.numel()), int(num_segments), F,
        _native.ptr(counts), _native.ptr(out), _native.stream_handle(stream)))
    return out


def batch_csr(batch, stream=None):
    """CSR over the batch nodes of a merged sampled batch (one node set, one
    edge set): rowptr int64 [capacity + 1] (rows past the batch's node count
    empty), col int32 [edge capacity], col = batch index of the sampled
    neighbour. No host synchronisation."""
    torch = _native.require_cuda()
    cap = int(batch.node_ids.numel())
    ecap = int(batch.edge_src.numel())
    rowptr = torch.empty(cap + 1, dtype=torch.int64, device=batch.node_ids.device)
    col = torch.empty(max(ecap, 1), dtype=torch.int32, device=batch.node_ids.device)[:ecap]
    _native.check(_native.lib().dgfx_batch_csr(
        _native.ptr(batch.node_offsets), _native.ptr(batch.edge_offsets), _native.ptr(batch.edge_src),
        _native.ptr(batch.edge_dst), int(batch.B), cap, _native.ptr(rowptr), _native.ptr(col),
        _native.stream_handle(stream)))
    return rowptr, col


def batch_mean_aggregate(batch, features, out=None, stream=None):
    """Mean aggregation over a merged sampled batch (jax.ops.segment_sum
    mean pooling of hetero_gnn.py:282-294, messages = the features of the
    sampled neighbours flowing to the node that sampled them): out[v] =
    mean of features[u] over the batch edges v -> u, zero rows for nodes
    without sampled neighbours; rows past the batch's node count are left
    as they are. features [capacity, F] in batch order (the rows gathered
    for batch.node_ids). One kernel (dgfx_batch_mean); the same values as
    csr_spmm(*batch_csr(batch), features, normalize=True)."""
    torch = _native.require_cuda()
    cap = int(batch.node_ids.numel())
    F = int(features.numel() // max(1, features.shape[0]))
    if out is None:
        out = torch.empty_like(features)
    _native.check(_native.lib().dgfx_batch_mean(
        _native.ptr(batch.node_offsets), _native.ptr(batch.edge_offsets), _native.ptr(batch.edge_src),
        _native.ptr(batch.edge_dst), int(batch.B), cap, _native.ptr(features), _dtype_code(features.dtype), F,
        _native.ptr(out), _native.stream_handle(stream)))
    return out
