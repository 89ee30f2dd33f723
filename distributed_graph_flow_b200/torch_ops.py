"""The aggregation boundary as torch custom operators (``torch.library``).

The reference's GNN layers call their aggregation inside trained models:
``jax.ops.segment_sum`` over an edge list
(dgf/src/learning/jax/layers/hetero_gnn.py:282-294) and ``SparseMatrix @
dense`` (homo_gnn_sparse_deferred.py:138-161, 292-297, 525-530). Here the
same operations are torch operators in the ``dgfx`` namespace, with fake
(meta) implementations for tracing and export, and autograd where the
reference's layers need gradients:

* ``dgfx::csr_spmm(rowptr, col, val, x, normalize, num_rows)`` —
  Y = S A X with A the CSR matrix (rows = message targets, columns =
  sources), S = diag(1 / max(deg, 1)) when normalize. Gradient with
  respect to x: A^T S dY, one SpMM over the transposed CSR (built on the
  device). The matrix values are constants (the reference's propagation
  matrices are built from the graph): a val that requires grad is rejected.
* ``dgfx::segment_sum(data, segment_ids, num_segments, mean)`` — gradient:
  d data[i] = dY[ids[i]] (/ max(count, 1) for the mean), a row gather.
  The two gradients are operators of their own (``dgfx::csr_spmm_grad_x``,
  ``dgfx::segment_sum_grad``), so backward graphs trace with fake tensors.
* ``dgfx::segment_softmax(logits, messages, segment_ids, num_segments)`` and
  ``dgfx::sage_mean_linear_relu(rowptr, col, x, weight, bias)`` — forward
  (inference) operators with fake implementations.

Every operator runs the library's sm_100a kernels (no fallback): the inputs
must be CUDA tensors.
"""

from __future__ import annotations

from typing import Optional

import torch

from distributed_graph_flow_b200 import aggregation

_LIB = "dgfx"


# ---------------------------------------------------------------------------
# csr_spmm
# ---------------------------------------------------------------------------
@torch.library.custom_op(f"{_LIB}::csr_spmm", mutates_args=())
def csr_spmm(rowptr: torch.Tensor, col: torch.Tensor, val: Optional[torch.Tensor], x: torch.Tensor,
             normalize: bool = False, num_rows: int = -1) -> torch.Tensor:
    rows = int(rowptr.numel()) - 1 if num_rows < 0 else int(num_rows)
    return aggregation.csr_spmm(rowptr, col, x.contiguous(), val=val, normalize=normalize, num_rows=rows)


@csr_spmm.register_fake
def _csr_spmm_fake(rowptr, col, val, x, normalize=False, num_rows=-1):
    rows = rowptr.shape[0] - 1 if num_rows < 0 else num_rows
    return x.new_empty((rows, x.shape[1]))


def _csr_spmm_setup(ctx, inputs, output):
    rowptr, col, val, x, normalize, num_rows = inputs
    if val is not None and val.requires_grad:
        raise RuntimeError("dgfx::csr_spmm: gradients with respect to the matrix values are not supported")
    ctx.save_for_backward(rowptr, col, val)
    ctx.normalize = normalize
    ctx.num_x_rows = x.shape[0]
    ctx.x_dtype = x.dtype


@torch.library.custom_op(f"{_LIB}::csr_spmm_grad_x", mutates_args=())
def csr_spmm_grad_x(rowptr: torch.Tensor, col: torch.Tensor, val: Optional[torch.Tensor], grad: torch.Tensor,
                    normalize: bool, num_x_rows: int) -> torch.Tensor:
    """A^T S dY: the transposed CSR (device build) times dY."""
    v = val
    if normalize:
        # Entry (r, c) of S A is val_rc / max(deg_r, 1).
        deg = (rowptr[1:] - rowptr[:-1]).clamp_min(1).to(torch.float32)
        scale = (1.0 / deg)[aggregation.csr_row_ids(rowptr)]
        v = scale if val is None else val * scale
    rp_t, col_t, val_t = aggregation.csr_transpose(rowptr, col, v, int(num_x_rows))
    return aggregation.csr_spmm(rp_t, col_t, grad.contiguous(), val=val_t, normalize=False, num_rows=int(num_x_rows))


@csr_spmm_grad_x.register_fake
def _csr_spmm_grad_x_fake(rowptr, col, val, grad, normalize, num_x_rows):
    return grad.new_empty((num_x_rows, grad.shape[1]))


def _csr_spmm_backward(ctx, grad):
    rowptr, col, val = ctx.saved_tensors
    dx = None
    if ctx.needs_input_grad[3]:
        dx = torch.ops.dgfx.csr_spmm_grad_x(rowptr, col, val, grad.to(ctx.x_dtype), ctx.normalize, ctx.num_x_rows)
    return None, None, None, dx, None, None


csr_spmm.register_autograd(_csr_spmm_backward, setup_context=_csr_spmm_setup)


# ---------------------------------------------------------------------------
# segment_sum
# ---------------------------------------------------------------------------
@torch.library.custom_op(f"{_LIB}::segment_sum", mutates_args=())
def segment_sum(data: torch.Tensor, segment_ids: torch.Tensor, num_segments: int, mean: bool = False) -> torch.Tensor:
    return aggregation.segment_sum(data.contiguous(), segment_ids, int(num_segments), mean=mean)


@segment_sum.register_fake
def _segment_sum_fake(data, segment_ids, num_segments, mean=False):
    return data.new_empty((num_segments, data.shape[1]))


def _segment_sum_setup(ctx, inputs, output):
    data, segment_ids, num_segments, mean = inputs
    ctx.save_for_backward(segment_ids)
    ctx.num_segments = int(num_segments)
    ctx.mean = bool(mean)
    ctx.data_dtype = data.dtype


@torch.library.custom_op(f"{_LIB}::segment_sum_grad", mutates_args=())
def segment_sum_grad(grad: torch.Tensor, segment_ids: torch.Tensor, num_segments: int, mean: bool) -> torch.Tensor:
    """d data[i] = dY[ids[i]] (/ max(count, 1) for the mean)."""
    counts = aggregation.segment_counts(segment_ids, int(num_segments)) if mean else None
    return aggregation.gather_rows_scaled(grad.contiguous(), segment_ids, int(num_segments), counts)


@segment_sum_grad.register_fake
def _segment_sum_grad_fake(grad, segment_ids, num_segments, mean):
    return grad.new_empty((segment_ids.shape[0], grad.shape[1]))


def _segment_sum_backward(ctx, grad):
    (ids,) = ctx.saved_tensors
    d = None
    if ctx.needs_input_grad[0]:
        d = torch.ops.dgfx.segment_sum_grad(grad.to(ctx.data_dtype), ids, ctx.num_segments, ctx.mean)
    return d, None, None, None


segment_sum.register_autograd(_segment_sum_backward, setup_context=_segment_sum_setup)


# ---------------------------------------------------------------------------
# Forward-only operators
# ---------------------------------------------------------------------------
@torch.library.custom_op(f"{_LIB}::segment_softmax", mutates_args=())
def segment_softmax(logits: torch.Tensor, messages: torch.Tensor, segment_ids: torch.Tensor,
                    num_segments: int) -> torch.Tensor:
    return aggregation.segment_softmax(logits.contiguous(), messages.contiguous(), segment_ids, int(num_segments))


@segment_softmax.register_fake
def _segment_softmax_fake(logits, messages, segment_ids, num_segments):
    return messages.new_empty((num_segments, messages.shape[1], messages.shape[2]))


@torch.library.custom_op(f"{_LIB}::sage_mean_linear_relu", mutates_args=())
def sage_mean_linear_relu(rowptr: torch.Tensor, col: torch.Tensor, x: torch.Tensor, weight: torch.Tensor,
                          bias: Optional[torch.Tensor]) -> torch.Tensor:
    return aggregation.sage_mean_linear_relu(rowptr, col, x.contiguous(), weight.contiguous(), bias)


@sage_mean_linear_relu.register_fake
def _sage_fake(rowptr, col, x, weight, bias):
    return x.new_empty((rowptr.shape[0] - 1, weight.shape[0]))


def gcn_propagate(x: torch.Tensor, matrix) -> torch.Tensor:
    """adj_symnorm @ x of the reference's GCN layer, matrix = (rowptr, col,
    val) from aggregation.gcn_matrix (differentiable in x)."""
    rowptr, col, val = matrix
    return torch.ops.dgfx.csr_spmm(rowptr, col, val, x, False, -1)


def gin_propagate(x: torch.Tensor, matrix) -> torch.Tensor:
    """(adj + adj^T + (1 + eps) I) @ x of the reference's GIN layer, matrix
    from aggregation.gin_matrix (differentiable in x)."""
    rowptr, col, val = matrix
    return torch.ops.dgfx.csr_spmm(rowptr, col, val, x, False, -1)
