"""Raw node id -> node index on the GPU.

``ByteIdToIdxMapper`` and ``PairMapping`` keep the interface and results of
dgf/src/io/io_ext.cc:26-170 (numpy in, numpy out: int64 indices, -1 for an
unknown id, plus the position of the last unknown id or -1); ``IdIndex`` is
the device form used by the graph loader: it indexes integer ids, numpy
fixed-width byte ids or Arrow binary columns where they lie on the GPU
(``dgfx_id_index_*``) and looks ids up into CUDA tensors.
"""

from __future__ import annotations

import ctypes
from typing import Tuple

import numpy as np

from distributed_graph_flow_b200 import _native

IDS_INT64, IDS_FIXED, IDS_VAR = 0, 1, 2


def _arrow_binary(column):
    """(offsets int64 numpy [n + 1], data uint8 numpy) of an Arrow binary /
    string column (Array or ChunkedArray), or None if it is not one."""
    try:
        import pyarrow as pa
    except ImportError:  # pragma: no cover
        return None
    if isinstance(column, pa.ChunkedArray):
        column = column.combine_chunks() if column.num_chunks != 1 else column.chunk(0)
    if not isinstance(column, pa.Array):
        return None
    t = column.type
    if not (pa.types.is_binary(t) or pa.types.is_large_binary(t) or pa.types.is_string(t)
            or pa.types.is_large_string(t)):
        return None
    if column.null_count:
        raise ValueError("null ids are not supported")
    large = pa.types.is_large_binary(t) or pa.types.is_large_string(t)
    bufs = column.buffers()
    off = np.frombuffer(bufs[1], dtype=np.int64 if large else np.int32)[column.offset:column.offset + len(column) + 1]
    data = np.frombuffer(bufs[2], dtype=np.uint8) if bufs[2] is not None else np.zeros(0, np.uint8)
    off = off.astype(np.int64)
    return off, data


class _DeviceIds:
    """Ids uploaded to the device in one of the three layouts."""

    def __init__(self, ids, device):
        torch = _native.require_cuda()
        self.offsets = None
        self.width = 0
        arrow = _arrow_binary(ids)
        if arrow is not None:
            off, data = arrow
            self.kind = IDS_VAR
            self.n = len(off) - 1
            base = int(off[0])
            self.offsets = torch.from_numpy(off - base).to(device)
            self.data = torch.from_numpy(np.ascontiguousarray(data[base:int(off[-1])])).to(device)
            return
        if isinstance(ids, torch.Tensor):
            if not ids.is_cuda:
                ids = ids.to(device)
            if ids.dtype == torch.uint8 and ids.dim() == 2:
                self.kind, self.n, self.width = IDS_FIXED, int(ids.shape[0]), int(ids.shape[1])
                self.data = ids.contiguous()
            else:
                self.kind, self.n = IDS_INT64, int(ids.numel())
                self.data = ids.reshape(-1).to(torch.int64).contiguous()
            return
        a = np.asarray(ids)
        if a.dtype.kind == "O":
            a = a.astype(np.bytes_)
        if a.ndim != 1:
            raise ValueError(f"ids must be a 1D array, got shape {a.shape}")
        self.n = a.shape[0]
        if a.dtype.kind == "S":
            self.kind = IDS_FIXED
            self.width = max(1, a.dtype.itemsize)
            if a.dtype.itemsize == 0:
                a = np.zeros(self.n, dtype="S1")
            raw = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
            self.data = torch.from_numpy(raw.copy() if raw.size else np.zeros(1, np.uint8)).to(device)
        elif a.dtype.kind == "U":
            return self.__init__(np.char.encode(a, "utf-8"), device)
        elif a.dtype.kind in "iub":
            self.kind = IDS_INT64
            self.data = torch.from_numpy(np.ascontiguousarray(a.astype(np.int64))).to(device)
        else:
            raise ValueError(f"unsupported id dtype {a.dtype}")

    def args(self):
        return (self.kind, _native.ptr(self.data), _native.ptr(self.offsets), int(self.width), int(self.n))


class IdIndex:
    """Device index of a node set's raw ids (last position wins for repeated
    ids; byte ids compare without trailing zero bytes)."""

    def __init__(self, ids, device=None):
        torch = _native.require_cuda()
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        with torch.cuda.device(self.device):
            self._ids = _DeviceIds(ids, self.device)
            need = ctypes.c_size_t()
            _native.check(_native.lib().dgfx_id_index_table_bytes(self._ids.n, ctypes.byref(need)))
            # The table comes from torch's caching allocator (no cudaMalloc per index).
            self._table = torch.empty(need.value, dtype=torch.uint8, device=self.device)
            h = ctypes.c_void_p()
            _native.check(_native.lib().dgfx_id_index_create(*self._ids.args(), _native.ptr(self._table),
                                                             need.value, _native.stream_handle(), ctypes.byref(h)))
        self._h = h.value
        self.num_ids = self._ids.n
        self.integer = self._ids.kind == IDS_INT64

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _native.lib().dgfx_id_index_destroy(h)
            except Exception:  # interpreter shutdown
                pass
            self._h = None

    def lookup(self, ids, out=None) -> Tuple[object, int]:
        """(int64 CUDA tensor of indices, -1 for unknown ids; position of the
        last unknown id or -1). ``out`` may be a preallocated int64 view."""
        torch = _native.require_cuda()
        with torch.cuda.device(self.device):
            q = ids if isinstance(ids, _DeviceIds) else _DeviceIds(ids, self.device)
            if out is None:
                out = torch.empty(max(1, q.n), dtype=torch.int64, device=self.device)[:q.n]
            mm = ctypes.c_int64(-1)
            _native.check(_native.lib().dgfx_id_index_lookup(self._h, *q.args(), _native.ptr(out), ctypes.byref(mm),
                                                             _native.stream_handle()))
        return out, int(mm.value)


class ByteIdToIdxMapper:
    """io_ext.ByteIdToIdxMapper: index byte ids; calling it maps an array of
    byte ids to (int64 indices with -1 for unknown ids, last unknown position
    or -1)."""

    def __init__(self, ids):
        a = np.asarray(ids)
        if a.dtype.kind not in "SO" and _arrow_binary(ids) is None:
            raise ValueError(f"Expecting a buffer of np.bytes (i.e. 's') array. Got a buffer of '{a.dtype}' instead")
        self._index = IdIndex(ids)

    def __call__(self, ids) -> Tuple[np.ndarray, int]:
        out, mismatch = self._index.lookup(ids)
        return out.cpu().numpy(), mismatch


def PairMapping(mapper1: ByteIdToIdxMapper, mapper2: ByteIdToIdxMapper, ids1, ids2,
                num_threads: int = 1) -> Tuple[np.ndarray, int, int]:
    """io_ext.PairMapping: both lookups stacked into one int64 [2, n] array,
    with each side's last unknown position (num_threads is accepted for
    compatibility; the GPU grid replaces the thread pool)."""
    torch = _native.require_cuda()
    n1 = len(ids1)
    if n1 != len(ids2):
        raise ValueError("Input arrays ids1 and ids2 must have the same size.")
    out = torch.empty((2, max(1, n1)), dtype=torch.int64, device=mapper1._index.device)
    _, m1 = mapper1._index.lookup(ids1, out=out[0, :n1])
    _, m2 = mapper2._index.lookup(ids2, out=out[1, :n1])
    return out[:, :n1].cpu().numpy(), m1, m2
