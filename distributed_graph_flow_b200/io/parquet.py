"""Sharded Parquet <-> numpy, as the GF format stores node and edge sets.

Column conversion follows dgf/src/io/parquet.py:63-135: binary columns become
fixed-width numpy bytes ('S<max length>', at least 1), string columns numpy
bytes, fixed-size lists reshape to [n, size, ...], variable-length lists
become object arrays of arrays; other columns convert with pyarrow's
to_numpy. Writes follow :215-355 (one Arrow type per feature format and
shape, shards named ``<name>-<shard:05d>-of-<num_shards:05d>.parquet``).
Reading and writing files is host IO (pyarrow); the id mapping that follows
runs on the GPU (``io.ids``).
"""

from __future__ import annotations

import concurrent.futures as futures
import glob
import os
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from distributed_graph_flow_b200.data import schema as schema_lib

PARQUET_EXTENSION = ".parquet"


def _pa():
    import pyarrow as pa
    import pyarrow.parquet as pq

    return pa, pq


def binary_to_fixed_bytes(column) -> np.ndarray:
    """Arrow binary (chunked) column -> numpy 'S<max length>' (zero padded)."""
    pa, _ = _pa()
    if isinstance(column, pa.Array):
        column = pa.chunked_array([column])
    n = len(column)
    lengths = [np.diff(np.frombuffer(c.buffers()[1], dtype=np.int64 if pa.types.is_large_binary(c.type) else np.int32)
                       [c.offset:c.offset + len(c) + 1]) for c in column.chunks]
    max_len = max([int(x.max()) for x in lengths if x.size] + [0]) or 1
    out = np.zeros((n, max_len), dtype=np.uint8)
    row = 0
    for c, ln in zip(column.chunks, lengths):
        large = pa.types.is_large_binary(c.type)
        off = np.frombuffer(c.buffers()[1], dtype=np.int64 if large else np.int32)[c.offset:c.offset + len(c) + 1]
        data = np.frombuffer(c.buffers()[2], dtype=np.uint8) if c.buffers()[2] is not None else np.zeros(0, np.uint8)
        if len(c):
            # Scatter every value's bytes into its padded row in one pass.
            starts = off[:-1].astype(np.int64)
            total = int(ln.sum())
            if total:
                rows = np.repeat(np.arange(len(c)), ln)
                within = np.arange(total) - np.repeat(np.cumsum(ln) - ln, ln)
                out[row + rows, within] = data[np.repeat(starts, ln) + within]
        row += len(c)
    return out.reshape(-1).view(f"S{max_len}")


def _array_to_numpy(arr) -> np.ndarray:
    pa, _ = _pa()
    t = arr.type
    if pa.types.is_binary(t) or pa.types.is_large_binary(t):
        return binary_to_fixed_bytes(pa.chunked_array([arr]))
    if pa.types.is_list(t) or pa.types.is_large_list(t):
        flat = _array_to_numpy(arr.flatten())
        offsets = arr.offsets.to_numpy()
        if len(offsets) < 2:
            return np.empty(0, dtype=object)
        parts = np.split(flat, offsets[1:-1] - offsets[0]) if offsets[0] else np.split(flat, offsets[1:-1])
        res = np.empty(len(parts), dtype=object)
        res[:] = parts
        return res
    if pa.types.is_fixed_size_list(t):
        flat = _array_to_numpy(arr.flatten())
        if len(flat) == 0:
            return flat.reshape((0, t.list_size) + flat.shape[1:])
        return flat.reshape((-1, t.list_size) + flat.shape[1:])
    values = arr.to_numpy(zero_copy_only=False)
    if pa.types.is_string(t) or pa.types.is_large_string(t):
        values = values.astype(np.bytes_)
    return values


def column_to_numpy(column) -> np.ndarray:
    pa, _ = _pa()
    t = column.type
    if pa.types.is_binary(t) or pa.types.is_large_binary(t):
        return binary_to_fixed_bytes(column)
    parts = [_array_to_numpy(c) for c in column.chunks]
    if not parts:
        values = column.to_numpy()
        if pa.types.is_string(t):
            values = values.astype(np.bytes_)
        return values
    return parts[0] if len(parts) == 1 else np.concatenate(parts, axis=0)


def list_shards(base_path: str) -> List[str]:
    """Shards ``<base_path>-*.parquet`` in name order (util/shard.py:134-260)."""
    return sorted(glob.glob(f"{glob.escape(base_path)}-*{PARQUET_EXTENSION}"))


def read_tables(paths: Sequence[str], columns: Optional[Sequence[str]] = None):
    """Reads the shards (threads) and concatenates them into one Arrow table."""
    pa, pq = _pa()

    def one(p):
        try:
            return pq.ParquetFile(p, pre_buffer=True).read(columns=list(columns) if columns is not None else None)
        except Exception as e:
            raise ValueError(f"Failed to read Parquet file {p!r}") from e

    with futures.ThreadPoolExecutor(max_workers=max(1, min(len(paths), 20))) as ex:
        tables = list(ex.map(one, paths))
    if not tables:
        return None
    return pa.concat_tables(tables)


def table_to_numpy_dict(table) -> Tuple[Dict[str, np.ndarray], int]:
    if table is None:
        return {}, 0
    out = {name: column_to_numpy(table[name]) for name in table.column_names}
    return out, table.num_rows


_FORMAT_TO_ARROW = {
    schema_lib.FeatureFormat.INTEGER_32: "int32",
    schema_lib.FeatureFormat.INTEGER_64: "int64",
    schema_lib.FeatureFormat.FLOAT_32: "float32",
    schema_lib.FeatureFormat.FLOAT_64: "float64",
    schema_lib.FeatureFormat.BYTES: "binary",
    schema_lib.FeatureFormat.BOOL: "bool_",
}


def arrow_type(fs: schema_lib.FeatureSchema):
    pa, _ = _pa()
    t = getattr(pa, _FORMAT_TO_ARROW[fs.format])()
    if fs.shape is None or fs.shape == ():
        return t
    for size in reversed(fs.shape):
        if size is None:
            t = pa.list_(t)
        elif isinstance(size, int) and size > 0:
            t = pa.list_(t, size)
        else:
            raise ValueError(f"Invalid dimension size in shape: {size}")
    return t


def sharded_filename(name: str, shard: int, num_shards: int) -> str:
    return f"{name}-{shard:05d}-of-{num_shards:05d}{PARQUET_EXTENSION}"


def write_numpy_dict(data: Dict[str, np.ndarray], name: str, base_path: str,
                     features: schema_lib.FeatureSetSchema, num_shards: int = 1, compression: str = "snappy"):
    """Writes the columns of ``features`` in ``num_shards`` row ranges."""
    pa, pq = _pa()
    if not data:
        raise ValueError("Input data dictionary is empty.")
    num_rows = next(iter(data.values())).shape[0]
    per = (num_rows + num_shards - 1) // max(1, num_shards)

    def to_arrow(key, values, fs):
        t = arrow_type(fs)
        try:
            if fs.shape is None or fs.shape == ():
                return pa.array(values, type=t)
            if all(d is not None for d in fs.shape):
                return pa.FixedSizeListArray.from_arrays(np.ravel(values, order="C"), type=t)
            return pa.array([x.tolist() for x in values], type=t)
        except Exception as e:
            raise ValueError(f"Failed to write feature {key!r} with values={values!r} and spec={fs!r}") from e

    def shard(i):
        lo, hi = i * per, min((i + 1) * per, num_rows)
        if lo >= hi:
            return
        cols = {k: to_arrow(k, data[k][lo:hi], fs) for k, fs in features.items()}
        pq.write_table(pa.Table.from_pydict(cols), os.path.join(base_path, sharded_filename(name, i, num_shards)),
                       compression=compression)

    with futures.ThreadPoolExecutor(max_workers=max(1, min(num_shards, 20))) as ex:
        list(ex.map(shard, range(num_shards)))


def estimate_num_shards(num_rows: int) -> int:
    """util/shard.py:263-300: 1000 rows per shard, at most 100 shards."""
    n = num_rows // 1000 + (num_rows % 1000 > 0)
    return n if n <= 100 else 100
