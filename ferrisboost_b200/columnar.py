"""Columnar ingest: Parquet / CSV files and pyarrow tables into device-resident bins.

The reference reads Parquet column chunks in Rust (src/source/parquet_source.rs,
decode rules in src/source/arrow_source.rs:121-200) and pyarrow tables in
Python (python/ferrisboost/__init__.py:798-880 ``_table_matrix``).  Here pyarrow
decodes the feature columns (multi-threaded) straight into one column-major
f32 buffer, F columns of n values back to back, and
``fb_dataset_on_device_columns`` copies that buffer to the device, where the
sketch and the binning read it column by column: no row-major copy is made
on the host.

Decode rules (the reference's, value for value):
- Parquet files: Float32, Float64, Int32 and Int64 columns convert with a
  single rounding to f32 (Rust ``as f32``); a dictionary column with numeric
  values decodes through f64 (``cast(.., Float64)`` then ``as f32``); nulls and
  values equal to ``missing`` are NaN; +-inf (also from an f64 outside the
  f32 range) is an error for features, labels and weights.  Without
  ``feature_types``, dictionary columns are categorical
  (parquet_source.rs:472-500).  Other column types are errors.
- CSV files (src/source/csv_source.rs): Arrow's CSV reader infers each
  column's type (integers -> Int64, decimals -> Float64) and only an empty
  field is null; the values then follow the Parquet rules above.  With
  ``header=False`` the label (and weight) are column indices and the model
  records no feature names.
- pyarrow tables: a dictionary column needs ``enable_categorical`` and
  contributes its dictionary indices as category codes (null -> NaN); other
  columns convert with ``to_numpy`` then ``float32``.
"""
from __future__ import annotations

import base64
import glob
import math
import os
from concurrent.futures import ThreadPoolExecutor
from typing import Any, NamedTuple, Sequence

import numpy as np


class Columns(NamedTuple):
    X: np.ndarray                  # (F, n) float32, C-contiguous: column f at X[f]
    names: list[str]
    categorical: np.ndarray | None  # (F,) uint8 or None
    label: np.ndarray | None
    weight: np.ndarray | None


def path_specs(data: Any) -> list[str] | None:
    """One path or a sequence of paths -> list of path strings; None when
    ``data`` is not a path (python/ferrisboost/__init__.py:496-508)."""
    if isinstance(data, (str, os.PathLike)):
        return [os.fspath(data)]
    if isinstance(data, (list, tuple)) and data and all(isinstance(d, (str, os.PathLike)) for d in data):
        return [os.fspath(d) for d in data]
    return None


def arrow_table(obj: Any):
    """A pyarrow Table as is, a RecordBatch or RecordBatchReader read into a
    Table; None for anything else (python/ferrisboost/__init__.py:520-535)."""
    mod = type(obj).__module__ or ""
    if not mod.startswith("pyarrow"):
        return None
    if hasattr(obj, "column_names"):
        if type(obj).__name__ == "RecordBatch":
            import pyarrow as pa
            return pa.Table.from_batches([obj])
        return obj
    if hasattr(obj, "read_all"):
        return obj.read_all()
    return None


def expand_paths(specs: Sequence[str]) -> list[str]:
    """Files of the given specs in order: a directory contributes its
    ``.parquet`` / ``.pq`` / ``.csv`` files sorted by name, a pattern with
    ``*``, ``?`` or ``[`` its sorted matches, anything else itself."""
    out: list[str] = []
    for s in specs:
        if os.path.isdir(s):
            files = sorted(f for f in os.listdir(s) if f.lower().endswith((".parquet", ".pq", ".csv")))
            if not files:
                raise ValueError(f"directory {s!r} holds no .parquet or .csv files")
            out.extend(os.path.join(s, f) for f in files)
        elif any(c in s for c in "*?["):
            files = sorted(glob.glob(s))
            if not files:
                raise ValueError(f"pattern {s!r} matches no files")
            out.extend(files)
        else:
            lower = s.lower()
            if not (lower.endswith(".parquet") or lower.endswith(".pq") or lower.endswith(".csv")):
                raise ValueError(f"cannot tell the format of {s!r} from its extension; supported: .parquet / .csv")
            if not os.path.exists(s):
                raise FileNotFoundError(s)
            out.append(s)
    return out


def _check_finite(v: np.ndarray, what: str) -> None:
    bad = np.flatnonzero(np.isinf(v))
    if bad.size:
        raise ValueError(f"{what} row {int(bad[0])} is {v[bad[0]]}: +-inf or values outside the f32 range are not "
                         "supported (XGBoost rejects them too); use null / NaN for missing values")


def file_schema(path: str):
    """The Arrow schema a Parquet file was written with (its ``ARROW:schema``
    metadata, as the reference's Rust reader applies it: an integer
    dictionary column reads as a dictionary), else the schema pyarrow infers."""
    import pyarrow as pa
    import pyarrow.parquet as pq

    md = pq.read_metadata(path).metadata or {}
    raw = md.get(b"ARROW:schema")
    if raw:
        try:
            return pa.ipc.read_schema(pa.py_buffer(base64.b64decode(raw)))
        except (ValueError, pa.ArrowException):
            pass
    return pq.read_schema(path)


def _is_csv(path: str) -> bool:
    return path.lower().endswith(".csv")


def _read_csv(path: str, header: bool = True):
    """A CSV file as a pyarrow Table with Arrow's type inference; only an empty
    field is null (csv_source.rs:193-195).  Headerless columns are named
    "0", "1", ... by position."""
    import pyarrow.csv as pcsv

    ro = pcsv.ReadOptions(autogenerate_column_names=not header, use_threads=True)
    co = pcsv.ConvertOptions(null_values=[""], strings_can_be_null=True, quoted_strings_can_be_null=True)
    table = pcsv.read_csv(path, read_options=ro, convert_options=co)
    if not header:
        table = table.rename_columns([str(i) for i in range(table.num_columns)])
    return table


def _open(path: str, header: bool = True):
    """(schema, reader of named columns) of a Parquet or CSV file."""
    import pyarrow.parquet as pq

    if _is_csv(path):
        table = _read_csv(path, header)
        return table.schema, (lambda cols: table.select(list(cols))), table.num_rows
    return file_schema(path), (lambda cols: pq.read_table(path, columns=list(cols), use_threads=True)), \
        pq.ParquetFile(path).metadata.num_rows


def _file_column_f32(col, name: str, missing: float, out: np.ndarray, allow_inf: bool = False,
                     file_type=None) -> None:
    """arrow_source.rs:121-200 visit_column_f32 of one Parquet column into
    ``out`` (n float32); prediction input keeps +-inf (arrow_source.rs:73-79
    column_as_f32_allow_inf).  ``file_type`` is the column's type in the
    file's Arrow schema (a dictionary there decodes through f64 even where
    pyarrow returns the plain values)."""
    import pyarrow as pa
    import pyarrow.compute as pc

    t = col.type
    dict_values = None  # value type of a dictionary column (in the file or as read)
    if pa.types.is_dictionary(t):
        dict_values = t.value_type
    elif file_type is not None and pa.types.is_dictionary(file_type):
        dict_values = file_type.value_type
    with np.errstate(over="ignore", invalid="ignore"):
        if dict_values is not None:
            if not (pa.types.is_integer(dict_values) or pa.types.is_floating(dict_values)):
                raise ValueError(f"column {name!r} is a dictionary of {dict_values} values, which can only be a "
                                 "categorical feature with category names; this engine trains on integer "
                                 "category codes: store the codes instead")
            if pa.types.is_dictionary(t):
                col = pa.chunked_array([c.dictionary_decode() for c in col.chunks], dict_values) \
                    if col.num_chunks else pa.chunked_array([], dict_values)
            out[:] = np.asarray(col.cast(pa.float64()).to_numpy(zero_copy_only=False), np.float64).astype(np.float32)
        elif t in (pa.float32(), pa.float64()):
            # chunk by chunk into place: a float chunk without nulls is read in
            # place, and the assignment is the one f64 -> f32 rounding
            pos = 0
            for ch in col.chunks:
                out[pos:pos + len(ch)] = ch.to_numpy(zero_copy_only=False)
                pos += len(ch)
        elif t in (pa.int32(), pa.int64()):
            pos = 0
            for ch in col.chunks:
                vals = (pc.fill_null(ch, 0) if ch.null_count else ch).to_numpy(zero_copy_only=False)
                out[pos:pos + len(ch)] = vals.astype(np.int64, copy=False)
                pos += len(ch)
        else:
            raise ValueError(f"column {name!r} is {t}; only numeric columns (float32, float64, int32, int64 or a "
                             "numeric dictionary) are supported")
    if col.null_count:
        out[np.asarray(col.is_null().to_numpy(zero_copy_only=False), bool)] = np.float32("nan")
    if not allow_inf:
        _check_finite(out, f"column {name!r}")
    if not math.isnan(missing):
        out[out == np.float32(missing)] = np.float32("nan")


def read_files(specs: Sequence[str], label: "str | int | None", weight: "str | int | None", feature_types=None,
               missing: float = float("nan"), header: bool = True) -> Columns:
    """Parquet / CSV file(s) -> feature columns, label and weight columns by
    name (parquet_source.rs:36-90 LabeledSource, 447-500 feature_columns and
    resolve_categorical_flags; a headerless CSV names them by index).  Files
    are concatenated in order; every file must hold the first file's columns
    (bound by name)."""
    import pyarrow as pa

    files = expand_paths(specs)
    if not header:
        if any(not _is_csv(f) for f in files):
            raise ValueError("header=False applies to CSV files only")
        label = None if label is None else str(int(label))
        weight = None if weight is None else str(int(weight))
    opened = [_open(f, header) for f in files]
    schema = opened[0][0]
    names_all = list(schema.names)
    if len(set(names_all)) != len(names_all):
        raise ValueError(f"{files[0]} has duplicate column names")
    for what, col in (("label", label), ("weight", weight)):
        if col is not None and col not in names_all:
            where = f"column index {col}" if not header else f"column {col!r}"
            raise ValueError(f"{what} {where} is not in {files[0]} (columns: {names_all})")
    if label is None:
        raise ValueError("label must name a column of the file")
    feats = [c for c in names_all if c not in (label, weight)]
    if not feats:
        raise ValueError("the file has no feature columns besides the label")
    counts = [o[2] for o in opened]
    n = int(sum(counts))
    if n == 0:
        raise ValueError("training data must have at least one row")
    F = len(feats)
    X = np.empty((F, n), np.float32)
    y = np.empty(n, np.float32)
    w = np.empty(n, np.float32) if weight is not None else None
    dict_cols = np.zeros(F, bool)
    r0 = 0
    for f_path, (sch, read, cnt) in zip(files, opened):
        want = feats + [label] + ([weight] if weight is not None else [])
        miss = [c for c in want if c not in sch.names]
        if miss:
            raise ValueError(f"{f_path} lacks the columns {miss} of {files[0]}")
        table = read(want)
        for i, name in enumerate(feats):
            dict_cols[i] |= pa.types.is_dictionary(sch.field(name).type)
        # columns convert in parallel (the numpy copies release the GIL)
        with ThreadPoolExecutor(max(1, min(F, os.cpu_count() or 1))) as ex:
            list(ex.map(lambda i: _file_column_f32(table.column(feats[i]), feats[i], missing, X[i, r0:r0 + cnt],
                                                   file_type=sch.field(feats[i]).type), range(F)))
        for name, out in ((label, y), (weight, w)):
            if name is None:
                continue
            _file_column_f32(table.column(name), name, float("nan"), out[r0:r0 + cnt],
                             file_type=sch.field(name).type)
        r0 += cnt
    if feature_types is not None:
        ft = list(feature_types)
        if len(ft) != F:
            raise ValueError(f"feature_types has {len(ft)} entries but the data has {F} feature columns")
        cat = np.array([t == "c" for t in ft], np.uint8)
    else:
        cat = dict_cols.astype(np.uint8)
    # a headerless CSV has no column names to record (tree.rs:247)
    return Columns(X, feats if header else [], cat if cat.any() else None, y, w)


def read_file_features(specs: Sequence[str], names: Sequence[str], missing: float = float("nan")) -> np.ndarray:
    """Prediction input from Parquet / CSV file(s): the named columns, bound
    by name, as (F, n) float32 with the file decode rules (+-inf kept)."""
    files = expand_paths(specs)
    opened = [_open(f) for f in files]
    X = np.empty((len(names), int(sum(o[2] for o in opened))), np.float32)
    r0 = 0
    for f_path, (sch, read, cnt) in zip(files, opened):
        miss = [c for c in names if c not in sch.names]
        if miss:
            raise ValueError(f"{f_path} lacks the model's feature columns {miss}")
        table = read(names)
        with ThreadPoolExecutor(max(1, min(len(names), os.cpu_count() or 1))) as ex:
            list(ex.map(lambda i: _file_column_f32(table.column(names[i]), names[i], missing, X[i, r0:r0 + cnt],
                                                   allow_inf=True, file_type=sch.field(names[i]).type),
                        range(len(names))))
        r0 += cnt
    return X


def read_table(table, enable_categorical: bool = False, feature_types=None, missing: float = float("nan"),
               order: Sequence[str] | None = None, what: str = "data", scoring: bool = False) -> Columns:
    """A pyarrow Table -> feature columns (python/ferrisboost/__init__.py:798-880
    ``_table_matrix``): columns in table order, or bound by name to ``order``.
    ``scoring`` (prediction input): an integer dictionary contributes its
    values (the codes, as a Parquet file's dictionary does) rather than its
    indices."""
    import pyarrow as pa

    names = list(table.column_names)
    dups = sorted({c for c in names if names.count(c) > 1})
    if dups:
        raise ValueError(f"{what} has duplicate column names {dups}; column names must be unique")
    if order is not None:
        missing_cols = [c for c in order if c not in names]
        extra = [c for c in names if c not in order]
        if missing_cols or extra:
            raise ValueError(f"{what} columns do not match the training data (bound by name): missing "
                             f"{missing_cols}, extra {extra}")
        names = list(order)
    if any(pa.types.is_dictionary(table.schema.field(c).type) for c in names):
        table = table.unify_dictionaries()
    n, F = table.num_rows, len(names)
    X = np.empty((F, n), np.float32)
    flags = np.zeros(F, np.uint8)
    for i, name in enumerate(names):
        col = table.column(name)
        if scoring and pa.types.is_dictionary(col.type) and pa.types.is_integer(col.type.value_type):
            dec = pa.chunked_array([c.dictionary_decode() for c in col.chunks], col.type.value_type)
            X[i] = np.asarray(dec.cast(pa.float64()).to_numpy(zero_copy_only=False), np.float64).astype(np.float32)
            flags[i] = 1
        elif pa.types.is_dictionary(col.type):
            if not enable_categorical and not scoring:
                raise ValueError(f"{what} column {name!r} has dictionary type; to train it as a categorical "
                                 "feature, set params['enable_categorical'] = True")
            codes = np.concatenate([np.asarray(c.indices.cast(pa.int64()).fill_null(-1).to_numpy(
                zero_copy_only=False), np.int64) for c in col.chunks]) if col.num_chunks else np.empty(0, np.int64)
            X[i] = np.where(codes < 0, np.float32("nan"), codes.astype(np.float32))
            flags[i] = 1
        else:
            with np.errstate(over="ignore", invalid="ignore"):
                X[i] = np.asarray(col.to_numpy(zero_copy_only=False), dtype=np.float32)
    if not math.isnan(missing):
        X[X == np.float32(missing)] = np.float32("nan")
    if feature_types is not None:
        ft = list(feature_types)
        if len(ft) != F:
            raise ValueError(f"feature_types has {len(ft)} entries, the data has {F} features")
        flags = np.array([t == "c" for t in ft], np.uint8)
    return Columns(X, names, flags if flags.any() else None, None, None)
