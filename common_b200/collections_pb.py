"""The reference's protobuf state-dictionary format, on the host, without a protobuf library.

Messages (engine/ml/src/main/proto/collections.proto):
  CollectionLibraryData  { repeated CollectionLibraryEntry collections = 1; }
  CollectionLibraryEntry { string key = 1; CollectionData collection = 2; }
  CollectionData         { TraversalPolicyData traversal_policy = 1; repeated double data = 2;
                           repeated float data_32 = 3; }
  TraversalPolicyData    { repeated int32 dims = 1; int32 traversal_axis = 2; }

read_library / read_directory index the entries of memory-mapped files and decode a tensor only when it is
asked for (StateDictionary.loadWeights, engine/ml/src/main/java/org/almostrealism/ml/StateDictionary.java:119-150,
with CollectionEncoder.decode, engine/ml/src/main/java/org/almostrealism/persist/assets/CollectionEncoder.java:150-185:
`data` doubles when present, else `data_32` floats; an entry without dimensions is null and dropped).
encode_library / save write the form StateDictionary.encode / save produce (StateDictionary.java:215-265,
CollectionEncoder.encode :55-95): entries in the map's order, dims then traversal_axis (omitted when 0, as
proto3 does), values packed as fp32 (`data_32`, the default) or fp64 (`data`).

The library loads the same files itself (qw_load_state_dict_pb); this module serves StateDictionary.get on
the host and writes files.
"""
from __future__ import annotations

import mmap
import os
import warnings

import numpy as np

__all__ = ["PbFormatError", "encode_library", "save", "read_library", "read_directory", "LazyEntry"]


class PbFormatError(ValueError):
    """Bytes that are not a CollectionLibraryData message."""


# ---------------------------------------------------------------- wire format

def _varint(buf, i: int, end: int):
    v = 0
    shift = 0
    while True:
        if i >= end or shift >= 64:
            raise PbFormatError("truncated varint")
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if not b & 0x80:
            return v, i
        shift += 7


def _fields(buf, i: int, end: int):
    """Yield (field, wire_type, value, start, stop) over one message; value is the varint, or None for
    length-delimited / fixed fields whose bytes are buf[start:stop]."""
    while i < end:
        tag, i = _varint(buf, i, end)
        field, wt = tag >> 3, tag & 7
        if wt == 0:
            v, i = _varint(buf, i, end)
            yield field, wt, v, i, i
        elif wt == 1 or wt == 5:
            n = 8 if wt == 1 else 4
            if i + n > end:
                raise PbFormatError("truncated fixed field")
            yield field, wt, None, i, i + n
            i += n
        elif wt == 2:
            n, i = _varint(buf, i, end)
            if i + n > end:
                raise PbFormatError("truncated length-delimited field")
            yield field, wt, None, i, i + n
            i += n
        else:
            raise PbFormatError(f"wire type {wt}")


def _int32(v: int) -> int:
    v &= 0xFFFFFFFF  # int32 fields carry the low 32 bits (negative values are sign-extended varints)
    return v - (1 << 32) if v & 0x80000000 else v


class LazyEntry:
    """One collection: its shape, and the byte ranges its values occupy in the mapped file."""

    __slots__ = ("key", "shape", "traversal_axis", "_buf", "_f64", "_f32")

    def __init__(self, key, shape, axis, buf, f64, f32):
        self.key, self.shape, self.traversal_axis, self._buf = key, tuple(shape), axis, buf
        self._f64, self._f32 = f64, f32  # lists of (start, stop, packed)

    @property
    def dtype(self):
        return np.float64 if self._has64() else np.float32

    def _has64(self):
        return any(b > a for a, b, _ in self._f64)

    def _values(self, ranges, dt):
        parts = [np.frombuffer(self._buf, dt, (b - a) // dt.itemsize, a) for a, b, _ in ranges]
        return np.concatenate(parts).astype(dt.newbyteorder("="))

    def numpy(self) -> np.ndarray:
        """The values in the precision stored (float64 from `data`, float32 from `data_32`)."""
        if self._has64():
            v = self._values(self._f64, np.dtype("<f8"))
        else:
            v = self._values(self._f32, np.dtype("<f4")) if self._f32 else np.zeros(0, np.float32)
        n = int(np.prod(self.shape, dtype=np.int64))
        if v.size != n:
            raise PbFormatError(f"'{self.key}': {v.size} values for shape {self.shape}")
        return v.reshape(self.shape)


def _parse_collection(buf, a, b):
    dims, axis, f64, f32 = [], 0, [], []
    for field, wt, v, s, e in _fields(buf, a, b):
        if field == 1 and wt == 2:
            for f2, wt2, v2, s2, e2 in _fields(buf, s, e):
                if f2 == 1 and wt2 == 2:
                    j = s2
                    while j < e2:
                        d, j = _varint(buf, j, e2)
                        dims.append(_int32(d))
                elif f2 == 1 and wt2 == 0:
                    dims.append(_int32(v2))
                elif f2 == 2 and wt2 == 0:
                    axis = _int32(v2)
        elif field == 2 and wt in (1, 2):
            if (e - s) % 8:
                raise PbFormatError("packed double field of odd length")
            f64.append((s, e, wt == 2))
        elif field == 3 and wt in (2, 5):
            if (e - s) % 4:
                raise PbFormatError("packed float field of odd length")
            f32.append((s, e, wt == 2))
    return dims, axis, f64, f32


def parse_library(buf) -> list:
    """Every non-null entry of one CollectionLibraryData message, in file order."""
    out = []
    end = len(buf)
    for field, wt, _, s, e in _fields(buf, 0, end):
        if field != 1 or wt != 2:
            continue
        key, coll = "", None
        for f2, wt2, _, s2, e2 in _fields(buf, s, e):
            if f2 == 1 and wt2 == 2:
                key = bytes(buf[s2:e2]).decode("utf-8")
            elif f2 == 2 and wt2 == 2:
                coll = _parse_collection(buf, s2, e2)
        if coll is None or not coll[0]:
            continue  # CollectionEncoder.decode returns null for a shape without dimensions
        dims, axis, f64, f32 = coll
        out.append(LazyEntry(key, dims, axis, buf, f64, f32))
    return out


def read_library(path: str) -> dict:
    """{key: LazyEntry} of one file (later entries with the same key replace earlier ones)."""
    with open(path, "rb") as f:
        size = os.fstat(f.fileno()).st_size
        if size == 0:
            return {}
        buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    return {e.key: e for e in parse_library(memoryview(buf))}


def read_directory(path: str) -> dict:
    """StateDictionary(weightsDirectory): every non-hidden regular file, in name order; a file that does not
    parse is skipped with a warning, as StateDictionary.loadWeights does."""
    if os.path.isfile(path):
        return read_library(path)
    out = {}
    for name in sorted(os.listdir(path)):
        full = os.path.join(path, name)
        if name.startswith(".") or not os.path.isfile(full):
            continue
        try:
            out.update(read_library(full))
        except (PbFormatError, UnicodeDecodeError) as e:
            warnings.warn(f"Error reading weights from file {name}: {e}")
    return out


# ---------------------------------------------------------------- writer

def _enc_varint(v: int) -> bytes:
    v &= 0xFFFFFFFFFFFFFFFF  # negative int32 values take ten bytes, as protobuf encodes them
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _len_field(field: int, payload: bytes) -> bytes:
    return _enc_varint(field << 3 | 2) + _enc_varint(len(payload)) + payload


def encode_collection(arr, precision: str = "fp32", traversal_axis: int = 0) -> bytes:
    """CollectionData bytes of one array (CollectionEncoder.encode(c, precision))."""
    a = np.asarray(arr)
    pol = b""
    if a.ndim:
        pol += _len_field(1, b"".join(_enc_varint(int(d)) for d in a.shape))
    if traversal_axis:
        pol += _enc_varint(2 << 3) + _enc_varint(int(traversal_axis))
    body = _len_field(1, pol)
    if a.size:
        if precision == "fp64":
            body += _len_field(2, np.ascontiguousarray(a, "<f8").tobytes())
        elif precision == "fp32":
            body += _len_field(3, np.ascontiguousarray(a, "<f4").tobytes())
        else:
            raise ValueError("precision must be 'fp32' or 'fp64'")
    return body


def encode_library(weights: dict, precision: str = "fp32") -> bytes:
    """CollectionLibraryData bytes for {key: array} (StateDictionary.encode(weights, precision))."""
    parts = []
    for k, v in weights.items():
        entry = _len_field(1, k.encode("utf-8")) + _len_field(2, encode_collection(v, precision))
        parts.append(_len_field(1, entry))
    return b"".join(parts)


def save(weights: dict, path: str, precision: str = "fp32") -> None:
    """StateDictionary.save: one file holding every entry."""
    with open(path, "wb") as f:
        for k, v in weights.items():  # entry by entry: no second copy of a large model in memory
            entry = _len_field(1, k.encode("utf-8")) + _len_field(2, encode_collection(v, precision))
            f.write(_len_field(1, entry))

