"""Reader and writer for .bf2 files (the reference's layer layout, opacc1ty/format/bf2.py).

Differences from the reference, all fixes that keep the on-disk layout:
  * Outlier row ids are written as int32, the width the header arithmetic and the reader assume
    (bf2.py:212, :280-283).  The reference writer emits whatever tensor it is given, and the
    quantizer produces int64 (torch.where), so its files misalign every layer after an outlier
    layer.  This reader accepts both widths: for each quantized layer with outliers it checks
    which candidate end position is followed by a valid layer header (or the end of file).
  * The layer index stores each layer's file position, so load_layer is O(1) instead of a
    rescan of the file per call (bf2.py:300-328).  The file is memory-mapped.
  * The file header is parsed from however many bytes it needs (the reference reads a fixed
    1024 bytes, bf2.py:181, and fails on longer model metadata).
  * Optionally (``BF2Writer.write(..., checksum=True)``) the file ends with the XXH64 checksum
    that the reference's format description promises (header.py:26) and the file header's flags
    say so; the reader then verifies it.  A reader that ignores the flag (the reference's) reads
    such a file unchanged: layers are found by their own offsets.
"""

from __future__ import annotations

import mmap
import os
from pathlib import Path
from typing import BinaryIO, Dict, Optional, Tuple

import numpy as np
import torch

import ctypes

from .header import CHECKSUM_BYTES, FLAG_CHECKSUM, HEADER_SIZE, BF2Header, LayerFormat, LayerType


def xxh64(data, seed: int = 0) -> int:
    """XXH64 of a bytes-like object or a contiguous numpy array (the C library's opc_xxh64)."""
    from .. import _lib

    a = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data.reshape(-1).view(np.uint8)
    ptr = a.ctypes.data_as(ctypes.c_void_p) if a.size else None
    return int(_lib.load().opc_xxh64(ptr, a.size, seed))


def _np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().contiguous().numpy()
    return np.ascontiguousarray(np.asarray(t))


class BF2Writer:
    """Writes quantized layer dicts to a .bf2 file (mirrors opacc1ty.format.bf2.BF2Writer)."""

    def __init__(self, path: str):
        self.path = Path(path)
        self.file: Optional[BinaryIO] = None

    def write(self, layers: Dict[str, dict], model_config: dict, quantize_config: dict, progress: bool = True,
              checksum: bool = False):
        """Write the layers; ``checksum`` appends the XXH64 trailer and sets FLAG_CHECKSUM."""
        items = [(k, v) for k, v in layers.items() if not k.startswith("_")]
        header = BF2Header(model_config=model_config, quantize_config=quantize_config, layer_count=len(items),
                           flags=FLAG_CHECKSUM if checksum else 0)
        self.file = open(self.path, "w+b")
        try:
            self.file.write(header.pack())
            for name, layer in items:
                self._write_layer(name, layer)
            size = self.file.tell()
            if checksum:
                self.file.flush()
                with mmap.mmap(self.file.fileno(), 0, access=mmap.ACCESS_READ) as mm:
                    digest = xxh64(mm)
                self.file.write(digest.to_bytes(CHECKSUM_BYTES, "little"))
                size += CHECKSUM_BYTES
        finally:
            self.file.close()
            self.file = None
        if progress:
            orig = sum(int(np.prod(v.get("shape", (0,)))) * 2 for k, v in layers.items() if not k.startswith("_"))
            ratio = size / orig if orig else 0.0
            print(f"\nWrote {self.path} ({size / 1e9:.2f} GB, {ratio:.1f}x compression)")

    def _write_layer(self, name: str, layer: dict):
        ltype = layer["type"]
        shape = tuple(layer["shape"])
        out_f, in_f = shape[0], (shape[1] if len(shape) > 1 else 1)
        name_bytes = name.encode("utf-8")
        data_start = HEADER_SIZE + len(name_bytes)
        f = self.file
        if ltype == "quantized":
            cb = _np(layer["codebooks"]).astype(np.float16, copy=False)
            idx = _np(layer["indices"]).astype(np.uint8, copy=False)
            ov = layer.get("outlier_values")
            oi = layer.get("outlier_indices")
            n_out = 0 if ov is None else len(ov)
            if n_out > 0xFFFF:
                raise ValueError(f"{name}: {n_out} outlier rows exceed the u16 header field")
            fmt = LayerFormat(
                name=name, layer_type=LayerType.QUANTIZED, out_features=out_f, in_features=in_f,
                n_groups=cb.shape[0], codebook_entries=cb.shape[1], sub_vector_size=cb.shape[2],
                n_outliers=n_out, cb_offset=data_start, idx_offset=data_start + cb.nbytes,
                out_val_offset=(data_start + cb.nbytes + idx.nbytes) if n_out else 0,
                out_idx_offset=(data_start + cb.nbytes + idx.nbytes + n_out * in_f * 2) if n_out else 0,
            )
            f.write(fmt.pack())
            f.write(name_bytes)
            f.write(cb.tobytes())
            f.write(idx.tobytes())
            if n_out:
                f.write(_np(ov).astype(np.float16, copy=False).tobytes())
                f.write(_np(oi).astype(np.int32).tobytes())
        elif ltype == "sparse_outlier":
            cb = _np(layer["codebooks"]).astype(np.float16, copy=False)
            idx = _np(layer["indices"]).astype(np.uint8, copy=False)
            ov = layer.get("outlier_values")
            oi = layer.get("outlier_indices")
            vals = np.zeros(0, np.float16) if ov is None else _np(ov).astype(np.float16, copy=False).reshape(-1)
            pos = np.zeros((0, 2), np.int32) if oi is None else _np(oi).astype(np.int32).reshape(-1, 2)
            if len(vals) != len(pos):
                raise ValueError(f"{name}: {len(vals)} outlier values for {len(pos)} positions")
            nnz = len(vals)
            fmt = LayerFormat(
                name=name, layer_type=LayerType.SPARSE_OUTLIER, out_features=out_f, in_features=in_f,
                n_groups=cb.shape[0], codebook_entries=cb.shape[1], sub_vector_size=cb.shape[2], n_outliers=0,
                cb_offset=data_start, idx_offset=data_start + cb.nbytes,
                out_val_offset=data_start + cb.nbytes + idx.nbytes,
                out_idx_offset=data_start + cb.nbytes + idx.nbytes + 2 * nnz, nnz=nnz,
            )
            f.write(fmt.pack())
            f.write(name_bytes)
            f.write(cb.tobytes())
            f.write(idx.tobytes())
            f.write(vals.tobytes())
            f.write(np.ascontiguousarray(pos).tobytes())
        elif ltype == "fp16_passthrough":
            data = _np(layer["data"]).astype(np.float16, copy=False)
            fmt = LayerFormat(name=name, layer_type=LayerType.FP16_PASSTHROUGH, out_features=out_f, in_features=in_f,
                              cb_offset=data_start)
            f.write(fmt.pack())
            f.write(name_bytes)
            f.write(data.tobytes())
        else:
            raise ValueError(f"{name}: cannot write layer type {ltype!r}")

    def close(self):
        if self.file:
            self.file.close()
            self.file = None


class BF2Reader:
    """Memory-mapped .bf2 reader (mirrors opacc1ty.format.bf2.BF2Reader)."""

    def __init__(self, path: str, verify_checksum: bool = True):
        self.path = Path(path)
        self._fh = open(self.path, "rb")
        size = os.fstat(self._fh.fileno()).st_size
        self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ) if size else b""
        self.header, self._data_start = BF2Header.unpack(self._mm[: min(size, 1 << 20)] if size else b"")
        self.has_checksum = bool(self.header.flags & FLAG_CHECKSUM)
        # the layers end where the checksum trailer (if any) begins
        self._size = size - CHECKSUM_BYTES if self.has_checksum else size
        if self._data_start > self._size:
            raise ValueError("BF2 header runs past the end of the file")
        # name -> (LayerFormat, header position, id width in bytes)
        self._index: Dict[str, Tuple[LayerFormat, int, int]] = {}
        self._build_index()
        self.checksum_ok: Optional[bool] = None
        if self.has_checksum and verify_checksum:
            self.verify()

    def checksum(self) -> Tuple[int, int]:
        """(stored, computed) XXH64 of a file written with FLAG_CHECKSUM."""
        if not self.has_checksum:
            raise ValueError(f"{self.path}: written without a checksum")
        stored = int.from_bytes(bytes(self._mm[self._size:self._size + CHECKSUM_BYTES]), "little")
        return stored, xxh64(memoryview(self._mm)[: self._size])

    def verify(self) -> bool:
        """Check the trailer; raises ValueError when the file does not match it."""
        stored, computed = self.checksum()
        self.checksum_ok = stored == computed
        if not self.checksum_ok:
            raise ValueError(f"{self.path}: checksum mismatch (stored {stored:016x}, computed {computed:016x})")
        return True

    # -- index ---------------------------------------------------------------------------
    def _parse_at(self, pos: int) -> Optional[Tuple[LayerFormat, int]]:
        if pos + HEADER_SIZE > self._size:
            return None
        raw = self._mm[pos:pos + HEADER_SIZE]
        try:
            fmt = LayerFormat.unpack(raw)
        except ValueError:
            return None
        nlen = LayerFormat.name_length(raw)
        if nlen == 0 or pos + HEADER_SIZE + nlen > self._size:
            return None
        try:
            fmt.name = bytes(self._mm[pos + HEADER_SIZE: pos + HEADER_SIZE + nlen]).decode("utf-8")
        except UnicodeDecodeError:
            return None
        return fmt, nlen

    def _build_index(self):
        pos = self._data_start
        n = self.header.layer_count
        for i in range(n):
            parsed = self._parse_at(pos)
            if parsed is None:
                raise ValueError(f"{self.path}: layer {i} header at byte {pos} is invalid or truncated")
            fmt, nlen = parsed
            base = pos + HEADER_SIZE + nlen
            id_bytes = 4
            if fmt.layer_type == LayerType.QUANTIZED and fmt.n_outliers > 0:
                end4 = base + fmt.payload_bytes(4)
                end8 = base + fmt.payload_bytes(8)
                last = i == n - 1
                ok4 = (end4 == self._size) if last else self._parse_at(end4) is not None
                ok8 = (end8 == self._size) if last else self._parse_at(end8) is not None
                if not ok4 and ok8:
                    id_bytes = 8
                elif not ok4 and not ok8 and not last:
                    raise ValueError(f"{self.path}: cannot locate the layer after {fmt.name!r}")
            end = base + fmt.payload_bytes(id_bytes)
            if end > self._size:
                raise ValueError(f"{self.path}: layer {fmt.name!r} is truncated")
            self._index[fmt.name] = (fmt, pos, id_bytes)
            pos = end

    # -- public API (opacc1ty/format/bf2.py:222-331) ----------------------------------------
    @property
    def model_config(self) -> dict:
        return self.header.model_config

    @property
    def quantize_config(self) -> dict:
        return self.header.quantize_config

    def layer_names(self) -> list:
        return list(self._index.keys())

    def layer_format(self, name: str) -> LayerFormat:
        return self._index[name][0]

    def _array(self, off: int, nbytes: int, dtype, shape) -> torch.Tensor:
        a = np.frombuffer(self._mm, dtype=dtype, count=nbytes // np.dtype(dtype).itemsize, offset=off)
        return torch.from_numpy(a.reshape(shape).copy())

    def load_layer(self, name: str) -> dict:
        if name not in self._index:
            raise KeyError(f"Layer '{name}' not found in BF2 file")
        fmt, pos, id_bytes = self._index[name]
        off = pos + HEADER_SIZE + len(name.encode("utf-8"))
        if fmt.layer_type == LayerType.QUANTIZED:
            ipr = fmt.in_features // fmt.sub_vector_size
            cb = self._array(off, fmt.codebook_bytes(), np.float16,
                             (fmt.n_groups, fmt.codebook_entries, fmt.sub_vector_size))
            off += fmt.codebook_bytes()
            idx = self._array(off, fmt.index_bytes(), np.uint8, (fmt.n_groups, ipr))
            off += fmt.index_bytes()
            out = {"type": "quantized", "shape": (fmt.out_features, fmt.in_features), "codebooks": cb,
                   "indices": idx}
            if fmt.n_outliers > 0:
                out["outlier_values"] = self._array(off, fmt.outlier_value_bytes(), np.float16,
                                                    (fmt.n_outliers, fmt.in_features))
                off += fmt.outlier_value_bytes()
                ids = self._array(off, fmt.n_outliers * id_bytes, np.int32 if id_bytes == 4 else np.int64,
                                  (fmt.n_outliers,))
                out["outlier_indices"] = ids.to(torch.int32)
            return out
        if fmt.layer_type == LayerType.SPARSE_OUTLIER:
            ipr = fmt.in_features // fmt.sub_vector_size
            cb = self._array(off, fmt.codebook_bytes(), np.float16,
                             (fmt.n_groups, fmt.codebook_entries, fmt.sub_vector_size))
            off += fmt.codebook_bytes()
            idx = self._array(off, fmt.index_bytes(), np.uint8, (fmt.n_groups, ipr))
            off += fmt.index_bytes()
            vals = self._array(off, 2 * fmt.nnz, np.float16, (fmt.nnz,))
            off += 2 * fmt.nnz
            pos = self._array(off, 8 * fmt.nnz, np.int32, (fmt.nnz, 2))
            return {"type": "sparse_outlier", "shape": (fmt.out_features, fmt.in_features), "codebooks": cb,
                    "indices": idx, "outlier_values": vals, "outlier_indices": pos.to(torch.int64)}
        if fmt.layer_type == LayerType.FP16_PASSTHROUGH:
            data = self._array(off, fmt.payload_bytes(), np.float16, (fmt.out_features, fmt.in_features))
            return {"type": "fp16_passthrough", "shape": (fmt.out_features, fmt.in_features), "data": data}
        raise ValueError(f"{name}: layer type {fmt.layer_type!r} has no payload reader")

    def close(self):
        if isinstance(self._mm, mmap.mmap):
            self._mm.close()
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
