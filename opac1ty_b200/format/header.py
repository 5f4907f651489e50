"""The .bf2 file and layer headers, byte-compatible with opacc1ty/format/header.py.

File layout (opacc1ty/format/header.py:7-43 and :131-148):
    magic "BF2\\0" | version u32 | flags u32 | model-JSON length u32 | model-JSON length u32
    (written twice) | model JSON | quant-JSON length u32 | quant JSON | layer count u32
    then per layer: 64-byte header | name | codebooks | indices | outlier values | outlier ids

Layer header, 64 bytes little-endian "<H B I I I B B H Q Q Q Q 13s" (header.py:82-97):
    name_len, type, out_features, in_features, n_groups, codebook_entries, sub_vector_size,
    n_outliers, cb_offset, idx_offset, out_val_offset, out_idx_offset, 13 reserved bytes.
The struct layout is the reference's (a format must match byte for byte to be a drop-in); the
code around it is this package's.

Element-wise outliers use the layer type the reference reserves for them, SPARSE_OUTLIER (1),
which its writer never emits (header.py:57-60): the payload is the quantized layer's codebooks and
indices, then the outlier values [nnz] fp16, then their positions [nnz][2] int32 (row, col).  The
entry count does not fit the u16 n_outliers field (1 % of a 4096 x 4096 layer is 167772), so it
is stored as a u64 in the first 8 reserved bytes and n_outliers is 0.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Tuple

MAGIC = b"BF2\x00"
VERSION = 1
HEADER_SIZE = 64
# File-header flag: the file ends with the XXH64 checksum (seed 0, little-endian u64) of every
# byte before it, the trailer the reference's format description lists (header.py:26) but its
# writer never emits.  Without the flag a file is byte-identical to the reference writer's.
FLAG_CHECKSUM = 0x1
CHECKSUM_BYTES = 8
_LAYER_STRUCT = struct.Struct("<H B I I I B B H Q Q Q Q 13s")
_FILE_PREFIX = struct.Struct("<4s I I I")
_U32 = struct.Struct("<I")
assert _LAYER_STRUCT.size == HEADER_SIZE


class LayerType(IntEnum):
    QUANTIZED = 0
    SPARSE_OUTLIER = 1
    FP16_PASSTHROUGH = 2


@dataclass
class LayerFormat:
    """On-disk description of one layer (mirrors opacc1ty.format.header.LayerFormat)."""

    name: str
    layer_type: LayerType
    out_features: int
    in_features: int
    n_groups: int = 0
    codebook_entries: int = 4
    sub_vector_size: int = 8
    n_outliers: int = 0
    cb_offset: int = 0
    idx_offset: int = 0
    out_val_offset: int = 0
    out_idx_offset: int = 0
    nnz: int = 0   # SPARSE_OUTLIER: element outliers (first 8 reserved bytes)

    def pack(self) -> bytes:
        name_bytes = self.name.encode("utf-8")[:256]
        return _LAYER_STRUCT.pack(
            len(name_bytes), int(self.layer_type), self.out_features, self.in_features, self.n_groups,
            self.codebook_entries, self.sub_vector_size, self.n_outliers, self.cb_offset, self.idx_offset,
            self.out_val_offset, self.out_idx_offset,
            (int(self.nnz).to_bytes(8, "little") + b"\x00" * 5) if self.layer_type == LayerType.SPARSE_OUTLIER
            else b"\x00" * 13,
        )

    @classmethod
    def unpack(cls, data: bytes) -> "LayerFormat":
        (_name_len, ltype, out_f, in_f, n_grp, cb_ent, svs, n_out, cb_off, idx_off, ov_off, oi_off,
         reserved) = _LAYER_STRUCT.unpack(data[:HEADER_SIZE])
        lt = LayerType(ltype)
        nnz = int.from_bytes(reserved[:8], "little") if lt == LayerType.SPARSE_OUTLIER else 0
        return cls(name="", layer_type=lt, out_features=out_f, in_features=in_f, n_groups=n_grp,
                   codebook_entries=cb_ent, sub_vector_size=svs, n_outliers=n_out, cb_offset=cb_off,
                   idx_offset=idx_off, out_val_offset=ov_off, out_idx_offset=oi_off, nnz=nnz)

    @staticmethod
    def name_length(data: bytes) -> int:
        return struct.unpack_from("<H", data, 0)[0]

    # Byte sizes of the payload regions (BF2Reader._build_index, bf2.py:204-218).
    def codebook_bytes(self) -> int:
        return self.n_groups * self.codebook_entries * self.sub_vector_size * 2

    def index_bytes(self) -> int:
        if self.sub_vector_size == 0:
            return 0
        return self.n_groups * (self.in_features // self.sub_vector_size)

    def outlier_value_bytes(self) -> int:
        return self.n_outliers * self.in_features * 2

    def payload_bytes(self, id_bytes: int = 4) -> int:
        if self.layer_type == LayerType.SPARSE_OUTLIER:
            return self.codebook_bytes() + self.index_bytes() + self.nnz * (2 + 8)
        if self.layer_type == LayerType.QUANTIZED:
            n = self.codebook_bytes() + self.index_bytes()
            if self.n_outliers > 0:
                n += self.outlier_value_bytes() + self.n_outliers * id_bytes
            return n
        if self.layer_type == LayerType.FP16_PASSTHROUGH:
            return self.out_features * self.in_features * 2
        return 0


@dataclass
class BF2Header:
    """Top-level file header (mirrors opacc1ty.format.header.BF2Header)."""

    version: int = VERSION
    flags: int = 0
    model_config: dict = field(default_factory=dict)
    quantize_config: dict = field(default_factory=dict)
    layer_count: int = 0

    def pack(self) -> bytes:
        model_json = json.dumps(self.model_config).encode("utf-8")
        quant_json = json.dumps(self.quantize_config).encode("utf-8")
        return b"".join([
            _FILE_PREFIX.pack(MAGIC, self.version, self.flags, len(model_json)),
            _U32.pack(len(model_json)), model_json,
            _U32.pack(len(quant_json)), quant_json,
            _U32.pack(self.layer_count),
        ])

    @classmethod
    def unpack(cls, data: bytes) -> Tuple["BF2Header", int]:
        """Parse the header; returns (header, bytes consumed).  Raises ValueError on a bad magic
        or a truncated header."""
        if len(data) < 24:
            raise ValueError("BF2 header truncated")
        magic, version, flags, _model_len = _FILE_PREFIX.unpack_from(data, 0)
        if magic != MAGIC:
            raise ValueError(f"Not a BF2 file: magic={magic!r}")
        pos = 16
        (mlen,) = _U32.unpack_from(data, pos)
        pos += 4
        if pos + mlen + 4 > len(data):
            raise ValueError("BF2 header truncated (model JSON)")
        model = json.loads(data[pos:pos + mlen].decode("utf-8"))
        pos += mlen
        (qlen,) = _U32.unpack_from(data, pos)
        pos += 4
        if pos + qlen + 4 > len(data):
            raise ValueError("BF2 header truncated (quantize JSON)")
        quant = json.loads(data[pos:pos + qlen].decode("utf-8"))
        pos += qlen
        (count,) = _U32.unpack_from(data, pos)
        pos += 4
        return cls(version=version, flags=flags, model_config=model, quantize_config=quant, layer_count=count), pos
