"""The .bf2 on-disk format (reference layout, opacc1ty/format/)."""

from .bf2 import BF2Reader, BF2Writer, xxh64
from .header import CHECKSUM_BYTES, FLAG_CHECKSUM, HEADER_SIZE, MAGIC, VERSION, BF2Header, LayerFormat, LayerType

__all__ = ["BF2Header", "LayerFormat", "LayerType", "BF2Writer", "BF2Reader", "MAGIC", "VERSION", "HEADER_SIZE",
           "FLAG_CHECKSUM", "CHECKSUM_BYTES", "xxh64"]
