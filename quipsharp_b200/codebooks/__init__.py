from .e8p import E8PCodebook, build_abs_table, decode_from_table, pack_code, unpack_code
from .e8_1bit import E8OneBitCodebook

__all__ = [
    "E8PCodebook", "E8OneBitCodebook", "build_abs_table", "decode_from_table",
    "pack_code", "unpack_code",
]
