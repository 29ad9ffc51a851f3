"""Shared helpers for the tests (input builders and error metrics)."""
from __future__ import annotations

import struct

import numpy as np

CELL_BYTES = 17408
HDR = 64
CODES = 16384
PAYLOAD = HDR + CODES


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.linalg.norm(a - b)
    n = np.linalg.norm(b)
    return float(d / n) if n > 0 else float(d)


def make_cell(bits: int, rows: int, cols: int, codes: bytes, scale: float = 0.0, bias: float = 0.0,
              flags: int = 0, group_scales: np.ndarray | None = None, outlier_w: np.ndarray | None = None,
              outlier_cols: np.ndarray | None = None) -> np.ndarray:
    """A 17408-byte Cell (src/geometry.zig:243-256) with TileMetadata at payload[0..32]
    (src/weight_archive.zig:92-105) and TileDims at payload[32..48] (src/chpe_engine.zig:146-151)."""
    cell = bytearray(CELL_BYTES)
    cell[HDR:HDR + len(codes)] = codes
    meta = struct.pack("<IIQIB3sQ", 0, 0, 0, rows * cols * 4, bits, b"\0\0\0", flags)
    cell[PAYLOAD:PAYLOAD + 32] = meta
    cell[PAYLOAD + 32:PAYLOAD + 48] = struct.pack("<ffII", scale, bias, rows, cols)
    if group_scales is not None:
        gs = np.asarray(group_scales, np.float16).tobytes()
        assert len(gs) <= 512
        cell[PAYLOAD + 48:PAYLOAD + 48 + len(gs)] = gs
    if outlier_w is not None:
        ow = np.asarray(outlier_w, np.float16).reshape(16, 8).tobytes()
        cell[PAYLOAD + 560:PAYLOAD + 816] = ow
        cell[PAYLOAD + 816:PAYLOAD + 832] = np.asarray(outlier_cols, np.uint16).tobytes()
    return np.frombuffer(bytes(cell), np.uint8).copy()


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack [rows, cols] codes LSB-first into bytes (the reference packer's order)."""
    codes = np.asarray(codes, np.uint8)
    rows, cols = codes.shape
    per = 8 // bits
    c = codes.reshape(rows, cols // per, per).astype(np.uint32)
    out = np.zeros((rows, cols // per), np.uint32)
    for i in range(per):
        out |= (c[:, :, i] & ((1 << bits) - 1)) << (bits * i)
    return out.astype(np.uint8)
