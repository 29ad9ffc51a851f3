"""CPU tests: the oracle against the reference's golden vectors and its own
known-answer tests, plus the bit-layout invariants the reference pins with
solver files.  No GPU needed."""
import itertools
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import make_cell, pack_codes, rel_l2

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pack_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


# --- scripts/pack_qwen72b_chpe.py golden vectors (made by importing the reference) ---

def test_quantize_4bit_block_matches_reference_packer(golden):
    p, s = O.quantize_4bit_block(golden["blocks"])
    assert np.array_equal(p, golden["q4_packed"])
    assert np.array_equal(s.view(np.uint16), golden["q4_scales"].view(np.uint16))


def test_quantize_2bit_block_matches_reference_packer(golden):
    p, s = O.quantize_2bit_block(golden["blocks"])
    assert np.array_equal(p, golden["q2_packed"])
    assert np.array_equal(s.view(np.uint16), golden["q2_scales"].view(np.uint16))


@pytest.mark.parametrize("bits,layout", [(4, "standard"), (4, "dense"), (2, "standard"), (2, "dense")])
def test_reference_records_layout(golden, bits, layout):
    """make_record output: codes at cell+64, TileDims at payload[32..48], group scales at payload[48..560]."""
    rec = golden[f"record_w{bits}_{layout}"]
    cell = rec[3072:] if layout == "standard" else rec
    assert cell.size == 17408
    w = golden["record_weights"]
    blk = w.reshape(-1, 128)
    packed, gs = (O.quantize_4bit_block if bits == 4 else O.quantize_2bit_block)(blk)
    assert np.array_equal(cell[64:64 + packed.size], packed)
    dims = np.frombuffer(cell[16448 + 32:16448 + 48].tobytes(), dtype=np.dtype([("s", "<f4"), ("b", "<f4"),
                                                                                 ("r", "<u4"), ("c", "<u4")]))[0]
    assert (dims["r"], dims["c"]) == (4, 8192)
    assert dims["s"] == np.float32(gs.astype(np.float16).mean())
    assert np.array_equal(cell[16448 + 48:16448 + 48 + 512].view(np.float16), gs)
    assert cell[16448 + 20] == bits


def test_reference_record_tile_gemv(golden):
    """gemvTileW4 on the packer's record uses the per-tile scale (mean of group scales), bias 0."""
    cell = golden["record_w4_standard"][3072:]
    rng = np.random.default_rng(3)
    x = rng.standard_normal(8192).astype(np.float32)
    y = O.gemv_tile_polymorphic(cell, x)
    packed = cell[64:64 + 4 * 4096]
    lo = (packed & 0xF).astype(np.int32) - 8
    hi = (packed >> 4).astype(np.int32) - 8
    q = np.stack([lo, hi], -1).reshape(4, 8192)
    scale = np.frombuffer(cell[16448 + 32:16448 + 36].tobytes(), np.float32)[0]
    ref = (q * scale).astype(np.float64) @ x.astype(np.float64)
    assert rel_l2(y, ref) < 1e-5


# --- src/kernels/neon.zig:714-841 known-answer and equivalence tests ---

def test_dot_symmetry():
    a = np.array([1, 2, 3, 4, 5, 6, 7, 8, -1, -2, -3, -4, -5, -6, -7, -8], np.int8)
    assert O.dot_i8(a, np.ones(16, np.int8), 1.0, 1.0) == 0.0


def test_activation_quant_known_answer():
    q, s = O.quantize_act_i8(np.array([-10.0, 0.0, 5.0, 10.0], np.float32))
    assert s > 0 and q[3] == 127 and q[0] == -127 and q[1] == 0 and q[2] == 64  # 5*12.7 = 63.5 -> 64 (half away)


def test_activation_quant_edges():
    q, s = O.quantize_act_i8(np.zeros(33, np.float32))
    assert s == 1.0 and not q.any()
    q, s = O.quantize_act_i8(np.full(5, 1e-10, np.float32))
    assert s == 1.0 and not q.any()


def _pat(n, mult, mod, off):
    return np.array([(i * mult) % mod - off for i in range(n)], np.int8)


def test_batch4_equivalence():
    w = _pat(64, 1, 15, 7)
    xs = np.stack([_pat(64, 1, 11, 5), _pat(64, 3, 17, 8), _pat(64, 5, 13, 6), _pat(64, 7, 19, 9)])
    sx = np.array([0.01, 0.02, 0.03, 0.04], np.float32)
    out = O.dot_i8_batch(w, xs, 0.05, sx)
    for b in range(4):
        assert abs(out[b] - O.dot_i8(w, xs[b], 0.05, sx[b])) <= 1e-4
        assert out[b] == np.float32(int(np.dot(w.astype(np.int64), xs[b].astype(np.int64)))) * np.float32(
            np.float32(0.05) * sx[b])


def test_batch8_equivalence():
    w = _pat(64, 1, 15, 7)
    xs = np.stack([_pat(64, (b + 1) * 2 + 1, 19, 9) for b in range(8)])
    sx = np.array([0.01 * (b + 1) for b in range(8)], np.float32)
    out = O.dot_i8_batch(w, xs, 0.05, sx)
    for b in range(8):
        assert abs(out[b] - O.dot_i8(w, xs[b], 0.05, sx[b])) <= 1e-4


def test_quadrow_equivalence():
    ws = np.stack([_pat(64, 1, 15, 7), _pat(64, 3, 17, 8), _pat(64, 5, 13, 6), _pat(64, 7, 19, 9)])
    x = _pat(64, 11, 23, 11)
    out = O.dot_i8_quadrow(ws, x, 0.05, 0.02)
    for r in range(4):
        assert abs(out[r] - O.dot_i8(ws[r], x, 0.05, 0.02)) <= 1e-4


def test_gateup_swiglu_equivalence():
    wg, wu, x = _pat(64, 1, 15, 7), _pat(64, 3, 17, 8), _pat(64, 5, 13, 6)
    fused = O.dot_i8_gateup_swiglu(wg, wu, x, 0.04, 0.06, 0.03)
    g = O.dot_i8(wg, x, 0.04, 0.03)
    u = O.dot_i8(wu, x, 0.06, 0.03)
    assert abs(fused - (g / (1 + np.exp(-g))) * u) <= 1e-4


# --- src/chpe_engine.zig:811-888 tile cells, with the known answers computed by hand ---

def test_tile_w2_known_answer():
    codes = bytes([0x55] * 8)  # 32 codes of 1 at the start of row 0
    cell = make_cell(2, 4, 128, codes, scale=0.5, bias=0.0)
    y = O.gemv_tile_polymorphic(cell, np.ones(128, np.float32))
    assert y[0] == 16.0 and y[1] == 0.0


def test_tile_w4_known_answer():
    cell = make_cell(4, 4, 128, bytes([0x99] * 64), scale=0.25, bias=0.0)
    y = O.gemv_tile_polymorphic(cell, np.ones(128, np.float32))
    assert y[0] == 32.0 and y[1] == -256.0  # zero bytes are nibble 0 -> -8 * 0.25


def test_tile_w8_known_answer():
    cell = make_cell(8, 4, 128, bytes([10] * 128), scale=0.1, bias=0.0)
    y = O.gemv_tile_polymorphic(cell, np.ones(128, np.float32))
    assert abs(y[0] - 128.0) < 1e-4 and y[1] == 0.0


def test_dot_tile_rows_match_cells():
    rng = np.random.default_rng(5)
    codes = rng.integers(0, 256, 512, dtype=np.uint8)
    x = rng.standard_normal(2048).astype(np.float32)
    r2 = O.dot_tile_row_2bit(codes, x, 0.3, 0.01)
    cell = make_cell(2, 1, 2048, codes.tobytes(), scale=0.3, bias=0.01)
    assert abs(O.gemv_tile_polymorphic(cell, x)[0] - r2) <= 1e-5 * max(1, abs(r2))
    r4 = O.dot_tile_row_4bit(codes, x[:1024], 0.3, 0.01)
    cell = make_cell(4, 1, 1024, codes.tobytes(), scale=0.3, bias=0.01)
    assert abs(O.gemv_tile_polymorphic(cell, x[:1024])[0] - r4) <= 1e-5 * max(1, abs(r4))


# --- tests/smt/qwen72b_2bit_group128_bounds.smt2 and qwen72b_uint4_coalesced_stride.smt2 ---

def test_two_bit_pack_order_is_injective():
    for c in itertools.product(range(4), repeat=4):
        b = c[0] | (c[1] << 2) | (c[2] << 4) | (c[3] << 6)
        assert tuple((b >> (2 * i)) & 3 for i in range(4)) == c
    # and the packer agrees: c0 sits in bits 1:0
    blk = np.zeros((1, 128), np.float32)
    blk[0, 0] = 2.0  # s = 1 -> first code 1 (>= 0.5); the rest 0
    p, s = O.quantize_2bit_block(blk)
    assert p[0] == 0x01 and s[0] == 1.0


def test_row_byte_alignment_invariants():
    assert 17408 + 3072 == 20480
    assert all((8192 // 4) % m == 0 for m in (16, 64, 512))
    assert all((29568 // 4) % m == 0 for m in (16, 32))


# --- the oracle's GEMV operators against plain numpy ---

def test_gemv_parallel_matches_integer_reference():
    rng = np.random.default_rng(0)
    w = rng.integers(-127, 128, (203, 333), dtype=np.int8)
    x = rng.integers(-128, 128, 333, dtype=np.int8)
    y = O.gemv_parallel(w, 0.003, x, 0.02, num_workers=8)
    acc = w.astype(np.int64) @ x.astype(np.int64)
    assert np.array_equal(y, acc.astype(np.float32) * np.float32(np.float32(0.003) * np.float32(0.02)))


def test_grouped_spec_degenerates_to_reference_paths():
    """Grouped formats with one group per row reduce to gemvTileW4 / gemvTileW8."""
    rng = np.random.default_rng(1)
    rows, cols = 4, 256
    nib = rng.integers(0, 16, (rows, cols), dtype=np.uint8)
    x = rng.standard_normal(cols).astype(np.float32)
    s = np.float16(0.0371)
    cell = make_cell(4, rows, cols, pack_codes(nib, 4).tobytes(), scale=float(s), bias=0.0)
    y_tile = O.gemv_tile_polymorphic(cell, x)
    y_spec = O.gemv_grouped(nib, np.full((rows, 1), s, np.float16), np.full((rows, 1), 8, np.float16), cols,
                            x[None])[0]
    assert rel_l2(y_spec, y_tile) < 1e-6
    q = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    cell = make_cell(8, rows, cols, q.tobytes(), scale=float(s), bias=0.0)
    y_tile = O.gemv_tile_polymorphic(cell, x)
    y_spec = O.gemv_grouped(q, np.full((rows, 1), s, np.float16), None, cols, x[None])[0]
    assert rel_l2(y_spec, y_tile) < 1e-6


def test_asym_quantizer_roundtrip_error():
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, (64, 512)).astype(np.float32)
    for bits in (4, 2):
        c, s, z = O.quantize_asym(w, bits, 64)
        assert c.max() <= (1 << bits) - 1
        deq = (c.reshape(64, 8, 64).astype(np.float32) - z.astype(np.float32)[..., None]) * s.astype(np.float32)[..., None]
        err = np.abs(deq.reshape(64, 512) - w).max()
        assert err <= 0.51 * s.astype(np.float32).max() + 1e-6
    c, s = O.quantize_sym8(w, 32)
    assert np.abs(c).max() <= 127
