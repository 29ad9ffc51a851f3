"""The device repack is lossless: every resident tensor read back out of the
strip layout (chpe_tensor_unpack) equals, bit for bit, the codes, scales and
zero-points it was uploaded from.

Covers the reference packer's own outputs (tests/golden: offset-8 nibbles
with fp16 block scales, scripts/pack_qwen72b_chpe.py:138-148, and the 2-bit
codebook, :110-135), the benchmark formats (Q8 with fp16 scale per 32
columns, Q4 and Q2 unsigned codes with fp16 scale + zero per 64 columns) at
config-2 shapes, W8A8 (the int8 MMA layout), reference cells with per-row
affine scales, and ragged shapes (rows not a multiple of 16, columns not a
multiple of a block: the padding must not leak into the read-back)."""
import os

import numpy as np
import pytest

from tests._util import make_cell, pack_codes

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "pack_golden.npz")


def test_reference_packed_q4_offset8_roundtrip(ctx):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_CONST_ZERO
    g = np.load(GOLDEN)
    codes = g["q4_packed"].reshape(64, 64)  # 64 blocks of 128 nibbles, low nibble = even element
    scales = g["q4_scales"].reshape(64, 1)
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_CONST_ZERO, codes, scales, rows=64, cols=128, group=128, zero=8.0)
    c, s, _ = t.unpack(n_groups=1)
    assert np.array_equal(c, codes)
    assert np.array_equal(s.view(np.uint16), scales.view(np.uint16))
    t.free()


def test_reference_packed_q2_codebook_roundtrip(ctx):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_W2_CODEBOOK_GROUP_F16
    g = np.load(GOLDEN)
    codes = g["q2_packed"].reshape(64, 32)  # 128 codes per block, element 4i in bits 1:0
    scales = g["q2_scales"].reshape(64, 1)
    t = ctx.upload_matrix(2, SCHEME_W2_CODEBOOK_GROUP_F16, codes, scales, rows=64, cols=128, group=128)
    c, s, _ = t.unpack(n_groups=1)
    assert np.array_equal(c, codes)
    assert np.array_equal(s.view(np.uint16), scales.view(np.uint16))
    t.free()


@pytest.mark.parametrize("bits", [4, 2])
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 12288), (12288, 4096), (4096, 151936), (1088, 37)])
def test_grouped_unsigned_roundtrip(ctx, bits, K, N):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(bits * 7 + K + N)
    codes = rng.integers(0, 256, (N, K * bits // 8), dtype=np.uint8)
    s = rng.random((N, K // 64)).astype(np.float16)
    z = rng.integers(0, 1 << bits, (N, K // 64)).astype(np.float16)
    t = ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, codes, s, z, rows=N, cols=K, group=64)
    c, s2, z2 = t.unpack(n_groups=K // 64, zeros=True)
    assert np.array_equal(c, codes)
    assert np.array_equal(s2.view(np.uint16), s.view(np.uint16))
    assert np.array_equal(z2.view(np.uint16), z.view(np.uint16))
    t.free()


@pytest.mark.parametrize("K,N", [(4096, 12288), (800, 21)])
def test_q8_group32_roundtrip(ctx, K, N):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16
    rng = np.random.default_rng(K + N)
    codes = rng.integers(-128, 128, (N, K), dtype=np.int8)
    s = (rng.random((N, K // 32)) * 1e-3).astype(np.float16)
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
    c, s2, _ = t.unpack(n_groups=K // 32)
    assert np.array_equal(c.view(np.int8), codes)
    assert np.array_equal(s2.view(np.uint16), s.view(np.uint16))
    t.free()


@pytest.mark.parametrize("K,N", [(4096, 1024), (2080, 777)])
def test_w8a8_roundtrip(ctx, K, N):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_TENSOR
    rng = np.random.default_rng(K * 3 + N)
    codes = rng.integers(-128, 128, (N, K), dtype=np.int8)
    t = ctx.upload_matrix(8, SCHEME_I8_TENSOR, codes, np.array([0.01], np.float32), rows=N, cols=K)
    c, _, _ = t.unpack()
    assert np.array_equal(c.view(np.int8), codes)
    t.free()


@pytest.mark.parametrize("bits", [8, 4, 2])
def test_cell_roundtrip(ctx, bits):
    """Reference cells (per-tile scale and bias): codes and per-row scales."""
    rng = np.random.default_rng(bits)
    rows, cols = 16, 1024 if bits == 8 else 2048
    codes = rng.integers(0, 256, rows * cols * bits // 8, dtype=np.uint8)
    cell = make_cell(bits, rows, cols, codes.tobytes(), scale=0.0123, bias=-0.5)
    t = ctx.upload_cells(cell, 1)
    c, s, _ = t.unpack(scales_f32=True)
    assert np.array_equal(c.reshape(-1), codes)
    assert np.all(s == np.float32(0.0123))
    t.free()


def test_unpack_rejects_zeros_without_zero_points(ctx):
    from chpe_qwen35_hybrid_engine_b200 import ChpeError, SCHEME_I8_GROUP_F16
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, np.zeros((16, 256), np.int8), np.ones((16, 8), np.float16),
                          rows=16, cols=256, group=32)
    with pytest.raises(ChpeError):
        t.unpack(n_groups=8, zeros=True)
    t.free()
