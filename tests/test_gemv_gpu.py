"""GPU parity tests: the sm_100a library through its C ABI against the oracle.

Integer paths (W8A8 GEMV, activation quantization, packing) must be
bit-exact; floating-point GEMVs must be within rel-L2 1e-3 of the oracle
(the tolerance the path is specified to), and in practice land near 1e-6.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import make_cell, pack_codes, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def torch_mod():
    import torch
    return torch


# --- W8A8 operators (src/engine.zig) : bit-exact ---

@pytest.mark.parametrize("rows,cols", [(1000, 4096), (333, 1000), (16, 32), (4096, 12288)])
def test_gemv_parallel_bit_exact(ctx, rows, cols):
    rng = np.random.default_rng(rows + cols)
    w = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    x = rng.integers(-128, 128, cols, dtype=np.int8)
    y = ctx.gemv_parallel(w, 0.0031, x, 0.017)
    ref = O.gemv_parallel(w, 0.0031, x, 0.017)
    assert np.array_equal(y, ref)


@pytest.mark.parametrize("nb", [4, 8])
def test_gemv_batch_bit_exact(ctx, nb):
    rng = np.random.default_rng(nb)
    rows, cols = 777, 2080
    w = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    xs = [rng.integers(-128, 128, cols, dtype=np.int8) for _ in range(nb)]
    sx = (rng.random(nb) * 0.05 + 0.001).astype(np.float32)
    f = ctx.gemv_batch4_parallel if nb == 4 else ctx.gemv_batch8_parallel
    outs = f(w, 0.002, xs, sx)
    ref = O.gemv_batch_parallel(w, 0.002, np.stack(xs), sx)
    for b in range(nb):
        assert np.array_equal(outs[b], ref[b])


def test_gate_up_swiglu(ctx):
    rng = np.random.default_rng(11)
    rows, cols = 1536, 4096
    wg = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    wu = rng.integers(-127, 128, (rows, cols), dtype=np.int8)
    x = rng.integers(-128, 128, cols, dtype=np.int8)
    y = ctx.gemv_gate_up_swiglu_parallel(wg, 0.0004, wu, 0.0005, x, 0.01)
    ref = O.gemv_gateup_swiglu_parallel(wg, 0.0004, wu, 0.0005, x, 0.01)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)


def test_neon_known_answers_on_gpu(ctx):
    """src/kernels/neon.zig:714-841 patterns through the GPU operators."""
    def pat(n, mult, mod, off):
        return np.array([(i * mult) % mod - off for i in range(n)], np.int8)
    w = np.stack([pat(64, 1, 15, 7), pat(64, 3, 17, 8), pat(64, 5, 13, 6), pat(64, 7, 19, 9)])
    x = pat(64, 11, 23, 11)
    y = ctx.gemv_parallel(w, 0.05, x, 0.02)
    for r in range(4):
        assert abs(y[r] - O.dot_i8(w[r], x, 0.05, 0.02)) <= 1e-4
    sym = np.array([[1, 2, 3, 4, 5, 6, 7, 8, -1, -2, -3, -4, -5, -6, -7, -8]], np.int8)
    assert ctx.gemv_parallel(sym, 1.0, np.ones(16, np.int8), 1.0)[0] == 0.0


def test_quantize_activation_int8(ctx):
    q, s = ctx.quantize_activation_int8(np.array([-10.0, 0.0, 5.0, 10.0], np.float32))
    assert q[3] == 127 and q[0] == -127 and q[2] == 64
    rng = np.random.default_rng(4)
    for n in (4096, 12288, 7, 1):
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        q, s = ctx.quantize_activation_int8(x)
        qr, sr = O.quantize_act_i8(x)
        assert s == sr and np.array_equal(q, qr)
    q, s = ctx.quantize_activation_int8(np.zeros(100, np.float32))
    assert s == 1.0 and not q.any()


# --- grouped formats (fp activations) ---

def _bf16(x):
    torch = torch_mod()
    t = torch.from_numpy(x).to(torch.bfloat16)
    return t, t.view(torch.int16).numpy().view(np.uint16)


def _q8_group32(rng, N, K):
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    scales = (0.02 / 127 * np.exp(rng.normal(0, 0.25, (N, K // 32)))).astype(np.float16)
    return codes, scales


@pytest.mark.parametrize("N,K,M", [(1000, 4096, 1), (2048, 1024, 1), (515, 2080, 3), (256, 4096, 8)])
def test_q8_group32_fp32_x(ctx, N, K, M):
    """Config-0 format: int8 codes, fp16 scale per 32 along K, fp32 x, fp32 y."""
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16
    rng = np.random.default_rng(N * 7 + K)
    codes, scales = _q8_group32(rng, N, K)
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, scales, rows=N, cols=K, group=32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = ctx.gemv(t, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = O.gemv_grouped(codes, scales, None, 32, x, num_workers=8)
    assert rel_l2(y, ref) < TOL
    t.free()


@pytest.mark.parametrize("bits", [4, 2])
@pytest.mark.parametrize("M", [1, 4, 8])
@pytest.mark.parametrize("N,K", [(1024, 4096), (1000, 960), (256, 12288)])
def test_q4_q2_group64_bf16_x(ctx, bits, M, N, K):
    """Config-2 format: unsigned codes, fp16 scale + zero per 64 along K, bf16 x."""
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(bits * 1000 + M * 100 + N)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    codes, s, z = O.quantize_asym(w, bits, 64)
    t = ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, bits), s, z, rows=N, cols=K, group=64)
    xt, xbits = _bf16(rng.standard_normal((M, K)).astype(np.float32))
    y = ctx.gemv(t, xt.cuda()).cpu().numpy()
    ref = O.gemv_grouped(codes, s, z, 64, xbits, num_workers=8)
    assert rel_l2(y, ref) < TOL
    t.free()


def test_full_size_config0_against_torch_fp64(ctx):
    """Config 0 at full size (y[1,12288] = x[1,4096] W^T): torch fp64 dequant-matmul as the reference."""
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16
    rng = np.random.default_rng(0)
    N, K = 12288, 4096
    codes, scales = _q8_group32(rng, N, K)
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, scales, rows=N, cols=K, group=32)
    x = torch.from_numpy(rng.standard_normal((1, K)).astype(np.float32)).cuda()
    y = ctx.gemv(t, x)
    wd = torch.from_numpy(codes).cuda().double() * torch.from_numpy(scales.astype(np.float32)).cuda().double(
    ).repeat_interleave(32, dim=1)
    ref = x.double() @ wd.T
    assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < TOL
    # deterministic: a second call is bitwise identical
    y2 = ctx.gemv(t, x)
    assert torch.equal(y, y2)
    t.free()


def test_many_rows_split_into_token_blocks(ctx):
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(9)
    N, K, M = 512, 1024, 13
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    codes, s, z = O.quantize_asym(w, 4, 64)
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K, group=64)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = ctx.gemv(t, torch.from_numpy(x).cuda()).cpu().numpy()
    ref = O.gemv_grouped(codes, s, z, 64, x, num_workers=8)
    assert rel_l2(y, ref) < TOL
    t.free()


def test_gateup_swiglu_grouped(ctx):
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(21)
    N, K, M = 1024, 2048, 4
    tens, refs = [], []
    xt, xbits = _bf16(rng.standard_normal((M, K)).astype(np.float32))
    for _ in range(2):
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        codes, s, z = O.quantize_asym(w, 4, 64)
        tens.append(ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K,
                                      group=64))
        refs.append(O.gemv_grouped(codes, s, z, 64, xbits, num_workers=8))
    y = ctx.gemv_gateup_swiglu(tens[0], tens[1], xt.cuda()).cpu().numpy()
    g, u = refs
    ref = g / (1 + np.exp(-g)) * u
    assert rel_l2(y, ref) < TOL


@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
def test_fp32_x_every_row_count_and_split(ctx, bits, M):
    """fp32 activations at every row count: M <= 4 feeds each activation's two
    fp16 halves to adjacent MMA columns, M > 4 to two MMAs; M > 2 sums split-K
    partials in a second kernel.  K = 12288 forces several K-slices and
    N = 520 leaves a ragged last strip group.  The fp32 split keeps ~22 bits
    (less where a 2-bit pre-scale pushes the lo half into fp16 subnormals), so
    the bound, 1e-4, is far tighter than the path's 1e-3.  Plain GEMV,
    accumulate into y, and the fused gate/up SwiGLU."""
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(bits * 100 + M)
    N, K = 520, 12288
    tens, refs = [], []
    x = rng.standard_normal((M, K)).astype(np.float32)
    for _ in range(2):
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        if bits == 8:
            codes, s = O.quantize_sym8(w, 32)
            tens.append(ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32))
            refs.append(O.gemv_grouped(codes, s, None, 32, x, num_workers=8))
        else:
            codes, s, z = O.quantize_asym(w, bits, 64)
            tens.append(ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, bits), s, z, rows=N,
                                          cols=K, group=64))
            refs.append(O.gemv_grouped(codes, s, z, 64, x, num_workers=8))
    xd = torch.from_numpy(x).cuda()
    y = ctx.gemv(tens[0], xd)
    assert rel_l2(y.cpu().numpy(), refs[0]) < 1e-4
    y0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).cuda()
    y1 = y0.clone()
    ctx.gemv(tens[0], xd, out=y1, accumulate=True)
    assert rel_l2(y1.cpu().numpy(), y0.cpu().numpy() + refs[0]) < 1e-4
    gu = ctx.gemv_gateup_swiglu(tens[0], tens[1], xd).cpu().numpy()
    g, u = refs
    assert rel_l2(gu, g / (1 + np.exp(-g)) * u) < 1e-4
    # deterministic
    assert torch.equal(ctx.gemv(tens[0], xd), y)
    for t in tens:
        t.free()


# --- device quantizers: bit-exact with the oracle ---

@pytest.mark.parametrize("bits,group,sym", [(4, 64, False), (2, 64, False), (8, 32, True), (4, 128, False)])
def test_device_quantizer_bit_exact(ctx, bits, group, sym):
    torch = torch_mod()
    rng = np.random.default_rng(bits + group)
    w = rng.normal(0, 0.02, (257, 1024)).astype(np.float32)
    w[3, :64] = 0.0        # degenerate group
    w[4, :group] = 1e-9    # below the floor
    c, s, z = ctx.quantize_group_dev(torch.from_numpy(w).cuda(), bits, group, sym)
    torch.cuda.synchronize()
    if sym:
        cr, sr = O.quantize_sym8(w, group)
        assert np.array_equal(c.cpu().numpy().view(np.int8), cr)
    else:
        cr, sr, zr = O.quantize_asym(w, bits, group)
        assert np.array_equal(c.cpu().numpy(), cr)
        assert np.array_equal(z.cpu().numpy().view(np.uint16), zr.view(np.uint16))
    assert np.array_equal(s.cpu().numpy().view(np.uint16), sr.view(np.uint16))


# --- CHPE cells (src/chpe_engine.zig gemvTile*) through gemv_tile_polymorphic ---

def _check_cell(ctx, cell, x, tol=TOL):
    rows = int(np.frombuffer(cell[16448 + 40:16448 + 44].tobytes(), np.uint32)[0])
    y = np.zeros(rows + 3, np.float32)
    ctx.gemv_tile_polymorphic(cell, x, y, row_base=3)
    ref = O.gemv_tile_polymorphic(cell, x, np.zeros(rows + 3, np.float32), row_base=3)
    assert rel_l2(y, ref) < tol, (rel_l2(y, ref))
    # accumulate adds into y
    y2 = y.copy()
    ctx.gemv_tile_polymorphic(cell, x, y2, row_base=3, accumulate=True)
    assert rel_l2(y2, 2 * ref) < tol


def test_cell_known_answers_on_gpu(ctx):
    y = np.zeros(4, np.float32)
    ctx.gemv_tile_polymorphic(make_cell(2, 4, 128, bytes([0x55] * 8), scale=0.5), np.ones(128, np.float32), y)
    assert abs(y[0] - 16.0) < 1e-4 and abs(y[1]) < 1e-4
    ctx.gemv_tile_polymorphic(make_cell(4, 4, 128, bytes([0x99] * 64), scale=0.25), np.ones(128, np.float32), y)
    assert abs(y[0] - 32.0) < 1e-4 and abs(y[1] + 256.0) < 1e-3
    ctx.gemv_tile_polymorphic(make_cell(8, 4, 128, bytes([10] * 128), scale=0.1), np.ones(128, np.float32), y)
    assert abs(y[0] - 128.0) < 1e-3 and abs(y[1]) < 1e-4


@pytest.mark.parametrize("bits,rows,cols", [(8, 4, 4096), (8, 16, 1024), (4, 16, 2048), (4, 4, 8192),
                                            (2, 16, 4096), (2, 4, 8192)])
def test_cells_per_tile_scale_bias(ctx, bits, rows, cols):
    rng = np.random.default_rng(bits * rows)
    nbytes = rows * cols * bits // 8
    codes = rng.integers(0, 256, nbytes, dtype=np.uint8).tobytes()
    cell = make_cell(bits, rows, cols, codes, scale=0.013, bias=0.002 if bits != 8 else 0.05)
    _check_cell(ctx, cell, rng.standard_normal(cols).astype(np.float32))


def test_cell_w2_group128_with_outliers(ctx):
    rng = np.random.default_rng(77)
    rows, cols = 16, 2048
    codes = rng.integers(0, 256, rows * cols // 4, dtype=np.uint8).tobytes()
    gs = (rng.random(rows * cols // 128) * 0.05 + 0.001).astype(np.float16)
    ow = rng.normal(0, 0.1, 128).astype(np.float16)
    oc = np.array([0, 5, 77, 2047, 3000, 1024, 9, 10], np.uint16)  # 3000 >= cols: ignored
    cell = make_cell(2, rows, cols, codes, scale=0.0, flags=1, group_scales=gs, outlier_w=ow, outlier_cols=oc)
    _check_cell(ctx, cell, rng.standard_normal(cols).astype(np.float32))


def test_reference_packer_records_on_gpu(ctx):
    """The 72B packer's own records (tests/golden, made by the reference packer)."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "pack_golden.npz"))
    rng = np.random.default_rng(8)
    x = rng.standard_normal(8192).astype(np.float32)
    for key in ("record_w4_standard", "record_w2_standard", "record_w4_dense", "record_w2_dense"):
        rec = g[key]
        cell = rec[3072:].copy() if rec.size == 20480 else rec.copy()
        _check_cell(ctx, cell, x)


def test_upload_cells_run_of_records(ctx):
    """A run of standard 20480-byte records uploaded as one tensor (stride = 20480)."""
    torch = torch_mod()
    rng = np.random.default_rng(12)
    n, rows, cols = 6, 4, 8192
    recs = np.zeros((n, 20480), np.uint8)
    cells = []
    for i in range(n):
        codes = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8).tobytes()
        c = make_cell(4, rows, cols, codes, scale=0.01 + i * 1e-3, bias=1e-3 * i)
        recs[i, 3072:] = c
        cells.append(c)
    t = ctx.upload_cells(recs.reshape(-1)[3072:], n, 20480)
    x = rng.standard_normal(cols).astype(np.float32)
    y = ctx.gemv(t, torch.from_numpy(x[None]).cuda()).cpu().numpy()[0]
    ref = np.concatenate([O.gemv_tile_polymorphic(c, x) for c in cells])
    assert rel_l2(y, ref) < TOL


def test_bad_arguments_return_errors(ctx):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO, ChpeError
    with pytest.raises(ChpeError):  # group 32 unsupported for 4-bit
        ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, np.zeros((16, 32), np.uint8), np.ones((16, 2), np.float16),
                          np.ones((16, 2), np.float16), rows=16, cols=64, group=32)
    with pytest.raises(ChpeError):  # K not a multiple of the group
        ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, np.zeros((16, 50), np.uint8), np.ones((16, 2), np.float16),
                          np.ones((16, 2), np.float16), rows=16, cols=100, group=64)
    with pytest.raises(ChpeError):  # fp16 cells are not quantized
        ctx.gemv_tile_polymorphic(make_cell(16, 4, 128, b""), np.ones(128, np.float32), np.zeros(4, np.float32))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_multi_source_launch(ctx, bits, M):
    """Three tensors of the same cols and format (q/k/v-like, ragged row
    counts) in one launch: each output matches the oracle, and matches its own
    single-tensor GEMV to fp32 summation order."""
    torch = torch_mod()
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO, X_F32
    rng = np.random.default_rng(bits + 10 * M)
    K = 4096
    tens, refs = [], []
    x = rng.standard_normal((M, K)).astype(np.float32)
    for N in (520, 100, 1000):
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        if bits == 8:
            codes, s = O.quantize_sym8(w, 32)
            tens.append(ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32))
            refs.append(O.gemv_grouped(codes, s, None, 32, x, num_workers=8))
        else:
            codes, s, z = O.quantize_asym(w, 4, 64)
            tens.append(ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K,
                                          group=64))
            refs.append(O.gemv_grouped(codes, s, z, 64, x, num_workers=8))
    xd = torch.from_numpy(x).cuda()
    xf = ctx.xfrag(tens[0], M, X_F32)
    ctx.xfrag_fill(xf, xd)
    outs = [torch.full((M, t.rows), float("nan"), device="cuda") for t in tens]
    ctx.gemv_multi_xfrag(tens, xf, outs)
    for t, o, ref in zip(tens, outs, refs):
        got = o.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, ref) < 1e-4
        single = torch.empty_like(o)
        ctx.gemv_xfrag(t, xf, single)
        assert rel_l2(got, single.cpu().numpy()) < 1e-6
    xf.free()
    for t in tens:
        t.free()

