"""Contexts on two GPUs in one process: each kernel's dynamic shared-memory
limit and occupancy are per device, so the first GEMV (and prefill GEMM) on
the second device must work after the first device has launched them.
Skipped with fewer than 2 GPUs."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import pack_codes, rel_l2

pytestmark = pytest.mark.gpu


def test_gemv_and_prefill_on_two_devices_in_one_process():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO, Context
    rng = np.random.default_rng(0)
    N, K = 1000, 4096
    codes, s, z = O.quantize_asym(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4, 64)
    x = rng.standard_normal((3, K)).astype(np.float32)
    want = O.gemv_grouped(codes, s, z, 64, x, num_workers=8)
    xp = rng.standard_normal((128, K)).astype(np.float32)
    want_p = O.gemv_grouped(codes, s, z, 64, xp, num_workers=8)
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            ctx = Context(dev)
            t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K, group=64)
            y = ctx.gemv(t, torch.from_numpy(x).to(f"cuda:{dev}"))
            yp = ctx.gemm_prefill(t, torch.from_numpy(xp).to(f"cuda:{dev}"))
            torch.cuda.synchronize(dev)
            assert rel_l2(y.cpu().numpy(), want) < 1e-4
            assert rel_l2(yp.cpu().numpy(), want_p) < 1e-3
            assert ctx.lib.chpe_sync(ctx.ptr) == 0
            t.free()
            ctx.close()
