"""Generate golden vectors by running the reference's own numpy packer.

Run in a container where the reference checkout is mounted (default
/root/reference; override with CHPE_REFERENCE).  It imports
scripts/pack_qwen72b_chpe.py from there and records, for seeded inputs and edge
cases, what `quantize_4bit_block`, `quantize_2bit_block` and `make_record`
return.  The output (tests/golden/pack_golden.npz) is committed; the tests read
only that file, so they run where the reference is absent.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

REF = os.environ.get("CHPE_REFERENCE", "/root/reference")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "pack_golden.npz")


def load_packer():
    path = os.path.join(REF, "scripts", "pack_qwen72b_chpe.py")
    spec = importlib.util.spec_from_file_location("ref_pack_qwen72b_chpe", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def blocks(seed: int) -> np.ndarray:
    """Seeded N(0,0.02) blocks plus hand-made edge cases, shape [n,128] f32."""
    rng = np.random.default_rng(seed)
    main = rng.normal(0.0, 0.02, size=(48, 128)).astype(np.float32)
    edge = np.zeros((16, 128), np.float32)
    edge[1] = 1e-9                                   # below the 1e-8 absmax floor
    edge[2] = np.linspace(-1.0, 1.0, 128)            # symmetric ramp
    edge[3, ::2] = 7.0; edge[3, 1::2] = -7.0         # exact 4-bit end points (s = 1)
    edge[4] = (np.arange(128) % 16 - 8) * 0.5 + 0.25  # 4-bit half ties
    edge[5] = np.array([0.5, -0.5, 1.5, -1.5] * 32) * 2.0 / 2.0  # 2-bit thresholds at s = 1
    edge[5, 0] = 2.0                                 # pins s = 1 for the 2-bit quantizer
    edge[6] = 65504.0 * np.sin(np.arange(128))       # fp16-range magnitudes
    edge[7] = 1e-5 * rng.standard_normal(128)        # fp16-subnormal scales
    edge[8, 0] = -3.0                                # single outlier
    edge[9] = rng.uniform(-1, 1, 128).astype(np.float32)
    edge[10] = -0.02
    edge[11] = 0.02
    edge[12] = rng.normal(0, 1e3, 128)
    edge[13] = rng.normal(0, 1e-4, 128)
    edge[14, 64:] = 1.0
    edge[15] = np.float32(np.pi) * ((np.arange(128) % 3) - 1)
    return np.concatenate([main, edge]).astype(np.float32)


def main():
    pk = load_packer()
    blk = blocks(0)
    p4, s4 = pk.quantize_4bit_block(blk)
    p2, s2 = pk.quantize_2bit_block(blk)

    # One 4-bit and one 2-bit record exactly as the packer writes them for a
    # [4, 8192] slice of a 72B-shape matrix (rows_per_tile = 32768 // 8192).
    rng = np.random.default_rng(1)
    w = rng.normal(0.0, 0.02, size=(4, 8192)).astype(np.float32)
    blk72 = w.reshape(-1, 128)
    rec = {}
    for bits in (4, 2):
        if bits == 2:
            packed, gs = pk.quantize_2bit_block(blk72)
            flags = pk.FLAG_GROUP128_OUTLIERS
        else:
            packed, gs = pk.quantize_4bit_block(blk72)
            flags = 0
        coded = bytearray(pk.TILE_CODE_BYTES)
        coded[: len(packed)] = packed.tobytes()
        aux = gs.tobytes().ljust(512, b"\x00")
        for dense in (False, True):
            r = pk.make_record(bytes(coded), 7, 4, 8192, float(gs.mean()), 0.0,
                               "model.layers.7.mlp.gate_proj.weight", quant_bits=bits,
                               custom_flags=flags, aux_payload=aux, dense=dense)
            rec[f"record_w{bits}_{'dense' if dense else 'standard'}"] = np.frombuffer(r, np.uint8)

    np.savez_compressed(
        OUT,
        blocks=blk,
        q4_packed=p4, q4_scales=s4.astype(np.float16),
        q2_packed=p2, q2_scales=s2.astype(np.float16),
        record_weights=w,
        **rec,
    )
    print("wrote", OUT, {k: v.shape for k, v in np.load(OUT).items()})


if __name__ == "__main__":
    sys.exit(main())
