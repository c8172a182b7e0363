"""The per-delta byte models of bench.py (its roofline) and of the C5 sweep
describe the same kernels: at the C1 shape (N = 16384, 4 limbs, 4 plaintext
batches, 5 columns, d = 1536, r = 16) they must agree kernel by kernel."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from provenloop_b200 import sweep  # noqa: E402


def test_bench_and_sweep_byte_models_agree_at_c1():
    names = ["enc_fused", "enc_a", "enc_u", "dec_limb1", "dec_fused", "encode", "gauss_gen", "encode_a",
             "encode_b", "decode_a", "decode_b"]
    for name in names:
        b = bench.kernel_bytes_per_delta(name, L=4, nb=4)
        s = sweep.kernel_bytes_per_delta(name, 16384, 4, 4, 5, bench.D, bench.R)
        assert b == s, (name, b, s)


def test_roofline_notes_cover_the_large_kernels():
    for name in ("enc_fused", "dec_fused"):
        assert bench.ROOF_NOTES.get(name)
