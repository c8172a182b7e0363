"""CPU checks of the C ABI: the library loads, exports every symbol the
header declares, fails loudly without a GPU, and its host-side parameter /
table construction equals the oracle's bit for bit."""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tsgpu.h")


def header_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ts_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def L():
    from provenloop_b200 import _lib
    return _lib.lib()


def test_exports_every_header_symbol(L):
    syms = header_symbols()
    assert len(syms) >= 40
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    from provenloop_b200._lib import SIGNATURES
    assert sorted(SIGNATURES) == syms


def test_no_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from provenloop_b200 import _lib, tensafe_he
    assert _lib.device_count() == 0
    with pytest.raises(_lib.TsError) as ei:
        tensafe_he.CkksContext(16384)
    assert "no CUDA device" in str(ei.value)
    assert tensafe_he.is_available() is False


def test_unsupported_degree_is_value_error():
    from provenloop_b200 import tensafe_he
    with pytest.raises(ValueError, match="Unsupported poly_mod_degree"):
        tensafe_he.CkksContext(4096)      # lib.rs:42-46
    with pytest.raises(ValueError, match="Unsupported depth"):
        tensafe_he.CkksContext.for_depth(9)  # lib.rs:69-73


def test_params_custom_matches_oracle(L, oracle):
    import ctypes as C
    for n, bits in ((16384, [60, 40, 40, 60]), (32768, [60, 40, 40, 40, 60]), (16384, [50, 50, 50])):
        b = np.asarray(bits, np.uint32)
        out = np.zeros(len(bits), np.uint64)
        assert L.ts_params_custom(n, b.ctypes.data_as(C.POINTER(C.c_uint32)), len(bits),
                                  out.ctypes.data_as(C.POINTER(C.c_uint64))) == 0
        assert [int(x) for x in out] == oracle.params_custom(n, bits)


@pytest.mark.parametrize("n,q", [(16384, 1152921504606748673), (16384, 1099510054913), (16384, 1099508121601),
                                 (16384, 1152921504606683137), (8192, 1099511480321), (16384, 1125899904679937)])
def test_host_tables_match_oracle(L, oracle, n, q):
    import ctypes as C
    fw, iw = np.zeros(n, np.uint64), np.zeros(n, np.uint64)
    t = [np.zeros(n) for _ in range(4)]
    P64, PD = C.POINTER(C.c_uint64), C.POINTER(C.c_double)
    assert L.ts_host_tables(n, q, fw.ctypes.data_as(P64), iw.ctypes.data_as(P64),
                            *[x.ctypes.data_as(PD) for x in t]) == 0
    ofw, oiw, _, _ = oracle.ntt_tables(n, q)
    assert np.array_equal(fw, ofw) and np.array_equal(iw, oiw)
    ctx = oracle.Ctx(n, [q])
    ot = ctx.fft_tables()
    for a, b in zip(t, ot):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))   # bit-identical doubles
