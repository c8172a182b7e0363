"""ts_decrypt_noalloc: decrypt for callers that cannot allocate device
memory while serving (their device heap is reserved or owned by another
allocator).  It must give exactly what ts_decrypt gives, call after call,
while taking its temporaries from the library's fixed device array.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _device_memory_state():
    """(free bytes of device 0, used and high-watermark bytes of its default
    stream-ordered pool) -- the two places an allocation would show.  The
    pool figures are None when cuda-python is not importable."""
    import torch
    free = torch.cuda.mem_get_info(0)[0]
    try:
        from cuda.bindings import runtime as rt
    except ImportError:
        return free, None, None
    err, pool = rt.cudaDeviceGetDefaultMemPool(0)
    assert err == rt.cudaError_t.cudaSuccess
    err, used = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent)
    assert err == rt.cudaError_t.cudaSuccess
    err, high = rt.cudaMemPoolGetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh)
    assert err == rt.cudaError_t.cudaSuccess
    return free, int(used), int(high)


def _reset_pool_high_watermark():
    try:
        from cuda.bindings import driver as dr
        from cuda.bindings import runtime as rt
    except ImportError:
        return
    err, pool = rt.cudaDeviceGetDefaultMemPool(0)
    assert err == rt.cudaError_t.cudaSuccess
    # the high watermark can only be reset, by writing zero
    (err,) = rt.cudaMemPoolSetAttribute(pool, rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh, dr.cuuint64_t(0))
    assert err == rt.cudaError_t.cudaSuccess


def test_decrypt_noalloc_matches_decrypt_twice():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from provenloop_b200 import tensafe_he
    from provenloop_b200._lib import check, lib

    ctx = tensafe_he.CkksContext(16384)
    sk = ctx.keygen(7)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 8192))
    fresh = ctx.encrypt_batch(x, sk, seeds=[11, 12])       # limb-0 decode path
    prod = fresh * rng.standard_normal(8192)                # CRT decode path (scale = Delta^2)
    for ct in (fresh, prod):
        cnt = ct._info()[0]
        ref = np.zeros(cnt * 8192)
        check(lib().ts_decrypt(ctx.handle, ct.handle, sk.handle, None, ref.ctypes.data, 0))
        for call in range(2):                               # two calls in a row share the array
            out = torch.full((cnt * 8192,), float("nan"), dtype=torch.float64, device="cuda:0")
            torch.cuda.synchronize()
            ctx.synchronize()
            _reset_pool_high_watermark()
            free0, used0, _ = _device_memory_state()
            check(lib().ts_decrypt_noalloc(ctx.handle, ct.handle, sk.handle, C.c_void_p(out.data_ptr())))
            ctx.synchronize()
            free1, used1, high1 = _device_memory_state()
            if call == 1:
                # nothing was allocated: no new device memory, and the
                # stream-ordered pool never held more than before the call
                assert free1 == free0
                if used0 is not None:
                    assert used1 == used0 and high1 <= used0
            got = out.cpu().numpy()
            assert np.abs(got - ref).max() <= 1e-12
            assert np.array_equal(got.view(np.uint64), ref.view(np.uint64))


def test_decrypt_noalloc_rejects_oversize():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from provenloop_b200 import tensafe_he
    from provenloop_b200._lib import check, lib

    ctx = tensafe_he.CkksContext(16384)
    sk = ctx.keygen(1)
    # 5 ciphertexts after ct x pt need 5 x 512 KiB > the 2 MiB array
    ct = ctx.encrypt_batch(np.zeros((5, 16)), sk, seeds=[1, 2, 3, 4, 5]) * np.ones(16)
    out = torch.empty(5 * 8192, dtype=torch.float64, device="cuda:0")
    with pytest.raises(ValueError, match="fixed"):
        check(lib().ts_decrypt_noalloc(ctx.handle, ct.handle, sk.handle, C.c_void_p(out.data_ptr())))
