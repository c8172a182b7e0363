"""GPU parity at N = 32768, where one poly-limb spans a cluster of two CTAs.

The preset chain (params.rs:106-126), the C4 chain custom(32768,
[60, 40, 40, 40, 60]) with its repeated primes (params.rs:142-162), and
moduli chosen so that range_u64 rejections occur in every stream.  Integer
results are bit-exact against the CPU oracle; deltas are held to 1e-4.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N = 32768
C4_BITS = [60, 40, 40, 40, 60]


def _dense_reject_primes(n, count):
    """61-bit primes q = 1 mod 2n just below 2^61 (1 - 2e-4): 2^64 mod q is
    2e-4 of 2^64, so one uniform draw in 5000 is rejected."""
    def is_prime(x):
        if x % 2 == 0:
            return False
        d, s = x - 1, 0
        while d % 2 == 0:
            d //= 2
            s += 1
        for a in (2, 3, 5, 7, 11, 13, 17, 19, 23, 29, 31, 37):
            y = pow(a, d, x)
            if y in (1, x - 1):
                continue
            for _ in range(s - 1):
                y = y * y % x
                if y == x - 1:
                    break
            else:
                return False
        return True
    q = (2 ** 64 * (10 ** 6 - 200)) // (8 * 10 ** 6)
    q -= (q - 1) % (2 * n)
    out = []
    while len(out) < count:
        if is_prime(q):
            out.append(q)
        q -= 2 * n
    return out


@pytest.fixture(scope="module")
def T():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from provenloop_b200 import tensafe_he
    return tensafe_he


@pytest.fixture(scope="module")
def ctx32(T):
    return T.CkksContext(N)


@pytest.fixture(scope="module")
def octx32(oracle):
    return oracle.Ctx(N)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def _host(t):
    return t.cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("chain", ["preset", "c4"])
def test_ntt_n32768_bit_exact(T, oracle, chain):
    from provenloop_b200._lib import lib, check
    ctx = T.CkksContext(N) if chain == "preset" else T.CkksContext.custom(N, C4_BITS)
    qs = ctx.moduli
    rng = np.random.default_rng(31)
    P = 2
    x = np.stack([np.stack([rng.integers(0, q, size=N, dtype=np.uint64) for q in qs]) for _ in range(P)])
    d = _dev(x)
    check(lib().ts_ntt_forward(ctx.handle, d.data_ptr(), P, len(qs), 0))
    ctx.synchronize()
    fwd = _host(d).reshape(x.shape)
    for p in range(P):
        for l, q in enumerate(qs):
            assert np.array_equal(fwd[p, l], oracle.ntt_forward(x[p, l], N, q)), (p, l)
    check(lib().ts_ntt_inverse(ctx.handle, d.data_ptr(), P, len(qs), 0))
    ctx.synchronize()
    assert np.array_equal(_host(d).reshape(x.shape), x)


@pytest.mark.parametrize("seed", [0, 7])
def test_keygen_n32768_bit_exact(T, ctx32, octx32, seed):
    assert np.array_equal(ctx32.keygen(seed).export(), octx32.keygen(seed))


def test_encrypt_decrypt_n32768_bit_exact(T, ctx32, octx32):
    rng = np.random.default_rng(32)
    z = rng.standard_normal(16384)
    sk, osk = ctx32.keygen(3), octx32.keygen(3)
    for seed in (5, 6):
        ct = ctx32.encrypt(z, sk, seed=seed)
        c0, c1 = ct.export()
        o0, o1, _ = octx32.encrypt(z, osk, seed=seed)
        assert np.array_equal(c1, o1) and np.array_equal(c0, o0), seed
        dec = ctx32.decrypt(ct, sk)
        ref = octx32.decrypt(c0, c1, ct.scale, osk)
        assert np.array_equal(dec.view(np.uint64), ref.view(np.uint64))
        assert np.abs(dec - z).max() < 1e-6


def test_ct_pt_mul_crt_decrypt_n32768(T, ctx32, octx32):
    rng = np.random.default_rng(33)
    a, b = rng.standard_normal(16384), rng.standard_normal(16384)
    sk, osk = ctx32.keygen(4), octx32.keygen(4)
    prod = ctx32.encrypt(a, sk, seed=9) * b
    p0, p1 = prod.export()
    dec = ctx32.decrypt(prod, sk)
    ref = octx32.decrypt(p0, p1, prod.scale, osk)
    assert np.array_equal(dec.view(np.uint64), ref.view(np.uint64))
    assert np.abs(dec - a * b).max() < 1e-6


def test_encrypt_n32768_dense_rejections(T, oracle):
    moduli = _dense_reject_primes(N, 2)
    ctx = T.CkksContext.from_moduli(N, moduli)
    o = oracle.Ctx(N, moduli)
    rng = np.random.default_rng(34)
    X = rng.standard_normal((20, 3000))
    seeds = list(range(2000, 2020))
    ct = ctx.encrypt_batch(X, ctx.keygen_batch([6]), seeds)
    osk = o.keygen(6)
    for i in range(20):
        c0, c1 = ct.export(i)
        o0, o1, _ = o.encrypt(X[i], osk, seed=seeds[i])
        assert np.array_equal(c1, o1) and np.array_equal(c0, o0), i
    st = ctx.stats()
    assert st["streams_repaired"] >= 18 and st["plan_overflow"] == 0


def test_lora_delta_c4_chain(T, oracle):
    """C4 shape: N = 32768 on [60, 40, 40, 40, 60], r = 32 (cols = 10,
    B = 4), one key per user; 24 users x 4 batches = 96 vectors, more than
    the 74 CTA pairs, so pairs take two vectors."""
    from provenloop_b200.backend import ZeroMoaiLora
    ctx = T.CkksContext.custom(N, C4_BITS)
    o = oracle.Ctx(N, oracle.params_custom(N, C4_BITS))
    rng = np.random.default_rng(35)
    r, d, n = 32, 1536, 24
    A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((n, d))
    keys = [3 + u for u in range(n)]
    seeds = [700 + u for u in range(n)]
    lora = ZeroMoaiLora(ctx, A, B)
    delta, inter = lora.delta(ctx.keygen_batch(keys), H, seeds, sk_index=list(range(n)))
    for i in range(0, n, 5):
        od, oi = o.lora_delta(o.keygen(keys[i]), H[i], A, B, enc_seed=seeds[i])
        assert np.abs(delta[i] - od).max() < 1e-4, i
        assert np.abs(inter[i] - oi).max() < 1e-8, i
    plain = (A.astype(np.float64) @ H.T).T @ B.astype(np.float64).T
    assert np.abs(delta - plain).max() < 1e-4


def test_lora_delta_c4_full_call(T, oracle):
    """The C4 benchmark call itself: custom(32768, [60,40,40,40,60]), 256
    users with their own keys (seed 3 + user) x 56 rank-32 adapters = 14336
    deltas in one ts_lora_delta_batch call (seven 2048-delta passes).  Rows
    of the first, a middle and the last user against the oracle; every row
    against float64 B (A h)."""
    from provenloop_b200.backend import ZeroMoaiLora
    users, adapters, r, d = 256, 56, 32, 1536
    ctx = T.CkksContext.custom(N, C4_BITS)
    o = oracle.Ctx(N, oracle.params_custom(N, C4_BITS))
    rng = np.random.default_rng(3)
    A = (rng.standard_normal((adapters, r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((adapters, d, r)) * 0.02).astype(np.float32)
    n = users * adapters
    H = np.random.default_rng(3000).standard_normal((n, d))
    adapter = np.tile(np.arange(adapters, dtype=np.int32), users)
    user = np.repeat(np.arange(users, dtype=np.int32), adapters)
    seeds = (np.arange(n, dtype=np.uint64) + 5_000_000).astype(np.uint64)
    lora = ZeroMoaiLora(ctx, A, B)
    delta, inter = lora.delta(ctx.keygen_batch([3 + u for u in range(users)]), H, seeds, expert=adapter,
                              sk_index=user)
    for u, a in ((0, 0), (0, 55), (127, 17), (128, 30), (255, 0), (255, 55)):
        i = u * adapters + a
        od, oi = o.lora_delta(o.keygen(3 + u), H[i], A[a], B[a], enc_seed=int(seeds[i]))
        assert np.abs(delta[i] - od).max() < 1e-4, (u, a)
        assert np.abs(inter[i] - oi).max() < 1e-8, (u, a)
    for a in range(adapters):
        rows = adapter == a
        plain = (H[rows] @ A[a].astype(np.float64).T) @ B[a].astype(np.float64).T
        assert np.abs(delta[rows] - plain).max() < 1e-4, a
