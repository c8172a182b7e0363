"""GPU parity for the public-key path, rescale and the shared-stream
batch_encrypt (the rows next to the delta path): bit-exact against the CPU
oracle (ciphertext.rs:114-154, :240-319, :476-535; lib.rs:231-258)."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))
DENSE_REJECT = [2305381840610885633, 2305381840610426881]  # one uniform draw in 5000 rejected


@pytest.fixture(scope="module")
def T():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from provenloop_b200 import tensafe_he
    return tensafe_he


@pytest.fixture(scope="module")
def ctx16(T):
    return T.CkksContext(16384)


@pytest.fixture(scope="module")
def octx16(oracle):
    return oracle.Ctx(16384)


@pytest.mark.parametrize("seed", [11, GOLD["encrypt_reject_seeds_n16384"][0]])
def test_keygen_public_bit_exact(T, ctx16, octx16, seed):
    sk, osk = ctx16.keygen(2), octx16.keygen(2)
    b, a = ctx16.keygen_public(sk, seed=seed).export()
    ob, oa = octx16.keygen_public(osk, seed)
    assert np.array_equal(a, oa) and np.array_equal(b, ob)


def test_keygen_public_from_key_batch(T, ctx16, octx16):
    skb = ctx16.keygen_batch([5, 6])
    b, a = ctx16.keygen_public(skb, seed=3, sk_index=1).export()
    ob, oa = octx16.keygen_public(octx16.keygen(6), 3)
    assert np.array_equal(a, oa) and np.array_equal(b, ob)


def test_encrypt_pk_bit_exact_and_decrypts(T, ctx16, octx16):
    rng = np.random.default_rng(41)
    z = rng.standard_normal(5000)
    sk, osk = ctx16.keygen(8), octx16.keygen(8)
    pk = ctx16.keygen_public(sk, seed=9)
    ob, oa = octx16.keygen_public(osk, 9)
    ct = ctx16.encrypt_pk(z, pk, seed=21)
    c0, c1 = ct.export()
    o0, o1, osc = octx16.encrypt_pk(z, ob, oa, 21)
    assert np.array_equal(c0, o0) and np.array_equal(c1, o1)
    assert ct.scale == osc
    dec = ctx16.decrypt(ct, sk)
    assert np.array_equal(dec.view(np.uint64), octx16.decrypt(c0, c1, ct.scale, osk).view(np.uint64))
    assert np.abs(dec[:5000] - z).max() < 1e-5


def test_encrypt_pk_batch_with_ternary_rejection(T, ctx16, octx16):
    """Seed whose ternary stream draws a 0 (rejected by range_u32(3)): the
    Gaussian segments after it shift, and the repair must follow them."""
    rng = np.random.default_rng(42)
    X = rng.standard_normal((3, 2000))
    seeds = [1, GOLD["keygen_reject_seed_n16384"], 2]
    sk, osk = ctx16.keygen(12), octx16.keygen(12)
    pk = ctx16.keygen_public(sk, seed=13)
    ob, oa = octx16.keygen_public(osk, 13)
    ct = ctx16.encrypt_pk_batch(X, pk, seeds)
    for i in range(3):
        c0, c1 = ct.export(i)
        o0, o1, _ = octx16.encrypt_pk(X[i], ob, oa, seeds[i])
        assert np.array_equal(c0, o0) and np.array_equal(c1, o1), i
    assert ctx16.stats()["streams_repaired"] >= 1


def test_rescale_bit_exact(T, ctx16, octx16):
    rng = np.random.default_rng(43)
    a, p = rng.standard_normal(8192), rng.standard_normal(8192)
    sk, osk = ctx16.keygen(14), octx16.keygen(14)
    prod = ctx16.encrypt(a, sk, seed=15) * p
    r = ctx16.rescale(prod)
    c0, c1 = r.export()
    p0, p1 = prod.export()
    o0, o1 = octx16.rescale(p0, p1)
    assert r.num_limbs == 3 and c0.shape == (3, 16384)
    assert np.array_equal(c0, o0) and np.array_equal(c1, o1)
    assert r.scale == prod.scale / float(ctx16.moduli[3])
    dec = ctx16.decrypt(r, sk)
    assert np.array_equal(dec.view(np.uint64), octx16.decrypt(o0, o1, r.scale, osk).view(np.uint64))
    assert np.abs(dec - a * p).max() < 1.0   # ciphertext.rs:790-797


def test_rescale_errors(T):
    one = T.CkksContext.from_moduli(16384, [1099510054913])
    ct = one.encrypt(np.ones(4), one.keygen(1), seed=1)
    with pytest.raises(ValueError, match="only 1 limb"):
        one.rescale(ct)
    c4 = T.CkksContext.custom(32768, [60, 40, 40, 40, 60])
    ct = c4.encrypt(np.ones(4), c4.keygen(1), seed=1)
    with pytest.raises(ValueError, match="Cannot invert zero"):
        c4.rescale(ct)


@pytest.mark.parametrize("moduli", [None, DENSE_REJECT])
def test_batch_encrypt_shares_one_stream(T, oracle, moduli):
    """lib.rs:231-258: array i continues the stream where array i-1 stopped;
    with frequent rejections every later array's start moves."""
    ctx = T.CkksContext(16384) if moduli is None else T.CkksContext.from_moduli(16384, moduli)
    o = oracle.Ctx(16384) if moduli is None else oracle.Ctx(16384, moduli)
    rng = np.random.default_rng(44)
    arrays = [rng.standard_normal(k) for k in (100, 8192, 3, 5000, 9000)]
    sk, osk = ctx.keygen(17), o.keygen(17)
    cts = ctx.batch_encrypt(arrays, sk, seed=99)
    r = oracle.Rng(99)
    for i, a in enumerate(arrays):
        c0, c1 = cts[i].export()
        o0, o1, _ = o.encrypt(a[:8192], osk, rng=r)
        assert np.array_equal(c0, o0) and np.array_equal(c1, o1), i
