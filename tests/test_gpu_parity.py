"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bit-exact for every integer result (NTT / INTT, Hadamard, keys,
ciphertexts, NTT(plaintext)); the f64 decode is compared bit-exactly too,
since it evaluates the reference's FFT with identical rounding.  Deltas are
held to the 1e-4 max-abs tolerance of the spec.
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))
C2 = GOLD["c2"]["primes"]


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


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def _host(t):
    return t.cpu().numpy().view(np.uint64)


# ------------------------------------------------------------------ NTT
@pytest.mark.parametrize("n,moduli", [(16384, None), (8192, None), (16384, C2), (4096, [1099510054913, 1125899904679937])])
def test_ntt_forward_inverse_bit_exact(T, oracle, n, moduli):
    import torch
    from provenloop_b200._lib import lib, check
    if moduli is None:
        ctx = T.CkksContext(n)
    else:
        ctx = T.CkksContext.from_moduli(n, moduli)
    qs = ctx.moduli
    rng = np.random.default_rng(n + len(qs))
    P = 3
    x = np.stack([np.stack([rng.integers(0, q, size=n, dtype=np.uint64) for q in qs]) for _ in range(P)])
    d = _dev(x)
    check(lib().ts_ntt_forward(ctx.handle, d.data_ptr(), P, len(qs), 0))
    ctx.synchronize()
    fwd = _host(d).reshape(x.shape)
    for p in range(P):
        for l, q in enumerate(qs):
            assert np.array_equal(fwd[p, l], oracle.ntt_forward(x[p, l], n, q)), (p, l)
    check(lib().ts_ntt_inverse(ctx.handle, d.data_ptr(), P, len(qs), 0))
    ctx.synchronize()
    assert np.array_equal(_host(d).reshape(x.shape), x)


def test_ntt_golden_c2(T, oracle):
    import hashlib
    from provenloop_b200._lib import lib, check
    ctx = T.CkksContext.from_moduli(16384, C2)
    sys_polys = __import__("tests.golden.make_golden", fromlist=["c2_polys"]).c2_polys()
    assert hashlib.sha256(sys_polys.tobytes()).hexdigest() == GOLD["c2"]["input_sha256"]
    d = _dev(sys_polys)
    check(lib().ts_ntt_forward(ctx.handle, d.data_ptr(), sys_polys.shape[0], 3, 0))
    ctx.synchronize()
    assert hashlib.sha256(_host(d).tobytes()).hexdigest() == GOLD["c2"]["forward_sha256"]


def test_ntt_limb_subset_and_extremes(T, oracle, ctx16):
    # limb_offset/limb_count selection; all-zero, all-(q-1) inputs
    from provenloop_b200._lib import lib, check
    n, qs = 16384, ctx16.moduli
    x = np.stack([np.zeros(n, np.uint64), np.full(n, qs[2] - 1, np.uint64)])
    d = _dev(x)
    check(lib().ts_ntt_forward(ctx16.handle, d.data_ptr(), 2, 1, 2))
    ctx16.synchronize()
    out = _host(d).reshape(2, n)
    assert np.array_equal(out[0], oracle.ntt_forward(x[0], n, qs[2]))
    assert np.array_equal(out[1], oracle.ntt_forward(x[1], n, qs[2]))


def test_hadamard_bit_exact(T, ctx16):
    from provenloop_b200._lib import lib, check
    n, qs = 16384, ctx16.moduli
    rng = np.random.default_rng(7)
    a = np.stack([np.stack([rng.integers(0, q, size=n, dtype=np.uint64) for q in qs]) for _ in range(4)])
    b = np.stack([rng.integers(0, q, size=n, dtype=np.uint64) for q in qs])
    da, db = _dev(a), _dev(b)
    out = _dev(np.zeros_like(a))
    check(lib().ts_hadamard(ctx16.handle, out.data_ptr(), da.data_ptr(), db.data_ptr(), 4, 4, 1))
    ctx16.synchronize()
    got = _host(out).reshape(a.shape)
    for p in range(4):
        for l, q in enumerate(qs):
            ref = np.array([(int(x) * int(y)) % q for x, y in zip(a[p, l, :257], b[l, :257])], np.uint64)
            assert np.array_equal(got[p, l, :257], ref)
    # full check via object arithmetic on one limb
    l = 2
    ref = (a[1, l].astype(object) * b[l].astype(object)) % qs[l]
    assert np.array_equal(got[1, l], ref.astype(np.uint64))


# ------------------------------------------------------------------ keys
@pytest.mark.parametrize("seed", [0, 42, GOLD["keygen_reject_seed_n16384"]])
def test_keygen_bit_exact(T, ctx16, octx16, seed):
    sk = ctx16.keygen(seed)
    assert np.array_equal(sk.export(), octx16.keygen(seed))


def test_keygen_batch_and_reject_golden(T, ctx16):
    import hashlib
    seeds = [GOLD["keygen_reject_seed_n16384"], 0]
    sk = ctx16.keygen_batch(seeds)
    assert hashlib.sha256(sk.export(0).tobytes()).hexdigest() == GOLD["keygen_reject_sk_sha256"]
    assert hashlib.sha256(sk.export(1).tobytes()).hexdigest() == GOLD["c1"]["sk_sha256"]


# ------------------------------------------------------------------ encode / encrypt
def _c1_rep():
    from tests.golden.make_golden import c1_inputs
    x, A, B = c1_inputs()
    rep = np.zeros(8192)
    for i in range(5):
        rep[i * 1536:(i + 1) * 1536] = x
    return rep, x, A, B


def test_encode_to_ntt_bit_exact(T, ctx16, octx16):
    rng = np.random.default_rng(11)
    z = np.stack([rng.standard_normal(8192), rng.standard_normal(8192) * 50, np.zeros(8192)])
    z[2, :7] = [1.0, -1.0, 0.5, 1e-9, 123.25, -7.5, 3.0]
    pt = ctx16.encode_to_ntt(z)
    for i in range(3):
        assert np.array_equal(pt.export(i), octx16.encode_to_ntt(z[i])), i


@pytest.mark.parametrize("seed", [0, 1, 123] + GOLD["encrypt_reject_seeds_n16384"])
def test_encrypt_bit_exact(T, ctx16, octx16, seed):
    rep, *_ = _c1_rep()
    sk = ctx16.keygen(0)
    osk = octx16.keygen(0)
    ct = ctx16.encrypt(rep, sk, seed=seed)
    c0, c1 = ct.export()
    o0, o1, osc = octx16.encrypt(rep, osk, seed=seed)
    assert np.array_equal(c1, o1) and np.array_equal(c0, o0)
    assert ct.scale == osc
    st = ctx16.stats()
    assert st["plan_overflow"] == 0 and st["near_tie_samples"] == 0


def test_encrypt_golden_c1(T, ctx16):
    import hashlib
    rep, *_ = _c1_rep()
    sk = ctx16.keygen(0)
    c0, c1 = ctx16.encrypt(rep, sk, seed=0).export()
    assert hashlib.sha256(c0.tobytes()).hexdigest() == GOLD["c1"]["ct_c0_sha256"]
    assert hashlib.sha256(c1.tobytes()).hexdigest() == GOLD["c1"]["ct_c1_sha256"]


def test_encrypt_batch_mixed_keys_and_rejections(T, ctx16, octx16):
    rng = np.random.default_rng(5)
    seeds = [9, GOLD["encrypt_reject_seeds_n16384"][1], 77, GOLD["encrypt_reject_seeds_n16384"][2]]
    X = rng.standard_normal((4, 3000))
    skb = ctx16.keygen_batch([0, 42])
    ski = [0, 1, 1, 0]
    ct = ctx16.encrypt_batch(X, skb, seeds, sk_index=ski)
    osk = {0: octx16.keygen(0), 1: octx16.keygen(42)}
    for i in range(4):
        c0, c1 = ct.export(i)
        o0, o1, _ = octx16.encrypt(X[i], osk[ski[i]], seed=seeds[i])
        assert np.array_equal(c0, o0) and np.array_equal(c1, o1), i


# 61-bit NTT primes just below 2^61 * (1 - 2e-4): 2^64 mod q is 2e-4 of 2^64,
# so range_u64 rejects one draw in 5000 and every N = 16384 limb segment
# holds a few rejections at scattered positions.
DENSE_REJECT = [2305381840610885633, 2305381840610426881]


def test_encrypt_dense_rejections(T, oracle):
    """Every stream needs the exact repair (more flagged streams than repair
    CTAs), with several rejections per limb anywhere in the segment."""
    ctx = T.CkksContext.from_moduli(16384, DENSE_REJECT)
    o = oracle.Ctx(16384, DENSE_REJECT)
    rng = np.random.default_rng(14)
    X = rng.standard_normal((24, 2000))
    seeds = list(range(1000, 1024))
    ct = ctx.encrypt_batch(X, ctx.keygen_batch([5]), seeds)
    osk = o.keygen(5)
    for i in range(24):
        c0, c1 = ct.export(i)
        o0, o1, _ = o.encrypt(X[i], osk, seed=seeds[i])
        assert np.array_equal(c1, o1) and np.array_equal(c0, o0), i
    st = ctx.stats()
    assert st["streams_repaired"] >= 20 and st["plan_overflow"] == 0


def test_encrypt_n8192_reject(T, oracle):
    ctx = T.CkksContext(8192)
    o = oracle.Ctx(8192)
    seed = GOLD["encrypt_reject_seeds_n8192"][0]
    z = np.linspace(-3, 3, 4096)
    c0, c1 = ctx.encrypt(z, ctx.keygen(1), seed=seed).export()
    o0, o1, _ = o.encrypt(z, o.keygen(1), seed=seed)
    assert np.array_equal(c0, o0) and np.array_equal(c1, o1)


def test_encrypt_pads_and_truncates(T, ctx16, octx16):
    sk, osk = ctx16.keygen(3), octx16.keygen(3)
    long = np.arange(9000) * 1e-3
    c0, _ = ctx16.encrypt(long, sk, seed=5).export()
    o0, _, _ = octx16.encrypt(long[:8192], osk, seed=5)
    assert np.array_equal(c0, o0)
    c0, _ = ctx16.encrypt(np.array([]), sk, seed=6).export()
    o0, _, _ = octx16.encrypt(np.array([]), osk, seed=6)
    assert np.array_equal(c0, o0)


# ------------------------------------------------------------------ decrypt / ct x pt
def test_decrypt_fresh_bit_exact(T, ctx16, octx16):
    rep, *_ = _c1_rep()
    sk, osk = ctx16.keygen(0), octx16.keygen(0)
    ct = ctx16.encrypt(rep, sk, seed=0)
    dec = ctx16.decrypt(ct, sk)
    c0, c1 = ct.export()
    ref = octx16.decrypt(c0, c1, ct.scale, osk)
    assert np.array_equal(dec.view(np.uint64), ref.view(np.uint64))
    assert np.abs(dec[:1536] - rep[:1536]).max() < 1e-6   # regression_gatelink.py:88


def test_ct_pt_mul_and_crt_decrypt_bit_exact(T, ctx16, octx16):
    rng = np.random.default_rng(2)
    a, b = rng.standard_normal(8192), rng.standard_normal(8192)
    sk, osk = ctx16.keygen(4), octx16.keygen(4)
    ct = ctx16.encrypt(a, sk, seed=8)
    prod = ct * b
    p0, p1 = prod.export()
    c0, c1 = ct.export()
    o0, o1 = octx16.ct_pt_mul(c0, c1, b)
    assert np.array_equal(p0, o0) and np.array_equal(p1, o1)
    assert prod.scale == ct.scale * ct.scale
    dec = ctx16.decrypt(prod, sk)
    ref = octx16.decrypt(o0, o1, prod.scale, osk)
    assert np.array_equal(dec.view(np.uint64), ref.view(np.uint64))
    assert np.abs(dec - a * b).max() < 1e-6


def test_ct_pt_mul_ntt_matches_uncached(T, ctx16):
    rng = np.random.default_rng(3)
    a, b = rng.standard_normal(8192), rng.standard_normal(8192)
    sk = ctx16.keygen(5)
    ct = ctx16.encrypt(a, sk, seed=1)
    pt = ctx16.encode_to_ntt(b)
    x0, x1 = ctx16.ct_pt_mul_ntt(ct, pt).export()
    y0, y1 = ctx16.ct_pt_mul(ct, b).export()
    assert np.array_equal(x0, y0) and np.array_equal(x1, y1)


def test_ct_add_sub_and_scale_mismatch(T, ctx16, octx16):
    sk = ctx16.keygen(42)
    a = np.arange(10) * 1.5
    b = 10.0 - np.arange(10) * 0.3
    ca, cb = ctx16.encrypt(a, sk, seed=111), ctx16.encrypt(b, sk, seed=112)
    s, d = ca + cb, ca - cb
    a0, a1 = ca.export()
    b0, b1 = cb.export()
    r0, r1 = octx16.ct_add(a0, a1, b0, b1)
    assert np.array_equal(s.export()[0], r0) and np.array_equal(s.export()[1], r1)
    r0, r1 = octx16.ct_add(a0, a1, b0, b1, sub=True)
    assert np.array_equal(d.export()[0], r0) and np.array_equal(d.export()[1], r1)
    assert np.abs(ctx16.decrypt(s, sk)[:10] - (a + b)).max() < 1e-4
    with pytest.raises(ValueError, match="Scale mismatch"):
        (ca * b) + cb


def test_serialize_bytes_match_oracle(T, ctx16, octx16, oracle):
    """serialize.rs:71-93 through the C ABI: the bytes of a GPU ciphertext
    equal the oracle's ct_to_bytes of the same (bit-exact) ciphertext, for a
    fresh one, a batch (blobs back to back), a ct x pt product (scale 2^80)
    and a rescaled one (3 limbs); bytes from the oracle load back and
    decrypt (the reference's KAT tolerance, serialize.rs:139-144)."""
    sk, osk = ctx16.keygen(42), octx16.keygen(42)
    z = np.arange(10, dtype=np.float64)
    ct = ctx16.encrypt(z, sk, seed=42)
    o0, o1, osc = octx16.encrypt(z, osk, seed=42)
    want = oracle.ct_to_bytes(osc, o0, o1)
    blob = ct.to_bytes()
    assert len(blob) == 8 + 2 * 4 * 16384 * 8 and blob == want
    ct2 = ctx16.ciphertext_from_bytes(want)
    assert ct2.to_bytes() == want
    assert np.abs(ctx16.decrypt(ct2, sk)[:10] - z).max() < 1e-4
    # a batch: each ciphertext's blob, back to back
    X = np.random.default_rng(31).standard_normal((3, 700))
    cts = ctx16.encrypt_batch(X, sk, seeds=[5, 6, 7])
    want3 = b""
    for i in range(3):
        e0, e1, esc = octx16.encrypt(X[i], osk, seed=5 + i)
        want3 += oracle.ct_to_bytes(esc, e0, e1)
    assert cts.to_bytes() == want3
    back = ctx16.ciphertext_from_bytes(want3)
    assert back._info()[0] == 3 and back.to_bytes() == want3
    # ct x pt (scale Delta^2) and its rescale (3 limbs)
    pt = np.random.default_rng(32).standard_normal(8192)
    prod = ct * pt
    p0, p1 = octx16.ct_pt_mul(o0, o1, pt)
    assert prod.to_bytes() == oracle.ct_to_bytes(prod.scale, p0, p1)
    r = ctx16.rescale(prod)
    r0, r1 = octx16.rescale(p0, p1)
    rb = r.to_bytes()
    assert rb == oracle.ct_to_bytes(r.scale, r0, r1) and len(rb) == 8 + 2 * 3 * 16384 * 8
    assert ctx16.ciphertext_from_bytes(rb, num_limbs=3).to_bytes() == rb
    # the reference's length assert, a word above q, mixed scales
    with pytest.raises(ValueError):
        ctx16.ciphertext_from_bytes(want[:-8])
    with pytest.raises(ValueError):
        ctx16.ciphertext_from_bytes(want, num_limbs=3)
    bad = bytearray(want)
    bad[8:16] = (ctx16.moduli[0] + 1).to_bytes(8, "little")
    with pytest.raises(ValueError, match="residue"):
        ctx16.ciphertext_from_bytes(bytes(bad))
    ok_q = bytearray(want)
    ok_q[8:16] = ctx16.moduli[0].to_bytes(8, "little")       # q itself: a word the reference's encode can emit
    ctx16.ciphertext_from_bytes(bytes(ok_q))
    mixed = want + bytes(prod.to_bytes()[:8]) + want[8:]
    with pytest.raises(ValueError, match="scale"):
        ctx16.ciphertext_from_bytes(mixed)


def test_pk_serialize_matches_oracle(T, ctx16, octx16, oracle):
    """serialize.rs:48-67 through the C ABI: pk bytes equal the oracle's
    pk_to_bytes of the same key; a key loaded from the oracle's bytes
    encrypts bit-identically to the original (Shoup companions rebuilt)."""
    sk, osk = ctx16.keygen(42), octx16.keygen(42)
    pk = ctx16.keygen_public(sk, seed=43)
    ob, oa = octx16.keygen_public(osk, 43)
    want = oracle.pk_to_bytes(ob, oa)
    assert pk.to_bytes() == want
    pk2 = ctx16.public_key_from_bytes(want)
    assert pk2.to_bytes() == want
    z = np.random.default_rng(33).standard_normal(3000)
    a = ctx16.encrypt_pk(z, pk, seed=44).to_bytes()
    b = ctx16.encrypt_pk(z, pk2, seed=44).to_bytes()
    assert a == b
    o0, o1, osc = octx16.encrypt_pk(z, ob, oa, 44)
    assert a == oracle.ct_to_bytes(osc, o0, o1)
    with pytest.raises(ValueError):
        ctx16.public_key_from_bytes(want[:-1])
    bad = bytearray(want)
    bad[-8:] = (2 ** 64 - 1).to_bytes(8, "little")
    with pytest.raises(ValueError, match="residue"):
        ctx16.public_key_from_bytes(bytes(bad))


# ------------------------------------------------------------------ ZeRo-MOAI delta
def test_lora_delta_c1(T, ctx16, octx16):
    from provenloop_b200.backend import ZeroMoaiLora
    rep, x, A, B = _c1_rep()
    sk = ctx16.keygen(0)
    lora = ZeroMoaiLora(ctx16, A, B)
    assert (lora.cols, lora.batches) == (5, 4)
    delta, inter = lora.delta(sk, x.astype(np.float64)[None], seeds=[0])
    odelta, ointer = octx16.lora_delta(octx16.keygen(0), x.astype(np.float64), A, B, enc_seed=0)
    assert np.abs(delta[0] - odelta).max() < 1e-4
    assert np.abs(inter[0] - ointer).max() < 1e-9
    assert np.allclose(inter[0], GOLD["c1"]["intermediate"], atol=1e-9, rtol=0)
    ref = B.astype(np.float64) @ (A.astype(np.float64) @ x.astype(np.float64))
    assert np.abs(delta[0] - ref).max() < 1e-4


def test_lora_delta_batch_experts_and_users(T, ctx16, octx16):
    from provenloop_b200.backend import ZeroMoaiLora
    rng = np.random.default_rng(9)
    E, r, d = 3, 16, 1536
    A = (rng.standard_normal((E, r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((E, d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((6, d))
    seeds = [10, 11, GOLD["encrypt_reject_seeds_n16384"][0], 13, 14, 15]
    expert = [0, 1, 2, 2, 1, 0]
    skb = ctx16.keygen_batch([0, 1])
    ski = [0, 1, 0, 1, 0, 1]
    lora = ZeroMoaiLora(ctx16, A, B)
    delta, inter = lora.delta(skb, H, seeds, expert=expert, sk_index=ski)
    osks = [octx16.keygen(0), octx16.keygen(1)]
    for i in range(6):
        od, oi = octx16.lora_delta(osks[ski[i]], H[i], A[expert[i]], B[expert[i]], enc_seed=seeds[i])
        assert np.abs(delta[i] - od).max() < 1e-4, i
        assert np.abs(inter[i] - oi).max() < 1e-8, i


def test_lora_delta_more_vectors_than_sms(T, ctx16, octx16):
    """80 users x 4 batches = 320 (delta, batch) vectors: the fused decrypt
    kernel's CTAs each take two or three of them."""
    from provenloop_b200.backend import ZeroMoaiLora
    rng = np.random.default_rng(12)
    r, d, n = 16, 1536, 80
    A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((n, d))
    seeds = list(range(500, 500 + n))
    lora = ZeroMoaiLora(ctx16, A, B)
    delta, inter = lora.delta(ctx16.keygen(4), H, seeds)
    osk = octx16.keygen(4)
    for i in range(n):
        od, oi = octx16.lora_delta(osk, H[i], A, B, enc_seed=seeds[i])
        assert np.abs(delta[i] - od).max() < 1e-4, i
        assert np.abs(inter[i] - oi).max() < 1e-8, i


def test_lora_delta_two_chunks_c1(T, ctx16, octx16):
    """The benchmarked shape and beyond: C1 with 2100 hidden states in one
    call: through host buffers, three pipelined passes (256, 1588, 256);
    through device buffers, two passes of 1050 (the bench's 2048 is one).  Rows from both passes, including
    the first and last of each, against the oracle; every row against
    float64 B (A h) (inference_engine.py:1244-1392)."""
    from provenloop_b200.backend import ZeroMoaiLora
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((16, 1536)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((1536, 16)) * 0.02).astype(np.float32)
    n = 2100
    H = np.random.default_rng(77).standard_normal((n, 1536)).astype(np.float32).astype(np.float64)
    seeds = np.arange(90_000, 90_000 + n, dtype=np.uint64)
    lora = ZeroMoaiLora(ctx16, A, B)
    delta, inter = lora.delta(ctx16.keygen(0), H, seeds)
    osk = octx16.keygen(0)
    pc = octx16.lora_pack(A)
    for i in (0, 1, 1023, 2046, 2047, 2048, 2049, 2099):
        od, oi = octx16.lora_delta(osk, H[i], A, B, enc_seed=int(seeds[i]), pt_cache=pc)
        assert np.abs(delta[i] - od).max() < 1e-4, i
        assert np.abs(inter[i] - oi).max() < 1e-8, i
    plain = (H @ A.astype(np.float64).T) @ B.astype(np.float64).T
    assert np.abs(delta - plain).max() < 1e-4
    # host buffers and device buffers run different passes: the same deltas
    # bit for bit
    import torch
    h_dev = torch.from_numpy(H).cuda()
    d_dev = torch.empty_like(h_dev)
    torch.cuda.synchronize()
    lora.delta_device(ctx16.keygen(0), h_dev, seeds, d_dev)
    ctx16.synchronize()
    assert np.array_equal(d_dev.cpu().numpy(), delta)


def test_lora_delta_eight_columns_fused(T, ctx16, octx16):
    """d = 1024 at N = 16384: 8 segment columns per plaintext, which takes
    the fused four-CTA decrypt sized for up to 10 columns (the benchmark's
    d = 1536 uses the 5-column form), in the batched regime (80 states x 2
    plaintext batches)."""
    from provenloop_b200.backend import ZeroMoaiLora
    rng = np.random.default_rng(14)
    r, d, n = 16, 1024, 80
    A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((n, d))
    seeds = list(range(800, 800 + n))
    lora = ZeroMoaiLora(ctx16, A, B)
    assert (lora.cols, lora.batches) == (8, 2)
    delta, inter = lora.delta(ctx16.keygen(5), H, seeds)
    osk = octx16.keygen(5)
    for i in (0, 1, 39, 78, 79):
        od, oi = octx16.lora_delta(osk, H[i], A, B, enc_seed=seeds[i])
        assert np.abs(delta[i] - od).max() < 1e-4, i
        assert np.abs(inter[i] - oi).max() < 1e-8, i
    plain = (H @ A.astype(np.float64).T) @ B.astype(np.float64).T
    assert np.abs(delta - plain).max() < 1e-4


def test_lora_delta_ragged_rank_and_small_d(T, ctx16, octx16):
    from provenloop_b200.backend import ZeroMoaiLora
    rng = np.random.default_rng(10)
    for r, d in ((7, 1536), (3, 64), (9, 3584)):
        A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
        B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
        h = rng.standard_normal(d)
        lora = ZeroMoaiLora(ctx16, A, B)
        delta, inter = lora.delta(ctx16.keygen(2), h, seeds=[21])
        od, oi = octx16.lora_delta(octx16.keygen(2), h, A, B, enc_seed=21)
        assert np.abs(delta[0] - od).max() < 1e-4 and np.abs(inter[0] - oi).max() < 1e-8, (r, d)


# ------------------------------------------------------------------ adapter surface
def test_adapter_surface_matches_engine_contract(T, ctx16):
    import torch
    from provenloop_b200.backend import TenSafeB200Adapter
    ad = TenSafeB200Adapter(ctx16, ctx16.keygen(0))
    v = np.random.default_rng(0).standard_normal(1536)
    ct = ad.encrypt_vector(v)
    assert np.abs(ad.decrypt_vector(ct)[:1536] - v).max() < 1e-6
    prod = ct * np.full(8192, 0.5)
    dg = ad.decrypt_to_gpu(prod)
    assert isinstance(dg, torch.Tensor) and dg.is_cuda and dg.dtype == torch.float64 and dg.numel() == 8192
    assert np.abs(dg.cpu().numpy()[:1536] - 0.5 * v).max() < 1e-6
    st = ad.status()
    for k in ("backend", "version", "initialized", "gpu_available", "gpu_enabled", "gpu_accelerated",
              "gpu_device", "poly_mod_degree", "emulated", "metrics"):
        assert k in st
    assert st["metrics"]["total_encryptions"] == 1 and st["metrics"]["total_decryptions"] == 2


def test_dp_noise(T, ctx16, oracle):
    from provenloop_b200.backend import add_dp_noise, dp_sigma
    sigma = dp_sigma(1.0, 1e-5, 1.0)
    assert abs(sigma - 4.8448) < 1e-3
    h = np.ones((2, 1536)) * 100.0
    out = add_dp_noise(ctx16, h, sigma, seeds=[7, 8], clip=1.0)
    clipped = h / np.linalg.norm(h[0])
    r = oracle.Rng(7)
    noise = np.array([r.gaussian(sigma) for _ in range(1536)])
    assert np.abs(out[0] - (clipped[0] + noise)).max() < 1e-9
    big = add_dp_noise(ctx16, np.zeros((1, 200000 // 100)), sigma, seeds=[1])
    assert abs(big.std() - sigma) < 0.3


# NTT-friendly primes on either side of 2^50, the bound of the FP64 butterfly
# mode (below: exact FP64 products; above: 64-bit integer Shoup products)
FP_EDGE = {8192: [1125899906826241, 1125899906990081], 16384: [1125899904679937, 1125899908022273],
           32768: [1125899904679937, 1125899908022273]}


@pytest.mark.parametrize("n", [8192, 16384, 32768])
def test_ntt_fp64_mode_edges_bit_exact(T, oracle, n):
    """Both transform modes at the largest values they admit: inputs of all
    q - 1, alternating 0 / q - 1, and uniform residues, on the primes just
    below and just above 2^50; forward and inverse bit-exact against the
    oracle (ntt.rs:79-141)."""
    from provenloop_b200._lib import lib, check
    qs = FP_EDGE[n]
    assert qs[0] < (1 << 50) < qs[1]
    ctx = T.CkksContext.from_moduli(n, qs)
    rng = np.random.default_rng(50 + n)
    polys = []
    for kind in range(3):
        rows = []
        for q in qs:
            if kind == 0:
                rows.append(np.full(n, q - 1, np.uint64))
            elif kind == 1:
                rows.append(np.where(np.arange(n) % 2 == 0, 0, q - 1).astype(np.uint64))
            else:
                rows.append(rng.integers(0, q, size=n, dtype=np.uint64))
        polys.append(np.stack(rows))
    x = np.stack(polys)
    d = _dev(x)
    check(lib().ts_ntt_forward(ctx.handle, d.data_ptr(), 3, 2, 0))
    ctx.synchronize()
    fwd = _host(d).reshape(x.shape)
    for p in range(3):
        for l, q in enumerate(qs):
            assert np.array_equal(fwd[p, l], oracle.ntt_forward(x[p, l], n, q)), (p, l)
    # inverse of the extreme inputs themselves (not a round trip)
    d2 = _dev(x)
    check(lib().ts_ntt_inverse(ctx.handle, d2.data_ptr(), 3, 2, 0))
    ctx.synchronize()
    inv = _host(d2).reshape(x.shape)
    for p in range(3):
        for l, q in enumerate(qs):
            assert np.array_equal(inv[p, l], oracle.ntt_inverse(x[p, l], n, q)), (p, l)


def test_lora_set_expert_between_graph_replays(T, oracle):
    """Adapter hot swap (inference_engine.py:879-959): a captured CUDA graph
    of ts_lora_delta_batch (device seeds and expert indexes) is replayed,
    expert 1 is replaced in place, and the next replay of the same graph
    gives expert 1's rows from the new adapter (against the oracle) while
    the other experts' rows are unchanged."""
    import torch
    from provenloop_b200 import _lib
    from provenloop_b200.backend import ZeroMoaiLora, lora_delta_graphable
    ctx = T.CkksContext(16384)
    octx = oracle.Ctx(16384)
    rng = np.random.default_rng(61)
    E, r, d, n = 3, 16, 1536, 6
    A = (rng.standard_normal((E, r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((E, d, r)) * 0.02).astype(np.float32)
    A2 = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
    B2 = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((n, d))
    seeds = np.arange(4000, 4000 + n, dtype=np.uint64)
    expert = np.array([0, 1, 2, 1, 0, 1], dtype=np.int32)
    sk = ctx.keygen(3)
    lora = ZeroMoaiLora(ctx, A, B)
    stream = torch.cuda.Stream()
    _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "set_stream")
    h = torch.from_numpy(H).cuda()
    out = torch.empty_like(h)
    sd = torch.from_numpy(seeds.view(np.int64)).cuda()
    ex = torch.from_numpy(expert).cuda()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        lora_delta_graphable(lora, sk, h, sd, out, expert_dev=ex)  # sizes the scratch
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            lora_delta_graphable(lora, sk, h, sd, out, expert_dev=ex)
    g.replay()
    torch.cuda.synchronize()
    before = out.cpu().numpy()
    osk = octx.keygen(3)
    for i in range(n):
        od, _ = octx.lora_delta(osk, H[i], A[expert[i]], B[expert[i]], enc_seed=int(seeds[i]))
        assert np.abs(before[i] - od).max() < 1e-4, i
    lora.set_expert(1, A2, B2)
    g.replay()
    torch.cuda.synchronize()
    after = out.cpu().numpy()
    for i in range(n):
        if expert[i] == 1:
            od, _ = octx.lora_delta(osk, H[i], A2, B2, enc_seed=int(seeds[i]))
            assert np.abs(after[i] - od).max() < 1e-4, i
            assert np.abs(after[i] - before[i]).max() > 1e-6, i
        else:
            assert np.array_equal(after[i], before[i]), i
    with pytest.raises(ValueError):
        lora.set_expert(3, A2, B2)
    with pytest.raises(ValueError):
        lora.set_expert(0, A2[:8], B2)
    del g
    _lib.check(_lib.lib().ts_ctx_reset_stream(ctx.handle), "reset_stream")
