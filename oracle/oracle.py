"""ctypes wrapper around the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a C restatement of the reference Rust crate
``tensafe-he/crates/tensafe-he-core`` (see ``tsoracle.c`` for the per-function
file:line citations).  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference arm of ``bench.py`` import this module; the product
package ``provenloop_b200`` never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libtsoracle.so")
_lib = None
_lock = threading.Lock()

U64P = C.POINTER(C.c_uint64)
I64P = C.POINTER(C.c_int64)
F64P = C.POINTER(C.c_double)
F32P = C.POINTER(C.c_float)
U32P = C.POINTER(C.c_uint32)


class OrRng(C.Structure):
    _fields_ = [("state", C.c_uint32 * 16), ("buffer", C.c_uint32 * 16), ("index", C.c_uint32)]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            L = C.CDLL(_LIB_PATH)
            sig = {
                "or_params_preset": (C.c_int, [C.c_uint32, U64P, U32P]),
                "or_find_ntt_friendly_prime": (C.c_uint64, [C.c_uint32, C.c_uint64]),
                "or_is_prime_u64": (C.c_int, [C.c_uint64]),
                "or_mod_add": (C.c_uint64, [C.c_uint64] * 3),
                "or_mod_sub": (C.c_uint64, [C.c_uint64] * 3),
                "or_mod_mul": (C.c_uint64, [C.c_uint64] * 3),
                "or_mod_pow": (C.c_uint64, [C.c_uint64] * 3),
                "or_mod_inv": (C.c_uint64, [C.c_uint64] * 2),
                "or_find_primitive_root": (C.c_uint64, [C.c_size_t, C.c_uint64]),
                "or_bit_reverse": (C.c_uint32, [C.c_uint32, C.c_uint32]),
                "or_ntt_forward_nq": (C.c_int, [U64P, C.c_size_t, C.c_uint64]),
                "or_ntt_inverse_nq": (C.c_int, [U64P, C.c_size_t, C.c_uint64]),
                "or_ntt_tables_export": (C.c_int, [C.c_size_t, C.c_uint64, U64P, U64P, U64P, U64P]),
                "or_chacha20_block": (None, [U32P, U32P]),
                "or_rng_from_seed": (None, [C.POINTER(OrRng), C.c_uint64]),
                "or_rng_next_u32": (C.c_uint32, [C.POINTER(OrRng)]),
                "or_rng_next_u64": (C.c_uint64, [C.POINTER(OrRng)]),
                "or_rng_range_u32": (C.c_uint32, [C.POINTER(OrRng), C.c_uint32]),
                "or_rng_range_u64": (C.c_uint64, [C.POINTER(OrRng), C.c_uint64]),
                "or_rng_next_f64": (C.c_double, [C.POINTER(OrRng)]),
                "or_rng_gaussian": (C.c_double, [C.POINTER(OrRng), C.c_double]),
                "or_sample_ternary": (None, [C.POINTER(OrRng), C.c_size_t, C.c_uint64, U64P]),
                "or_sample_gaussian_signed": (None, [C.POINTER(OrRng), C.c_size_t, C.c_double, I64P]),
                "or_sample_uniform": (None, [C.POINTER(OrRng), C.c_size_t, C.c_uint64, U64P]),
                "or_ctx_new": (C.c_void_p, [C.c_uint32, U64P, C.c_uint32, C.c_uint32]),
                "or_ctx_free": (None, [C.c_void_p]),
                "or_ctx_fft_tables": (C.c_int, [C.c_void_p, F64P, F64P, F64P, F64P]),
                "or_encode": (C.c_int, [C.c_void_p, F64P, C.c_size_t, U64P]),
                "or_encode_coeffs": (C.c_int, [C.c_void_p, F64P, C.c_size_t, I64P]),
                "or_decode": (None, [C.c_void_p, U64P, C.c_double, F64P]),
                "or_decode_coefficients": (None, [C.c_void_p, F64P, F64P]),
                "or_fft": (None, [C.c_void_p, F64P, F64P]),
                "or_keygen": (None, [C.c_void_p, C.POINTER(OrRng), U64P]),
                "or_keygen_public": (None, [C.c_void_p, U64P, C.POINTER(OrRng), U64P, U64P]),
                "or_encrypt": (C.c_int, [C.c_void_p, F64P, C.c_size_t, U64P, C.POINTER(OrRng), U64P, U64P, F64P]),
                "or_encrypt_pk": (C.c_int, [C.c_void_p, F64P, C.c_size_t, U64P, U64P, C.POINTER(OrRng), U64P, U64P, F64P]),
                "or_decrypt": (None, [C.c_void_p, U64P, U64P, C.c_uint32, C.c_double, U64P, F64P]),
                "or_decrypt_coeffs": (None, [C.c_void_p, U64P, U64P, C.c_uint32, C.c_double, U64P, F64P]),
                "or_encode_to_ntt": (C.c_int, [C.c_void_p, F64P, C.c_size_t, U64P]),
                "or_ct_pt_mul_ntt": (None, [C.c_void_p, U64P, U64P, C.c_uint32, U64P, U64P, U64P]),
                "or_ct_pt_mul": (C.c_int, [C.c_void_p, U64P, U64P, C.c_uint32, F64P, C.c_size_t, U64P, U64P]),
                "or_ct_add": (None, [C.c_void_p, U64P, U64P, U64P, U64P, C.c_uint32, U64P, U64P]),
                "or_ct_sub": (None, [C.c_void_p, U64P, U64P, U64P, U64P, C.c_uint32, U64P, U64P]),
                "or_rescale": (C.c_int, [C.c_void_p, U64P, U64P, C.c_uint32, U64P, U64P]),
                "or_u128_to_f64": (C.c_double, [C.c_uint64, C.c_uint64]),
                "or_find_reject_seed": (C.c_uint64, [U64P, C.c_uint32, C.c_size_t, C.c_uint64, C.c_uint64, C.c_int]),
                "or_rns_poly_to_bytes": (None, [U64P, C.c_size_t, C.c_uint32, C.c_char_p]),
                "or_rns_poly_from_bytes": (C.c_int, [C.c_char_p, C.c_size_t, C.c_size_t, C.c_uint32, U64P]),
                "or_pk_to_bytes": (None, [U64P, U64P, C.c_size_t, C.c_uint32, C.c_char_p]),
                "or_pk_from_bytes": (C.c_int, [C.c_char_p, C.c_size_t, C.c_size_t, C.c_uint32, U64P, U64P]),
                "or_ct_to_bytes": (None, [C.c_double, U64P, U64P, C.c_size_t, C.c_uint32, C.c_char_p]),
                "or_ct_from_bytes": (C.c_int, [C.c_char_p, C.c_size_t, C.c_size_t, C.c_uint32, F64P, U64P, U64P]),
                "or_lora_delta": (C.c_int, [C.c_void_p, U64P, F64P, C.c_uint32, F32P, F32P, C.c_uint32,
                                            C.c_uint64, C.c_int, F64P, F64P]),
                "or_lora_pack": (C.c_int, [C.c_void_p, F32P, C.c_uint32, C.c_uint32, U64P]),
                "or_lora_delta_cached": (C.c_int, [C.c_void_p, U64P, F64P, C.c_uint32, F32P, F32P, C.c_uint32,
                                                   C.c_uint64, C.c_int, U64P, F64P, F64P]),
            }
            for name, (res, args) in sig.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _u64(a):
    a = np.ascontiguousarray(a, dtype=np.uint64)
    return a


# ---------------------------------------------------------------- params / rns
def params_preset(n: int):
    m = np.zeros(4, np.uint64)
    b = np.zeros(4, np.uint32)
    L = lib().or_params_preset(n, _p(m, U64P), _p(b, U32P))
    if L < 0:
        raise ValueError(f"Unsupported polynomial degree {n}")
    return [int(x) for x in m[:L]], [int(x) for x in b[:L]]


def params_custom(n: int, bits):
    """CkksParams::custom (params.rs:142-162): one descending search per width."""
    return [int(lib().or_find_ntt_friendly_prime(int(b), 2 * n)) for b in bits]


def find_primitive_root(n, q):
    return int(lib().or_find_primitive_root(n, q))


def ntt_forward(a, n, q):
    a = _u64(a).copy()
    rc = lib().or_ntt_forward_nq(_p(a, U64P), n, q)
    if rc:
        raise RuntimeError(f"ntt tables rc={rc}")
    return a


def ntt_inverse(a, n, q):
    a = _u64(a).copy()
    rc = lib().or_ntt_inverse_nq(_p(a, U64P), n, q)
    if rc:
        raise RuntimeError(f"ntt tables rc={rc}")
    return a


def ntt_tables(n, q):
    fw = np.zeros(n, np.uint64)
    iw = np.zeros(n, np.uint64)
    psi = C.c_uint64()
    ninv = C.c_uint64()
    rc = lib().or_ntt_tables_export(n, q, _p(fw, U64P), _p(iw, U64P), C.byref(psi), C.byref(ninv))
    if rc:
        raise RuntimeError(f"ntt tables rc={rc}")
    return fw, iw, int(psi.value), int(ninv.value)


# ---------------------------------------------------------------- rng
class Rng:
    """TenSafeRng (rng.rs:22-158)."""

    def __init__(self, seed: int):
        self._s = OrRng()
        lib().or_rng_from_seed(C.byref(self._s), seed & 0xFFFFFFFFFFFFFFFF)

    @property
    def ref(self):
        return C.byref(self._s)

    def next_u32(self):
        return int(lib().or_rng_next_u32(self.ref))

    def next_u64(self):
        return int(lib().or_rng_next_u64(self.ref))

    def range_u32(self, m):
        return int(lib().or_rng_range_u32(self.ref, m))

    def range_u64(self, m):
        return int(lib().or_rng_range_u64(self.ref, m))

    def next_f64(self):
        return float(lib().or_rng_next_f64(self.ref))

    def gaussian(self, sigma):
        return float(lib().or_rng_gaussian(self.ref, sigma))

    def sample_ternary(self, n, q):
        out = np.zeros(n, np.uint64)
        lib().or_sample_ternary(self.ref, n, q, _p(out, U64P))
        return out

    def sample_gaussian_signed(self, n, sigma=3.19):
        out = np.zeros(n, np.int64)
        lib().or_sample_gaussian_signed(self.ref, n, sigma, _p(out, I64P))
        return out

    def sample_uniform(self, n, q):
        out = np.zeros(n, np.uint64)
        lib().or_sample_uniform(self.ref, n, q, _p(out, U64P))
        return out


def chacha20_block(state):
    st = np.ascontiguousarray(state, dtype=np.uint32)
    out = np.zeros(16, np.uint32)
    lib().or_chacha20_block(_p(st, U32P), _p(out, U32P))
    return out


def find_reject_seed(moduli, n, start, count, kind):
    """First seed in [start, start+count) whose encrypt (kind 0) or keygen
    (kind 1) stream rejects a candidate, or None."""
    m = np.asarray(moduli, dtype=np.uint64)
    s = int(lib().or_find_reject_seed(_p(m, U64P), m.size, n, start, count, kind))
    return None if s == 0xFFFFFFFFFFFFFFFF else s


# ---------------------------------------------------------------- wire format
def rns_poly_to_bytes(poly) -> bytes:
    """serialize.rs:14-23: limb-major, u64 little-endian."""
    p = _u64(poly)
    L, n = p.shape
    out = C.create_string_buffer(L * n * 8)
    lib().or_rns_poly_to_bytes(_p(p, U64P), n, L, out)
    return out.raw


def rns_poly_from_bytes(blob: bytes, n: int, L: int):
    out = np.zeros((L, n), np.uint64)
    if lib().or_rns_poly_from_bytes(blob, len(blob), n, L, _p(out, U64P)):
        raise ValueError(f"Expected {L * n * 8} bytes for RnsPoly(n={n}, L={L}), got {len(blob)}")
    return out


def pk_to_bytes(b, a) -> bytes:
    """serialize.rs:48-52: [b | a]."""
    b, a = _u64(b), _u64(a)
    L, n = b.shape
    out = C.create_string_buffer(2 * L * n * 8)
    lib().or_pk_to_bytes(_p(b, U64P), _p(a, U64P), n, L, out)
    return out.raw


def pk_from_bytes(blob: bytes, n: int, L: int):
    b = np.zeros((L, n), np.uint64)
    a = np.zeros((L, n), np.uint64)
    if lib().or_pk_from_bytes(blob, len(blob), n, L, _p(b, U64P), _p(a, U64P)):
        raise ValueError(f"Expected {2 * L * n * 8} bytes for PublicKey, got {len(blob)}")
    return b, a


def ct_to_bytes(scale: float, c0, c1) -> bytes:
    """serialize.rs:71-77: [scale f64 LE | c0 | c1]."""
    c0, c1 = _u64(c0), _u64(c1)
    L, n = c0.shape
    out = C.create_string_buffer(8 + 2 * L * n * 8)
    lib().or_ct_to_bytes(float(scale), _p(c0, U64P), _p(c1, U64P), n, L, out)
    return out.raw


def ct_from_bytes(blob: bytes, n: int, L: int):
    """serialize.rs:80-93; returns (scale, c0, c1)."""
    c0 = np.zeros((L, n), np.uint64)
    c1 = np.zeros((L, n), np.uint64)
    sc = C.c_double()
    if lib().or_ct_from_bytes(blob, len(blob), n, L, C.byref(sc), _p(c0, U64P), _p(c1, U64P)):
        raise ValueError(f"Expected {8 + 2 * L * n * 8} bytes for Ciphertext, got {len(blob)}")
    return sc.value, c0, c1


def u128_to_f64(v: int) -> float:
    return float(lib().or_u128_to_f64((v >> 64) & 0xFFFFFFFFFFFFFFFF, v & 0xFFFFFFFFFFFFFFFF))


# ---------------------------------------------------------------- context
class Ctx:
    """CkksContext (ciphertext.rs:61-74) for a preset or explicit chain."""

    def __init__(self, n: int, moduli=None, scale_bits: int = 40):
        if moduli is None:
            moduli, _ = params_preset(n)
        self.n = n
        self.S = n // 2
        self.moduli = [int(q) for q in moduli]
        self.L = len(self.moduli)
        m = np.asarray(self.moduli, dtype=np.uint64)
        self._h = lib().or_ctx_new(n, _p(m, U64P), self.L, scale_bits)
        if not self._h:
            raise RuntimeError("or_ctx_new failed")
        self.scale = float(2.0 ** 40)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().or_ctx_free(h)
            self._h = None

    # encoding
    def fft_tables(self):
        a = [np.zeros(self.n) for _ in range(4)]
        lib().or_ctx_fft_tables(self._h, *[_p(x, F64P) for x in a])
        return a

    def encode(self, z):
        z = np.ascontiguousarray(z, dtype=np.float64)
        out = np.zeros(self.L * self.n, np.uint64)
        if lib().or_encode(self._h, _p(z, F64P), z.size, _p(out, U64P)):
            raise ValueError("encode: input longer than slot count")
        return out.reshape(self.L, self.n)

    def encode_coeffs(self, z):
        z = np.ascontiguousarray(z, dtype=np.float64)
        out = np.zeros(self.n, np.int64)
        if lib().or_encode_coeffs(self._h, _p(z, F64P), z.size, _p(out, I64P)):
            raise ValueError("encode: input longer than slot count")
        return out

    def encode_to_ntt(self, z):
        z = np.ascontiguousarray(z, dtype=np.float64)
        out = np.zeros(self.L * self.n, np.uint64)
        if lib().or_encode_to_ntt(self._h, _p(z, F64P), z.size, _p(out, U64P)):
            raise ValueError("encode: input longer than slot count")
        return out.reshape(self.L, self.n)

    def decode(self, poly, scale):
        poly = _u64(poly)
        out = np.zeros(self.S)
        lib().or_decode(self._h, _p(poly, U64P), scale, _p(out, F64P))
        return out

    def decode_coefficients(self, coeffs):
        coeffs = np.ascontiguousarray(coeffs, dtype=np.float64)
        out = np.zeros(self.S)
        lib().or_decode_coefficients(self._h, _p(coeffs, F64P), _p(out, F64P))
        return out

    def fft(self, re, im):
        re = np.ascontiguousarray(re, dtype=np.float64).copy()
        im = np.ascontiguousarray(im, dtype=np.float64).copy()
        lib().or_fft(self._h, _p(re, F64P), _p(im, F64P))
        return re, im

    # keys / ciphertexts (polys returned as [L, n] uint64)
    def keygen(self, seed: int = None, rng: Rng = None):
        r = rng if rng is not None else Rng(seed)
        sk = np.zeros(self.L * self.n, np.uint64)
        lib().or_keygen(self._h, r.ref, _p(sk, U64P))
        return sk.reshape(self.L, self.n)

    def keygen_public(self, sk, seed: int = None, rng: Rng = None):
        r = rng if rng is not None else Rng(seed)
        sk = _u64(sk)
        b = np.zeros(self.L * self.n, np.uint64)
        a = np.zeros(self.L * self.n, np.uint64)
        lib().or_keygen_public(self._h, _p(sk, U64P), r.ref, _p(b, U64P), _p(a, U64P))
        return b.reshape(self.L, self.n), a.reshape(self.L, self.n)

    def encrypt(self, z, sk, seed: int = None, rng: Rng = None):
        r = rng if rng is not None else Rng(seed)
        z = np.ascontiguousarray(z, dtype=np.float64)
        sk = _u64(sk)
        c0 = np.zeros(self.L * self.n, np.uint64)
        c1 = np.zeros(self.L * self.n, np.uint64)
        sc = C.c_double()
        if lib().or_encrypt(self._h, _p(z, F64P), z.size, _p(sk, U64P), r.ref, _p(c0, U64P),
                            _p(c1, U64P), C.byref(sc)):
            raise ValueError("encode: input longer than slot count")
        return c0.reshape(self.L, self.n), c1.reshape(self.L, self.n), sc.value

    def encrypt_pk(self, z, pk_b, pk_a, seed: int):
        r = Rng(seed)
        z = np.ascontiguousarray(z, dtype=np.float64)
        b, a = _u64(pk_b), _u64(pk_a)
        c0 = np.zeros(self.L * self.n, np.uint64)
        c1 = np.zeros(self.L * self.n, np.uint64)
        sc = C.c_double()
        if lib().or_encrypt_pk(self._h, _p(z, F64P), z.size, _p(b, U64P), _p(a, U64P), r.ref,
                               _p(c0, U64P), _p(c1, U64P), C.byref(sc)):
            raise ValueError("encode: input longer than slot count")
        return c0.reshape(self.L, self.n), c1.reshape(self.L, self.n), sc.value

    def decrypt(self, c0, c1, scale, sk):
        c0, c1, sk = _u64(c0), _u64(c1), _u64(sk)
        nl = c0.size // self.n
        out = np.zeros(self.S)
        lib().or_decrypt(self._h, _p(c0, U64P), _p(c1, U64P), nl, scale, _p(sk, U64P), _p(out, F64P))
        return out

    def decrypt_coeffs(self, c0, c1, scale, sk):
        c0, c1, sk = _u64(c0), _u64(c1), _u64(sk)
        nl = c0.size // self.n
        out = np.zeros(self.n)
        lib().or_decrypt_coeffs(self._h, _p(c0, U64P), _p(c1, U64P), nl, scale, _p(sk, U64P),
                                _p(out, F64P))
        return out

    def ct_pt_mul_ntt(self, c0, c1, pt_ntt):
        c0, c1, p = _u64(c0), _u64(c1), _u64(pt_ntt)
        nl = c0.size // self.n
        o0 = np.zeros_like(c0)
        o1 = np.zeros_like(c1)
        lib().or_ct_pt_mul_ntt(self._h, _p(c0, U64P), _p(c1, U64P), nl, _p(p, U64P), _p(o0, U64P),
                               _p(o1, U64P))
        return o0.reshape(nl, self.n), o1.reshape(nl, self.n)

    def ct_pt_mul(self, c0, c1, pt):
        c0, c1 = _u64(c0), _u64(c1)
        pt = np.ascontiguousarray(pt, dtype=np.float64)
        nl = c0.size // self.n
        o0 = np.zeros_like(c0)
        o1 = np.zeros_like(c1)
        if lib().or_ct_pt_mul(self._h, _p(c0, U64P), _p(c1, U64P), nl, _p(pt, F64P), pt.size,
                              _p(o0, U64P), _p(o1, U64P)):
            raise ValueError("encode: input longer than slot count")
        return o0.reshape(nl, self.n), o1.reshape(nl, self.n)

    def ct_add(self, a0, a1, b0, b1, sub=False):
        a0, a1, b0, b1 = map(_u64, (a0, a1, b0, b1))
        nl = a0.size // self.n
        o0 = np.zeros_like(a0)
        o1 = np.zeros_like(a1)
        f = lib().or_ct_sub if sub else lib().or_ct_add
        f(self._h, _p(a0, U64P), _p(a1, U64P), _p(b0, U64P), _p(b1, U64P), nl, _p(o0, U64P), _p(o1, U64P))
        return o0.reshape(nl, self.n), o1.reshape(nl, self.n)

    def rescale(self, c0, c1):
        c0, c1 = _u64(c0), _u64(c1)
        nl = c0.size // self.n
        o0 = np.zeros((nl - 1) * self.n, np.uint64)
        o1 = np.zeros((nl - 1) * self.n, np.uint64)
        if lib().or_rescale(self._h, _p(c0, U64P), _p(c1, U64P), nl, _p(o0, U64P), _p(o1, U64P)):
            raise ValueError("Cannot rescale: only 1 limb left")
        return o0.reshape(nl - 1, self.n), o1.reshape(nl - 1, self.n)

    def lora_pack(self, lora_a):
        """NTT(encode(packed A rows)) per batch: [n_batches, L, n]."""
        A = np.ascontiguousarray(lora_a, dtype=np.float32)
        r, d = A.shape
        cols = max(1, self.S // d)
        nb = -(-r // cols)
        out = np.zeros((nb, self.L, self.n), np.uint64)
        if lib().or_lora_pack(self._h, _p(A, F32P), r, d, _p(out, U64P)):
            raise ValueError("or_lora_pack failed")
        return out

    def lora_delta(self, sk, h, lora_a, lora_b, enc_seed: int, mode: int = 0, pt_cache=None):
        """ZeRo-MOAI delta (inference_engine.py:1244-1392). Returns (delta, intermediate).

        mode 0 + pt_cache: cached NTT(pt) (fastest CPU form); mode 0: encode
        per call; mode 1: as the PyO3 binding invokes it."""
        sk = _u64(sk)
        h = np.ascontiguousarray(h, dtype=np.float64)
        A = np.ascontiguousarray(lora_a, dtype=np.float32)
        B = np.ascontiguousarray(lora_b, dtype=np.float32)
        r, d = A.shape
        delta = np.zeros(d)
        inter = np.zeros(r)
        pc = None if pt_cache is None else _u64(pt_cache)
        rc = lib().or_lora_delta_cached(self._h, _p(sk, U64P), _p(h, F64P), d, _p(A, F32P), _p(B, F32P), r,
                                        enc_seed, mode, None if pc is None else _p(pc, U64P), _p(delta, F64P),
                                        _p(inter, F64P))
        if rc:
            raise ValueError(f"or_lora_delta rc={rc}")
        return delta, inter
