"""Drop-in replacement for the PyO3 module ``tensafe_he``.

Mirrors tensafe-he/crates/tensafe-he-python/src/lib.rs class for class:
``CkksContext``, ``TenSafeCiphertext``, ``TenSafeSecretKey``,
``TenSafePublicKey`` -- same constructor arguments, getters, methods,
padding / truncation rules and error types -- but every operation runs on a
B200 through libtsgpu.so.  A ciphertext object keeps its residues in device
memory; numpy arrays go in and come out exactly as with the Rust binding.

Use it where the inference engine does ``import tensafe_he``
(demonstrator/server/inference_engine.py:630-652)::

    import provenloop_b200.tensafe_he as tensafe_he
"""
from __future__ import annotations

import ctypes as C
import sys
import os
import struct

import numpy as np

from . import _lib
from ._lib import check, lib, ptr

__all__ = ["CkksContext", "TenSafeCiphertext", "TenSafeSecretKey", "TenSafePublicKey", "is_available"]

VERSION = "0.1.0"
SCALE = float(2 ** 40)


def _entropy_seed() -> int:
    # TenSafeRng::from_entropy (rng.rs:73-76, :210-221): 8 bytes of
    # /dev/urandom, little endian.
    return struct.unpack("<Q", os.urandom(8))[0]


def _seed(seed):
    return _entropy_seed() if seed is None else int(seed) & 0xFFFFFFFFFFFFFFFF


def _f64(data) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(data, dtype=np.float64).ravel())


def is_available() -> bool:
    """True when libtsgpu.so loads and a CUDA device is visible."""
    try:
        return _lib.device_count() > 0
    except Exception:
        return False


class _Handle:
    __slots__ = ("_h", "_destroy", "_keep")

    def __init__(self, h, destroy, keep=None):
        self._h = h
        self._destroy = destroy
        self._keep = keep  # keeps the context alive while the object lives

    def close(self):
        h, self._h = self._h, None
        if h:
            self._destroy(h)

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit the CUDA runtime may already be torn down (and
        # module globals cleared); the process releases everything anyway
        if _finalizing():
            return
        try:
            self.close()
        except Exception:
            pass


class TenSafeSecretKey:
    """Secret key s (NTT domain) held on the device (lib.rs:297-301)."""

    def __init__(self, ctx: "CkksContext", h):
        self._ctx = ctx
        self._hd = _Handle(h, lib().ts_sk_destroy, ctx)

    @property
    def handle(self):
        return self._hd._h

    def export(self, index: int = 0) -> np.ndarray:
        """NTT-domain residues [L, N] (tests)."""
        out = np.zeros(self._ctx._L * self._ctx._n, np.uint64)
        check(lib().ts_sk_export(self.handle, index, ptr(out, C.c_uint64)), "ts_sk_export")
        return out.reshape(self._ctx._L, self._ctx._n)


class TenSafePublicKey:
    """Public key pk = (b, a), NTT domain, on the device (lib.rs:303-307)."""

    def __init__(self, ctx: "CkksContext", h):
        self._ctx = ctx
        self._hd = _Handle(h, lib().ts_pk_destroy, ctx)

    @property
    def handle(self):
        return self._hd._h

    def export(self):
        """(b, a) residues, each [L, N] uint64 (tests)."""
        n = self._ctx._L * self._ctx._n
        b, a = np.zeros(n, np.uint64), np.zeros(n, np.uint64)
        check(lib().ts_pk_export(self.handle, ptr(b, C.c_uint64), ptr(a, C.c_uint64)), "ts_pk_export")
        return b.reshape(self._ctx._L, self._ctx._n), a.reshape(self._ctx._L, self._ctx._n)

    def to_bytes(self) -> bytes:
        """serialize.rs:48-52 pk_to_bytes: [b | a], limb-major u64 LE."""
        size = 2 * self._ctx._L * self._ctx._n * 8
        buf = C.create_string_buffer(size)
        check(lib().ts_pk_to_bytes(self.handle, buf, size, None), "ts_pk_to_bytes")
        return buf.raw


class TenSafeCiphertext:
    """CKKS ciphertext with operator overloading (lib.rs:309-395)."""

    def __init__(self, ctx: "CkksContext", h):
        self._ctx = ctx
        self._hd = _Handle(h, lib().ts_ct_destroy, ctx)

    @property
    def handle(self):
        return self._hd._h

    def _info(self):
        cnt, nl, sc = C.c_uint32(), C.c_uint32(), C.c_double()
        check(lib().ts_ct_info(self.handle, C.byref(cnt), C.byref(nl), C.byref(sc)), "ts_ct_info")
        return cnt.value, nl.value, sc.value

    @property
    def scale(self) -> float:
        return self._info()[2]

    @property
    def num_limbs(self) -> int:
        return self._info()[1]

    def __mul__(self, other):
        # lib.rs:336-356: ct * numpy plaintext (the ZeRo-MOAI hot path)
        return self._ctx.ct_pt_mul(self, other)

    def __add__(self, other: "TenSafeCiphertext"):
        return self._ctx.ct_add(self, other)

    def __sub__(self, other: "TenSafeCiphertext"):
        return self._ctx.ct_sub(self, other)

    def export(self, index: int = 0):
        """(c0, c1) residues, each [num_limbs, N] uint64 (tests / wire format)."""
        _, nl, _ = self._info()
        n = self._ctx._n
        c0 = np.zeros(nl * n, np.uint64)
        c1 = np.zeros(nl * n, np.uint64)
        check(lib().ts_ct_export(self.handle, index, ptr(c0, C.c_uint64), ptr(c1, C.c_uint64)), "ts_ct_export")
        return c0.reshape(nl, n), c1.reshape(nl, n)

    def to_bytes(self) -> bytes:
        """serialize.rs:71-77 ct_to_bytes: [scale f64 LE | c0 | c1], limb-major
        u64 LE (ts_ct_to_bytes).  A batch gives its ciphertexts' blobs back to
        back."""
        count, nl, _ = self._info()
        size = count * (8 + 2 * nl * self._ctx._n * 8)
        buf = C.create_string_buffer(size)
        written = C.c_size_t()
        check(lib().ts_ct_to_bytes(self.handle, buf, size, C.byref(written)), "ts_ct_to_bytes")
        return buf.raw[: written.value]


class CkksContext:
    """CKKS context on a B200 (lib.rs:19-295)."""

    def __init__(self, poly_mod_degree: int = 16384, device: int = 0):
        h = C.c_void_p()
        check(lib().ts_ctx_create(int(poly_mod_degree), int(device), C.byref(h)), "ts_ctx_create")
        self._init_from(h, device)

    def _init_from(self, h, device: int = 0):
        self._device = int(device)
        self._hd = _Handle(h, lib().ts_ctx_destroy)
        n, s, L = C.c_uint32(), C.c_uint32(), C.c_uint32()
        mod = np.zeros(16, np.uint64)
        check(lib().ts_ctx_info(h, C.byref(n), C.byref(s), C.byref(L), ptr(mod, C.c_uint64)), "ts_ctx_info")
        self._n, self._slots, self._L = n.value, s.value, L.value
        self._moduli = [int(x) for x in mod[: self._L]]

    @classmethod
    def custom(cls, poly_degree: int, modulus_bits, scale_bits: int = 40, device: int = 0):
        """CkksParams::custom (params.rs:142-162)."""
        bits = np.asarray(modulus_bits, dtype=np.uint32)
        h = C.c_void_p()
        check(lib().ts_ctx_create_custom(int(poly_degree), ptr(bits, C.c_uint32), bits.size, int(scale_bits),
                                         int(device), C.byref(h)), "ts_ctx_create_custom")
        obj = cls.__new__(cls)
        obj._init_from(h, device)
        return obj

    @classmethod
    def from_moduli(cls, poly_degree: int, moduli, device: int = 0):
        m = np.asarray(moduli, dtype=np.uint64)
        h = C.c_void_p()
        check(lib().ts_ctx_create_moduli(int(poly_degree), ptr(m, C.c_uint64), m.size, int(device), C.byref(h)),
              "ts_ctx_create_moduli")
        obj = cls.__new__(cls)
        obj._init_from(h, device)
        return obj

    @staticmethod
    def for_depth(depth: int = 3):
        # lib.rs:62-76
        table = {1: 8192, 2: 16384, 3: 32768, 4: 32768, 5: 32768}
        if depth not in table:
            raise ValueError(f"Unsupported depth: {depth}. Use 1-5.")
        return CkksContext(table[depth])

    @property
    def handle(self):
        return self._hd._h

    @property
    def num_slots(self) -> int:
        return self._slots

    @property
    def poly_mod_degree(self) -> int:
        return self._n

    @property
    def moduli(self):
        return list(self._moduli)

    # -------------------------------------------------------------- keys
    def keygen(self, seed=None) -> TenSafeSecretKey:
        h = C.c_void_p()
        check(lib().ts_keygen(self.handle, _seed(seed), C.byref(h)), "ts_keygen")
        return TenSafeSecretKey(self, h)

    def keygen_batch(self, seeds) -> TenSafeSecretKey:
        s = np.ascontiguousarray(seeds, dtype=np.uint64)
        h = C.c_void_p()
        check(lib().ts_keygen_batch(self.handle, ptr(s, C.c_uint64), s.size, C.byref(h)), "ts_keygen_batch")
        return TenSafeSecretKey(self, h)

    # -------------------------------------------------------------- encrypt
    def keygen_public(self, sk: TenSafeSecretKey, seed=None, sk_index: int = 0) -> TenSafePublicKey:
        """lib.rs:102-110 (ciphertext.rs:114-154): pk = (-a*s + e, a)."""
        h = C.c_void_p()
        check(lib().ts_keygen_public(self.handle, sk.handle, int(sk_index), _seed(seed), C.byref(h)),
              "ts_keygen_public")
        return TenSafePublicKey(self, h)

    def encrypt_pk(self, data, pk: TenSafePublicKey, seed=None) -> TenSafeCiphertext:
        """lib.rs:142-164 (ciphertext.rs:240-319); pads / truncates to num_slots."""
        return self.encrypt_pk_batch(np.atleast_2d(_f64(data)[: self._slots]), pk, [_seed(seed)])

    def encrypt_pk_batch(self, data, pk: TenSafePublicKey, seeds) -> TenSafeCiphertext:
        """Public-key encryption of each row with its own seed (B200 batch API)."""
        x = np.ascontiguousarray(np.atleast_2d(np.asarray(data, dtype=np.float64)))
        s = np.ascontiguousarray(seeds, dtype=np.uint64)
        if s.size != x.shape[0]:
            raise ValueError("one seed per row required")
        h = C.c_void_p()
        check(lib().ts_encrypt_pk(self.handle, pk.handle, x.ctypes.data if x.size else None, x.shape[0], x.shape[1],
                                  x.shape[1], ptr(s, C.c_uint64), 0, C.byref(h)), "ts_encrypt_pk")
        return TenSafeCiphertext(self, h)

    def rescale(self, ct: "TenSafeCiphertext") -> "TenSafeCiphertext":
        """lib.rs:218-225 (ciphertext.rs:476-535): drop the last limb, scale / q_last.
        ValueError with one limb (the reference panics)."""
        h = C.c_void_p()
        check(lib().ts_rescale(self.handle, ct.handle, C.byref(h)), "ts_rescale")
        return TenSafeCiphertext(self, h)

    def encrypt(self, data, sk: TenSafeSecretKey, seed=None) -> TenSafeCiphertext:
        x = _f64(data)
        h = C.c_void_p()
        check(lib().ts_encrypt(self.handle, sk.handle, ptr(x, C.c_double), x.size, _seed(seed), C.byref(h)),
              "ts_encrypt")
        return TenSafeCiphertext(self, h)

    def encrypt_batch(self, data, sk: TenSafeSecretKey, seeds, sk_index=None) -> TenSafeCiphertext:
        """Independent streams per row (B200 batch API)."""
        x = np.ascontiguousarray(np.atleast_2d(np.asarray(data, dtype=np.float64)))
        s = np.ascontiguousarray(seeds, dtype=np.uint64)
        if s.size != x.shape[0]:
            raise ValueError("one seed per row required")
        ski = None if sk_index is None else np.ascontiguousarray(sk_index, dtype=np.int32)
        h = C.c_void_p()
        check(lib().ts_encrypt_batch(self.handle, sk.handle, x.ctypes.data, x.shape[0], x.shape[1], x.shape[1],
                                     ptr(s, C.c_uint64), ptr(ski, C.c_int32), 0, C.byref(h)), "ts_encrypt_batch")
        return TenSafeCiphertext(self, h)

    def batch_encrypt(self, arrays, sk: TenSafeSecretKey, seed=None):
        """lib.rs:231-258: one RNG shared by all arrays, in order."""
        if not arrays:
            return []
        rows = [_f64(a)[: self._slots] for a in arrays]
        width = max(1, max(r.size for r in rows))
        x = np.zeros((len(rows), width))
        for i, r in enumerate(rows):
            x[i, : r.size] = r
        h = C.c_void_p()
        check(lib().ts_encrypt_stream(self.handle, sk.handle, ptr(x, C.c_double), x.shape[0], width, width,
                                      _seed(seed), C.byref(h)), "ts_encrypt_stream")
        batch = TenSafeCiphertext(self, h)
        return [self._select(batch, i) for i in range(len(rows))]

    def _select(self, ct: TenSafeCiphertext, i: int) -> TenSafeCiphertext:
        h = C.c_void_p()
        check(lib().ts_ct_select(self.handle, ct.handle, i, C.byref(h)), "ts_ct_select")
        return TenSafeCiphertext(self, h)

    # -------------------------------------------------------------- decrypt
    def decrypt(self, ct: TenSafeCiphertext, sk: TenSafeSecretKey) -> np.ndarray:
        cnt, _, _ = ct._info()
        out = np.zeros(cnt * self._slots)
        check(lib().ts_decrypt(self.handle, ct.handle, sk.handle, None, out.ctypes.data, 0), "ts_decrypt")
        return out if cnt == 1 else out.reshape(cnt, self._slots)

    def decrypt_to_device(self, ct: TenSafeCiphertext, sk: TenSafeSecretKey):
        """Decrypt into a CUDA tensor (float64 [slots] or [count, slots]) -- the
        engine's ``decrypt_to_gpu`` (inference_engine.py:190-205)."""
        import torch

        cnt, _, _ = ct._info()
        out = torch.empty(cnt * self._slots, dtype=torch.float64, device=f"cuda:{self._device}")
        # ts_decrypt returns after its stream has finished writing `out`
        torch.cuda.current_stream(self._device).synchronize()
        check(lib().ts_decrypt(self.handle, ct.handle, sk.handle, None, out.data_ptr(), 1), "ts_decrypt")
        return out if cnt == 1 else out.view(cnt, self._slots)

    def batch_decrypt(self, cts, sk: TenSafeSecretKey):
        return [self.decrypt(ct, sk) for ct in cts]

    @property
    def device(self) -> int:
        return self._device

    # -------------------------------------------------------------- ct x pt
    def ct_pt_mul(self, ct: TenSafeCiphertext, plaintext) -> TenSafeCiphertext:
        p = _f64(plaintext)
        h = C.c_void_p()
        check(lib().ts_ct_pt_mul(self.handle, ct.handle, ptr(p, C.c_double), p.size, C.byref(h)), "ts_ct_pt_mul")
        return TenSafeCiphertext(self, h)

    def encode_to_ntt(self, plaintexts) -> "NttPlaintext":
        x = np.ascontiguousarray(np.atleast_2d(np.asarray(plaintexts, dtype=np.float64)))
        h = C.c_void_p()
        check(lib().ts_encode_ntt(self.handle, x.ctypes.data, x.shape[0], x.shape[1], x.shape[1], 0, C.byref(h)),
              "ts_encode_ntt")
        return NttPlaintext(self, h, x.shape[0])

    def ct_pt_mul_ntt(self, ct: TenSafeCiphertext, pt: "NttPlaintext", index: int = 0) -> TenSafeCiphertext:
        h = C.c_void_p()
        check(lib().ts_ct_pt_mul_ntt(self.handle, ct.handle, pt.handle, index, C.byref(h)), "ts_ct_pt_mul_ntt")
        return TenSafeCiphertext(self, h)

    def ct_add(self, a: TenSafeCiphertext, b: TenSafeCiphertext) -> TenSafeCiphertext:
        h = C.c_void_p()
        check(lib().ts_ct_add(self.handle, a.handle, b.handle, C.byref(h)), "ts_ct_add")
        return TenSafeCiphertext(self, h)

    def ct_sub(self, a: TenSafeCiphertext, b: TenSafeCiphertext) -> TenSafeCiphertext:
        h = C.c_void_p()
        check(lib().ts_ct_sub(self.handle, a.handle, b.handle, C.byref(h)), "ts_ct_sub")
        return TenSafeCiphertext(self, h)

    def import_ciphertext(self, c0, c1, scale: float) -> TenSafeCiphertext:
        c0 = np.ascontiguousarray(c0, dtype=np.uint64)
        c1 = np.ascontiguousarray(c1, dtype=np.uint64)
        nl = c0.size // self._n
        h = C.c_void_p()
        check(lib().ts_ct_import(self.handle, ptr(c0, C.c_uint64), ptr(c1, C.c_uint64), nl, float(scale),
                                 C.byref(h)), "ts_ct_import")
        return TenSafeCiphertext(self, h)

    def ciphertext_from_bytes(self, blob: bytes, num_limbs: int = None) -> TenSafeCiphertext:
        """serialize.rs:80-93 ct_from_bytes (ts_ct_from_bytes); the length is
        checked like the reference's assert_eq!.  num_limbs defaults to what
        the length of one blob implies (the reference passes it explicitly)."""
        blob = bytes(blob)
        if num_limbs is None:
            # the largest limb count whose blob size divides the length (one
            # blob, or several back to back)
            fits = [nl for nl in range(self._L, 0, -1) if len(blob) % (8 + 2 * nl * self._n * 8) == 0]
            if not blob or not fits:
                raise ValueError(f"Expected 8 + 2*L*{self._n * 8} bytes for Ciphertext, got {len(blob)}")
            num_limbs = fits[0]
        h = C.c_void_p()
        check(lib().ts_ct_from_bytes(self.handle, blob, len(blob), int(num_limbs), C.byref(h)), "ts_ct_from_bytes")
        return TenSafeCiphertext(self, h)

    def public_key_from_bytes(self, blob: bytes) -> "TenSafePublicKey":
        """serialize.rs:55-67 pk_from_bytes (ts_pk_from_bytes)."""
        blob = bytes(blob)
        h = C.c_void_p()
        check(lib().ts_pk_from_bytes(self.handle, blob, len(blob), C.byref(h)), "ts_pk_from_bytes")
        return TenSafePublicKey(self, h)

    # -------------------------------------------------------------- info
    @staticmethod
    def is_available() -> bool:
        return is_available()

    def get_backend_info(self) -> dict:
        # lib.rs:282-294
        return {
            "backend": "tensafe-he-b200",
            "version": VERSION,
            "language": "CUDA (sm_100a) + C ABI",
            "gpu_accelerated": True,
            "poly_mod_degree": self._n,
            "num_slots": self._slots,
            "num_limbs": self._L,
        }

    def stats(self) -> dict:
        out = np.zeros(4, np.uint64)
        check(lib().ts_ctx_stats(self.handle, ptr(out, C.c_uint64)), "ts_ctx_stats")
        return {"near_tie_samples": int(out[0]), "streams_repaired": int(out[1]), "plan_overflow": int(out[2])}

    def synchronize(self):
        check(lib().ts_ctx_synchronize(self.handle), "ts_ctx_synchronize")


class NttPlaintext:
    """Cached NTT(plaintext) rows on the device (ciphertext.rs:539-545)."""

    def __init__(self, ctx: CkksContext, h, count: int):
        self._ctx = ctx
        self.count = count
        self._hd = _Handle(h, lib().ts_pt_destroy, ctx)

    @property
    def handle(self):
        return self._hd._h

    def export(self, index: int = 0) -> np.ndarray:
        out = np.zeros(self._ctx._L * self._ctx._n, np.uint64)
        check(lib().ts_pt_export(self.handle, index, ptr(out, C.c_uint64)), "ts_pt_export")
        return out.reshape(self._ctx._L, self._ctx._n)
