"""Engine-facing side of the B200 CKKS backend.

* ``TenSafeB200Adapter`` -- the duck-typed backend the inference engine calls
  (``encrypt_vector``, ``ct * pt``, ``decrypt_vector``, ``decrypt_to_gpu``,
  ``status``), same surface and metrics schema as ``_TenSafeHEAdapter``
  (demonstrator/server/inference_engine.py:148-220).
* ``ZeroMoaiLora`` -- device-resident ZeRo-MOAI LoRA adapters for one or more
  CryptoMOE experts, computing whole batches of encrypted deltas in one call
  (inference_engine.py:1197-1405, plaintext cache :1037-1074).
* ``dp_sigma`` / ``add_dp_noise`` -- post-transformer Gaussian-mechanism noise
  (inference_engine.py:792-798, :1411-1465) on the device.
* ``route_expert`` -- the keyword step-gate (inference_engine.py:1155-1171).
"""
from __future__ import annotations

import ctypes as C
import math
import time

import numpy as np

from . import tensafe_he
from ._lib import check, lib, ptr


class TenSafeB200Adapter:
    """Drop-in for ``_TenSafeHEAdapter`` backed by libtsgpu.so."""

    def __init__(self, ctx: "tensafe_he.CkksContext", sk: "tensafe_he.TenSafeSecretKey"):
        self._ctx = ctx
        self._sk = sk
        self._slots = ctx.num_slots
        self._metrics = {
            "total_encryptions": 0,
            "total_decryptions": 0,
            "total_encrypt_ms": 0.0,
            "total_decrypt_ms": 0.0,
        }

    def encrypt_vector(self, data: np.ndarray):
        # inference_engine.py:166-176 -- pad / truncate to the slot count
        self._metrics["total_encryptions"] += 1
        t0 = time.perf_counter()
        padded = np.zeros(self._slots, dtype=np.float64)
        flat = np.asarray(data).flatten().astype(np.float64)
        n = min(len(flat), self._slots)
        padded[:n] = flat[:n]
        ct = self._ctx.encrypt(padded, self._sk)
        self._metrics["total_encrypt_ms"] += (time.perf_counter() - t0) * 1000
        return ct

    def decrypt_vector(self, ct) -> np.ndarray:
        self._metrics["total_decryptions"] += 1
        t0 = time.perf_counter()
        result = np.asarray(self._ctx.decrypt(ct, self._sk), dtype=np.float64)
        self._metrics["total_decrypt_ms"] += (time.perf_counter() - t0) * 1000
        return result

    def decrypt_to_gpu(self, ct):
        """Decrypt into a CUDA float64 tensor; the engine then stacks all
        batches and makes one host transfer (inference_engine.py:1328-1377)."""
        self._metrics["total_decryptions"] += 1
        t0 = time.perf_counter()
        result = self._ctx.decrypt_to_device(ct, self._sk)
        self._metrics["total_decrypt_ms"] += (time.perf_counter() - t0) * 1000
        return result

    def status(self) -> dict:
        info = self._ctx.get_backend_info()
        return {
            "backend": info["backend"],
            "version": info["version"],
            "initialized": True,
            "gpu_available": True,
            "gpu_enabled": True,
            "gpu_accelerated": True,
            "gpu_device": self._ctx.device,
            "poly_mod_degree": self._slots * 2,
            "emulated": False,
            "metrics": dict(self._metrics),
        }


class ZeroMoaiLora:
    """Packed LoRA plaintexts of ``experts`` adapters cached as NTT residues on
    the device, plus their B matrices.

    lora_a: [experts, r, d] (or [r, d]); lora_b: [experts, d, r] (or [d, r]).
    """

    def __init__(self, ctx: "tensafe_he.CkksContext", lora_a, lora_b):
        A = np.asarray(lora_a, dtype=np.float32)
        B = np.asarray(lora_b, dtype=np.float32)
        if A.ndim == 2:
            A = A[None]
        if B.ndim == 2:
            B = B[None]
        if A.shape[0] != B.shape[0] or A.shape[1] != B.shape[2] or A.shape[2] != B.shape[1]:
            raise ValueError(f"LoRA shapes do not match: A {A.shape}, B {B.shape}")
        self._ctx = ctx
        self.experts, self.r, self.d = (int(x) for x in A.shape)
        A = np.ascontiguousarray(A)
        B = np.ascontiguousarray(B)
        h = C.c_void_p()
        check(lib().ts_lora_load(ctx.handle, ptr(A, C.c_float), ptr(B, C.c_float), self.experts, self.r, self.d,
                                 C.byref(h)), "ts_lora_load")
        self._hd = tensafe_he._Handle(h, lib().ts_lora_destroy, ctx)
        cols, nb = C.c_uint32(), C.c_uint32()
        check(lib().ts_lora_info(h, None, None, None, C.byref(cols), C.byref(nb)), "ts_lora_info")
        self.cols, self.batches = cols.value, nb.value

    @property
    def handle(self):
        return self._hd._h

    def set_expert(self, expert: int, lora_a, lora_b):
        """Hot-swap one expert's adapter in place (swap_adapter,
        inference_engine.py:879-959): A [r, d], B [d, r] with this object's r
        and d.  Device pointers stay the same, so a captured decode-step graph
        uses the new adapter on its next replay."""
        A = np.ascontiguousarray(np.asarray(lora_a, dtype=np.float32))
        B = np.ascontiguousarray(np.asarray(lora_b, dtype=np.float32))
        if A.shape != (self.r, self.d) or B.shape != (self.d, self.r):
            raise ValueError(f"expected A {(self.r, self.d)} and B {(self.d, self.r)}, got {A.shape} and {B.shape}")
        check(lib().ts_lora_set_expert(self._ctx.handle, self.handle, int(expert), ptr(A, C.c_float),
                                       ptr(B, C.c_float)), "ts_lora_set_expert")

    def delta(self, sk, h, seeds, expert=None, sk_index=None, out=None, out_inter=None, want_inter=True):
        """Encrypted deltas for hidden states h [n, d] (host arrays).

        ``out`` / ``out_inter`` may be preallocated (e.g. pinned) float64
        arrays.  Returns (delta [n, d] f64, intermediate [n, r] f64 or None)."""
        H = np.ascontiguousarray(np.atleast_2d(np.asarray(h, dtype=np.float64)))
        n = H.shape[0]
        if H.shape[1] != self.d:
            raise ValueError(f"hidden size {H.shape[1]} != adapter d {self.d}")
        s = np.ascontiguousarray(np.broadcast_to(np.asarray(seeds, dtype=np.uint64), (n,)))
        ex = None if expert is None else np.ascontiguousarray(np.broadcast_to(np.asarray(expert, np.int32), (n,)))
        ski = None if sk_index is None else np.ascontiguousarray(np.broadcast_to(np.asarray(sk_index, np.int32), (n,)))
        delta = np.zeros((n, self.d)) if out is None else out
        if delta.shape != (n, self.d) or delta.dtype != np.float64 or not delta.flags.c_contiguous:
            raise ValueError("out must be a C-contiguous float64 array of shape (n, d)")
        inter = None
        if want_inter or out_inter is not None:
            inter = np.zeros((n, self.r)) if out_inter is None else out_inter
        check(lib().ts_lora_delta_batch(self._ctx.handle, sk.handle, self.handle, H.ctypes.data, n,
                                        ptr(ex, C.c_int32), ptr(ski, C.c_int32), ptr(s, C.c_uint64),
                                        delta.ctypes.data, None if inter is None else inter.ctypes.data, 0),
              "ts_lora_delta_batch")
        return delta, inter

    def delta_device(self, sk, h_dev, seeds, delta_dev, expert=None, sk_index=None, inter_dev=None):
        """Same, with h / delta (/ intermediate) as CUDA tensors (float64,
        contiguous).  Completes on the context's stream; call
        ``ctx.synchronize()`` (or order streams) before reading delta."""
        n = int(h_dev.shape[0])
        s = np.ascontiguousarray(np.broadcast_to(np.asarray(seeds, dtype=np.uint64), (n,)))
        ex = None if expert is None else np.ascontiguousarray(np.broadcast_to(np.asarray(expert, np.int32), (n,)))
        ski = None if sk_index is None else np.ascontiguousarray(np.broadcast_to(np.asarray(sk_index, np.int32), (n,)))
        check(lib().ts_lora_delta_batch(self._ctx.handle, sk.handle, self.handle, h_dev.data_ptr(), n,
                                        ptr(ex, C.c_int32), ptr(ski, C.c_int32), ptr(s, C.c_uint64),
                                        delta_dev.data_ptr(), None if inter_dev is None else inter_dev.data_ptr(),
                                        1), "ts_lora_delta_batch")


def _dptr(t, ctype=None):
    if t is None:
        return None
    return t.data_ptr() if ctype is None else C.cast(t.data_ptr(), C.POINTER(ctype))


def lora_delta_graphable(lora: "ZeroMoaiLora", sk, h_dev, seeds_dev, delta_dev, expert_dev=None, sk_index_dev=None,
                         inter_dev=None):
    """``ZeroMoaiLora.delta_device`` with the seeds (int64 / uint64 CUDA
    tensor) and the optional expert / key indexes (int32 CUDA tensors) on the
    device as well: the call only enqueues work on the context's stream, so
    it can be captured in a CUDA graph after one uncaptured call of the same
    size.  Indexes are not range-checked."""
    n = int(h_dev.shape[0])
    check(lib().ts_lora_delta_batch(lora._ctx.handle, sk.handle, lora.handle, h_dev.data_ptr(), n,
                                    _dptr(expert_dev, C.c_int32), _dptr(sk_index_dev, C.c_int32),
                                    _dptr(seeds_dev, C.c_uint64), delta_dev.data_ptr(), _dptr(inter_dev), 2),
          "ts_lora_delta_batch")


def he_lora_delta(ctx, sk, lora: ZeroMoaiLora, h_plain, seed=None, expert: int = 0):
    """``_he_lora_delta``'s encrypted branch for one hidden state
    (inference_engine.py:1244-1392).  Returns (delta, compute_ms, decrypt_ms,
    ops) with the reference's op count (1 encrypt + r ct x pt rows + B
    segment-sum passes)."""
    t0 = time.perf_counter()
    seed = tensafe_he._seed(seed)
    delta, _ = lora.delta(sk, np.asarray(h_plain, dtype=np.float64)[: lora.d], [seed], expert=[expert])
    ms = (time.perf_counter() - t0) * 1000
    ops = 1 + lora.r + lora.batches
    return delta[0], ms, 0.0, ops


def dp_sigma(epsilon: float = 1.0, delta: float = 1e-5, sensitivity: float = 1.0) -> float:
    """Gaussian mechanism sigma = sensitivity * sqrt(2 ln(1.25/delta)) / epsilon
    (inference_engine.py:792-798)."""
    return sensitivity * math.sqrt(2 * math.log(1.25 / delta)) / epsilon


def add_dp_noise(ctx, hidden, sigma: float, seeds, clip: float = 1.0):
    """Clip each row of ``hidden`` [n, d] to L2 norm <= clip and add
    N(0, sigma^2) noise on the device (inference_engine.py:1436-1456).  The
    noise comes from the ChaCha20 stream of each row's seed (Box-Muller,
    rng.rs:152-157) instead of numpy's global generator, so it is
    reproducible per seed."""
    H = np.ascontiguousarray(np.atleast_2d(np.asarray(hidden, dtype=np.float64))).copy()
    n, d = H.shape
    s = np.ascontiguousarray(np.broadcast_to(np.asarray(seeds, dtype=np.uint64), (n,)))
    check(lib().ts_dp_noise(ctx.handle, H.ctypes.data, n, d, float(clip), float(sigma), ptr(s, C.c_uint64), 0),
          "ts_dp_noise")
    return H


def route_expert(query: str, experts: dict, default: str = "shared_attention") -> str:
    """Keyword step-gate over non-always-active experts
    (inference_engine.py:1155-1171)."""
    q = query.lower()
    best, best_score = default, 0
    for name, adp in experts.items():
        if adp.get("always_active"):
            continue
        score = sum(1 for kw in adp.get("gate_keywords", []) if kw in q)
        if score > best_score:
            best, best_score = name, score
    if best not in experts and experts:
        return next(iter(experts))
    return best
