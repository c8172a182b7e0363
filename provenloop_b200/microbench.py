"""Microbenchmarks of single kernels through the C ABI (also the small cases
used for ncu captures).

    python -m provenloop_b200.microbench ntt [--polys 1024] [--reps 10]
    python -m provenloop_b200.microbench hadamard [--polys 1024] [--reps 4]
    python -m provenloop_b200.microbench delta [--batch 256] [--reps 3]
    python -m provenloop_b200.microbench latency [--batch 1] [--reps 50]
    python -m provenloop_b200.microbench kernels

`ntt` is the C2 configuration: `polys` polynomials x 3 limbs x N = 16384 with
the three largest distinct 50-bit primes == 1 mod 2N, forward then inverse
negacyclic NTT (checked to round-trip), timed with CUDA events on the
library's stream.  Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

N_POLY = 16384
C2_PRIMES = [1125899904679937, 1125899903991809, 1125899903827969]


def _ctx(moduli=None, device=0):
    import torch

    from . import _lib, tensafe_he

    ctx = (tensafe_he.CkksContext(N_POLY, device=device) if moduli is None
           else tensafe_he.CkksContext.from_moduli(N_POLY, moduli, device=device))
    stream = torch.cuda.Stream(device=device)
    _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "ts_ctx_set_stream")
    return ctx, stream


def _polys(P, dev, seed=1):
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = torch.tensor(C2_PRIMES, dtype=torch.int64, device=dev).view(1, 3, 1)
    return (torch.randint(0, 1 << 62, (P, 3, N_POLY), device=dev, generator=g) % q).contiguous()


def ntt(polys=1024, reps=10, device=0, peak_gbs=None):
    import torch

    from . import _lib

    dev = torch.device("cuda", device)
    ctx, stream = _ctx(C2_PRIMES, device)
    L = _lib.lib()
    with torch.cuda.stream(stream):
        x = _polys(polys, dev)
        ref = x.clone()
        for _ in range(2):
            _lib.check(L.ts_ntt_forward(ctx.handle, x.data_ptr(), polys, 3, 0))
            _lib.check(L.ts_ntt_inverse(ctx.handle, x.data_ptr(), polys, 3, 0))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        fw = iv = 0.0
        for _ in range(reps):
            ev[0].record(stream)
            _lib.check(L.ts_ntt_forward(ctx.handle, x.data_ptr(), polys, 3, 0))
            ev[1].record(stream)
            _lib.check(L.ts_ntt_inverse(ctx.handle, x.data_ptr(), polys, 3, 0))
            ev[2].record(stream)
            stream.synchronize()
            fw += ev[0].elapsed_time(ev[1])
            iv += ev[1].elapsed_time(ev[2])
        ok = bool(torch.equal(x, ref))
    byt = polys * 3 * N_POLY * 16  # one read + one write of every 8-byte word
    out = {"kernel": "ntt", "polys": polys, "limbs": 3, "n": N_POLY, "roundtrip_bit_exact": ok,
           "forward_ms": fw / reps, "inverse_ms": iv / reps,
           "forward_gbs": byt / (fw / reps / 1e3) / 1e9, "inverse_gbs": byt / (iv / reps / 1e3) / 1e9,
           "bytes_per_direction": byt,
           "butterflies_per_s_forward": polys * 3 * (N_POLY // 2) * 14 / (fw / reps / 1e3)}
    if peak_gbs:
        out["forward_frac"] = out["forward_gbs"] / peak_gbs
        out["inverse_frac"] = out["inverse_gbs"] / peak_gbs
    return out


def hadamard(polys=1024, reps=4, device=0, peak_gbs=None):
    import torch

    from . import _lib

    dev = torch.device("cuda", device)
    ctx, stream = _ctx(C2_PRIMES, device)
    L = _lib.lib()
    with torch.cuda.stream(stream):
        a = _polys(polys, dev, 1)
        b = _polys(polys, dev, 2)
        out = torch.empty_like(a)
        for _ in range(2):
            _lib.check(L.ts_hadamard(ctx.handle, out.data_ptr(), a.data_ptr(), b.data_ptr(), polys, 3, 0))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        for _ in range(reps):
            _lib.check(L.ts_hadamard(ctx.handle, out.data_ptr(), a.data_ptr(), b.data_ptr(), polys, 3, 0))
        ev[1].record(stream)
        stream.synchronize()
        ms = ev[0].elapsed_time(ev[1])
        qa = torch.tensor(C2_PRIMES, dtype=torch.int64, device=dev).view(1, 3, 1)
        # spot check a slice exactly with Python integers
        aa, bb, oo = (t[0, :, :64].cpu().numpy().astype(object) for t in (a, b, out))
        ok = all(int(oo[l, i]) == int(aa[l, i]) * int(bb[l, i]) % C2_PRIMES[l] for l in range(3) for i in range(64))
        del qa
    byt = reps * polys * 3 * N_POLY * 24
    o = {"kernel": "hadamard", "products": reps * polys, "limbs": 3, "ms": ms, "gbs": byt / (ms / 1e3) / 1e9,
         "spot_check_exact": ok}
    if peak_gbs:
        o["frac"] = o["gbs"] / peak_gbs
    return o


def delta(batch=256, reps=3, device=0, c4=False):
    """The delta pipeline on `batch` hidden states: C1 (N = 16384, r = 16), or
    with c4 the C4 chain (N = 32768, [60, 40, 40, 40, 60], r = 32) on one key."""
    import torch

    from . import _lib, tensafe_he
    from .backend import ZeroMoaiLora

    dev = torch.device("cuda", device)
    if c4:
        ctx = tensafe_he.CkksContext.custom(32768, [60, 40, 40, 40, 60], device=device)
        stream = torch.cuda.Stream(device=device)
        _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "ts_ctx_set_stream")
    else:
        ctx, stream = _ctx(None, device)
    r = 32 if c4 else 16
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((r, 1536)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((1536, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((batch, 1536))
    with torch.cuda.stream(stream):
        sk = ctx.keygen(0)
        lora = ZeroMoaiLora(ctx, A, B)
        h = torch.from_numpy(H).to(dev)
        d = torch.empty_like(h)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        lora.delta_device(sk, h, np.arange(batch, dtype=np.uint64), d)
        ev[0].record(stream)
        for i in range(reps):
            lora.delta_device(sk, h, np.arange((i + 1) * batch, (i + 2) * batch, dtype=np.uint64), d)
        ev[1].record(stream)
        stream.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / reps
    return {"kernel": "lora_delta_pipeline", "config": "c4" if c4 else "c1", "batch": batch, "ms_per_batch": ms,
            "deltas_per_s": batch / (ms / 1e3),
            "launches_total": _lib.launch_count()}


def latency(batch=1, reps=50, rank=32, device=0):
    """Latency of one small delta batch (the decode-step case: rank 2r = 32
    stacked q/v rows, 7 plaintext batches, 3 experts), device-resident
    inputs with device seeds: per-call time from CUDA events, and per-kernel
    time from the library's event-bracketed profile."""
    import torch

    from . import _lib
    from .backend import ZeroMoaiLora, lora_delta_graphable

    dev = torch.device("cuda", device)
    ctx, stream = _ctx(None, device)
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((3, rank, 1536)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((3, 1536, rank)) * 0.02).astype(np.float32)
    with torch.cuda.stream(stream):
        sk = ctx.keygen(0)
        lora = ZeroMoaiLora(ctx, A, B)
        h = torch.from_numpy(rng.standard_normal((batch, 1536))).to(dev)
        d = torch.empty_like(h)
        inter = torch.empty((batch, rank), dtype=torch.float64, device=dev)
        seeds = torch.arange(batch, dtype=torch.int64, device=dev)
        ex = torch.ones(batch, dtype=torch.int32, device=dev)
        for _ in range(3):
            lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        stream.synchronize()
        ev[0].record(stream)
        for i in range(reps):
            seeds.add_(batch)
            lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
        ev[1].record(stream)
        stream.synchronize()
        per_call = ev[0].elapsed_time(ev[1]) / reps
        # the same calls replayed from one CUDA graph (the decode step's form)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(8):
                seeds.add_(batch)
                lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
        graph.replay()
        stream.synchronize()
        ev[0].record(stream)
        for i in range(reps):
            graph.replay()
        ev[1].record(stream)
        stream.synchronize()
        per_call_graph = ev[0].elapsed_time(ev[1]) / (reps * 8)
        # cold L2: a 256 MiB write between calls (as a decode step's weight
        # stream evicts the tables between layers), minus the writes alone
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

        def graph_of(with_delta):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(8):
                    flush.fill_(i)
                    if with_delta:
                        seeds.add_(batch)
                        lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
            return g

        cold = []
        for g in (graph_of(True), graph_of(False)):
            g.replay()
            stream.synchronize()
            ev[0].record(stream)
            for i in range(reps):
                g.replay()
            ev[1].record(stream)
            stream.synchronize()
            cold.append(ev[0].elapsed_time(ev[1]) / (reps * 8))
        per_call_cold = cold[0] - cold[1]
        _lib.profile_reset()
        _lib.profile_enable(True)
        for i in range(reps):
            lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
        stream.synchronize()
        _lib.profile_enable(False)
    names = ("prefetch_l2", "gauss_gen", "encode", "enc_fused", "enc_a", "enc_x", "enc_combine", "enc_u", "plan", "gauss_fix",
             "enc_a_fix", "enc_u_fix", "dec_fused", "decrypt_limb", "crt_seg", "gather_inter", "bmat",
             "warm_decrypt_limb", "warm_crt_seg")

    def read():
        out = {}
        for name in names:
            ms, n = _lib.profile_read(name)
            if n:
                out[name] = ms / reps
        return out

    kern = read()
    # the same with L2 flushed before every call
    with torch.cuda.stream(stream):
        _lib.profile_reset()
        _lib.profile_enable(True)
        for i in range(reps):
            flush.fill_(i)
            lora_delta_graphable(lora, sk, h, seeds, d, expert_dev=ex, inter_dev=inter)
        stream.synchronize()
        _lib.profile_enable(False)
    kern_cold = read()
    return {"kernel": "lora_delta_latency", "batch": batch, "rank": rank, "ms_per_call": per_call,
            "graph_ms_per_call": per_call_graph, "graph_cold_l2_ms_per_call": per_call_cold,
            "kernels_ms_per_call": kern, "kernels_cold_l2_ms_per_call": kern_cold}


def kernels(device=0):
    """One call of every path of the library at sizes whose data exceed L2
    where the path allows (the case the per-kernel ncu summary is captured
    on): batched keygen, secret- and public-key encryption, decrypt of fresh
    and ct x pt ciphertexts, rescale, DP noise, the small-batch delta (the
    decode step's latency form), and an N = 32768 delta batch."""
    import torch

    from . import _lib, tensafe_he
    from .backend import ZeroMoaiLora, add_dp_noise, dp_sigma

    rng = np.random.default_rng(0)
    ctx, stream = _ctx(None, device)
    with torch.cuda.stream(stream):
        skb = ctx.keygen_batch(list(range(128)))                     # 128 keys (64 MiB)
        sk = ctx.keygen(7)
        X = rng.standard_normal((128, 8192))
        ct = ctx.encrypt_batch(X, sk, list(range(128)))              # 128 MiB of ciphertexts
        ctx.decrypt(ct, sk)                                          # fresh: limb 0, decode
        prod = ct * rng.standard_normal(8192)                        # encode_to_ntt + Hadamard
        ctx.decrypt(prod, sk)                                        # CRT decode
        ctx.rescale(prod)
        pk = ctx.keygen_public(sk, seed=3)
        ctx.encrypt_pk_batch(X[:64], pk, list(range(64)))
        add_dp_noise(ctx, rng.standard_normal((8192, 1536)), dp_sigma(), list(range(8192)))
        A = (rng.standard_normal((3, 32, 1536)) * 0.02).astype(np.float32)
        B = (rng.standard_normal((3, 1536, 32)) * 0.02).astype(np.float32)
        lora = ZeroMoaiLora(ctx, A, B)
        lora.delta(sk, rng.standard_normal((1, 1536)), [5], expert=[1])   # small-batch form
        c32 = tensafe_he.CkksContext.custom(32768, [60, 40, 40, 40, 60], device=device)
        _lib.check(_lib.lib().ts_ctx_set_stream(c32.handle, stream.cuda_stream), "ts_ctx_set_stream")
        l32 = ZeroMoaiLora(c32, A[0], B[0])
        l32.delta(c32.keygen(3), rng.standard_normal((64, 1536)), list(range(64)))
        stream.synchronize()
    return {"kernel": "all_paths", "launches_total": _lib.launch_count()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["ntt", "hadamard", "delta", "latency", "kernels"])
    ap.add_argument("--polys", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--reps", type=int, default=None)
    ap.add_argument("--c4", action="store_true", help="delta: the C4 chain at N = 32768, rank 32")
    a = ap.parse_args()
    if a.what == "ntt":
        r = ntt(a.polys, a.reps or 10)
    elif a.what == "hadamard":
        r = hadamard(a.polys, a.reps or 4)
    elif a.what == "latency":
        r = latency(a.batch if a.batch != 256 else 1, a.reps or 50)
    elif a.what == "kernels":
        r = kernels()
    else:
        r = delta(a.batch, a.reps or 3, c4=a.c4)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
