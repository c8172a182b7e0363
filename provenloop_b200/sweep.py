"""C5: encode / encrypt / ct x pt / decrypt / decode throughput sweep of the
ZeRo-MOAI delta path over ring degree, batch, hidden size and LoRA rank.

    python -m provenloop_b200.sweep [--steps 3] [--warmup 3] [--quick]

Grid (seed 4): N in {8192, 16384, 32768} (the preset 4-prime chains,
params.rs:66-162), batch in {1, 16, 256, 4096} hidden states, d in
{1536, 3584} (x ~ N(0, 1)), r in {8, 16, 32, 64} (A, B ~ N(0, 0.02^2)).
cols = floor(N / 2 / d) copies of x per ciphertext and ceil(r / cols)
plaintext batches (inference_engine.py:1244-1272).  Each point times whole
delta steps (encrypt -> ct x pt -> batched decrypt -> segment sums -> B
product) on device-resident inputs with CUDA events, L2 flushed between
steps, then repeats the steps with every launch event-timed to give each
kernel's time and its algorithmic bytes / time as a fraction of the measured
HBM copy bandwidth.  Under torchrun every rank runs the grid on its own users
(weak scaling); times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

NS = (8192, 16384, 32768)
BATCHES = (1, 16, 256, 4096)
DS = (1536, 3584)
RS = (8, 16, 32, 64)

KERNELS = ("encode", "encode_a", "encode_b", "gauss_gen", "enc_fused", "enc_a", "enc_u", "enc_x", "enc_combine", "plan",
           "gauss_fix", "enc_a_fix", "enc_u_fix", "dec_limb1", "dec_fused", "decrypt_limb", "crt_seg", "decode_a", "decode_b",
           "gather_inter", "bmat")


def kernel_bytes_per_delta(name: str, n: int, L: int, nb: int, cols: int, d: int, r: int) -> float:
    """Algorithmic bytes one delta moves through kernel `name`: its compulsory
    reads and writes, shared tables (keys, plaintexts, twiddles) counted once
    per delta as the per-delta traffic model does.

    encode        h in (8d); m (8N) out (the error e comes from gauss_gen)
    encode_a/b    the two-kernel encode: 16N (+8d) and 25N
    gauss_gen     e out (N)
    enc_a         c1 out (8NL)
    enc_u         per limb: m, e, s, c1 in, c0 out (33N)
    enc_fused     per limb: m, e, s in, c1 and c0 out (33N; N = 8192, 16384)
    enc_x         per limb: m, e in, c0 out (17N)
    enc_combine   per limb: c0, c1, s in, c0 out (32N)
    dec_limb1     (N >= 8192) ct limbs 0-1 and s limbs 0-1 in, the u
                  rows of limbs 0-1 out, NTT(pt) limb 1 per batch in, limb 1's
                  INTT per batch out: 8N(8 + 2B)
    dec_fused     N >= 8192 (k_dec_pair): limb 0's u row, NTT(pt) limb 0
                  and limb 1's INTT per batch in, segment sums out:
                  8N(1 + 2B) + 8B*cols; other N (k_dec_fused): ct limbs 0-1,
                  s limbs 0-1, NTT(pt) limbs 0-1 per batch in, segment sums
                  out: 8N(6 + 2B) + 8B*cols
    decrypt_limb  per (batch, limb 0/1): c0, c1, s, pt in, INTT out (40N)
    crt_seg       per batch: both INTT limbs in (16N)
    decode_a/b    per batch: 32N and 16N
    gather_inter  segment sums in, intermediate out
    bmat          intermediate in, delta out (8r + 8d)
    """
    table = {
        "encode": 8 * n + 8 * d,
        "encode_a": 16 * n + 8 * d,
        "encode_b": 25 * n,
        "gauss_gen": n,
        "enc_a": 8 * n * L,
        "enc_u": 33 * n * L,
        "enc_fused": 33 * n * L,
        "enc_x": 17 * n * L,
        "enc_combine": 32 * n * L,
        "dec_limb1": 8 * n * (8 + 2 * nb),
        "dec_fused": (8 * n * (1 + 2 * nb) if n >= 8192 else 8 * n * (6 + 2 * nb)) + 8 * nb * cols,
        "decrypt_limb": 80 * n * nb,
        "crt_seg": 16 * n * nb,
        "decode_a": 32 * n * nb,
        "decode_b": 16 * n * nb,
        "gather_inter": 8 * nb * cols + 8 * r,
        "bmat": 8 * r + 8 * d,
    }
    return float(table.get(name, 0))


def grid(quick: bool = False):
    if quick:
        return [(16384, b, 1536, 16) for b in (1, 256)]
    return [(n, b, d, r) for n in NS for d in DS for r in RS for b in BATCHES]


def run(steps: int = 3, warmup: int = 3, points=None, peak_gbs: float = 6650.0, device: int | None = None):
    """Runs the grid; returns the list of per-point dicts (on every rank)."""
    import torch
    import torch.distributed as dist

    from . import _lib, multigpu, tensafe_he
    from .backend import ZeroMoaiLora

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    local = device if device is not None else int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    points = points if points is not None else grid()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    out = []
    for n in sorted({p[0] for p in points}):
        ctx = tensafe_he.CkksContext(n, device=local)
        _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "ts_ctx_set_stream")
        L = 4
        with torch.cuda.stream(stream):
            sk = ctx.keygen(4)
            for (_, batch, d, r) in [p for p in points if p[0] == n]:
                cols = (n // 2) // d
                nb = -(-r // cols)
                rng = np.random.default_rng(4)
                A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
                B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
                H = np.random.default_rng(4000 + rank).standard_normal((batch, d))
                lora = ZeroMoaiLora(ctx, A, B)
                h_dev = torch.from_numpy(H).to(dev)
                delta_dev = torch.empty((batch, d), dtype=torch.float64, device=dev)
                users = np.arange(rank * batch, (rank + 1) * batch, dtype=np.uint64)

                def step(i):
                    seeds = multigpu.stream_seeds(users, i, world * batch)
                    lora.delta_device(sk, h_dev, seeds, delta_dev)

                for i in range(warmup):
                    step(i)
                stream.synchronize()
                if world > 1:
                    dist.barrier()
                ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                      for _ in range(steps)]
                for k in range(steps):
                    flush.zero_()
                    ev[k][0].record(stream)
                    step(warmup + k)
                    ev[k][1].record(stream)
                stream.synchronize()
                t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
                _lib.profile_reset()
                _lib.profile_enable(True)
                for k in range(steps):
                    flush.zero_()
                    step(warmup + steps + k)
                stream.synchronize()
                _lib.profile_enable(False)
                kern = {}
                for name in KERNELS:
                    ms, cnt = _lib.profile_read(name)
                    if cnt:
                        by = kernel_bytes_per_delta(name, n, L, nb, cols, d, r) * batch
                        gbs = by * steps / (ms / 1e3) / 1e9 if ms > 0 else 0.0
                        kern[name] = {"ms_per_step": ms / steps, "gbs": gbs, "hbm_frac": gbs / peak_gbs}
                if world > 1:
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item()) / steps
                out.append({"n": n, "batch": batch, "d": d, "r": r, "cols": cols, "pt_batches": nb,
                            "ms_per_step": ms, "deltas_per_s": world * batch / (ms / 1e3), "kernels": kern})
                del lora, h_dev, delta_dev
        del sk
        stream.synchronize()
        del ctx
        torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--quick", action="store_true", help="two points only (a smoke run of the sweep)")
    a = ap.parse_args()
    pts = run(a.steps, a.warmup, grid(a.quick))
    for p in pts:
        print(json.dumps(p))


if __name__ == "__main__":
    main()
