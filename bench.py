#!/usr/bin/env python
"""Benchmark: encrypted ZeRo-MOAI LoRA deltas per second on B200.

Workload (C1, batched): CKKS N = 16384 with the reference's 4-prime chain
[60, 40, 40, 60] (params.rs:88-105), scale 2^40, ternary key (seed 0),
hidden size d = 1536, LoRA rank r = 16 (cols = 5 rows per plaintext, 4
plaintext batches), one expert.  A step encrypts `batch` independent hidden
states (5-fold slot replication), multiplies each by the 4 packed LoRA-A
plaintexts, decrypts, segment-sums and applies B -- one call of
ts_lora_delta_batch.  Synthetic data: h ~ N(0,1) (fp32 values), A, B ~
N(0, 0.02^2), numpy default_rng(0); fresh encryption seeds every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank holds `batch` hidden states of its own
users (weak scaling) and rank 0 gathers the decrypted deltas (fp32) over
NCCL; the gather of step k overlaps the compute of step k + 1.  The line
also carries a `c4` object: the multi-user N = 32768 workload (256 users x
56 adapters, a fixed total sharded over the ranks: strong scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # NCCL's init lines name every rank's communicator size; set before torch
    # loads NCCL, which reads these once
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"

_RESULT_FD = None


def quiet_stdout():
    """Points this process's stdout at stderr from here on and keeps the
    original stdout for the result line.  Every rank calls it before the last
    barrier: the lines NCCL prints at teardown then go to stderr, and the JSON
    result stays the last line of stdout."""
    global _RESULT_FD
    import ctypes
    sys.stdout.flush()
    try:
        ctypes.CDLL(None).fflush(None)   # C-level buffers (NCCL's log) first
    except (OSError, AttributeError):
        pass
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def emit(line):
    """Prints the JSON result line on the original stdout."""
    text = json.dumps(line)
    if _RESULT_FD is None:
        print(text, flush=True)
        return
    data = (text + "\n").encode()
    while data:
        data = data[os.write(_RESULT_FD, data):]


N_POLY, D, R = 16384, 1536, 16
METRIC = "encrypted LoRA deltas/sec (CKKS N=16384, d=1536, r=16, ZeRo-MOAI)"
UNIT = "deltas/s"
C2_PRIMES = [1125899904679937, 1125899903991809, 1125899903827969]
C4_USERS, C4_ADAPTERS, C4_R, C4_N = 256, 56, 32, 32768
C4_BITS = [60, 40, 40, 40, 60]
C4_METRIC = "encrypted LoRA deltas/sec (CKKS N=32768, [60,40,40,40,60], r=32, 256 users x 56 adapters)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=2048, help="hidden states per GPU per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-micro", action="store_true", help="skip the NTT / Hadamard microbenchmarks")
    ap.add_argument("--no-c3", action="store_true", help="skip the HE decode-step (Qwen-shaped) measurement")
    ap.add_argument("--no-c4", action="store_true", help="skip the multi-user N=32768 leg of the default line")
    ap.add_argument("--config", default="c1", choices=["c1", "c4", "c5"],
                    help="c1: the headline single-key N=16384 workload; c4: 256 users with their own keys, "
                         "N=32768 on [60,40,40,40,60], 28 layers x 2 projections of rank-32 adapters; c5: the "
                         "sweep over N, batch, d and r (one JSON line with every point)")
    return ap.parse_args()


def inputs(batch: int, rank: int = 0):
    rng = np.random.default_rng(0)
    A = (rng.standard_normal((R, D)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((D, R)) * 0.02).astype(np.float32)
    H = np.random.default_rng(1000 + rank).standard_normal((batch, D)).astype(np.float32).astype(np.float64)
    return H, A, B


def workload(batch, world):
    return {
        "workload": "C1 batched: encrypt -> 4x ct*pt -> batched decrypt -> segment sums -> B matmul per hidden state",
        "poly_degree": N_POLY, "limbs": 4, "moduli_bits": [60, 40, 40, 60], "scale_bits": 40,
        "d": D, "r": R, "cols_per_ct": 5, "pt_batches": 4, "experts": 1,
        "batch_per_gpu": batch, "global_batch": batch * world,
        "l2": "flushed between timed steps (256 MiB write); per-step ciphertext working set >> 126 MB L2",
        "parallelism": ("replicas" if world == 1 else
                        f"users sharded over {world} ranks, NCCL gather of fp32 deltas to rank 0"),
    }


# ----------------------------------------------------------------- helpers
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        j = json.load(open(p))
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons during the timed region.

    nvidia-smi's start-up touches every GPU of the node and stalls work
    running on them for tens of milliseconds (up to 130 ms measured on an
    8-GPU box).  So every rank starts its sampler, and waits for its first
    samples, before the barrier that opens the timed region: no rank's start-up
    then falls inside another rank's timed steps."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self, samples: int = 2):
        """Starts sampling every 100 ms; returns after `samples` samples (or
        5 s), so that the start-up is over before the timed region, and drops
        those samples (taken on an idle GPU)."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()
            while len(self.lines) < samples and time.time() - t0 < 5.0:
                time.sleep(0.02)
            self.lines.clear()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t0 = time.time()
        while not self.lines and time.time() - t0 < 0.3:   # a timed region shorter than the period
            time.sleep(0.01)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ----------------------------------------------------------------- CPU legs
class CpuDeltas:
    """The oracle restatement of tensafe-he-core (the reference's CPU CKKS
    backend) computing C1 deltas on host threads.  mode "cached": cached
    context and NTT(pt), ct_pt_mul_ntt (the fastest CPU form); mode
    "as_invoked": a context rebuilt per ciphertext object and the plaintext
    re-encoded on every `*`, as the PyO3 binding does (lib.rs:322-356).
    The pool persists across steps, so no thread start-up is timed."""

    def __init__(self, threads: int, n_inputs: int = 64):
        from concurrent.futures import ThreadPoolExecutor

        from oracle import oracle as O

        self.threads = threads
        self.H, self.A, self.B = inputs(n_inputs)
        self.octx = O.Ctx(N_POLY)
        self.osk = self.octx.keygen(0)
        self.pc = self.octx.lora_pack(self.A)
        self.pool = ThreadPoolExecutor(max_workers=threads)
        self.next_seed = 10_000

    def one(self, i: int, seed: int, mode: str = "cached", h=None):
        hv = self.H[i % len(self.H)] if h is None else h
        if mode == "as_invoked":
            return self.octx.lora_delta(self.osk, hv, self.A, self.B, enc_seed=seed, mode=1)
        return self.octx.lora_delta(self.osk, hv, self.A, self.B, enc_seed=seed, mode=0, pt_cache=self.pc)

    def run(self, n: int, mode: str = "cached", threads: int | None = None):
        """n deltas on `threads` workers (default all); returns wall seconds."""
        s0 = self.next_seed
        self.next_seed += n
        t0 = time.perf_counter()
        if (threads or self.threads) == 1:
            for i in range(n):
                self.one(i, s0 + i, mode)
        else:
            list(self.pool.map(lambda i: self.one(i, s0 + i, mode), range(n)))
        return time.perf_counter() - t0

    def rate(self, seconds: float, mode: str = "cached", threads: int | None = None):
        """(deltas/s, deltas, wall s) over about `seconds` of work."""
        t = threads or self.threads
        wall = self.run(t, mode, t)                   # calibration round
        n = max(t, int(t / wall * seconds) // t * t)
        wall = self.run(n, mode, t)
        return n / wall, n, wall

    def close(self):
        self.pool.shutdown(wait=True)


def cpu_c3_layer(cd: CpuDeltas, threads: int):
    """Seconds of CKKS work for one decode-step layer of C3 on the CPU
    restatement: one encryption of the layer input (shared by q and v), then
    for q and v each 4 batches of ct x cached NTT(pt) and a decrypt (the B
    product and segment sums are negligible).  With threads > 1 the 8
    products-and-decrypts of the layer run in parallel (the layers
    themselves are sequential)."""
    o, sk = cd.octx, cd.osk
    cols = (N_POLY // 2) // D
    z = np.zeros(N_POLY // 2)
    for i in range(cols):
        z[i * D:(i + 1) * D] = cd.H[0]
    t0 = time.perf_counter()
    c0, c1, scale = o.encrypt(z, sk, seed=cd.next_seed)
    cd.next_seed += 1

    def mul_dec(b):
        p0, p1 = o.ct_pt_mul_ntt(c0, c1, cd.pc[b % len(cd.pc)])
        return o.decrypt(p0, p1, scale * scale, sk)

    if threads == 1:
        for b in range(8):
            mul_dec(b)
    else:
        list(cd.pool.map(mul_dec, range(8)))
    return time.perf_counter() - t0


def oracle_spot_check(rows, seeds, got):
    """The CPU leg's checker: the oracle recomputes the deltas of the given
    hidden-state rows and encryption seeds (cached NTT(pt), as the GPU arm's
    adapter); max-abs error against the GPU deltas, tolerance 1e-4."""
    from oracle import oracle as O

    H, A, B = inputs(1)
    octx = O.Ctx(N_POLY)
    osk = octx.keygen(0)
    pc = octx.lora_pack(A)
    errs = [float(np.abs(octx.lora_delta(osk, h, A, B, enc_seed=int(s), mode=0, pt_cache=pc)[0] - g).max())
            for h, s, g in zip(rows, seeds, got)]
    return {"rows": len(errs), "max_abs_err_vs_oracle": max(errs), "tolerance": 1e-4, "ok": max(errs) < 1e-4}


def cpu_baseline_leg(seconds: float = 10.0, check=None):
    """CPU baseline on the box's host cores (rank 0, N = 1): the oracle
    restatement of tensafe-he-core.  The headline `value` is the all-core
    cached form (the fastest CPU figure); `variants` adds one core, the
    as-invoked form and C3's CKKS-only HE tok/s.  `check` = (H rows, seeds,
    GPU deltas) of the last timed GPU step: the same deltas recomputed here
    and compared (1e-4 max-abs), returned as the parity record."""
    threads = cpu_threads()
    cd = CpuDeltas(threads)
    try:
        parity = oracle_spot_check(*check) if check is not None else None
        rate, n, wall = cd.rate(seconds, "cached")
        r1, n1, w1 = cd.rate(3.0, "cached", 1)
        ra, na, wa = cd.rate(3.0, "as_invoked")
        r1a, n1a, w1a = cd.rate(2.0, "as_invoked", 1)
        cpu_c3_layer(cd, 1)                           # warm
        lay1 = min(cpu_c3_layer(cd, 1) for _ in range(2))
        layt = min(cpu_c3_layer(cd, threads) for _ in range(2))
    finally:
        cd.close()
    base = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} C1 deltas ({wall:.1f} s wall) on {threads} threads of {cpu_model()}; C oracle "
                      "restating tensafe-he-core, cached context and NTT(pt) (its fastest form); the Rust crate "
                      "cannot be built here",
            "variants": {
                "cached_1_core": {"value": r1, "unit": UNIT, "cores": 1, "sample": f"{n1} deltas, {w1:.1f} s"},
                "as_invoked_all_cores": {"value": ra, "unit": UNIT, "cores": threads,
                                         "sample": f"{na} deltas, {wa:.1f} s; context rebuilt per ciphertext "
                                                   "object and plaintext re-encoded per ct*pt (lib.rs:322-356)"},
                "as_invoked_1_core": {"value": r1a, "unit": UNIT, "cores": 1, "sample": f"{n1a} deltas, {w1a:.1f} s"},
                "c3_he_tok_s_1_core": {"value": 1.0 / (28 * lay1), "unit": "HE tok/s", "cores": 1,
                                       "sample": f"one layer = encrypt + 8 x (ct*pt + decrypt) in {lay1 * 1e3:.1f} ms,"
                                                 " x 28 layers; CKKS work only"},
                "c3_he_tok_s_all_cores": {"value": 1.0 / (28 * layt), "unit": "HE tok/s", "cores": threads,
                                          "sample": f"the layer's 8 ct*pt + decrypt in parallel: {layt * 1e3:.1f} ms"},
            }}
    return base, parity


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's CKKS backend
    (cached NTT(pt), all host threads, persistent pool) on the GPU arm's C1
    config.  Each step is a bounded sample of the step's deltas, about 1.5 s
    of CPU work, so that a run of K steps ends in a few minutes."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = cpu_threads()
    cd = CpuDeltas(threads)
    try:
        wall = cd.run(threads)                                          # calibration
        per_s = threads / wall
        step_s = min(1.5, 90.0 / max(args.steps, 1))
        per_step = max(threads, int(per_s * step_s) // threads * threads)
        for _ in range(args.warmup):
            cd.run(threads)
        total_wall = 0.0
        for _ in range(args.steps):
            total_wall += cd.run(per_step)
    finally:
        cd.close()
    value = per_step * args.steps / total_wall
    sample = (f"{per_step} of each step's {args.batch} C1 deltas (about {step_s:.1f} s of CPU work per step) on "
              f"{threads} threads of {cpu_model()}; C restatement of tensafe-he-core with cached NTT(pt) (the "
              "Rust crate cannot be built here)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total_wall / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
        "config": workload(args.batch, 1),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ----------------------------------------------------------------- GPU leg
# Algorithmic HBM bytes per unit of work of each kernel (N = 16384 words of
# 8 bytes per poly-limb):
#   enc_a         per (ct, limb):        write c1 (8N)
#   enc_u         per (ct, limb):        read m (8N) + e (N) + s (8N) + c1 (8N), write c0 (8N) = 33N
#   enc_fused     per (ct, limb):        read m (8N) + e (N) + s (8N), write c1 (8N) + c0 (8N) = 33N
#   decrypt_limb  per (ct, batch, limb): read c0, c1 (16N) + s (8N) + NTT(pt) (8N), write M (8N) = 40N
#   decode_a      per (ct, batch):       read M (2 x 8N), write 16N = 32N
#   decode_b      per (ct, batch):       read 16N
#   encode        per ct (N = 16384, one kernel): read h (d*8), write m (8N) (+ e (N) when fused)
#   gauss_gen     per ct:                write e (N)
#   encode_a      per ct:                write 16N (+ d*8 read)
#   encode_b      per ct:                read 16N, write m (8N) + e (N) = 25N
#   dec_limb1     per delta:             the split decrypt's first kernel: read ct limbs 0-1
#                                        (4 x 8N) + s limbs 0-1 (2 x 8N), write the u rows of
#                                        limbs 0-1 (2 x 8N), read NTT(pt) limb 1 per batch (B x 8N),
#                                        write limb 1's INTT per batch (B x 8N) = 8N(8 + 2B)
#   dec_fused     per delta:             the second (limb 0, CRT, functionals): read limb 0's u
#                                        row (8N) + NTT(pt) limb 0 per batch (B x 8N) + limb 1's
#                                        INTT per batch (B x 8N), write B*cols segment sums
#                                        = 8N(1 + 2B) + 8*B*cols
#   ntt_*         per poly-limb:         read 8N + write 8N = 16N
def kernel_bytes_per_delta(name: str, L: int = 4, nb: int = 4) -> float:
    n = N_POLY
    table = {
        "enc_a": 8 * n * L,
        "enc_u": 33 * n * L,
        "enc_fused": 33 * n * L,
        "decrypt_limb": 40 * n * nb * 2,
        "decode_a": 32 * n * nb,
        "decode_b": 16 * n * nb,
        "encode": 8 * n + D * 8,
        "gauss_gen": n,
        "encode_a": 16 * n + D * 8,
        "encode_b": 25 * n,
        "dec_fused": 8 * n * (1 + 2 * nb) + 8 * nb * 5,
        "dec_limb1": 8 * n * (8 + 2 * nb),
    }
    return float(table.get(name, 0))


KERNEL_NAMES = ("prefetch_l2", "gauss_gen", "encode", "encode_a", "encode_b", "enc_fused", "enc_a", "enc_u", "enc_x",
                "enc_combine", "plan", "gauss_fix", "enc_a_fix", "enc_u_fix", "decrypt_limb", "crt_seg", "decode_a",
                "decode_b", "dec_limb1", "dec_fused", "gather_inter", "bmat", "warm_decrypt_limb", "warm_crt_seg")


def profiled_kernels(_lib, run_steps):
    """Per-kernel CUDA-event time: the steps again, every launch of the
    library bracketed by events on its stream.  {name: (ms, launches)}."""
    _lib.profile_reset()
    _lib.profile_enable(True)
    run_steps()
    _lib.profile_enable(False)
    kern = {}
    for name in KERNEL_NAMES:
        ms, n = _lib.profile_read(name)
        if n:
            kern[name] = (ms, n)
    return kern


ROOF_NOTES = {
    "dec_fused": "compute-bound, not HBM-bound: the fused decrypt runs the 60-bit limb's INTT on the IMAD pipe "
                 "and the 40-bit limb's on the FP64 pipe, and its DRAM traffic is below the compulsory model "
                 "because the key and cached plaintexts stay in L2; `compute` is the binding roofline",
    "enc_fused": "compute-bound, not HBM-bound: both forward NTTs of a (ciphertext, limb) run on one CTA pair "
                 "(the 60-bit limbs' butterflies on the IMAD pipe, the 40-bit limbs' on the FP64 pipe) beside "
                 "ChaCha20 on the ALU pipe; `compute` is the binding roofline",
}


def roofline(kern, batch, steps, peak, peak_kind, sm_mhz, sms):
    """HBM roofline of the dominant kernel (algorithmic bytes per launch /
    its event-timed duration) and, beside it, its compute roofline: warp
    instructions issued per second (ncu's instruction count per delta x
    deltas / event time) against the SMs' issue limit of one warp
    instruction per scheduler per clock (4 per SM) at the sampled clock."""
    dom = max(kern, key=lambda k: kern[k][0]) if kern else None
    if not dom or kernel_bytes_per_delta(dom) <= 0:
        return None
    ms, n = kern[dom]
    total_bytes = kernel_bytes_per_delta(dom) * batch * steps
    achieved = total_bytes / (ms / 1000.0) / 1e9
    tr = {}
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "traffic.json"))).get(dom, {})
    except Exception:
        tr = {}
    traffic = tr["dram_bytes_per_delta"] * batch * steps / n if "dram_bytes_per_delta" in tr else None
    roof = {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak,
            "peak_kind": ("measured (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                          else "fallback 6650 GB/s"),
            "traffic": traffic, "algorithmic_bytes_per_launch": total_bytes / n, "avg_launch_ms": ms / n,
            "binding": "compute", "note": ROOF_NOTES.get(dom, "")}
    if "warp_inst_per_delta" in tr and sm_mhz:
        inst = tr["warp_inst_per_delta"] * batch * steps / (ms / 1000.0)
        ipeak = sms * 4 * sm_mhz * 1e6
        roof["compute"] = {"metric": "warp instructions issued", "achieved": inst / 1e9, "peak": ipeak / 1e9,
                           "unit": "G warp-inst/s", "frac": inst / ipeak,
                           "peak_kind": f"{sms} SMs x 4 schedulers x 1 warp-inst/clk at the sampled {sm_mhz:.0f} MHz",
                           "inst_source": tr.get("inst_source", "ncu sm__inst_executed.sum per delta")}
    if "pipes" in tr:
        roof["pipes"] = tr["pipes"]
    return roof


def plain_check(H, A, B, got):
    """Max-abs error of the GPU deltas against float64 B (A h) for every row
    (the spec's plaintext check, tolerance 1e-4)."""
    ref = (H @ A.astype(np.float64).T) @ B.astype(np.float64).T
    return float(np.abs(ref - got).max())


def run_ours(args):
    import torch
    import torch.distributed as dist

    from provenloop_b200 import _lib, multigpu, tensafe_he
    from provenloop_b200.backend import ZeroMoaiLora

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    batch = args.batch
    H, A, B = inputs(batch, rank)

    ctx = tensafe_he.CkksContext(N_POLY, device=local)
    # one dedicated stream for the library, the L2 flush and the timing events
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "set_stream")
    sk = ctx.keygen(0)
    lora = ZeroMoaiLora(ctx, A, B)
    h_dev = torch.from_numpy(H).to(dev)
    # two delta buffers: step k's gather (N > 1) overlaps step k + 1
    delta_dev = [torch.empty((batch, D), dtype=torch.float64, device=dev) for _ in range(2)]
    d32 = [torch.empty((batch, D), dtype=torch.float32, device=dev) for _ in range(2)]
    recv = [([torch.empty((batch, D), dtype=torch.float32, device=dev) for _ in range(world)] if rank == 0 else None)
            for _ in range(2)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    # users are sharded in blocks over ranks; seeds depend on (user, step) only
    n_users = batch * world
    u0, u1 = multigpu.user_block(n_users, world, rank)
    users = np.arange(u0, u1, dtype=np.uint64)
    pending = [None]

    def seeds_of(i):
        return multigpu.stream_seeds(users, i, n_users)

    def step(i, last=False):
        b = i & 1
        lora.delta_device(sk, h_dev, seeds_of(i), delta_dev[b])
        if world > 1:
            d32[b].copy_(delta_dev[b])                         # fp32 deltas for the gather
            if pending[0] is not None:
                pending[0].wait()                              # step i-1's gather (its buffer is reused at i+1)
            pending[0] = dist.gather(d32[b], gather_list=recv[b], dst=0, async_op=True)
            if last:
                pending[0].wait()
                pending[0] = None

    for i in range(args.warmup):
        step(i, last=i == args.warmup - 1)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    # ---- timed region
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for k in range(args.steps):
        flush.zero_()
        ev[k][0].record(stream)
        step(args.warmup + k, last=k == args.steps - 1)
        ev[k][1].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches = _lib.launch_count() - launches0
    clk = clocks.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in ev)
    last_i = args.warmup + args.steps - 1
    last_rows = [0, batch // 3, (2 * batch) // 3, batch - 1]
    last_delta = delta_dev[last_i & 1].cpu().numpy()
    plain_err = plain_check(H, A, B, last_delta)
    last_seeds = seeds_of(last_i)

    # ---- per-kernel event time (the same steps again, every launch bracketed)
    def prof_steps():
        for k in range(args.steps):
            flush.zero_()
            step(args.warmup + args.steps + k, last=k == args.steps - 1)
        torch.cuda.synchronize(dev)

    kern = profiled_kernels(_lib, prof_steps)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = world * batch * args.steps / (max_ms / 1000.0)

    # ---- NCCL gather alone (not overlapped), for the record of what it costs
    gather_ms = None
    if world > 1:
        ge = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        dist.barrier()
        torch.cuda.synchronize(dev)
        ge[0].record(stream)
        for _ in range(5):
            dist.gather(d32[0], gather_list=recv[0], dst=0)
        ge[1].record(stream)
        torch.cuda.synchronize(dev)
        g = torch.tensor([ge[0].elapsed_time(ge[1]) / 5], dtype=torch.float64, device=dev)
        dist.all_reduce(g, op=dist.ReduceOp.MAX)
        gather_ms = float(g.item())

    # ---- end to end through the public host API (pinned host buffers)
    h_pin = torch.from_numpy(H).pin_memory()
    d_pin = torch.empty((batch, D), dtype=torch.float64).pin_memory()
    hv, dv = h_pin.numpy(), d_pin.numpy()
    if world == 1:
        for i in range(2):
            lora.delta(sk, hv, np.arange(i * batch, (i + 1) * batch, dtype=np.uint64) + 7, out=dv, want_inter=False)
    e2e_ms = 0.0
    h2d, d2h = batch * D * 8, batch * D * 8
    if world == 1:
        for k in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            lora.delta(sk, hv, seeds_of(1000 + k), out=dv, want_inter=False)   # H2D, GPU pipeline, D2H, sync
            e2e_ms += (time.perf_counter() - t0) * 1000.0
    else:
        # each rank streams its users' steps the way a serving loop would:
        # step k's hidden states go host -> device on a copy stream while
        # step k-1 computes, the fp32 deltas are gathered to rank 0 over NCCL,
        # and rank 0 copies every rank's deltas to pinned host memory on a
        # second copy stream while step k+1 computes.  Every step's copies
        # are inside the wall-clock region, which ends when the last step's
        # deltas are in host memory.
        s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        h_in = [torch.empty_like(h_dev) for _ in range(2)]
        g_pin = ([torch.empty((world * batch, D), dtype=torch.float32).pin_memory() for _ in range(2)]
                 if rank == 0 else None)
        d2h = world * batch * D * 4 if rank == 0 else 0
        ev_in = [torch.cuda.Event() for _ in range(2)]     # h_in[b] holds step k's inputs
        ev_read = [torch.cuda.Event() for _ in range(2)]   # step k's kernels are done with h_in[b]
        ev_out = [torch.cuda.Event() for _ in range(2)]    # step k's deltas have left recv[b]
        work = [None, None]

        def e2e_steps(k0, nsteps):
            for k in range(k0, k0 + nsteps):
                b = k & 1
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_read[b])
                    h_in[b].copy_(h_pin, non_blocking=True)
                    ev_in[b].record(s_in)
                stream.wait_event(ev_in[b])
                flush.zero_()
                if work[b] is not None:
                    work[b].wait()                     # step k-2's gather is done with d32[b] and recv[b]
                lora.delta_device(sk, h_in[b], seeds_of(1000 + k), delta_dev[b])
                ev_read[b].record(stream)
                d32[b].copy_(delta_dev[b])
                if rank == 0:
                    stream.wait_event(ev_out[b])       # step k-2's deltas have been copied out
                work[b] = dist.gather(d32[b], gather_list=recv[b], dst=0, async_op=True)
                if rank == 0:
                    with torch.cuda.stream(s_out):
                        work[b].wait()
                        for r_ in range(world):
                            g_pin[b][r_ * batch:(r_ + 1) * batch].copy_(recv[b][r_], non_blocking=True)
                        ev_out[b].record(s_out)
            for b in range(2):
                if work[b] is not None:
                    work[b].wait()
                    work[b] = None
            torch.cuda.synchronize(dev)

        e2e_steps(0, 2)                                  # warms the path (untimed)
        dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        e2e_steps(2, args.steps)
        e2e_ms = (time.perf_counter() - t0) * 1000.0
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = world * batch * args.steps / (float(t.item()) / 1000.0)

    peak, peak_kind = measured_peaks()
    roof = roofline(kern, batch, args.steps, peak, peak_kind, clk.get("sm_mhz") or clk.get("sm_max_mhz") or 1965.0,
                    ctx_sms(dev))

    c4 = None
    if not args.no_c4:
        c4 = c4_leg(args, dev, world, rank, local, steps=min(args.steps, 5), warmup=3, print_line=False)

    micro = None
    if rank == 0 and not args.no_micro:
        micro = ntt_micro(dev, peak)

    c3 = None
    if rank == 0 and world == 1 and not args.no_c3:
        c3 = c3_leg(dev)

    base, parity = None, None
    check = (H[last_rows], last_seeds[last_rows], last_delta[last_rows])
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        base, parity = cpu_baseline_leg(check=check)
    elif rank == 0:
        parity = oracle_spot_check(*check)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": workload(batch, world),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roof, "cpu_baseline": base, "clocks": clk,
            "gpu_launches": launches,
            "parity_checked": bool(parity and parity["ok"] and plain_err < 1e-4),
            "parity": {"last_timed_step_rows_vs_oracle": parity, "all_rows_vs_float64_plaintext": plain_err,
                       "rows": last_rows, "tolerance": 1e-4},
            "kernels_ms_per_step": {k: v[0] / args.steps for k, v in kern.items()},
        }
        if world > 1:
            line["gather_ms_per_step_unoverlapped"] = gather_ms
            line["kernel_ms_per_step_sum"] = sum(v[0] for v in kern.values()) / args.steps
        if micro:
            line["ntt_c2"] = micro
        if c3:
            line["c3"] = c3
        if c4:
            line["c4"] = c4
    if world > 1:
        quiet_stdout()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


def ctx_sms(dev):
    import torch
    return torch.cuda.get_device_properties(dev).multi_processor_count


def ntt_micro(dev, peak):
    """C2 microbenchmarks: NTT round trip of 1024 x 3 x N=16384 and 4096
    pointwise products of 3-limb polys (provenloop_b200.microbench)."""
    from provenloop_b200 import microbench

    out = microbench.ntt(1024, 10, dev.index, peak)
    out["hadamard"] = microbench.hadamard(1024, 4, dev.index, peak)
    return out


def c3_leg(dev, tokens: int = 16):
    """C3: HE tok/s of greedy decode on a random-init Qwen2.5-1.5B-shaped
    model (28 layers, bf16) with encrypted LoRA (rank 16, 3 CryptoMOE
    experts, top-1 router over uniform logits) on q_proj and v_proj of every
    layer and post-transformer DP noise (C = 1, eps = 1, delta = 1e-5),
    N = 16384.  The whole decode step (transformer, 28 HE-LoRA calls, DP
    noise, greedy pick) is one CUDA graph replayed per token; timed with CUDA
    events on its stream, beside the same graph without HE and the eager
    (uncaptured) HE decode."""
    import torch

    from provenloop_b200 import tensafe_he
    from provenloop_b200.decode_step import HeLoraDecoder, build_model

    with torch.cuda.device(dev):
        model = build_model(device=dev, seed=2)
        ctx = tensafe_he.CkksContext(16384, device=dev.index)
        dec = HeLoraDecoder(model, ctx, ctx.keygen(2), rank=16, experts=3, seed=2)
        prompt = 151643

        def timed(run):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            torch.cuda.synchronize(dev)
            ev[0].record(run.stream)
            run(prompt, tokens)
            ev[1].record(run.stream)
            torch.cuda.synchronize(dev)
            return ev[0].elapsed_time(ev[1])

        he_run = dec.capture(max_len=tokens + 8)
        timed(he_run)                        # warm replay
        he_ms = timed(he_run)
        dec.enabled = False
        plain_run = dec.capture(max_len=tokens + 8)
        timed(plain_run)
        plain_ms = timed(plain_run)
        dec.enabled = True
        dec.generate([prompt], tokens=2)     # eager warm-up
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        torch.cuda.synchronize(dev)
        ev[0].record()
        dec.generate([prompt], tokens=tokens)
        ev[1].record()
        torch.cuda.synchronize(dev)
        eager_ms = ev[0].elapsed_time(ev[1])
        dec.remove()
        del he_run, plain_run, model
        torch.cuda.empty_cache()
    he_ms_layer = (he_ms - plain_ms) / tokens / 28
    return {"workload": "Qwen2.5-1.5B-shaped greedy decode, random init bf16, 28 layers; HE-LoRA r=16 on q_proj "
                        "and v_proj of every layer (one encryption per layer shared by q and v), 3 experts, "
                        "post-transformer DP noise; CKKS N=16384; one CUDA graph per decode step",
            "tokens": tokens, "batch": 1, "he_tok_s": tokens / (he_ms / 1e3),
            "plain_tok_s": tokens / (plain_ms / 1e3), "he_ms_per_token": he_ms / tokens,
            "plain_ms_per_token": plain_ms / tokens, "he_ms_per_layer": he_ms_layer,
            "he_only_tok_s": 1.0 / (28 * he_ms_layer / 1e3) if he_ms_layer > 0 else None,
            "eager_he_tok_s": tokens / (eager_ms / 1e3)}


def c4_leg(args, dev, world, rank, local, steps, warmup, print_line):
    """C4: multi-user batched HE-LoRA at N = 32768 (custom [60,40,40,40,60],
    scale 2^40).  256 users, each with an independent secret key (seed 3 +
    user id) and 28 layers x 2 projections of rank-32 adapters (d = 1536,
    cols = 10, 4 plaintext batches); every step computes all 256 x 56 deltas
    once.  Users are block-sharded over the ranks (the total is fixed:
    strong scaling), and rank 0 gathers the decrypted deltas (fp32) over
    NCCL inside the step.  Returns the measurement (rank 0) as a dict."""
    import torch
    import torch.distributed as dist

    from provenloop_b200 import _lib, multigpu, tensafe_he
    from provenloop_b200.backend import ZeroMoaiLora

    u0, u1 = multigpu.user_block(C4_USERS, world, rank)
    nu = u1 - u0
    nmax = -(-C4_USERS // world) * C4_ADAPTERS      # gather buffers sized for the largest block
    batch = nu * C4_ADAPTERS
    rng = np.random.default_rng(3)
    A = (rng.standard_normal((C4_ADAPTERS, C4_R, D)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((C4_ADAPTERS, D, C4_R)) * 0.02).astype(np.float32)
    H = np.random.default_rng(3000 + rank).standard_normal((batch, D))
    ctx = tensafe_he.CkksContext.custom(C4_N, C4_BITS, device=local)
    stream = torch.cuda.Stream(device=dev)
    prev_stream = torch.cuda.current_stream(dev)
    torch.cuda.set_stream(stream)
    _lib.check(_lib.lib().ts_ctx_set_stream(ctx.handle, stream.cuda_stream), "set_stream")
    sk = ctx.keygen_batch([3 + u for u in range(u0, u1)])
    lora = ZeroMoaiLora(ctx, A, B)
    h_dev = torch.from_numpy(H).to(dev)
    delta_dev = torch.empty((batch, D), dtype=torch.float64, device=dev)
    d32 = torch.zeros((nmax, D), dtype=torch.float32, device=dev)
    recv = [torch.empty((nmax, D), dtype=torch.float32, device=dev) for _ in range(world)] if rank == 0 else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    adapter = np.tile(np.arange(C4_ADAPTERS, dtype=np.int32), nu)
    user_ix = np.repeat(np.arange(nu, dtype=np.int32), C4_ADAPTERS)
    gid = (u0 + user_ix.astype(np.int64)) * C4_ADAPTERS + adapter   # global delta id

    def step(i):
        seeds = multigpu.stream_seeds(gid, i, C4_USERS * C4_ADAPTERS)
        lora.delta_device(sk, h_dev, seeds, delta_dev, expert=adapter, sk_index=user_ix)
        if world > 1:
            d32[:batch].copy_(delta_dev)
            dist.gather(d32, gather_list=recv, dst=0)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = _lib.launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for k in range(steps):
        flush.zero_()
        ev[k][0].record(stream)
        step(warmup + k)
        ev[k][1].record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    launches = _lib.launch_count() - launches0
    clk = clocks.stop()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
    got = delta_dev.cpu().numpy()
    plain_err = 0.0
    for a in range(C4_ADAPTERS):
        rows = adapter == a
        if rows.any():
            ref = (H[rows] @ A[a].astype(np.float64).T) @ B[a].astype(np.float64).T
            plain_err = max(plain_err, float(np.abs(ref - got[rows]).max()))

    def prof_steps():
        for k in range(steps):
            flush.zero_()
            step(warmup + steps + k)
        torch.cuda.synchronize(dev)

    kern = profiled_kernels(_lib, prof_steps)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    total = C4_USERS * C4_ADAPTERS
    value = total * steps / (max_ms / 1000.0)
    # end to end, one step after a warm one: N = 1 through the host API
    # (pinned host buffers in and out); N > 1 from pinned host hidden states
    # through the pipeline and the NCCL gather to rank 0's pinned host memory
    h_pin = torch.from_numpy(H).pin_memory()
    d_pin = torch.empty((batch, D), dtype=torch.float64).pin_memory()
    g_pin = torch.empty((world * nmax, D), dtype=torch.float32).pin_memory() if (world > 1 and rank == 0) else None
    e2e_ms = 0.0
    for k in range(2):
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        seeds = multigpu.stream_seeds(gid, 999 + k, total)
        if world == 1:
            lora.delta(sk, h_pin.numpy(), seeds, expert=adapter, sk_index=user_ix, out=d_pin.numpy(),
                       want_inter=False)
        else:
            h_dev.copy_(h_pin, non_blocking=True)
            lora.delta_device(sk, h_dev, seeds, delta_dev, expert=adapter, sk_index=user_ix)
            d32[:batch].copy_(delta_dev)
            dist.gather(d32, gather_list=recv, dst=0)
            if rank == 0:
                for r_ in range(world):
                    g_pin[r_ * nmax:(r_ + 1) * nmax].copy_(recv[r_], non_blocking=True)
            torch.cuda.synchronize(dev)
        e2e_ms = (time.perf_counter() - t0) * 1000.0
    e2e = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    torch.cuda.set_stream(prev_stream)
    out = {
        "metric": C4_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": max_ms / steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u64", "data": "synthetic",
        "config": {"workload": "C4 multi-user: 256 users (own keys) x 28 layers x 2 projections, one delta each "
                               "per step", "poly_degree": C4_N, "moduli_bits": C4_BITS, "scale_bits": 40,
                   "d": D, "r": C4_R, "cols_per_ct": 10, "pt_batches": 4, "adapters": C4_ADAPTERS,
                   "users": C4_USERS, "global_batch": total, "batch_per_gpu": batch,
                   "parallelism": "replicas" if world == 1 else
                   f"users sharded over {world} ranks, NCCL gather of fp32 deltas to rank 0"},
        "e2e": {"value": total / (float(e2e.item()) / 1000.0), "unit": UNIT,
                "h2d_bytes_per_step": batch * D * 8,
                "d2h_bytes_per_step": batch * D * 8 if world == 1 else world * nmax * D * 4},
        "clocks": clk, "gpu_launches": launches,
        "kernels_ms_per_step": {k: v[0] / steps for k, v in kern.items()},
        "rank0_rows_vs_float64_plaintext": plain_err,
    }
    del lora, sk, ctx
    if print_line and rank == 0:
        print(json.dumps(out))
    return out if rank == 0 else None


def run_c4(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    out = c4_leg(args, torch.device("cuda", local), world, rank, local, args.steps, args.warmup, print_line=False)
    if world > 1:
        quiet_stdout()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(out)


def run_c5(args):
    """C5: the sweep of provenloop_b200/sweep.py (N x batch x d x r), one
    JSON line; `value` is its N = 16384, batch 4096, d = 1536, r = 16 point."""
    import torch
    import torch.distributed as dist

    from provenloop_b200 import _lib, sweep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    peak, peak_kind = measured_peaks()
    launches0 = _lib.launch_count()
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    pts = sweep.run(args.steps, args.warmup, peak_gbs=peak, device=local)
    clk = clocks.stop()
    head = next(p for p in pts if (p["n"], p["batch"], p["d"], p["r"]) == (16384, 4096, 1536, 16))
    if rank == 0:
        line = {
            "metric": "encrypted LoRA deltas/sec, sweep over N, batch, d and r (C5)",
            "value": head["deltas_per_s"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": "C5 sweep: N in {8192,16384,32768} x batch in {1,16,256,4096} per GPU x d in "
                                   "{1536,3584} x r in {8,16,32,64}; value = the N=16384/4096/1536/16 point",
                       "l2": "flushed between timed steps (256 MiB write)", "seed": 4,
                       "parallelism": "replicas" if world == 1 else f"users sharded over {world} ranks"},
            "peak_gbs": peak, "peak_kind": peak_kind, "clocks": clk,
            "gpu_launches": _lib.launch_count() - launches0, "points": pts,
        }
    if world > 1:
        quiet_stdout()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c4":
        run_c4(args)
    elif args.config == "c5":
        run_c5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
