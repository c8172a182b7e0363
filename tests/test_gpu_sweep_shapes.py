"""GPU parity at the corners of the C5 sweep (N, batch, d, r), through the
C ABI against the CPU oracle's ZeRo-MOAI delta (inference_engine.py:1244-1392):
one column per ciphertext (N = 8192, d = 3584: 64 plaintext batches at
r = 64), the N = 32768 preset chain with d = 3584, and batches of 1 and 16,
which take the small-batch forms (forked encryption, per-limb decrypt plus
the cluster CRT kernel) where 256 (and 40 at N = 32768, whose four-batch
vectors fill the GPU) takes the fused encryption and the split decrypt.
Deltas within 1e-4 max-abs, intermediates within 1e-8.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def T():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from provenloop_b200 import tensafe_he
    return tensafe_he


def _check(T, oracle, n, d, r, batch, check_rows, seed0=40):
    from provenloop_b200.backend import ZeroMoaiLora
    ctx = T.CkksContext(n)
    octx = oracle.Ctx(n)
    rng = np.random.default_rng(4)
    A = (rng.standard_normal((r, d)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((d, r)) * 0.02).astype(np.float32)
    H = rng.standard_normal((batch, d))
    seeds = list(range(seed0, seed0 + batch))
    lora = ZeroMoaiLora(ctx, A, B)
    cols = (n // 2) // d
    assert (lora.cols, lora.batches) == (cols, -(-r // cols))
    sk = ctx.keygen(4)
    delta, inter = lora.delta(sk, H, seeds)
    osk = octx.keygen(4)
    for i in check_rows:
        od, oi = octx.lora_delta(osk, H[i], A, B, enc_seed=seeds[i])
        assert np.abs(delta[i] - od).max() < 1e-4, (n, d, r, batch, i)
        assert np.abs(inter[i] - oi).max() < 1e-8, (n, d, r, batch, i)
    ref = (B.astype(np.float64) @ (A.astype(np.float64) @ H.T)).T
    assert np.abs(delta - ref).max() < 1e-4


@pytest.mark.parametrize("batch", [1, 16])
def test_n8192_one_column_r64(T, oracle, batch):
    _check(T, oracle, 8192, 3584, 64, batch, [0, batch - 1])


def test_n8192_d1536_r8_batch256(T, oracle):
    _check(T, oracle, 8192, 1536, 8, 256, [0, 131, 255])


@pytest.mark.parametrize("batch", [1, 16])
def test_n16384_d3584_r64(T, oracle, batch):
    _check(T, oracle, 16384, 3584, 64, batch, [0, batch - 1])


@pytest.mark.parametrize("batch", [1, 16])
def test_n32768_d3584_r8(T, oracle, batch):
    _check(T, oracle, 32768, 3584, 8, batch, [0, batch - 1])


def test_n32768_d1536_r32_batch40(T, oracle):
    # 40 deltas x 4 plaintext batches: enough vectors for the split decrypt
    # and the fused encryption at N = 32768 on the preset chain
    _check(T, oracle, 32768, 1536, 32, 40, [0, 20, 39])
