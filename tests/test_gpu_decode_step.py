"""GPU check of the encrypted-LoRA decode step (q_proj / v_proj on every
layer of a Qwen2.5-1.5B-shaped model, random init): the deltas the hooks add
equal the float64 plaintext LoRA B(A h) within the 1e-4 delta tolerance, and
the device DP noise equals the host path's for the same seed."""
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


def test_decode_step_deltas_match_plaintext(T):
    import torch
    from provenloop_b200.decode_step import HeLoraDecoder, build_model
    model = build_model(layers=2)
    ctx = T.CkksContext(16384)
    dec = HeLoraDecoder(model, ctx, ctx.keygen(0), rank=16, experts=3, seed=2)
    seen = []

    def probe(module, inp, out):
        # runs after the HE hook of the same q_proj (registered later)
        seen.append((inp[0][:, -1, :].double().cpu().numpy()[0], dec._dq.cpu().numpy()[0],
                     dec._dv.cpu().numpy()[0], dec._expert))
    model.model.layers[1].self_attn.q_proj.register_forward_hook(probe)
    toks = dec.generate([151643], tokens=3)
    torch.cuda.synchronize()
    assert toks.shape == (1, 3)
    aq, av, bq, bv = dec.weights[1]
    for h, dq, dv, e in seen:
        ref_q = bq[e].astype(np.float64) @ (aq[e].astype(np.float64) @ h)
        ref_v = bv[e].astype(np.float64) @ (av[e].astype(np.float64) @ h)
        assert np.abs(dq - ref_q).max() < 1e-4
        assert np.abs(dv - ref_v).max() < 1e-4
    assert len(seen) == 3
    dec.remove()


def test_device_dp_noise_matches_host(T):
    import ctypes as C
    import torch
    from provenloop_b200._lib import check, lib, ptr
    from provenloop_b200.backend import add_dp_noise, dp_sigma
    ctx = T.CkksContext(16384)
    sigma = dp_sigma(1.0, 1e-5, 1.0)
    h = np.random.default_rng(5).standard_normal((2, 1536)) * 3
    ref = add_dp_noise(ctx, h, sigma, seeds=[11, 12], clip=1.0)
    d = torch.from_numpy(h.copy()).cuda()
    torch.cuda.synchronize()  # the copy is on torch's stream, the noise on the context's
    s = np.array([11, 12], dtype=np.uint64)
    check(lib().ts_dp_noise(ctx.handle, d.data_ptr(), 2, 1536, 1.0, float(sigma), ptr(s, C.c_uint64), 1), "dp")
    ctx.synchronize()
    assert np.array_equal(d.cpu().numpy(), ref)
