"""Encrypted-LoRA decode steps on a Qwen2.5-1.5B-shaped model.

The reference applies ZeRo-MOAI encrypted LoRA while it generates tokens
(demonstrator/server/inference_engine.py:1197-1405): the hidden state is
encrypted, multiplied by the packed LoRA-A plaintexts of the routed CryptoMOE
expert (:832-877, :1155-1171), decrypted in one batch, multiplied by B and
added to the projection, and the post-transformer hidden state gets clipped
Gaussian DP noise (:1411-1465).  It does this for one representative
projection pair on the final hidden state (:987-997).  This module runs the
same arithmetic at every layer, on q_proj and v_proj, of a random-init model
with Qwen2.5-1.5B's shape (28 layers, d = 1536, 12 / 2 heads, FFN 8960;
demonstrator/frontend/weights/config.json:2-7).

Per layer and token:
- ONE encryption of the layer input, shared by q and v: the q and v A
  matrices are stacked into one rank-2r adapter;
- ceil(2r / cols) ct x pt products and one batched decrypt, all in
  ``ts_lora_delta_batch`` on the model's CUDA stream;
- the q delta applied by the library (B_q), the v delta from the decrypted
  intermediate (B_v has 256 outputs, not d).

Everything stays on the device, so a token costs no host synchronisation.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import tensafe_he
from ._lib import check, lib, ptr
from .backend import ZeroMoaiLora, dp_sigma

QWEN25_15B = dict(hidden_size=1536, intermediate_size=8960, num_hidden_layers=28, num_attention_heads=12,
                  num_key_value_heads=2, vocab_size=151936, max_position_embeddings=32768, rope_theta=1000000.0,
                  rms_norm_eps=1e-6, tie_word_embeddings=True)


def build_model(device="cuda", seed: int = 2, layers: int = 28):
    """Random-init bf16 Qwen2ForCausalLM of the 1.5B shape (no checkpoint)."""
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(**dict(QWEN25_15B, num_hidden_layers=layers))
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


class HeLoraDecoder:
    """HE-LoRA (q_proj, v_proj) on every layer of ``model``, CryptoMOE
    experts chosen per token by a top-1 router over random logits."""

    def __init__(self, model, ctx: "tensafe_he.CkksContext", sk, rank: int = 16, experts: int = 3, seed: int = 2,
                 dp=(1.0, 1.0, 1e-5)):
        import torch

        self.model, self.ctx, self.sk = model, ctx, sk
        self.rank, self.experts = rank, experts
        cfg = model.config
        d = cfg.hidden_size
        dv = cfg.num_key_value_heads * (cfg.hidden_size // cfg.num_attention_heads)
        self.dev = next(model.parameters()).device
        rng = np.random.default_rng(seed)
        self.loras, self.bv = [], []
        self.weights = []  # per layer (A_q, A_v, B_q, B_v), float32 as loaded
        for _ in range(cfg.num_hidden_layers):
            aq = (rng.standard_normal((experts, rank, d)) * 0.02).astype(np.float32)
            av = (rng.standard_normal((experts, rank, d)) * 0.02).astype(np.float32)
            bq = (rng.standard_normal((experts, d, rank)) * 0.02).astype(np.float32)
            bv = (rng.standard_normal((experts, dv, rank)) * 0.02).astype(np.float32)
            self.weights.append((aq, av, bq, bv))
            b_lib = np.zeros((experts, d, 2 * rank))
            b_lib[:, :, :rank] = bq
            self.loras.append(ZeroMoaiLora(ctx, np.concatenate([aq, av], axis=1).astype(np.float32),
                                           b_lib.astype(np.float32)))
            self.bv.append(torch.from_numpy(bv.astype(np.float64)).to(self.dev))
        self.clip, eps, delta = dp
        self.sigma = dp_sigma(eps, delta, self.clip)
        self._h = torch.zeros((1, d), dtype=torch.float64, device=self.dev)
        self._dq = torch.zeros((1, d), dtype=torch.float64, device=self.dev)
        self._inter = torch.zeros((1, 2 * rank), dtype=torch.float64, device=self.dev)
        self._fin = torch.zeros((1, d), dtype=torch.float64, device=self.dev)
        self._dv = None
        self._token = 0
        self._expert = 0
        self._rng = np.random.default_rng(seed + 1)
        self._hooks = []
        self.enabled = True
        for li, layer in enumerate(model.model.layers):
            self._hooks.append(layer.self_attn.q_proj.register_forward_hook(self._q_hook(li)))
            self._hooks.append(layer.self_attn.v_proj.register_forward_hook(self._v_hook))
        self._hooks.append(model.model.norm.register_forward_hook(self._dp_hook))
        # the library works on torch's stream: no host synchronisation per layer
        self._stream = None

    def _seed(self, layer: int) -> int:
        return (self._token * 1_000_003 + layer * 7919 + 17) & 0xFFFFFFFFFFFFFFFF

    def _q_hook(self, li):
        def hook(module, inp, out):
            if not self.enabled:
                return out
            self._h.copy_(inp[0][:, -1, :])
            self.loras[li].delta_device(self.sk, self._h, [self._seed(li)], self._dq, expert=[self._expert],
                                        inter_dev=self._inter)
            self._dv = self._inter[:, self.rank:] @ self.bv[li][self._expert].T
            out[:, -1, :] += self._dq.to(out.dtype)
            return out
        return hook

    def _v_hook(self, module, inp, out):
        if self.enabled:
            out[:, -1, :] += self._dv.to(out.dtype)
        return out

    def _dp_hook(self, module, inp, out):
        # post-transformer clip + Gaussian noise (inference_engine.py:1436-1456)
        if not self.enabled:
            return out
        self._fin.copy_(out[:, -1, :])
        s = np.array([self._seed(10_000)], dtype=np.uint64)
        check(lib().ts_dp_noise(self.ctx.handle, self._fin.data_ptr(), 1, self._fin.shape[1], float(self.clip),
                                float(self.sigma), ptr(s, C.c_uint64), 1), "ts_dp_noise")
        out[:, -1, :] = self._fin.to(out.dtype)
        return out

    def bind_stream(self):
        import torch
        check(lib().ts_ctx_set_stream(self.ctx.handle, torch.cuda.current_stream(self.dev).cuda_stream),
              "ts_ctx_set_stream")

    def generate(self, prompt_ids, tokens: int = 16):
        """Greedy decode of ``tokens`` tokens; every forward pass (the prompt
        step and each decode step) runs HE-LoRA on all layers."""
        import torch
        from transformers import DynamicCache

        self.bind_stream()
        ids = torch.as_tensor(prompt_ids, device=self.dev).view(1, -1)
        cache = DynamicCache()
        out_ids = []
        with torch.no_grad():
            for t in range(tokens):
                self._expert = int(np.argmax(self._rng.random(self.experts)))  # top-1 over uniform logits
                res = self.model(input_ids=ids, past_key_values=cache, use_cache=True)
                nxt = res.logits[:, -1, :].argmax(dim=-1, keepdim=True)
                out_ids.append(nxt)
                ids = nxt
                self._token += 1
        return torch.cat(out_ids, dim=1)

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
