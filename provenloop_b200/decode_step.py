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

Seeds, the routed expert and the DP seed are derived on the device from a
token counter, so a decode step issues stream work only: ``capture`` records
the whole step -- transformer, 28 HE-LoRA calls, DP noise, greedy pick -- as
one CUDA graph that is replayed per token.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import tensafe_he
from ._lib import check, lib
from .backend import ZeroMoaiLora, dp_sigma, lora_delta_graphable

QWEN25_15B = dict(hidden_size=1536, intermediate_size=8960, num_hidden_layers=28, num_attention_heads=12,
                  num_key_value_heads=2, vocab_size=151936, max_position_embeddings=32768, rope_theta=1000000.0,
                  rms_norm_eps=1e-6, tie_word_embeddings=True)

_SEED_TOKEN, _SEED_LAYER, _SEED_BASE, _DP_LAYER = 1_000_003, 7919, 17, 10_000


def build_model(device="cuda", seed: int = 2, layers: int = 28):
    """Random-init bf16 Qwen2ForCausalLM of the 1.5B shape (no checkpoint)."""
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen2Config(**dict(QWEN25_15B, num_hidden_layers=layers))
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


def encryption_seed(token: int, layer: int) -> int:
    """Seed of (token, layer)'s encryption (the device computes the same)."""
    return token * _SEED_TOKEN + layer * _SEED_LAYER + _SEED_BASE


class HeLoraDecoder:
    """HE-LoRA (q_proj, v_proj) on every layer of ``model``, CryptoMOE
    experts chosen per token by a top-1 router over hash-uniform logits."""

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
        f64 = dict(dtype=torch.float64, device=self.dev)
        self._h = torch.zeros((1, d), **f64)
        self._dq = torch.zeros((1, d), **f64)
        self._dv = torch.zeros((1, dv), **f64)
        self._inter = torch.zeros((1, 2 * rank), **f64)
        self._fin = torch.zeros((1, d), **f64)
        self.token = torch.zeros((1,), dtype=torch.int64, device=self.dev)   # device token counter
        self.expert = torch.zeros((1,), dtype=torch.int32, device=self.dev)
        self._seed = torch.zeros((1,), dtype=torch.int64, device=self.dev)
        self._eidx = torch.arange(experts, dtype=torch.float64, device=self.dev)
        self._hooks = []
        self.enabled = True
        self._hooks.append(model.model.embed_tokens.register_forward_hook(self._route_hook))
        for li, layer in enumerate(model.model.layers):
            self._hooks.append(layer.self_attn.q_proj.register_forward_hook(self._q_hook(li)))
            self._hooks.append(layer.self_attn.v_proj.register_forward_hook(self._v_hook))
        self._hooks.append(model.model.norm.register_forward_hook(self._dp_hook))

    # ---------------------------------------------------------------- hooks
    def _route_hook(self, module, inp, out):
        # top-1 router over uniform logits: hash-uniform values of (token, e)
        import torch
        if self.enabled:
            x = torch.sin(self.token.double() * 12.9898 + self._eidx * 78.233) * 43758.5453
            self.expert.copy_(torch.argmax(x - torch.floor(x)).view(1).to(torch.int32))
        return out

    def _q_hook(self, li):
        def hook(module, inp, out):
            if not self.enabled:
                return out
            self._h.copy_(inp[0][:, -1, :])
            self._seed.copy_(self.token * _SEED_TOKEN + (li * _SEED_LAYER + _SEED_BASE))
            lora_delta_graphable(self.loras[li], self.sk, self._h, self._seed, self._dq, expert_dev=self.expert,
                                 inter_dev=self._inter)
            bv = self.bv[li].index_select(0, self.expert.long())[0]
            self._dv.copy_(self._inter[:, self.rank:] @ bv.T)
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
        self._seed.copy_(self.token * _SEED_TOKEN + (_DP_LAYER * _SEED_LAYER + _SEED_BASE))
        check(lib().ts_dp_noise(self.ctx.handle, self._fin.data_ptr(), 1, self._fin.shape[1], float(self.clip),
                                float(self.sigma), C.cast(self._seed.data_ptr(), C.POINTER(C.c_uint64)), 2),
              "ts_dp_noise")
        out[:, -1, :] = self._fin.to(out.dtype)
        return out

    # ---------------------------------------------------------------- decode
    def bind_stream(self, stream=None):
        """Run the library on ``stream`` (default: torch's current stream)."""
        import torch
        s = stream if stream is not None else torch.cuda.current_stream(self.dev)
        check(lib().ts_ctx_set_stream(self.ctx.handle, s.cuda_stream), "ts_ctx_set_stream")

    def generate(self, prompt_ids, tokens: int = 16):
        """Greedy decode, eager (DynamicCache); every forward pass runs
        HE-LoRA on all layers."""
        import torch
        from transformers import DynamicCache

        self.bind_stream()
        ids = torch.as_tensor(prompt_ids, device=self.dev).view(1, -1)
        cache = DynamicCache()
        out_ids = []
        with torch.no_grad():
            for _ in range(tokens):
                res = self.model(input_ids=ids, past_key_values=cache, use_cache=True)
                ids = res.logits[:, -1, :].argmax(dim=-1, keepdim=True)
                out_ids.append(ids)
                self.token += 1
        return torch.cat(out_ids, dim=1)

    def capture(self, max_len: int = 64, warmup: int = 2):
        """Capture one decode step (static KV cache) as a CUDA graph on a
        side stream; returns run(prompt_id, n) that decodes n tokens from a
        one-token prompt by replaying it."""
        import torch
        from transformers import StaticCache

        cfg = self.model.config
        cache = StaticCache(config=cfg, max_batch_size=1, max_cache_len=max_len, device=self.dev,
                            dtype=torch.bfloat16)
        ids = torch.zeros((1, 1), dtype=torch.long, device=self.dev)
        pos = torch.zeros((1,), dtype=torch.long, device=self.dev)
        outs = torch.zeros((1, max_len), dtype=torch.long, device=self.dev)
        stream = torch.cuda.Stream(device=self.dev)
        self.bind_stream(stream)

        def step():
            r = self.model(input_ids=ids, cache_position=pos, position_ids=pos.view(1, 1), past_key_values=cache,
                           use_cache=True)
            nxt = r.logits[:, -1, :].argmax(dim=-1, keepdim=True)
            outs.index_copy_(1, pos, nxt)
            ids.copy_(nxt)
            pos.add_(1)
            self.token.add_(1)

        stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(warmup):  # sizes the library's scratch, loads kernels
                step()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
        torch.cuda.synchronize(self.dev)

        def run(prompt_id: int, n: int, start_token: int = 0):
            if n > max_len:
                raise ValueError(f"at most {max_len} tokens per capture")
            with torch.cuda.stream(stream):
                # the static cache keeps its own device write position
                # (cumulative_length), which must restart with pos
                cache.reset()
                ids.fill_(int(prompt_id))
                pos.zero_()
                self.token.fill_(int(start_token))
                for _ in range(n):
                    graph.replay()
            return outs[:, :n]

        run.stream = stream
        run.graph = graph
        return run

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
