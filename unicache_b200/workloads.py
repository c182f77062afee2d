"""Seeded builders of the benchmark configurations' caches, assembled through
the public API (the same calls an engine makes), shared by ``bench.py`` and
the parity tests.

Config 4 (an image-editing layer, the shape the reference's long-query patch
targets, unicache/adapters/bagel.py:1598-1858): 28 query / 4 KV heads,
head_dim 128, bf16 K, V ~ N(0, 1) with 4 outlier key channels x10.  The cache
holds 256 instruction tokens and 4900 ViT tokens, each compressed by H2O to
20% (51 and 980 per KV head, scored by the attention of the current 1024-token
latent block over the full dense cache: the reference's "full_kv_first_call"
observation, operators/physical.py:51-101), 1024 source-VAE tokens in 2-bit
KIVI, group 32, with a 32-token bf16 residual (992 packed), and 16 boundary
tokens in bf16; the latent block's own 1024 keys/values stay dense.  The
query is the latent block: Lq = 1024 positions x 28 heads.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import kernels
from .adapters.attention import long_query_attention_summary
from .storage.physical import GQAH2OCache, PackedKIVICache
from .synthetic import make_kv, make_query

CONFIG4 = {"instruction": 256, "vit": 4900, "vae": 1024, "boundary": 16, "latent": 1024, "lq": 1024,
           "q_heads": 28, "kv_heads": 4, "head_dim": 128, "ratio": 0.2, "recent_fraction": 0.25,
           "bits": 2, "group": 32, "residual": 32}


def h2o_budget(tokens: int, ratio: float, recent_fraction: float) -> tuple[int, int]:
    """(target, recent) per KV head, as the reference's storage backend
    computes them (Python rounding, tensor_backend.py:199-210)."""

    target = max(1, int(round(tokens * ratio)))
    return target, int(round(target * recent_fraction))


@dataclass
class Config4Layer:
    query: torch.Tensor            # [Lq, Hq, D] bf16
    dense: dict                    # name -> (key, value) [N, Hkv, D] bf16, the raw segments
    scores: dict                   # name -> [Hkv, N] fp32 H2O scores of the H2O segments
    first_call_lse: torch.Tensor   # [Hq, Lq] LSE of the latent block over the full dense cache
    segments: list                 # [instruction H2O, ViT H2O, VAE packed]
    dense_key: torch.Tensor        # boundary + latent rows [16 + 1024, Hkv, D]
    dense_value: torch.Tensor

    @property
    def key_tokens(self) -> int:
        n = int(self.dense_key.shape[0])
        for seg in self.segments:
            n += seg.retained_tokens if isinstance(seg, GQAH2OCache) else \
                seg.quantized_tokens + int(seg.residual_key.shape[0])
        return n


def config4_layer(device, seed: int = 1) -> Config4Layer:
    c = CONFIG4
    hkv, d = c["kv_heads"], c["head_dim"]
    names = ("instruction", "vit", "vae", "boundary", "latent")
    dense = {name: make_kv(c[name], hkv, d, seed=seed * 10 + i, device=device) for i, name in enumerate(names)}
    query = make_query(c["lq"], c["q_heads"], d, seed=seed, device=device)
    # First call: the latent block attends to the whole dense cache; its LSE
    # drives the H2O scores of the instruction and ViT segments.
    full_k = torch.cat([dense[n][0] for n in names])
    full_v = torch.cat([dense[n][1] for n in names])
    _, lse = long_query_attention_summary(query, [], dense_key=full_k, dense_value=full_v)
    scale = 1.0 / math.sqrt(d)
    scores, segments = {}, []
    for name in ("instruction", "vit"):
        k, v = dense[name]
        scores[name] = kernels.h2o_scores(query, k, lse, kv_heads=hkv, softmax_scale=scale)
        target, recent = h2o_budget(c[name], c["ratio"], c["recent_fraction"])
        segments.append(GQAH2OCache.from_dense(k, v, logical_token_ids=torch.arange(c[name], device=device),
                                               token_type_id=1, per_kv_head_scores=scores[name],
                                               target_tokens=target, recent_tokens=recent, selection_frozen=True))
    vk, vv = dense["vae"]
    segments.append(PackedKIVICache.from_dense(vk, vv, logical_token_ids=torch.arange(c["vae"], device=device),
                                               token_type_id=3, k_bits=c["bits"], v_bits=c["bits"],
                                               group_size=c["group"], residual_length=c["residual"]))
    dense_key = torch.cat([dense["boundary"][0], dense["latent"][0]])
    dense_value = torch.cat([dense["boundary"][1], dense["latent"][1]])
    return Config4Layer(query, dense, scores, lse, segments, dense_key, dense_value)


# ---------------------------------------------------------------- config 5
QWEN2_7B = {"hidden": 3584, "layers": 28, "q_heads": 28, "kv_heads": 4, "head_dim": 128, "ffn": 18944,
            "vocab": 151936, "rope_theta": 1.0e6, "eps": 1.0e-6}


class Qwen2PackedDecode:
    """a Qwen2-7B-shaped decoder (hidden 3584, 28 layers, 28
    query / 4 KV heads, head_dim 128, FFN 18944, untied 151936-token head:
    modeling/qwen2/configuration_qwen2.py:123-134 of the reference) with
    seeded random bf16 weights, decoding ``batch`` sequences greedily.

    Each layer's prompt cache of ``prompt`` tokens per sequence is synthetic
    (seeded K/V with the benchmark's distribution and seeded H2O scores, in
    place of a prefill), compressed by H2O to ``ratio`` of the tokens per KV
    head (the reference's recent fraction 0.25) and the retained rows packed
    in ``bits``-bit KIVI (group ``group``, ``residual`` bf16 tokens) -- the
    composition the reference refuses on one request (tensor_backend.py:
    137-144) applied as two steps.  New tokens go to a dense bf16 suffix of
    capacity ``new_tokens`` (the reference appends decode tokens to its dense
    cache).  Attention is the packed decode kernel over [packed prompt +
    residual + live suffix]; the projections are cuBLAS GEMMs through torch
    (residual adds in their epilogues), and RMSNorm, the rotary embedding
    fused with the suffix append, and the SwiGLU gate are one library kernel
    each (``kernels.rms_norm``, ``qkv_rope_append``, ``silu_mul``): ten
    launches per layer.  One decode step is captured once as a CUDA graph:
    the suffix length, the RoPE position and the append index live on the
    device.
    """

    def __init__(self, device, *, batch: int = 32, prompt: int = 16384, new_tokens: int = 512,
                 ratio: float = 0.2, recent_fraction: float = 0.25, bits: int = 2, group: int = 32,
                 residual: int = 32, layers: int | None = None, prefilled: int = 0, seed: int = 5):
        from .kernels import GrowingSuffix

        c = QWEN2_7B
        self.device = torch.device(device)
        self.batch, self.prompt, self.capacity = batch, prompt, new_tokens
        self.layers = c["layers"] if layers is None else layers
        hid, hq, hkv, d, ffn = c["hidden"], c["q_heads"], c["kv_heads"], c["head_dim"], c["ffn"]
        self.hq, self.hkv, self.d, self.ffn, self.eps = hq, hkv, d, ffn, c["eps"]
        gen = torch.Generator(device=self.device).manual_seed(seed)

        def weight(*shape, std=0.02):
            return (torch.randn(*shape, generator=gen, device=self.device) * std).to(torch.bfloat16)

        qkv_out = (hq + 2 * hkv) * d
        self.w = []
        for _ in range(self.layers):
            self.w.append({
                "in_norm": torch.ones(hid, device=self.device, dtype=torch.bfloat16),
                "qkv": weight(hid, qkv_out), "qkv_bias": weight(qkv_out),
                "o": weight(hq * d, hid),
                "post_norm": torch.ones(hid, device=self.device, dtype=torch.bfloat16),
                "gate_up": weight(hid, 2 * ffn), "down": weight(ffn, hid),
            })
        self.embed = weight(c["vocab"], hid)
        self.final_norm = torch.ones(hid, device=self.device, dtype=torch.bfloat16)
        self.lm_head = weight(hid, c["vocab"])
        half = d // 2
        self.inv_freq = 1.0 / (c["rope_theta"] ** (torch.arange(half, device=self.device, dtype=torch.float32) / half))

        # caches: H2O 20% of the prompt per KV head, then KIVI on the retained rows
        target, recent = h2o_budget(prompt, ratio, recent_fraction)
        self.retained = target
        self.length = torch.full((1,), prefilled, device=self.device, dtype=torch.int32)
        self.plans, self.suffixes, self.packed = [], [], []
        outliers = torch.randperm(d, generator=torch.Generator().manual_seed(seed))[:4].to(self.device)
        for layer in range(self.layers):
            sk = torch.zeros(batch, new_tokens, hkv, d, device=self.device, dtype=torch.bfloat16)
            sv = torch.zeros_like(sk)
            if prefilled:
                sk[:, :prefilled] = weight(batch, prefilled, hkv, d, std=1.0)
                sv[:, :prefilled] = weight(batch, prefilled, hkv, d, std=1.0)
            self.suffixes.append((sk, sv))
            seqs = []
            for b in range(batch):
                # generated on the device (the prompt caches are tens of GB in total)
                k = torch.randn(prompt, hkv, d, generator=gen, device=self.device)
                k[:, :, outliers] *= 10.0
                k = k.to(torch.bfloat16)
                v = torch.randn(prompt, hkv, d, generator=gen, device=self.device).to(torch.bfloat16)
                scores = torch.rand(hkv, prompt, generator=gen, device=self.device)
                kept = GQAH2OCache.from_dense(k, v, logical_token_ids=torch.arange(prompt, device=self.device),
                                              token_type_id=0, per_kv_head_scores=scores, target_tokens=target,
                                              recent_tokens=recent, selection_frozen=True)
                packed = PackedKIVICache.from_dense(kept.key.transpose(0, 1), kept.value.transpose(0, 1),
                                                    logical_token_ids=kept.logical_token_ids[0], token_type_id=0,
                                                    k_bits=bits, v_bits=bits, group_size=group,
                                                    residual_length=residual)
                del k, v, kept
                seqs.append([packed, GrowingSuffix(sk[b], sv[b], self.length)])
                self.packed.append(packed)
            from .kernels import build_decode_plan

            self.plans.append(build_decode_plan(seqs, num_kv_heads=hkv, head_dim=d))
        torch.cuda.empty_cache()
        self.ids = torch.zeros(batch, device=self.device, dtype=torch.int64)
        self.x = self.embed[self.ids].clone()
        self.q_buf = torch.empty(batch, hq, d, device=self.device, dtype=torch.bfloat16)
        self.attn_out = torch.empty(batch, hq, d, device=self.device, dtype=torch.bfloat16)
        self.attn_lse = torch.empty(batch, hq, device=self.device, dtype=torch.float32)
        self.graph = None

    # bytes one decode step must read: every weight matrix once (the embedding
    # gather is a few rows), the packed prompt of every layer and sequence,
    # and the live suffix rows.
    def weight_bytes(self) -> int:
        per_layer = sum(t.numel() * t.element_size() for t in self.w[0].values())
        return per_layer * self.layers + self.lm_head.numel() * 2 + self.final_norm.numel() * 2

    def cache_bytes(self, suffix_len: int) -> int:
        prompt = sum(p.bytes_per_step for p in self.plans)
        grown = self.layers * self.batch * self.hkv * self.d * 4 * suffix_len  # bf16 K and V rows
        capacity = self.layers * self.batch * self.hkv * self.d * 4 * self.capacity
        return prompt - capacity // 2 + grown  # the plans weight the suffix at half its capacity

    def step(self) -> torch.Tensor:
        """One greedy decode step of every sequence (device-only, capturable):
        returns the next token ids [batch]."""

        from . import kernels

        b, hq, hkv, d = self.batch, self.hq, self.hkv, self.d
        self.length += 1  # this step's token is row length - 1 of every suffix
        x = self.x
        for layer in range(self.layers):
            w = self.w[layer]
            h = kernels.rms_norm(x, w["in_norm"], self.eps)
            qkv = torch.addmm(w["qkv_bias"], h, w["qkv"])
            sk, sv = self.suffixes[layer]
            # rotary embedding, the query for the decode kernel, the key and
            # value appended to the suffix row the device-side length names
            kernels.qkv_rope_append(qkv, hq=hq, hkv=hkv, length=self.length, prompt=self.prompt,
                                    inv_freq=self.inv_freq, q_out=self.q_buf, suffix_k=sk, suffix_v=sv)
            self.plans[layer].run(self.q_buf, out=self.attn_out, lse=self.attn_lse)
            x = torch.addmm(x, self.attn_out.view(b, hq * d), w["o"])
            h = kernels.rms_norm(x, w["post_norm"], self.eps)
            x = torch.addmm(x, kernels.silu_mul(h @ w["gate_up"]), w["down"])
        logits = kernels.rms_norm(x, self.final_norm, self.eps) @ self.lm_head
        self.ids.copy_(torch.argmax(logits, dim=-1))
        self.x.copy_(self.embed[self.ids])
        return self.ids

    def capture(self) -> None:
        """Capture one decode step as a CUDA graph (after a first eager step has
        done every first-call set-up); ``replay`` then runs a step."""

        stream = torch.cuda.Stream(device=self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        self.graph = torch.cuda.CUDAGraph()
        saved = self.length.clone()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(self.graph, stream=stream):
                self.step()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        self.length.copy_(saved)  # capture does not run the step

    def replay(self) -> None:
        self.graph.replay()
