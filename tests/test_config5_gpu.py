"""BASELINE config 5 pieces on the GPU.

* A decode plan over [packed prompt + residual + growing dense suffix]: the
  suffix's live length is a device scalar, so one plan serves every step;
  after each length change the decode matches the float64 oracle over the
  live rows (max-abs 2e-2, mean-abs 1e-3).
* The Qwen2-shaped decoder of ``workloads.Qwen2PackedDecode`` at a reduced
  size: an eager step, a captured step and its replays agree, the suffix
  grows by one row per step, and layer 0's attention of a replayed step
  matches the oracle over that layer's cache.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention, kivi
from unicache_b200 import PackedKIVICache, kernels
from unicache_b200.kernels import GrowingSuffix, build_decode_plan
from unicache_b200.synthetic import make_kv, make_query

from .gpu_util import assert_attention_close, host, need_gpu

pytestmark = pytest.mark.gpu


def test_growing_suffix_plan_follows_the_live_length():
    need_gpu()
    heads, cap = 4, 64
    caches, refs, suffixes = [], [], []
    length = torch.zeros(1, device="cuda", dtype=torch.int32)
    for b in range(3):
        k, v = make_kv(700, heads, 128, seed=40 + b, device="cuda")
        packed = PackedKIVICache.from_dense(k, v, logical_token_ids=torch.arange(700, device="cuda"), token_type_id=0,
                                            k_bits=2, v_bits=2, group_size=32, residual_length=16)
        sk, sv = make_kv(cap, heads, 128, seed=50 + b, device="cuda")
        caches.append([packed, GrowingSuffix(sk, sv, length)])
        refs.append(kivi.packed_dequantize(kivi.packed_from_dense(host(k), host(v), "bfloat16", k_bits=2, v_bits=2,
                                                                   group_size=32, residual_length=16)))
        suffixes.append((host(sk), host(sv)))
    plan = build_decode_plan(caches, num_kv_heads=heads)
    query = make_query(3, 28, 128, seed=60, device="cuda")
    for live in (0, 1, 13, 64):
        length.fill_(live)
        out, lse = plan.run(query)
        torch.cuda.synchronize()
        for b in range(3):
            rk, rv = refs[b]
            keys = np.concatenate([rk, suffixes[b][0][:live]])
            vals = np.concatenate([rv, suffixes[b][1][:live]])
            e_out, e_lse = attention.attention_summary(host(query[b:b + 1]), keys, vals)
            assert_attention_close(out[b:b + 1], e_out, what=f"live {live}, sequence {b}")
            assert np.abs(host(lse[b]) - e_lse[:, 0]).max() <= 2e-2
    assert kernels.device_status() == 0


def test_qwen2_shaped_decode_steps_and_replays():
    need_gpu()
    from unicache_b200.workloads import Qwen2PackedDecode

    model = Qwen2PackedDecode("cuda", batch=4, prompt=1024, new_tokens=32, layers=2, seed=7)
    assert model.retained == 205
    model.step()  # eager: first-call set-up, suffix length 1
    torch.cuda.synchronize()
    assert int(model.length) == 1
    model.capture()
    assert int(model.length) == 1
    for _ in range(3):
        model.replay()
    torch.cuda.synchronize()
    assert int(model.length) == 4
    ids = model.ids.clone()
    assert bool(((ids >= 0) & (ids < 151936)).all())
    assert torch.isfinite(model.attn_out.float()).all()

    # layer 0's attention of the next step against the oracle over its cache
    length = int(model.length) + 1
    sk, sv = model.suffixes[0]
    x = model.x.clone()
    model.replay()
    torch.cuda.synchronize()
    w = model.w[0]
    h = _rms_norm_ref(x, w["in_norm"], model.eps)
    qkv = torch.addmm(w["qkv_bias"], h, w["qkv"])
    pos = torch.tensor([length - 1 + model.prompt], device="cuda", dtype=torch.float32)
    angle = pos * model.inv_freq
    q = _rope_ref(qkv[:, :28 * 128].view(4, 28, 128), torch.cos(angle), torch.sin(angle))
    for b in range(4):
        packed = model.packed[b]  # layer 0's caches are the first `batch` entries
        ref = packed.reference_layout()
        keys_p, vals_p = packed.dequantize(dtype=torch.bfloat16)
        keys = np.concatenate([host(keys_p), host(sk[b, :length])])
        vals = np.concatenate([host(vals_p), host(sv[b, :length])])
        e_out, _ = attention.attention_summary(host(q[b:b + 1]), keys, vals)
        del ref
        plan_out, _ = model.plans[0].run(q.contiguous())
        torch.cuda.synchronize()
        assert_attention_close(plan_out[b:b + 1], e_out, what=f"config-5 layer 0, sequence {b}")
    assert kernels.device_status() == 0


# torch fp32 references of the decoder's element-wise steps (Qwen2's RMSNorm,
# half-split rotary embedding and SwiGLU gate, rounding where torch rounds)
def _rms_norm_ref(x, weight, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * weight


def _rope_ref(x, cos, sin):
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


def _ulps_bf16(a, b):
    """Largest difference between two bf16 tensors in units of the larger value's last place."""

    a, b = a.float(), b.float()
    scale = torch.maximum(a.abs(), b.abs()).clamp_min(1e-30)
    ulp = torch.exp2(torch.floor(torch.log2(scale)) - 7)
    return float(((a - b).abs() / ulp).max())


def test_decoder_glue_kernels_match_torch_reference():
    need_gpu()
    gen = torch.Generator(device="cuda").manual_seed(11)
    x = (torch.randn(32, 3584, generator=gen, device="cuda") * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(3584, generator=gen, device="cuda")).to(torch.bfloat16)
    assert _ulps_bf16(kernels.rms_norm(x, w, 1e-6), _rms_norm_ref(x, w, 1e-6)) <= 1.0

    gu = torch.randn(32, 2 * 512, generator=gen, device="cuda").to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gu[:, :512]) * gu[:, 512:])
    assert _ulps_bf16(kernels.silu_mul(gu), ref) <= 1.0

    hq, hkv, d, cap, prompt = 28, 4, 128, 16, 1000
    qkv = torch.randn(32, (hq + 2 * hkv) * d, generator=gen, device="cuda").to(torch.bfloat16)
    inv_freq = 1.0 / (1000000.0 ** (torch.arange(d // 2, device="cuda", dtype=torch.float32) / (d // 2)))
    sk = torch.zeros(32, cap, hkv, d, device="cuda", dtype=torch.bfloat16)
    sv = torch.zeros_like(sk)
    q_out = torch.empty(32, hq, d, device="cuda", dtype=torch.bfloat16)
    length = torch.tensor([6], device="cuda", dtype=torch.int32)
    kernels.qkv_rope_append(qkv, hq=hq, hkv=hkv, length=length, prompt=prompt, inv_freq=inv_freq, q_out=q_out,
                            suffix_k=sk, suffix_v=sv)
    angle = torch.tensor([prompt + 5.0], device="cuda") * inv_freq
    cos, sin = torch.cos(angle), torch.sin(angle)
    assert _ulps_bf16(q_out, _rope_ref(qkv[:, :hq * d].view(32, hq, d), cos, sin)) <= 1.0
    k_ref = _rope_ref(qkv[:, hq * d:(hq + hkv) * d].view(32, hkv, d), cos, sin)
    assert _ulps_bf16(sk[:, 5], k_ref) <= 1.0
    assert torch.equal(sv[:, 5], qkv[:, (hq + hkv) * d:].view(32, hkv, d))
    others = torch.ones(cap, dtype=torch.bool)
    others[5] = False
    assert not sk[:, others].any() and not sv[:, others].any()
    assert kernels.device_status() == 0
    # a full suffix: the kernel's own bound check appends nothing and sets flag 2
    length.fill_(cap + 1)
    kernels.qkv_rope_append(qkv, hq=hq, hkv=hkv, length=length, prompt=prompt, inv_freq=inv_freq, q_out=q_out,
                            suffix_k=sk, suffix_v=sv)
    assert kernels.device_status() == 2
    assert not sk[:, others].any()
