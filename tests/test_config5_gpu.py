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
    from unicache_b200.workloads import _rms_norm

    h = _rms_norm(x, w["in_norm"], model.eps)
    qkv = torch.addmm(w["qkv_bias"], h, w["qkv"])
    pos = torch.tensor([length - 1 + model.prompt], device="cuda", dtype=torch.float32)
    angle = pos * model.inv_freq
    q = model._rope(qkv[:, :28 * 128].view(4, 28, 128), torch.cos(angle), torch.sin(angle))
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
