"""Tensor-level wrappers over the C ABI (include/unicache_b200.h).

PyTorch only supplies device memory and the current CUDA stream; every
computation runs in ``libunicache_b200.so``.  All inputs must be CUDA tensors:
there is no CPU path, and a CPU tensor raises ``RuntimeError`` exactly like the
reference's fail-closed CUDA backend (unicache/storage/kivi_cuda.py:174-175,
242-243).
"""

from __future__ import annotations

import ctypes
import functools
import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _capi
from ._capi import UcbDecodeCta, UcbDecodePair, UcbSpan, call

_DTYPE_CODES = {torch.bfloat16: _capi.UCB_BF16, torch.float16: _capi.UCB_F16, torch.float32: _capi.UCB_F32}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected bfloat16, float16 or float32") from None


def require_cuda(tensor: torch.Tensor, name: str) -> None:
    if not isinstance(tensor, torch.Tensor) or tensor.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor: the b200 backend has no CPU path")


# The current stream's raw handle without building a torch Stream object
# (0.15 vs 2.25 us per call on the B200 hosts; torch's generated code reads
# it the same way), with the public call where that accessor is missing.
_current_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(tensor: torch.Tensor) -> int:
    if _current_raw_stream is not None:
        return _current_raw_stream(tensor.device.index)
    return torch.cuda.current_stream(tensor.device).cuda_stream


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def codes_per_word(bits: int) -> int:
    return 32 // bits


# ---------------------------------------------------------------- KIVI pack / dequant
def kivi_pack_key(key: torch.Tensor, *, bits: int, group_size: int):
    """Quantize and pack keys [T, H, D] along tokens -> b200 layout
    (codes [H, T/f, D] int32 or [H, T, D] uint8; scale/min [H, T/G, D])."""

    require_cuda(key, "key")
    if key.dim() != 3 or key.stride(2) != 1:
        raise ValueError("key must be [tokens, heads, head_dim] with unit channel stride")
    tokens, heads, head_dim = map(int, key.shape)
    if tokens % group_size:
        raise ValueError("key tokens must be a multiple of group_size")
    if bits == 8:
        codes = torch.empty((heads, tokens, head_dim), device=key.device, dtype=torch.uint8)
    else:
        codes = torch.empty((heads, tokens // codes_per_word(bits), head_dim), device=key.device, dtype=torch.int32)
    scale = torch.empty((heads, tokens // group_size, head_dim), device=key.device, dtype=key.dtype)
    minimum = torch.empty_like(scale)
    call("ucb_kivi_pack_key", key.data_ptr(), dtype_code(key.dtype), tokens, heads, head_dim,
         key.stride(0), key.stride(1), bits, group_size, codes.data_ptr(), scale.data_ptr(),
         minimum.data_ptr(), stream_of(key))
    return codes, scale, minimum


def kivi_pack_value(value: torch.Tensor, *, bits: int, group_size: int):
    """Quantize and pack values [T, H, D] along channels -> b200 layout
    (codes [H, T, D/f] int32 or [H, T, D] uint8; scale/min [H, T, D/G])."""

    require_cuda(value, "value")
    if value.dim() != 3 or value.stride(2) != 1:
        raise ValueError("value must be [tokens, heads, head_dim] with unit channel stride")
    tokens, heads, head_dim = map(int, value.shape)
    if head_dim % group_size:
        raise ValueError("value head_dim must be a multiple of group_size")
    if bits == 8:
        codes = torch.empty((heads, tokens, head_dim), device=value.device, dtype=torch.uint8)
    else:
        codes = torch.empty((heads, tokens, head_dim // codes_per_word(bits)), device=value.device, dtype=torch.int32)
    scale = torch.empty((heads, tokens, head_dim // group_size), device=value.device, dtype=value.dtype)
    minimum = torch.empty_like(scale)
    call("ucb_kivi_pack_value", value.data_ptr(), dtype_code(value.dtype), tokens, heads, head_dim,
         value.stride(0), value.stride(1), bits, group_size, codes.data_ptr(), scale.data_ptr(),
         minimum.data_ptr(), stream_of(value))
    return codes, scale, minimum


def kivi_pack_kv(key: torch.Tensor, value: torch.Tensor, *, k_bits: int, v_bits: int, group_size: int):
    """Quantize and pack keys and values [T, H, D] of one segment: (key codes,
    key scale, key min, value codes, value scale, value min) in the b200
    layout, identical to ``kivi_pack_key`` + ``kivi_pack_value``.  bf16 inputs
    with head_dim 128 and group 32 take one fused launch; other shapes the two
    separate kernels."""

    require_cuda(key, "key")
    require_cuda(value, "value")
    if key.shape != value.shape or key.dim() != 3 or key.stride(2) != 1 or value.stride(2) != 1:
        raise ValueError("key and value must be matching [tokens, heads, head_dim] with unit channel stride")
    tokens, heads, head_dim = map(int, key.shape)
    fused = (key.dtype == torch.bfloat16 and value.dtype == torch.bfloat16 and head_dim == 128 and group_size == 32
             and value.data_ptr() % 16 == 0 and value.stride(0) % 8 == 0 and value.stride(1) % 8 == 0
             and tokens > 0 and tokens % group_size == 0)
    if not fused:
        return (*kivi_pack_key(key, bits=k_bits, group_size=group_size),
                *kivi_pack_value(value, bits=v_bits, group_size=group_size))
    dev = key.device
    kc = (torch.empty((heads, tokens, head_dim), device=dev, dtype=torch.uint8) if k_bits == 8 else
          torch.empty((heads, tokens // codes_per_word(k_bits), head_dim), device=dev, dtype=torch.int32))
    vc = (torch.empty((heads, tokens, head_dim), device=dev, dtype=torch.uint8) if v_bits == 8 else
          torch.empty((heads, tokens, head_dim // codes_per_word(v_bits)), device=dev, dtype=torch.int32))
    ks = torch.empty((heads, tokens // group_size, head_dim), device=dev, dtype=key.dtype)
    km = torch.empty_like(ks)
    vs = torch.empty((heads, tokens, head_dim // group_size), device=dev, dtype=value.dtype)
    vm = torch.empty_like(vs)
    call("ucb_kivi_pack_kv", key.data_ptr(), value.data_ptr(), dtype_code(key.dtype), tokens, heads, head_dim,
         key.stride(0), key.stride(1), value.stride(0), value.stride(1), k_bits, v_bits, group_size,
         kc.data_ptr(), ks.data_ptr(), km.data_ptr(), vc.data_ptr(), vs.data_ptr(), vm.data_ptr(), stream_of(key))
    return kc, ks, km, vc, vs, vm


class KiviPackBatch:
    """``kivi_pack_kv`` of several segments (key, value [T_i, H, 128] bf16
    pairs, the same H) as one launch over a device job table.  The outputs
    and the table are allocated when the batch is built, so ``run`` is a
    single launch that a CUDA graph can capture; ``outputs`` holds one 6-tuple
    of b200-layout tensors per pair.  Pairs the fused kernel does not take
    (group other than 32, unaligned value rows) fall back to one
    ``kivi_pack_kv`` call each inside ``run``."""

    def __init__(self, pairs: list, *, k_bits: int, v_bits: int, group_size: int):
        if not pairs:
            raise ValueError("a pack batch needs at least one segment")
        self.pairs, self.k_bits, self.v_bits, self.group_size = pairs, k_bits, v_bits, group_size
        self.fused = group_size == 32 and all(
            k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16 and k.shape == v.shape and k.dim() == 3
            and int(k.shape[2]) == 128 and k.stride(2) == 1 and v.stride(2) == 1 and int(k.shape[0]) > 0
            and int(k.shape[0]) % 32 == 0 and v.data_ptr() % 16 == 0 and v.stride(0) % 8 == 0
            and v.stride(1) % 8 == 0 and k.is_cuda and k.device == pairs[0][0].device
            and int(k.shape[1]) == int(pairs[0][0].shape[1]) for k, v in pairs)
        self.outputs: list = []
        if not self.fused:
            return
        heads = int(pairs[0][0].shape[1])
        dev = pairs[0][0].device
        jobs, max_blocks = [], 0
        for key, value in pairs:
            tokens = int(key.shape[0])
            kc = (torch.empty((heads, tokens, 128), device=dev, dtype=torch.uint8) if k_bits == 8 else
                  torch.empty((heads, tokens // codes_per_word(k_bits), 128), device=dev, dtype=torch.int32))
            vc = (torch.empty((heads, tokens, 128), device=dev, dtype=torch.uint8) if v_bits == 8 else
                  torch.empty((heads, tokens, 128 // codes_per_word(v_bits)), device=dev, dtype=torch.int32))
            ks = torch.empty((heads, tokens // 32, 128), device=dev, dtype=torch.bfloat16)
            km = torch.empty_like(ks)
            vs = torch.empty((heads, tokens, 4), device=dev, dtype=torch.bfloat16)
            vm = torch.empty_like(vs)
            job = _capi.UcbPackJob()
            job.k = _capi.UcbPackSide(key.data_ptr(), key.stride(0), key.stride(1), kc.data_ptr(), ks.data_ptr(),
                                      km.data_ptr())
            job.v = _capi.UcbPackSide(value.data_ptr(), value.stride(0), value.stride(1), vc.data_ptr(),
                                      vs.data_ptr(), vm.data_ptr())
            job.tokens = tokens
            job.key_blocks = -(-(tokens // 32) * heads // 2)
            job.blocks = job.key_blocks + -(-tokens * heads * 4 // 256)
            max_blocks = max(max_blocks, job.blocks)
            jobs.append(job)
            self.outputs.append((kc, ks, km, vc, vs, vm))
        if int(_capi.load().ucb_kivi_pack_job_bytes()) != ctypes.sizeof(_capi.UcbPackJob):
            raise RuntimeError("pack job layout mismatch between the library and its binding")
        self.table = torch.frombuffer(bytearray(_capi.struct_array_bytes(jobs)), dtype=torch.uint8).to(dev)
        self.heads, self.max_blocks, self.jobs = heads, max_blocks, len(jobs)

    def run(self) -> list:
        if not self.fused:
            self.outputs = [kivi_pack_kv(k, v, k_bits=self.k_bits, v_bits=self.v_bits, group_size=self.group_size)
                            for k, v in self.pairs]
            return self.outputs
        call("ucb_kivi_pack_kv_batched", self.table.data_ptr(), self.jobs, self.max_blocks, self.heads, self.k_bits,
             self.v_bits, self.group_size, stream_of(self.pairs[0][0]))
        return self.outputs


def kivi_pack_kv_batch(pairs: list, *, k_bits: int, v_bits: int, group_size: int) -> list:
    """One-shot ``KiviPackBatch``: the packed 6-tuples of every (key, value) pair."""

    batch = KiviPackBatch(pairs, k_bits=k_bits, v_bits=v_bits, group_size=group_size)
    out = batch.run()
    for t in out:  # the job table must outlive the launch on its stream
        t[0].__dict__.setdefault("_ucb_pack_batch", batch)
    return out


def kivi_dequant(which: str, codes, scale, minimum, *, bits: int, group_size: int, quantized_tokens: int,
                 heads: int, head_dim: int, start: int, stop: int, out: torch.Tensor) -> torch.Tensor:
    """Dequantize tokens [start, stop) into ``out`` rows [0, stop-start) ([N, H, D] view)."""

    require_cuda(codes, "codes")
    require_cuda(out, "out")
    if out.dim() != 3 or out.stride(2) != 1 or tuple(out.shape[1:]) != (heads, head_dim):
        raise ValueError("dequantization output must be [tokens, heads, head_dim] with unit channel stride")
    if int(out.shape[0]) < stop - start:
        raise ValueError("dequantization output has too few rows")
    name = "ucb_kivi_dequant_key" if which == "key" else "ucb_kivi_dequant_value"
    call(name, codes.data_ptr(), scale.data_ptr(), minimum.data_ptr(), dtype_code(scale.dtype), quantized_tokens,
         heads, head_dim, bits, group_size, start, stop, out.data_ptr(), dtype_code(out.dtype), out.stride(0),
         out.stride(1), stream_of(out))
    return out


def fake_quant(data: torch.Tensor, *, bits: int, dim: int, group_size: int) -> torch.Tensor:
    """asymmetric_fake_quant (unicache/operators/builtin.py:31-53) on the GPU."""

    require_cuda(data, "data")
    if data.numel() == 0 or bits >= 16:
        return data
    if bits not in (2, 3, 4, 8):
        raise ValueError(f"Unsupported fake quant bits: {bits}")
    x = data.contiguous()
    dim = dim if dim >= 0 else x.dim() + dim
    outer = math.prod(x.shape[:dim])
    length = int(x.shape[dim])
    inner = math.prod(x.shape[dim + 1:])
    out = torch.empty_like(x)
    call("ucb_fake_quant", x.data_ptr(), out.data_ptr(), dtype_code(x.dtype), outer, length, inner, bits,
         int(group_size), stream_of(x))
    return out


# ---------------------------------------------------------------- LSE merge
def lse_merge(summaries: list[tuple[torch.Tensor, torch.Tensor]]):
    """merge_attention_summaries (unicache/adapters/bagel.py:57-72): summaries of
    (out [rows, heads, D], lse [heads, rows] fp32) -> merged (out, lse)."""

    if not summaries:
        raise ValueError("At least one attention summary is required")
    o0, _ = summaries[0]
    require_cuda(o0, "summary output")
    rows, heads, head_dim = map(int, o0.shape)
    outs, lses = [], []
    for o, lse in summaries:
        if tuple(o.shape) != (rows, heads, head_dim) or tuple(lse.shape) != (heads, rows):
            raise ValueError("attention summaries must share [rows, heads, head_dim] / [heads, rows] shapes")
        outs.append(o.to(o0.dtype).contiguous())
        lses.append(lse.float().contiguous())
    merged = torch.empty_like(outs[0])
    total = torch.empty((heads, rows), device=o0.device, dtype=torch.float32)
    n = len(outs)
    optrs = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
    lptrs = (ctypes.c_void_p * n)(*[l.data_ptr() for l in lses])
    call("ucb_lse_merge", n, optrs, lptrs, dtype_code(o0.dtype), rows, heads, head_dim, merged.data_ptr(),
         total.data_ptr(), stream_of(o0))
    return merged, total


# ---------------------------------------------------------------- H2O
def h2o_select(scores: torch.Tensor, *, history_end: int, heavy_k: int, recent: int) -> torch.Tensor:
    """Per-row heavy top-k (ascending indices) followed by the recent window
    (unicache/storage/physical.py:508-532).  scores: fp32 [H, T]."""

    require_cuda(scores, "scores")
    if scores.dim() != 2 or scores.dtype != torch.float32 or scores.stride(1) != 1:
        raise ValueError("scores must be float32 [heads, tokens] with unit token stride")
    heads, tokens = map(int, scores.shape)
    index = torch.empty((heads, heavy_k + recent), device=scores.device, dtype=torch.int64)
    call("ucb_h2o_select", scores.data_ptr(), scores.stride(0), heads, tokens, history_end, heavy_k, recent,
         index.data_ptr(), stream_of(scores))
    return index


def gather_rows(src: torch.Tensor, index: torch.Tensor, *, head_stride: int, token_stride: int,
                row_elems: int, out: torch.Tensor) -> torch.Tensor:
    """out[h, j, :] = src[h*head_stride + index[h, j]*token_stride : ... + row_elems]."""

    require_cuda(src, "src")
    heads, keep = map(int, index.shape)
    call("ucb_gather_rows", src.data_ptr(), head_stride, token_stride, row_elems, src.element_size(),
         index.data_ptr(), heads, keep, out.data_ptr(), stream_of(src))
    return out


def accumulate_probs(probs: torch.Tensor, kv_heads: int, scores: torch.Tensor | None = None) -> torch.Tensor:
    """Per-KV-head received attention (unicache/operators/physical.py:63-65):
    probs [Hq, Lq, N] -> [Hkv, N]; added into ``scores`` when given."""

    require_cuda(probs, "probabilities")
    if probs.dim() != 3:
        raise ValueError("H2O probabilities must be [query_heads, queries, tokens]")
    q_heads, queries, tokens = map(int, probs.shape)
    if q_heads % kv_heads:
        raise ValueError("Query heads must be divisible by KV heads for GQA H2O")
    probs = probs.contiguous()
    accumulate = scores is not None
    if scores is None:
        scores = torch.empty((kv_heads, tokens), device=probs.device, dtype=torch.float32)
    call("ucb_h2o_accumulate_probs", probs.data_ptr(), dtype_code(probs.dtype), q_heads, queries, tokens,
         kv_heads, scores.data_ptr(), int(accumulate), stream_of(probs))
    return scores


def h2o_scores(query: torch.Tensor, key: torch.Tensor, lse: torch.Tensor | None, *, kv_heads: int,
               softmax_scale: float, scores: torch.Tensor | None = None, head_major: bool = False) -> torch.Tensor:
    """Per-KV-head received attention without materialised probabilities
    (operators/physical.py:63-65 and storage/physical.py:598-610 reduce the
    softmax probabilities; here each probability is recomputed from the
    row's LSE): scores[kv, t] (+)= sum over the kv head's query heads h and
    queries i of exp(scale * q[i, h] . key[t, kv] - lse[h, i]).

    query [Lq, Hq, D] and key rows share a dtype (bf16: tensor cores; fp32:
    CUDA cores).  key is [N, Hkv, D] (token-major, any strides) or, with
    ``head_major``, [Hkv, N, D].  lse fp32 [Hq, Lq] (natural log) is the
    normaliser over every key of the attention; None means the attention
    covers exactly ``key`` and the LSE is computed first.  Adds into
    ``scores`` (fp32 [Hkv, N]) when it is given."""

    require_cuda(query, "query")
    require_cuda(key, "key")
    if query.dtype != key.dtype or query.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("H2O scoring takes bfloat16 or float32 query and keys of one dtype")
    q = query.contiguous()
    queries, q_heads, head_dim = map(int, q.shape)
    if head_major:
        tokens, stride_t, stride_h = int(key.shape[1]), key.stride(1), key.stride(0)
    else:
        tokens, stride_t, stride_h = int(key.shape[0]), key.stride(0), key.stride(1)
    if key.stride(-1) != 1 or int(key.shape[-1]) != head_dim:
        raise ValueError("key rows must have a unit channel stride and the query's head_dim")
    accumulate = scores is not None
    if scores is None:
        scores = torch.empty((kv_heads, tokens), device=q.device, dtype=torch.float32)
    elif scores.dtype != torch.float32 or tuple(scores.shape) != (kv_heads, tokens) or not scores.is_contiguous():
        raise ValueError("scores must be contiguous float32 [kv_heads, tokens]")
    workspace = None
    if lse is None:
        floats = int(_capi.load().ucb_h2o_scores_workspace_floats(queries, q_heads, tokens))
        workspace = torch.empty(floats, device=q.device, dtype=torch.float32)
    else:
        lse = lse.float().contiguous()
    call("ucb_h2o_scores", q.data_ptr(), dtype_code(q.dtype), queries, q_heads, key.data_ptr(), stride_t, stride_h,
         tokens, kv_heads, head_dim, ptr(lse), ptr(workspace), float(softmax_scale), scores.data_ptr(),
         int(accumulate), stream_of(q))
    return scores


def scores_from_lse(query: torch.Tensor, key: torch.Tensor, lse: torch.Tensor, *, kv_heads: int,
                    softmax_scale: float, scores: torch.Tensor | None = None) -> torch.Tensor:
    """``h2o_scores`` for token-major keys [N, Hkv, D] and a given LSE."""

    return h2o_scores(query, key, lse, kv_heads=kv_heads, softmax_scale=softmax_scale, scores=scores)


# ---------------------------------------------------------------- dense compaction
def compact_rows(src: torch.Tensor, mask: torch.Tensor, types: torch.Tensor | None = None):
    """Keep rows of ``src`` (first axis) where ``mask`` is true, in order."""

    require_cuda(src, "src")
    rows = int(src.shape[0])
    src = src.contiguous()
    m = mask.to(device=src.device, dtype=torch.uint8).contiguous()
    prefix = torch.empty(rows + 1, device=src.device, dtype=torch.int64)
    dst = torch.empty_like(src)
    types_out = None
    if types is not None:
        types = types.to(device=src.device, dtype=torch.int64).contiguous()
        types_out = torch.empty_like(types)
    kept = ctypes.c_int64(0)
    row_bytes = src[0].numel() * src.element_size() if rows else 1
    call("ucb_compact_rows", src.data_ptr(), row_bytes, m.data_ptr(), rows, ptr(types), dst.data_ptr(),
         ptr(types_out), prefix.data_ptr(), ctypes.byref(kept), stream_of(src))
    n = int(kept.value)
    return dst[:n], (types_out[:n] if types_out is not None else None)


# ---------------------------------------------------------------- decode attention
PACKED_STAGE = 64   # tokens per packed unit (decode kernel stage)
DENSE_STAGE = 8     # tokens per dense unit
MAX_PAIRS_PER_CTA = 4
MAX_SPANS_PER_CTA = 16
# Warp time model fitted to per-warp loop times on B200 (2-bit K/V, G32):
# a dense 8-token stage costs 0.55 of a full packed stage (0.83 per byte of a
# 2-bit packed stage) and entering a new segment costs 0.4 packed stages.
DENSE_UNIT_COST = 0.83
SEGMENT_SWITCH_STAGES = 0.4
# A unit past a growing suffix's live length copies and computes nothing but
# still passes through its warp's loop: about this fraction of a dense unit.
EMPTY_UNIT_COST = 0.1


@dataclass
class DenseRows:
    """A dense bf16 K/V span for one KV head: row i at base + i*stride.  With
    ``live`` (a device int32 scalar) the span is a growing suffix of capacity
    ``tokens`` whose first ``live`` rows are read."""

    key: torch.Tensor
    value: torch.Tensor
    key_offset: int
    value_offset: int
    key_stride: int
    value_stride: int
    tokens: int
    live: torch.Tensor | None = None


@dataclass
class DecodePlan:
    """Device tables of a decode batch over immutable (frozen) physical caches.

    Built once per cache layout and reused for every decode step: pairs are
    (sequence, KV head), spans are a pair's packed or dense token ranges, and
    CTA records give every persistent CTA an equal-bytes range of stage units
    (see include/unicache_b200.h).
    """

    device: torch.device
    num_seqs: int
    num_kv_heads: int
    head_dim: int
    k_bits: int
    v_bits: int
    group_size: int
    spans: torch.Tensor
    ctas: torch.Tensor
    warp_bounds: torch.Tensor
    pairs: torch.Tensor
    num_spans: int
    num_ctas: int
    num_pairs: int
    partials: torch.Tensor
    warp_slots: torch.Tensor
    num_partials: int = 0
    keepalive: list = field(default_factory=list)
    bytes_per_step: int = 0

    def launch(self, query_ptr: int, query_stride: int, q_heads: int, out_ptr: int, out_stride: int, lse_ptr: int,
               stream: int, softmax_scale: float | None = None) -> None:
        """Launch on raw device-visible addresses (device memory or mapped
        pinned host memory): query rows [B, q_heads, D] bf16 with row stride
        ``query_stride`` elements, out likewise, lse fp32 [B, q_heads] or 0."""

        scale = (1.0 / math.sqrt(self.head_dim)) if softmax_scale is None else float(softmax_scale)
        call("ucb_decode_attention", query_ptr, query_stride, q_heads, self.num_kv_heads, self.head_dim,
             self.spans.data_ptr(), self.num_spans, self.ctas.data_ptr(), self.num_ctas, self.warp_bounds.data_ptr(),
             self.pairs.data_ptr(), self.num_pairs, self.k_bits, self.v_bits, self.group_size, _capi.UCB_BF16,
             scale, self.partials.data_ptr(), self.warp_slots.data_ptr(), out_ptr, out_stride, lse_ptr or None,
             stream)

    def run(self, query: torch.Tensor, *, softmax_scale: float | None = None, out: torch.Tensor | None = None,
            lse: torch.Tensor | None = None):
        """query [B, Hq, D] bf16 -> (out [B, Hq, D] bf16, lse [B, Hq] fp32)."""

        require_cuda(query, "query")
        if query.dtype != torch.bfloat16:
            raise ValueError("decode attention expects a bfloat16 query")
        if query.dim() != 3 or int(query.shape[0]) != self.num_seqs or int(query.shape[2]) != self.head_dim:
            raise ValueError("query must be [num_seqs, q_heads, head_dim]")
        if query.stride(2) != 1 or query.stride(1) != self.head_dim:
            query = query.contiguous()
        q_heads = int(query.shape[1])
        if q_heads % self.num_kv_heads:
            raise ValueError("Query heads must be divisible by KV heads")
        scale = (1.0 / math.sqrt(self.head_dim)) if softmax_scale is None else float(softmax_scale)
        if out is None:
            out = torch.empty_like(query)
        if lse is None:
            lse = torch.empty((self.num_seqs, q_heads), device=query.device, dtype=torch.float32)
        call("ucb_decode_attention", query.data_ptr(), query.stride(0), q_heads, self.num_kv_heads,
             self.head_dim, self.spans.data_ptr(), self.num_spans, self.ctas.data_ptr(), self.num_ctas,
             self.warp_bounds.data_ptr(), self.pairs.data_ptr(), self.num_pairs, self.k_bits, self.v_bits,
             self.group_size, _capi.UCB_BF16,
             scale, self.partials.data_ptr(), self.warp_slots.data_ptr(), out.data_ptr(), out.stride(0),
             lse.data_ptr(), stream_of(query))
        return out, lse


def decode_config(k_bits: int, v_bits: int, group_size: int) -> tuple[int, int]:
    """(CTAs that run at once, warps per CTA) of the decode kernel on this device."""

    ctas = ctypes.c_int(0)
    warps = ctypes.c_int(0)
    call("ucb_decode_config", k_bits, v_bits, group_size, _capi.UCB_BF16, ctypes.byref(ctas), ctypes.byref(warps))
    return int(ctas.value), int(warps.value)


def _packed_span(cache, head: int) -> UcbSpan:
    sp = UcbSpan()
    sp.key_code = cache.key_code[head].data_ptr()
    sp.key_scale = cache.key_scale[head].data_ptr()
    sp.key_minimum = cache.key_minimum[head].data_ptr()
    sp.value_code = cache.value_code[head].data_ptr()
    sp.value_scale = cache.value_scale[head].data_ptr()
    sp.value_minimum = cache.value_minimum[head].data_ptr()
    sp.kind = 0
    sp.tokens = int(cache.quantized_tokens)
    return sp


def _dense_span(rows: DenseRows) -> UcbSpan:
    sp = UcbSpan()
    es = rows.key.element_size()
    sp.key_code = rows.key.data_ptr() + rows.key_offset * es
    sp.value_code = rows.value.data_ptr() + rows.value_offset * es
    sp.key_stride = rows.key_stride
    sp.value_stride = rows.value_stride
    sp.kind = 1
    sp.tokens = rows.tokens
    if rows.live is not None:
        if not rows.live.is_cuda or rows.live.dtype != torch.int32 or rows.live.numel() != 1:
            raise ValueError("a growing span's live length must be a CUDA int32 scalar")
        sp.key_scale = rows.live.data_ptr()
    for name, base, off, stride in (("key", rows.key, rows.key_offset, rows.key_stride),
                                    ("value", rows.value, rows.value_offset, rows.value_stride)):
        if base.dtype != torch.bfloat16:
            raise ValueError(f"dense {name} rows must be bfloat16")
        if base.stride(-1) != 1:
            raise ValueError(f"dense {name} rows must have a unit channel stride")
        if (base.data_ptr() + off * es) % 16 or (stride * es) % 16:
            raise ValueError(f"dense {name} rows must start on 16-byte boundaries")
    return sp


def dense_rows_token_major(key: torch.Tensor, value: torch.Tensor, head: int,
                           live: torch.Tensor | None = None) -> DenseRows:
    """[N, H, D] tensors (dense cache, KIVI residual, or a growing suffix of
    capacity N whose live length is the device scalar ``live``)."""

    return DenseRows(key, value, head * key.stride(1), head * value.stride(1), key.stride(0), value.stride(0),
                     int(key.shape[0]), live)


@dataclass
class GrowingSuffix:
    """Dense bf16 rows appended one decode step at a time: key/value
    [capacity, H, D] and the device int32 ``length``; a decode plan reads the
    first ``length`` rows (the reference appends decode tokens to its dense
    cache, unicache/adapters/bagel.py:1199-1297)."""

    key: torch.Tensor
    value: torch.Tensor
    length: torch.Tensor


def dense_rows_head_major(key: torch.Tensor, value: torch.Tensor, head: int) -> DenseRows:
    """[H, N, D] tensors (compacted H2O segment)."""

    return DenseRows(key, value, head * key.stride(0), head * value.stride(0), key.stride(1), value.stride(1),
                     int(key.shape[1]))


def packed_bytes_per_token(k_bits: int, v_bits: int, group_size: int, head_dim: int, stat_bytes: int = 2) -> float:
    return head_dim * (k_bits + v_bits) / 8 + 2 * stat_bytes * head_dim / group_size * 2


def _split_warps(weights: list[float], segs: list[int], u0: int, u1: int, warps: int) -> list[int] | None:
    """Cut [u0, u1) into ``warps`` contiguous ranges of about equal weight, each
    crossing at most one segment boundary; None if that is impossible."""

    total = sum(weights[u0:u1])
    bounds = [u0]
    u, acc = u0, 0.0
    for w in range(warps - 1):
        target = total * (w + 1) / warps
        start, crossed = u, 0
        while u < u1 and acc + weights[u] / 2 <= target:
            if u > start and segs[u] != segs[u - 1]:
                if crossed:
                    break
                crossed = 1
            acc += weights[u]
            u += 1
        bounds.append(u)
    bounds.append(u1)
    last = bounds[-2]
    if sum(1 for k in range(last + 1, u1) if segs[k] != segs[k - 1]) > 1:
        return None
    return bounds


def _assign_ctas(unit_weights: list[float], unit_pair: list[int], unit_seg: list[int], num_ctas: int,
                 warps: int, unit_span: list[int] | None = None) -> list[list[int]]:
    """Cut the unit sequence into about ``num_ctas`` contiguous ranges of equal
    weight, each touching at most MAX_PAIRS_PER_CTA pairs, and split every range
    into per-warp bounds.  Returns one bounds list (warps + 1 entries) per CTA."""

    total = sum(unit_weights)
    n = len(unit_weights)
    ranges = []
    u, acc = 0, 0.0
    for c in range(num_ctas):
        if u >= n:
            break
        target = total * (c + 1) / num_ctas
        begin = u
        pairs = {unit_pair[u]}
        acc += unit_weights[u]
        u += 1
        while u < n and acc + unit_weights[u] / 2 <= target:
            if unit_pair[u] not in pairs and len(pairs) == MAX_PAIRS_PER_CTA:
                break
            pairs.add(unit_pair[u])
            acc += unit_weights[u]
            u += 1
        ranges.append((begin, u))
    while u < n:  # leftovers, only when the pair cap cut ranges short
        begin, pairs = u, set()
        while u < n and (unit_pair[u] in pairs or len(pairs) < MAX_PAIRS_PER_CTA):
            pairs.add(unit_pair[u])
            u += 1
        ranges.append((begin, u))
    out = []
    stack = list(reversed(ranges))
    while stack:
        u0, u1 = stack.pop()
        too_many_spans = unit_span is not None and unit_span[u1 - 1] - unit_span[u0] + 1 > MAX_SPANS_PER_CTA
        bounds = None if too_many_spans else _split_warps(unit_weights, unit_seg, u0, u1, warps)
        if bounds is None:
            mid = (u0 + u1) // 2
            stack.append((mid, u1))
            stack.append((u0, mid))
            continue
        out.append(bounds)
    return out


def build_decode_plan(sequences: list[list], *, num_kv_heads: int, head_dim: int = 128,
                      target_ctas: int | None = None) -> DecodePlan:
    """Build device tables for decode over ``sequences``: one list of segments
    per sequence, each segment a b200 ``PackedKIVICache`` (its residual rides
    along as a dense span), a ``GQAH2OCache`` or a ``(key, value)`` pair of dense
    [N, H, D] bf16 tensors."""

    from .storage.physical import GQAH2OCache, PackedKIVICache

    spans: list[UcbSpan] = []
    span_bytes: list[float] = []
    growing: set[int] = set()  # spans that are growing suffixes
    keepalive: list = []
    pairs_info: list[tuple[int, int]] = []
    cfg = None
    device = None

    def add(sp: UcbSpan, pair: int, nbytes: float):
        sp.pair = pair
        spans.append(sp)
        span_bytes.append(nbytes)

    for b, segments in enumerate(sequences):
        for h in range(num_kv_heads):
            pair = len(pairs_info)
            pairs_info.append((b, h))
            for seg in segments:
                if isinstance(seg, PackedKIVICache):
                    if seg.backend != "b200":
                        raise ValueError("decode plans need b200-layout packed segments")
                    if seg.quantized_tokens:
                        key = (seg.k_bits, seg.v_bits, seg.group_size, seg.key_scale.dtype)
                        if cfg is None:
                            cfg = key
                        elif cfg != key:
                            raise ValueError("all packed segments of a decode plan must share bits, group and dtype")
                        if seg.k_bits == 8 or seg.v_bits == 8:
                            raise ValueError("8-bit packed segments are not supported by the decode kernel")
                        if seg.head_dim != head_dim:
                            raise ValueError("packed segment head_dim mismatch")
                        add(_packed_span(seg, h), pair, seg.quantized_tokens * packed_bytes_per_token(
                            seg.k_bits, seg.v_bits, seg.group_size, head_dim))
                        keepalive.append(seg)
                        device = seg.key_code.device
                    if int(seg.residual_key.shape[0]):
                        rows = dense_rows_token_major(seg.residual_key, seg.residual_value, h)
                        add(_dense_span(rows), pair, rows.tokens * head_dim * 4)
                        keepalive.append(seg)
                        device = seg.residual_key.device
                elif isinstance(seg, GQAH2OCache):
                    rows = dense_rows_head_major(seg.key, seg.value, h)
                    add(_dense_span(rows), pair, rows.tokens * head_dim * 4)
                    keepalive.append(seg)
                    device = seg.key.device
                elif isinstance(seg, GrowingSuffix):
                    rows = dense_rows_token_major(seg.key, seg.value, h, seg.length)
                    # counted at half its capacity (its average fill over a decode run);
                    # its units are weighted by how often each is live (below)
                    add(_dense_span(rows), pair, rows.tokens * head_dim * 4 * 0.5)
                    growing.add(len(spans) - 1)
                    keepalive.append(seg)
                    device = seg.key.device
                else:
                    key, value = seg
                    if int(key.shape[0]) == 0:
                        continue
                    rows = dense_rows_token_major(key, value, h)
                    add(_dense_span(rows), pair, rows.tokens * head_dim * 4)
                    keepalive.append((key, value))
                    device = key.device
    if device is None:
        raise ValueError("decode plan has no tokens")
    k_bits, v_bits, group, stat_dtype = cfg if cfg is not None else (2, 2, 64, torch.bfloat16)
    if stat_dtype != torch.bfloat16:
        raise ValueError("the decode kernel reads bfloat16 packed statistics")
    covered = {sp.pair for sp in spans}
    for p, (b, h) in enumerate(pairs_info):
        if p not in covered:
            raise ValueError(f"sequence {b} has no tokens for KV head {h}")

    # Units: 64-token packed stages and 8-token dense stages, in span order; a
    # segment is a run of units with the same (pair, kind).
    unit_weights: list[float] = []
    unit_pair: list[int] = []
    unit_seg: list[int] = []
    unit_span: list[int] = []
    seg_id, last_key = -1, None
    packed_stage_bytes = packed_bytes_per_token(k_bits, v_bits, group, head_dim) * PACKED_STAGE
    for s, sp in enumerate(spans):
        stage = PACKED_STAGE if sp.kind == 0 else DENSE_STAGE
        units = math.ceil(sp.tokens / stage)
        sp.unit_begin = len(unit_weights)
        new_segment = (sp.pair, sp.kind) != last_key
        if new_segment:
            seg_id += 1
            last_key = (sp.pair, sp.kind)
        per_token = span_bytes[s] / sp.tokens
        # Weights are time estimates in bytes of packed stream (see the model
        # above DENSE_UNIT_COST).
        cost = 1.0 if sp.kind == 0 else DENSE_UNIT_COST
        for k in range(units):
            n = min(stage, sp.tokens - k * stage)
            w = per_token * n * cost
            if s in growing:
                # unit k is live over the last (capacity - first row) / capacity
                # of the decode steps: weight it by that share (live units sit at
                # the suffix's front, so a uniform weight would overload the warps
                # that hold them), plus the pass of an empty unit
                live = (sp.tokens - k * stage) / sp.tokens
                full = (head_dim * 4) * n * cost
                w = full * (live + (1.0 - live) * EMPTY_UNIT_COST)
            if k == 0 and new_segment:
                w += SEGMENT_SWITCH_STAGES * packed_stage_bytes
            unit_weights.append(w)
            unit_pair.append(sp.pair)
            unit_seg.append(seg_id)
            unit_span.append(s)
    with torch.cuda.device(device):
        slots, warps = decode_config(k_bits, v_bits, group)
    if target_ctas is None:
        # every SM for a full-size batch; a small problem gets about one unit
        # per warp (fewer CTAs plan faster and leave fewer states to merge)
        target_ctas = min(slots, max(1, -(-len(unit_weights) // warps)))
    cta_bounds = _assign_ctas(unit_weights, unit_pair, unit_seg, target_ctas, warps, unit_span)

    span_starts = [sp.unit_begin for sp in spans]
    ctas: list[UcbDecodeCta] = []
    touched: dict[int, list[int]] = {}
    flat_bounds: list[int] = []
    for c, bounds in enumerate(cta_bounds):
        u0, u1 = bounds[0], bounds[-1]
        flat_bounds.extend(bounds)
        rec = UcbDecodeCta()
        rec.unit_begin, rec.unit_end = u0, u1
        rec.span_begin = unit_span[u0]
        rec.reserved[0] = unit_span[u1 - 1] + 1
        p0, p1 = unit_pair[u0], unit_pair[u1 - 1]
        rec.pair_begin, rec.num_pairs = p0, p1 - p0 + 1
        if rec.num_pairs > MAX_PAIRS_PER_CTA:
            raise AssertionError("decode planner produced a CTA range over too many pairs")
        ctas.append(rec)
        for p in range(p0, p1 + 1):
            touched.setdefault(p, []).append(c)
    # Warp states: a warp writes one state per segment it processed (its first
    # segment only when it crosses a boundary, its last segment always).  The
    # slots of a pair are contiguous, in CTA and warp order.
    states_by_pair: dict[int, list[int]] = {}
    warp_slots = [-1] * (2 * warps * len(cta_bounds))
    for c, bounds in enumerate(cta_bounds):
        for w in range(warps):
            a, b = bounds[w], bounds[w + 1]
            if a == b:
                continue
            if unit_seg[a] != unit_seg[b - 1]:
                states_by_pair.setdefault(unit_pair[a], []).append(2 * (c * warps + w))
            states_by_pair.setdefault(unit_pair[b - 1], []).append(2 * (c * warps + w) + 1)
    pairs: list[UcbDecodePair] = []
    partial_total = 0
    for p, (b, h) in enumerate(pairs_info):
        cs = touched[p]
        if cs != list(range(cs[0], cs[0] + len(cs))):
            raise AssertionError("CTAs of a pair must be consecutive")
        pr = UcbDecodePair()
        pr.seq, pr.kv_head = b, h
        pr.partial_begin, pr.cta_first = partial_total, cs[0]
        for idx in states_by_pair.get(p, []):
            warp_slots[idx] = partial_total
            partial_total += 1
        pr.partial_count = partial_total - pr.partial_begin
        if pr.partial_count == 0:
            raise AssertionError("every pair needs at least one warp state")
        pairs.append(pr)

    # the five tables in one host -> device copy, each at a 256-byte offset
    parts = [_capi.struct_array_bytes(spans), _capi.struct_array_bytes(ctas),
             np.asarray(flat_bounds, dtype=np.int32).tobytes(), _capi.struct_array_bytes(pairs),
             np.asarray(warp_slots, dtype=np.int32).tobytes()]
    offsets, total = [], 0
    for raw in parts:
        offsets.append(total)
        total += -(-len(raw) // 256) * 256
    blob = bytearray(total)
    for off, raw in zip(offsets, parts):
        blob[off:off + len(raw)] = raw
    dev_blob = torch.frombuffer(blob, dtype=torch.uint8).to(device)
    table = [dev_blob[off:off + len(raw)] for off, raw in zip(offsets, parts)]

    partial_bytes = int(_capi.load().ucb_decode_partial_bytes(head_dim))
    return DecodePlan(
        device=device,
        num_seqs=len(sequences),
        num_kv_heads=num_kv_heads,
        head_dim=head_dim,
        k_bits=k_bits,
        v_bits=v_bits,
        group_size=group,
        spans=table[0],
        ctas=table[1],
        warp_bounds=table[2].view(torch.int32),
        pairs=table[3],
        num_spans=len(spans),
        num_ctas=len(ctas),
        num_pairs=len(pairs),
        partials=torch.empty(partial_total * partial_bytes, device=device, dtype=torch.uint8),
        warp_slots=table[4].view(torch.int32),
        num_partials=partial_total,
        keepalive=keepalive,
        bytes_per_step=int(sum(span_bytes)),
    )


# ---------------------------------------------------------------- long-query attention
def prefill_attention(q: torch.Tensor, k: torch.Tensor, vt: torch.Tensor, n_tokens: int, *,
                      softmax_scale: float | None = None, out: torch.Tensor | None = None,
                      lse: torch.Tensor | None = None):
    """Non-causal attention per KV head on the tcgen05 tensor cores.

    q [H, M, 128] bf16, k [H, Np, 128] bf16, vt [H, 128, Np] bf16 with
    Np >= n_tokens a multiple of 8 and finite padding -> (out [H, M, 128] bf16,
    lse [H, M] fp32, natural log)."""

    for name, t in (("q", q), ("k", k), ("vt", vt)):
        require_cuda(t, name)
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.dim() != 3:
            raise ValueError(f"{name} must be a contiguous 3-D bfloat16 tensor")
    heads, m_rows, d = map(int, q.shape)
    n_padded = int(k.shape[1])
    if d != 128 or tuple(k.shape) != (heads, n_padded, d) or tuple(vt.shape) != (heads, d, n_padded):
        raise ValueError("prefill attention expects q [H,M,128], k [H,Np,128], vt [H,128,Np]")
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((heads, m_rows), device=q.device, dtype=torch.float32)
    split = _key_split_launch(q.device, heads, m_rows, int(n_tokens), n_padded, stream_of(q))
    if split is None:
        call("ucb_prefill_attention", q.data_ptr(), k.data_ptr(), vt.data_ptr(), heads, m_rows, int(n_tokens),
             n_padded, scale, out.data_ptr(), lse.data_ptr(), stream_of(q))
    else:
        items, partials, flags = split
        call("ucb_prefill_attention_items", q.data_ptr(), k.data_ptr(), vt.data_ptr(), heads, m_rows, n_padded,
             items.data_ptr(), int(items.shape[0]), scale, out.data_ptr(), lse.data_ptr(), partials.data_ptr(),
             flags.data_ptr(), stream_of(q))
    return out, lse



# ------------------------------------------------------------------ decoder glue (configuration 5)
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of bf16 rows [rows, hidden]: bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight)."""

    require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or x.dim() != 2 or not x.is_contiguous():
        raise ValueError("rms_norm takes contiguous bfloat16 [rows, hidden] rows and a bfloat16 weight")
    out = torch.empty_like(x) if out is None else out
    call("ucb_rms_norm", x.data_ptr(), weight.data_ptr(), int(x.shape[0]), int(x.shape[1]), float(eps),
         out.data_ptr(), stream_of(x))
    return out


def qkv_rope_append(qkv: torch.Tensor, *, hq: int, hkv: int, length: torch.Tensor, prompt: int,
                    inv_freq: torch.Tensor, q_out: torch.Tensor, suffix_k: torch.Tensor,
                    suffix_v: torch.Tensor) -> torch.Tensor:
    """Rotary embedding of the new token's query and key heads at position
    prompt + length - 1 (``length`` a device int32 [1]); the query goes to
    ``q_out`` [batch, hq, d], the key and value heads to row length - 1 of
    the dense suffixes [batch, capacity, hkv, d]."""

    for name, t in (("qkv", qkv), ("q_out", q_out), ("suffix_k", suffix_k), ("suffix_v", suffix_v)):
        require_cuda(t, name)
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous bfloat16 tensor")
    batch, capacity, _, d = map(int, suffix_k.shape)
    if tuple(qkv.shape) != (batch, (hq + 2 * hkv) * d) or tuple(q_out.shape) != (batch, hq, d) or \
            tuple(suffix_v.shape) != tuple(suffix_k.shape) or int(suffix_k.shape[2]) != hkv:
        raise ValueError("qkv, q_out and the suffixes disagree in shape")
    if length.dtype != torch.int32 or inv_freq.dtype != torch.float32 or int(inv_freq.numel()) != d // 2:
        raise ValueError("length must be int32 and inv_freq float32 [head_dim / 2]")
    call("ucb_qkv_rope_append", qkv.data_ptr(), batch, hq, hkv, d, length.data_ptr(), int(prompt),
         inv_freq.data_ptr(), q_out.data_ptr(), suffix_k.data_ptr(), suffix_v.data_ptr(), capacity, stream_of(qkv))
    return q_out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """SwiGLU gate of [rows, 2 * ffn] bf16: bf16(bf16(silu(gate)) * up) [rows, ffn]."""

    require_cuda(gate_up, "gate_up")
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or not gate_up.is_contiguous() or gate_up.shape[1] % 2:
        raise ValueError("silu_mul takes contiguous bfloat16 [rows, 2 * ffn]")
    rows, ffn = int(gate_up.shape[0]), int(gate_up.shape[1]) // 2
    out = torch.empty(rows, ffn, device=gate_up.device, dtype=gate_up.dtype) if out is None else out
    call("ucb_silu_mul", gate_up.data_ptr(), rows, ffn, out.data_ptr(), stream_of(gate_up))
    return out

PREFILL_ROWS_PER_CTA = 256
PREFILL_KEY_TILE = 128
_KEY_SPLITS: dict = {}


PREFILL_CTA_FIXED_TILES = 4.0  # a CTA's set-up, pipeline fill and epilogue, in key-tile times (measured)


@functools.lru_cache(maxsize=4096)
def plan_key_split(row_blocks: int, key_tiles: int, sms: int) -> int | None:
    """Key tiles of the first part when splitting every row block's keys in
    two fills the GPU better than one CTA per row block, else None.

    With R < SMs row blocks of T key tiles, one CTA each leaves SMs idle for
    its whole F + T tile times (F: a CTA's fixed cost, about 4 tile times on
    B200).  Split, the R first parts (L tiles) start at once and the R second
    parts (T - L tiles) run on the SMs - R others in ceil(R / (SMs - R))
    rounds; the first parts then merge their partner's result (about half a
    tile).  The plan minimises max(F + L + 1/2, rounds * (F + T - L)) and is
    kept only if it saves at least one tile time."""

    free = sms - row_blocks
    if free <= 0 or key_tiles < 2 or row_blocks <= 0:
        return None
    rounds = -(-row_blocks // free)
    fixed = PREFILL_CTA_FIXED_TILES
    whole = fixed + key_tiles
    best_l, best = None, whole
    for first in range(1, key_tiles):
        cost = max(fixed + first + 0.5, rounds * (fixed + key_tiles - first))
        if cost < best:
            best, best_l = cost, first
    return best_l if best_l is not None and best <= whole - 1 else None


_KEY_SPLITS_MAX = 64  # item tables kept; the workspace itself is shared per (device, stream)


def _key_split_launch(device, heads: int, m_rows: int, n_tokens: int, n_padded: int, stream: int):
    """(items, partials, flags) of a key-split launch, or None.

    Only the item table (a few hundred bytes) is cached per shape, and at most
    ``_KEY_SPLITS_MAX`` of them; partials and flags come from the per-(device,
    stream) workspace of ``prefill_split_workspace``, which only grows to the
    largest row-block count seen, so a session whose key count changes every
    call does not accumulate device memory."""

    key = (device.index, heads, m_rows, n_tokens, n_padded)
    if key in _KEY_SPLITS:
        items = _KEY_SPLITS[key]
    else:
        blocks_per_head = -(-m_rows // PREFILL_ROWS_PER_CTA)
        row_blocks = heads * blocks_per_head
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        first = plan_key_split(row_blocks, -(-n_tokens // PREFILL_KEY_TILE), sms)
        items = None
        if first is not None:
            split_at = first * PREFILL_KEY_TILE
            merge_items, partial_items = [], []
            for h in range(heads):
                for b in range(blocks_per_head):
                    slot = len(merge_items)
                    q0 = b * PREFILL_ROWS_PER_CTA
                    rows = min(PREFILL_ROWS_PER_CTA, m_rows - q0)
                    merge_items.append([h, q0, rows, 0, split_at, 2, slot, 0])
                    partial_items.append([h, q0, rows, split_at, n_tokens - split_at, 1, slot, 0])
            items = torch.tensor(merge_items + partial_items, dtype=torch.int32).to(device)
        if len(_KEY_SPLITS) >= _KEY_SPLITS_MAX:
            _KEY_SPLITS.pop(next(iter(_KEY_SPLITS)))
        _KEY_SPLITS[key] = items
    if items is None:
        return None
    partials, flags = prefill_split_workspace(device, int(items.shape[0]) // 2, stream)
    return items, partials, flags


def split_prefill_items(items: list, sms: int) -> tuple[list, int]:
    """Item rows (head, q_row0, q_rows, k_row0, n_tokens, 0, 0, ...; any
    further columns, such as a segment-table item's span range, are kept)
    with each row block's keys split in two where ``plan_key_split`` says it pays
    (fewer row blocks than SMs): the first parts as merge items (mode 2)
    first, then the unsplit items, then the second parts as partial items
    (mode 1), slot i shared by the i-th pair.  Returns (rows, slots)."""

    if len(items) >= sms:
        return [list(r) for r in items], 0
    merges, whole, partials = [], [], []
    for row in items:
        row = [int(x) for x in row]
        k0, n = row[3], row[4]
        first = plan_key_split(len(items), -(-n // PREFILL_KEY_TILE), sms)
        if first is None:
            whole.append(row[:5] + [0, 0] + row[7:])
            continue
        cut = first * PREFILL_KEY_TILE
        slot = len(merges)
        merges.append(row[:3] + [k0, cut, 2, slot] + row[7:])
        partials.append(row[:3] + [k0 + cut, n - cut, 1, slot] + row[7:])
    return merges + whole + partials, len(merges)


PERSIST_MIN_TILES = 6  # smallest share of key tiles a persistent CTA is given (fewer, larger pieces:
#                        a merge item folds its partials in with chains of L2 loads)


def plan_stream_k(blocks: list, sms: int, min_tiles: int = PERSIST_MIN_TILES) -> tuple[list, list, int]:
    """Split the (row block, key tile) units of ``blocks`` (segment-table
    item rows, one per row block: head, q_row0, q_rows, k_row0 = 0, n_tokens,
    0, 0, span_begin, span_count, pos0, ws_row0, 0) into at most ``sms``
    contiguous ranges of equal size, one per persistent CTA.  A row block
    that a range boundary cuts becomes pieces: its first piece a merge item
    (mode 2; the last item of its CTA) folding in the others, partial items
    (mode 1; each the first item of its CTA) in consecutive slots [slot, slot
    + reserved[1]).  Returns (item rows, cta_items offsets, slots)."""

    tiles = [-(-int(b[4]) // PREFILL_KEY_TILE) for b in blocks]
    total = sum(tiles)
    if total == 0:
        raise ValueError("every row block needs at least one key")
    ctas = max(1, min(sms, total // max(1, min_tiles)))
    cuts = [(c * total) // ctas for c in range(ctas + 1)]
    starts, acc = [], 0
    for t in tiles:
        starts.append(acc)
        acc += t
    pieces = [[] for _ in blocks]      # per block: [item index, tile_begin, tile_end]
    order = []                         # item index -> (block, piece number)
    offsets = [0]
    b = 0
    for c in range(ctas):
        lo, hi = cuts[c], cuts[c + 1]
        while b < len(blocks) and starts[b] + tiles[b] <= lo:
            b += 1
        bb = b
        while bb < len(blocks) and starts[bb] < hi:
            t0, t1 = max(lo, starts[bb]) - starts[bb], min(hi, starts[bb] + tiles[bb]) - starts[bb]
            if t1 > t0:
                pieces[bb].append([len(order), t0, t1])
                order.append((bb, len(pieces[bb]) - 1))
            bb += 1
        offsets.append(len(order))
    rows, slots = [None] * len(order), 0
    for bi, plist in enumerate(pieces):
        blk = [int(x) for x in blocks[bi]]
        tokens = blk[4]
        first_slot = slots
        if len(plist) > 1:
            slots += len(plist) - 1
        for pi, (idx, t0, t1) in enumerate(plist):
            k0 = t0 * PREFILL_KEY_TILE
            n = min(tokens, t1 * PREFILL_KEY_TILE) - k0
            if len(plist) == 1:
                mode, slot, nparts = 0, 0, 0
            elif pi == 0:
                mode, slot, nparts = 2, first_slot, len(plist) - 1
            else:
                mode, slot, nparts = 1, first_slot + pi - 1, 0
            rows[idx] = blk[:3] + [k0, n, mode, slot] + blk[7:11] + [nparts]
    return rows, offsets, slots


_SPLIT_WORKSPACES: dict = {}
_RETIRED_WORKSPACES: list = []  # outgrown workspaces stay alive: a captured CUDA graph may still use them


def prefill_split_workspace(device, slots: int, stream: int):
    """(partials, flags) for ``slots`` split row blocks, cached per device and
    stream.  Every launch leaves each flag even (each split item adds 1), so
    one workspace serves every later launch on that stream."""

    key = (device.index, stream)
    ws = _SPLIT_WORKSPACES.get(key)
    if ws is None or int(ws[1].numel()) < slots:
        if ws is not None:
            _RETIRED_WORKSPACES.append(ws)
        slot_floats = int(_capi.load().ucb_prefill_partial_bytes()) // 4
        ws = (torch.empty(slots * slot_floats, device=device, dtype=torch.float32),
              torch.zeros(slots, device=device, dtype=torch.int32))
        _SPLIT_WORKSPACES[key] = ws
    return ws


def prefill_attention_batched(q: torch.Tensor, k: torch.Tensor, vt: torch.Tensor, items: torch.Tensor, *,
                              softmax_scale: float | None = None, out: torch.Tensor | None = None,
                              lse: torch.Tensor | None = None, split_workspace=None):
    """One launch over several non-causal attention problems sharing the
    tensors q [H, M, 128], k [H, Np, 128], vt [H, 128, Np] (bf16):
    ``items`` is an int32 device tensor [num_items, 8] of (head, q_row0,
    q_rows <= 256, k_row0 (multiple of 64), n_tokens, mode, slot, 0), one per
    CTA; items of modes 1 and 2 (see ``split_prefill_items``) need
    ``split_workspace`` = (partials, flags).  Returns (out [H, M, 128] bf16,
    lse [H, M] fp32); rows no item covers are left unwritten."""

    for name, t in (("q", q), ("k", k), ("vt", vt), ("items", items)):
        require_cuda(t, name)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or vt.dtype != torch.bfloat16:
        raise ValueError("q, k and vt must be bfloat16")
    if items.dtype != torch.int32 or items.dim() != 2 or int(items.shape[1]) != 8:
        raise ValueError("items must be int32 [num_items, 8]")
    heads, m_rows, d = map(int, q.shape)
    n_padded = int(k.shape[1])
    if d != 128 or tuple(k.shape) != (heads, n_padded, d) or tuple(vt.shape) != (heads, d, n_padded):
        raise ValueError("batched prefill expects q [H,M,128], k [H,Np,128], vt [H,128,Np]")
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty((heads, m_rows), device=q.device, dtype=torch.float32)
    if split_workspace is None:
        call("ucb_prefill_attention_batched", q.data_ptr(), k.data_ptr(), vt.data_ptr(), heads, m_rows, n_padded,
             items.data_ptr(), int(items.shape[0]), scale, out.data_ptr(), lse.data_ptr(), stream_of(q))
    else:
        partials, flags = split_workspace
        call("ucb_prefill_attention_items", q.data_ptr(), k.data_ptr(), vt.data_ptr(), heads, m_rows, n_padded,
             items.data_ptr(), int(items.shape[0]), scale, out.data_ptr(), lse.data_ptr(), partials.data_ptr(),
             flags.data_ptr(), stream_of(q))
    return out, lse


# ---------------------------------------------------------------- host transfers
def host_device_pointer(host: torch.Tensor) -> int:
    """Device-visible address of a pinned host tensor (mapped pinned memory)."""

    if host.is_cuda or not host.is_pinned():
        raise ValueError("expected a pinned host tensor")
    dev = ctypes.c_void_p()
    call("ucb_host_device_pointer", host.data_ptr(), ctypes.byref(dev))
    return int(dev.value)


def copy_ranges(ranges: list[tuple[int, int, int]], stream: int) -> None:
    """One kernel copies every (dst, src, nbytes) range between device-visible
    addresses (device memory or mapped pinned host memory), 16-byte aligned."""

    n = len(ranges)
    dst = (ctypes.c_void_p * n)(*[r[0] for r in ranges])
    src = (ctypes.c_void_p * n)(*[r[1] for r in ranges])
    size = (ctypes.c_int64 * n)(*[int(r[2]) for r in ranges])
    call("ucb_copy_ranges", n, dst, src, size, stream)


def device_status(device: torch.device | None = None) -> int:
    flags = ctypes.c_uint(0)
    stream = torch.cuda.current_stream(device).cuda_stream
    call("ucb_device_status", ctypes.byref(flags), stream)
    return int(flags.value)


def selftest_mma_subnormal() -> float:
    err = ctypes.c_float(-1.0)
    call("ucb_selftest_mma_subnormal", ctypes.byref(err), torch.cuda.current_stream().cuda_stream)
    return float(err.value)


# ---------------------------------------------------------------- long-query over spans
LQ_ITEM_INTS = 12  # ucb_lq_item


@dataclass
class LongQueryTables:
    """Device tables of a segment-table long-query launch: the spans every KV
    head of every sample reads in place, and one item per CTA."""

    spans: torch.Tensor         # ucb_span structs (raw bytes)
    items: torch.Tensor         # int32 [num_items, 12]
    num_spans: int
    num_items: int
    k_bits: int
    v_bits: int
    group_size: int
    slots: int                  # key-split slots (partials/flags) the items use
    jobs: torch.Tensor | None = None  # int32 [num_jobs, 8] ucb_lq_stage_job: one per (sample, KV head) key space
    p_items: torch.Tensor | None = None  # persistent staged launch: item rows (plan_stream_k)
    p_ctas: torch.Tensor | None = None   # int32 [num_ctas + 1] item offsets per CTA
    num_p_items: int = 0
    num_ctas: int = 0
    p_slots: int = 0
    num_jobs: int = 0
    max_chunks: int = 0         # 64-token staging blocks of the largest key space
    ws_rows: int = 0            # staging workspace rows per KV head (samples at 128-aligned bases)
    row_blocks: int = 0         # row blocks (items before key splits) per key space, at most
    keepalive: list = field(default_factory=list)


def long_query_spans(segments: list, num_kv_heads: int, head: int, include_residual: bool = True):
    """The spans of one KV head of one sample: (list of UcbSpan with
    ``unit_begin`` = first token, tokens, (k_bits, v_bits, group) of its
    packed spans or None, objects to keep alive).  Packed spans come first,
    then the dense, H2O and residual rows in segment order: attention does not
    depend on the order of its keys, and a key split hands the last key tiles
    of a row block to the CTAs that run in several rounds, so those should be
    the cheap dense tiles rather than the tiles restored from codes."""

    from .storage.physical import GQAH2OCache, PackedKIVICache

    packed, dense, keep, cfg = [], [], [], None

    def add(sp):
        sp.pair = 0
        (packed if sp.kind == 0 else dense).append(sp)

    for seg in segments:
        if isinstance(seg, PackedKIVICache):
            if seg.backend != "b200":
                raise ValueError("long-query spans need b200-layout packed segments")
            if seg.quantized_tokens:
                if seg.k_bits not in (2, 4) or seg.v_bits not in (2, 4):
                    raise ValueError("the long-query kernel reads 2- or 4-bit packed segments")
                if seg.key_scale.dtype != torch.bfloat16 or seg.head_dim != 128:
                    raise ValueError("the long-query kernel reads bf16 statistics and head_dim 128")
                this = (seg.k_bits, seg.v_bits, seg.group_size)
                if cfg is not None and cfg != this:
                    raise ValueError("all packed segments of a long-query launch must share bits and group")
                cfg = this
                add(_packed_span(seg, head))
            if include_residual and int(seg.residual_key.shape[0]):
                add(_dense_span(dense_rows_token_major(seg.residual_key, seg.residual_value, head)))
            keep.append(seg)
        elif isinstance(seg, GQAH2OCache):
            if seg.retained_tokens:
                add(_dense_span(dense_rows_head_major(seg.key, seg.value, head)))
            keep.append(seg)
        else:
            key, value = seg
            if int(key.shape[0]):
                add(_dense_span(dense_rows_token_major(key, value, head)))
            keep.append((key, value))
    spans, t0 = packed + dense, 0
    for sp in spans:
        sp.unit_begin = t0
        t0 += int(sp.tokens)
    return spans, t0, cfg, keep


@functools.lru_cache(maxsize=64)
def _sm_count(index: int) -> int:
    return torch.cuda.get_device_properties(index).multi_processor_count


def _segment_signature(seg) -> tuple:
    """Everything a span table records about a segment: its identity, the
    addresses and strides of its tensors and its token counts."""

    from .storage.physical import GQAH2OCache, PackedKIVICache

    if isinstance(seg, PackedKIVICache):
        packed = (seg.key_code.data_ptr(), seg.value_code.data_ptr()) if seg.quantized_tokens else (0, 0)
        return (id(seg), *packed, seg.quantized_tokens,
                seg.residual_key.data_ptr(), seg.residual_value.data_ptr(), int(seg.residual_key.shape[0]),
                tuple(seg.residual_key.stride()), tuple(seg.residual_value.stride()), seg.k_bits, seg.v_bits,
                seg.group_size)
    if isinstance(seg, GQAH2OCache):
        return (id(seg), seg.key.data_ptr(), seg.value.data_ptr(), tuple(seg.key.shape), tuple(seg.key.stride()),
                tuple(seg.value.stride()))
    key, value = seg
    return (key.data_ptr(), value.data_ptr(), tuple(key.shape), tuple(key.stride()), tuple(value.stride()),
            key.dtype, value.dtype)


_LQ_BY_SIGNATURE: dict = {}


def long_query_tables(samples: list, num_kv_heads: int, pos0: list, q_rows: list, device,
                      include_residual: bool = True) -> LongQueryTables:
    """Segment-table launch tables for several samples: sample i's queries are
    positions [pos0[i], pos0[i] + q_rows[i] / grp) of the launch's query
    tensor (q_rows[i] = its positions x query heads per KV head), its keys the
    concatenation of its segments.  Tables are cached
    on the segments' signatures (identity, addresses, strides, lengths), so a
    layer called again over the same frozen segments costs a dictionary
    lookup on the host."""

    index = torch.device(device).index
    signature = (index, num_kv_heads, bool(include_residual), tuple(pos0), tuple(q_rows),
                 tuple(tuple(_segment_signature(seg) for seg in segs) for segs in samples))
    hit = _LQ_BY_SIGNATURE.get(signature)
    if hit is not None:
        return hit
    tables = _build_long_query_tables(samples, num_kv_heads, pos0, q_rows, device, include_residual)
    if len(_LQ_BY_SIGNATURE) >= _LQ_TABLES_MAX:
        _LQ_BY_SIGNATURE.pop(next(iter(_LQ_BY_SIGNATURE)))
    _LQ_BY_SIGNATURE[signature] = tables
    return tables


def _build_long_query_tables(samples: list, num_kv_heads: int, pos0: list, q_rows: list, device,
                             include_residual: bool) -> LongQueryTables:
    all_spans, rows, jobs, cfg, base, row_blocks = [], [], [], None, 0, 0
    for segs, p0, nrows in zip(samples, pos0, q_rows):
        extent = 0
        for h in range(num_kv_heads):
            spans, tokens, this, _ = long_query_spans(segs, num_kv_heads, h, include_residual)
            if tokens == 0:
                raise ValueError("every sample needs at least one key token")
            if this is not None:
                if cfg is not None and cfg != this:
                    raise ValueError("all packed segments of a long-query launch must share bits and group")
                cfg = this
            begin = len(all_spans)
            all_spans.extend(spans)
            padded = -(-tokens // PREFILL_KEY_TILE) * PREFILL_KEY_TILE
            extent = max(extent, padded)
            # staging job: this key space at workspace rows [base, base + padded) of head h
            jobs.append([h, begin, len(spans), tokens, base, padded, 0, 0])
            blocks = 0
            for r in range(0, nrows, PREFILL_ROWS_PER_CTA):
                rows.append([h, r, min(PREFILL_ROWS_PER_CTA, nrows - r), 0, tokens, 0, 0, begin, len(spans),
                             p0, base, 0])
                blocks += 1
            row_blocks = max(row_blocks, blocks)
        base += extent
    sms = _sm_count(torch.device(device).index)
    p_rows, p_offsets, p_slots = plan_stream_k(rows, sms, PERSIST_MIN_TILES)
    rows, slots = split_prefill_items(rows, sms)
    k_bits, v_bits, group = cfg if cfg is not None else (2, 2, 32)
    raw = _capi.struct_array_bytes(all_spans)
    # Device tables are reused while the spans (addresses, strides, lengths)
    # and items are the same, so a layer called again over the same segments
    # uploads nothing.
    key = (torch.device(device).index, raw, tuple(tuple(r) for r in rows), tuple(tuple(j) for j in jobs),
           tuple(tuple(r) for r in p_rows), tuple(p_offsets))
    cached = _LQ_TABLES.get(key)
    if cached is None:
        spans_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)
        items_dev = torch.tensor(rows, dtype=torch.int32).to(device)
        jobs_dev = torch.tensor(jobs, dtype=torch.int32).to(device)
        p_items_dev = torch.tensor(p_rows, dtype=torch.int32).to(device)
        p_ctas_dev = torch.tensor(p_offsets, dtype=torch.int32).to(device)
        if len(_LQ_TABLES) >= _LQ_TABLES_MAX:
            _LQ_TABLES.pop(next(iter(_LQ_TABLES)))
        cached = _LQ_TABLES[key] = (spans_dev, items_dev, jobs_dev, p_items_dev, p_ctas_dev)
    # The tables hold addresses only: the caller keeps the segments alive for
    # the launch, and a cached entry whose tensors were freed is never stale
    # in content, because its signature records every address it holds.
    max_rows = max(j[5] for j in jobs)
    return LongQueryTables(cached[0], cached[1], len(all_spans), len(rows), k_bits, v_bits, group, slots,
                           jobs=cached[2], num_jobs=len(jobs), max_chunks=max_rows // LQ_STAGE_TOKENS,
                           ws_rows=base, row_blocks=row_blocks, p_items=cached[3], p_ctas=cached[4],
                           num_p_items=len(p_rows), num_ctas=len(p_offsets) - 1, p_slots=p_slots)


_LQ_TABLES: dict = {}
_LQ_TABLES_MAX = 64


LQ_STAGE_TOKENS = 32          # tokens per staging block (ucb_long_query_stage)
LQ_STAGE_MIN_ROW_BLOCKS = 1   # stage the keys when at least this many row blocks read each key space
# (measured on the configuration-4 segment mix, CUDA graphs: staged 45-70 us
# against 64-100 us in place from 8 to 1024 query positions, so always)


def long_query_stage(tables: LongQueryTables, num_kv_heads: int, device, stream=None):
    """Gather every key space of ``tables`` into a bf16 workspace (K rows
    [num_kv_heads, ws_rows, 128], V transposed [num_kv_heads, 128, ws_rows]):
    dense spans copied, packed spans restored as in the kernel's tiles."""

    k_ws = torch.empty((num_kv_heads, tables.ws_rows, 128), device=device, dtype=torch.bfloat16)
    vt_ws = torch.empty((num_kv_heads, 128, tables.ws_rows), device=device, dtype=torch.bfloat16)
    call("ucb_long_query_stage", tables.spans.data_ptr(), tables.num_spans, tables.jobs.data_ptr(), tables.num_jobs,
         tables.max_chunks, tables.k_bits, tables.v_bits, tables.group_size, k_ws.data_ptr(), vt_ws.data_ptr(),
         tables.ws_rows, stream if stream is not None else stream_of(k_ws))
    return k_ws, vt_ws


def long_query_attention(query: torch.Tensor, tables: LongQueryTables, *, num_kv_heads: int,
                         softmax_scale: float | None = None, out: torch.Tensor | None = None,
                         lse: torch.Tensor | None = None, staged: bool | None = None,
                         persistent: bool = True):
    """Non-causal attention of query [positions, Hq, 128] (bf16, the caller's
    layout) over the spans of ``tables``: (out [positions, Hq, 128] bf16, lse
    [Hq, positions] fp32 natural log); positions no item covers are left
    unwritten.

    ``staged=False`` reads the spans in place (packed KIVI tiles restored in
    shared memory by every row block); ``staged=True`` first gathers each key
    space once into a bf16 workspace (``ucb_long_query_stage``) and streams it
    by TMA, which is faster once several row blocks read the same keys;
    ``None`` stages when every key space has at least
    ``LQ_STAGE_MIN_ROW_BLOCKS`` row blocks.  A staged launch is persistent
    by default: at most one CTA per SM, each running an equal contiguous
    share of the (row block, key tile) units (``plan_stream_k``);
    ``persistent=False`` runs one CTA per row block (or per key-split part)."""

    require_cuda(query, "query")
    if query.dtype != torch.bfloat16 or not query.is_contiguous() or query.dim() != 3 or int(query.shape[2]) != 128:
        raise ValueError("query must be a contiguous bfloat16 [positions, q_heads, 128] tensor")
    positions, q_heads, d = map(int, query.shape)
    if q_heads % num_kv_heads:
        raise ValueError("Query heads must be divisible by KV heads")
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    if out is None:
        out = torch.empty_like(query)
    if lse is None:
        lse = torch.empty((q_heads, positions), device=query.device, dtype=torch.float32)
    if staged is None:
        staged = tables.jobs is not None and tables.row_blocks >= LQ_STAGE_MIN_ROW_BLOCKS
    persistent = bool(staged and persistent and tables.p_items is not None)
    slots = tables.p_slots if persistent else tables.slots
    partials = flags = None
    if slots:
        partials, flags = prefill_split_workspace(query.device, slots, stream_of(query))
    if staged:
        if tables.jobs is None:
            raise ValueError("these tables carry no staging jobs")
        k_ws = torch.empty((num_kv_heads, tables.ws_rows, 128), device=query.device, dtype=torch.bfloat16)
        vt_ws = torch.empty((num_kv_heads, 128, tables.ws_rows), device=query.device, dtype=torch.bfloat16)
        items, n_items = (tables.p_items, tables.num_p_items) if persistent else (tables.items, tables.num_items)
        call("ucb_long_query_attention_staged", query.data_ptr(), positions, q_heads, num_kv_heads,
             items.data_ptr(), n_items, tables.p_ctas.data_ptr() if persistent else None,
             tables.num_ctas if persistent else 0, tables.spans.data_ptr(), tables.num_spans,
             tables.jobs.data_ptr(), tables.num_jobs, tables.max_chunks, tables.k_bits, tables.v_bits,
             tables.group_size, scale, k_ws.data_ptr(), vt_ws.data_ptr(), tables.ws_rows, out.data_ptr(),
             lse.data_ptr(), ptr(partials), ptr(flags), stream_of(query))
        return out, lse
    call("ucb_long_query_attention", query.data_ptr(), positions, q_heads, num_kv_heads, tables.items.data_ptr(),
         tables.num_items, tables.spans.data_ptr(), tables.num_spans, tables.k_bits, tables.v_bits,
         tables.group_size, scale, out.data_ptr(), lse.data_ptr(), ptr(partials), ptr(flags), stream_of(query))
    return out, lse
