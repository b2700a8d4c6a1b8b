"""Decoder-only LLM oracle on the CPU -- TEST INFRASTRUCTURE ONLY.

A restatement, in PyTorch CPU ops, of the reference's whole-model oracle
``workloads/pytorch/decoder_llm.py`` (reference project) with the exact storage
rounding points of that module:

- RMSNorm in fp32, result cast to the storage dtype (decoder_llm.py:8-16);
- interleaved RoPE in fp32 with fp32 cos/sin tables, cast back (decoder_llm.py:19-31);
- attention: fp32 scores / sqrt(D), causal mask, fp32 softmax, fp32
  probabilities x values, context cast to storage (decoder_llm.py:61-90);
- SwiGLU MLP on storage-dtype linears (decoder_llm.py:93-101);
- pre-norm residual blocks (decoder_llm.py:104-118), LM head + greedy argmax on
  the storage-dtype logits (export_decoder_llm.py:538-549).

Extensions the reference lacks, each reducing to it exactly when unused:
- grouped-query attention: ``kv_heads`` < ``heads``; query head h reads KV head
  h // (heads // kv_heads) (the reference rejects GQA, export_decoder_llm.py:217-218);
- ``rope_theta`` for random-init models (the reference hard-codes 10000 unless a
  Llama checkpoint supplies it, decoder_llm.py:48-55, export_decoder_llm.py:420-431);
- batch > 1 with independent per-sequence caches and positions (the exporter
  rejects batch != 1, export_decoder_llm.py:367-368).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline import it.
"""

from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F


@dataclass
class DecoderSpec:
    hidden: int
    heads: int
    kv_heads: int
    intermediate: int
    vocab: int
    layers: int
    capacity: int
    epsilon: float = 1e-5
    rope_theta: float = 10000.0
    dtype: torch.dtype = torch.float16

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def rope_tables(capacity: int, head_dim: int, theta: float):
    """fp32 cos/sin tables [capacity, head_dim/2] (decoder_llm.py:48-55)."""
    positions = torch.arange(capacity, dtype=torch.float32).unsqueeze(1)
    frequencies = torch.exp(torch.arange(0, head_dim, 2, dtype=torch.float32)
                            * (-math.log(theta) / head_dim))
    angles = positions * frequencies.unsqueeze(0)
    return torch.cos(angles), torch.sin(angles)


def _rms_norm(value, weight, eps):
    scale = torch.rsqrt(value.float().pow(2).mean(dim=-1, keepdim=True) + eps)
    return (value.float() * scale * weight.float()).to(value.dtype)


def _rope(value, cosine, sine, positions):
    # value [B, H, S, D]; positions [B, S] absolute positions.
    cos = cosine[positions].unsqueeze(1)  # [B, 1, S, D/2]
    sin = sine[positions].unsqueeze(1)
    even = value[..., 0::2].float()
    odd = value[..., 1::2].float()
    rotated = torch.stack((even * cos - odd * sin, even * sin + odd * cos), dim=-1)
    return rotated.flatten(-2).to(value.dtype)


@dataclass
class DecoderOracle:
    """Stateful oracle: weights by the reference manifest names, KV caches per sequence."""

    spec: DecoderSpec
    weights: dict
    rope_cos: torch.Tensor | None = None
    rope_sin: torch.Tensor | None = None
    caches: dict = field(default_factory=dict)  # seq -> list[(K [Hkv,L,D], V)] per layer
    # When set, every linear layer sums its inputs in a fixed permuted order:
    # mathematically the same model, a different fp32 summation order. The
    # spread between two such oracles is the order-of-operations noise floor
    # that any other correct implementation (e.g. a GPU kernel) also shows.
    summation_order_seed: int | None = None

    def __post_init__(self):
        dt = self.spec.dtype
        self.w = {k: torch.as_tensor(np.asarray(v, dtype=np.float32)).to(dt) for k, v in self.weights.items()
                  if not k.startswith("rope.")}
        if self.rope_cos is None:
            self.rope_cos, self.rope_sin = rope_tables(self.spec.capacity, self.spec.head_dim,
                                                       self.spec.rope_theta)

    def _linear(self, x, weight):
        if self.summation_order_seed is None:
            return F.linear(x, weight)
        k = weight.shape[1]
        perm = torch.from_numpy(np.random.default_rng(self.summation_order_seed + k).permutation(k))
        return F.linear(x[..., perm], weight[:, perm])

    def fork(self, summation_order_seed=None, caches=None):
        """A new oracle over the same weight tensors (shared, not copied) with
        its own caches (a shallow copy of `caches`, else empty) and summation
        order -- full-width models hold gigabytes of weights."""
        other = copy.copy(self)
        other.caches = dict(caches) if caches is not None else {}
        other.summation_order_seed = summation_order_seed
        return other

    def length(self, seq) -> int:
        c = self.caches.get(seq)
        return 0 if c is None else c[0][0].shape[1]

    @torch.no_grad()
    def forward(self, seq, token_ids):
        """Run S new tokens of one sequence (prefill if its cache is empty).
        Returns (logits [S, vocab] in storage dtype, next token int)."""
        s = self.spec
        dt = s.dtype
        ids = torch.as_tensor(np.asarray(token_ids, dtype=np.int64)).view(1, -1)
        S = ids.shape[1]
        past = self.caches.get(seq)
        start = self.length(seq)
        if start + S > s.capacity:
            raise ValueError("decoder KV cache capacity exceeded")
        positions = torch.arange(start, start + S).view(1, S)
        x = F.embedding(ids, self.w["embedding.weight"])
        new_cache = []
        D = s.head_dim
        for layer in range(s.layers):
            p = f"layer{layer}."
            h = _rms_norm(x, self.w[p + "input_norm.weight"], s.epsilon)
            q = self._linear(h, self.w[p + "q.weight"]).view(1, S, s.heads, D).transpose(1, 2)
            k = self._linear(h, self.w[p + "k.weight"]).view(1, S, s.kv_heads, D).transpose(1, 2)
            v = self._linear(h, self.w[p + "v.weight"]).view(1, S, s.kv_heads, D).transpose(1, 2)
            q = _rope(q, self.rope_cos, self.rope_sin, positions)
            k = _rope(k, self.rope_cos, self.rope_sin, positions)
            if past is not None:
                k = torch.cat((past[layer][0].unsqueeze(0), k), dim=2)
                v = torch.cat((past[layer][1].unsqueeze(0), v), dim=2)
            new_cache.append((k[0], v[0]))
            ctx = causal_gqa_attention(q, k, v, start).to(dt)
            ctx = ctx.transpose(1, 2).contiguous().view(1, S, -1)
            x = x + self._linear(ctx, self.w[p + "o.weight"])
            h = _rms_norm(x, self.w[p + "post_norm.weight"], s.epsilon)
            mlp = self._linear(F.silu(self._linear(h, self.w[p + "gate.weight"])) * self._linear(h, self.w[p + "up.weight"]),
                           self.w[p + "down.weight"])
            x = x + mlp
        logits = self._linear(_rms_norm(x, self.w["final_norm.weight"], s.epsilon), self.w["lm_head.weight"])
        self.caches[seq] = new_cache
        nxt = int(logits[0, -1].argmax().item())
        return logits[0], nxt


def causal_gqa_attention(q, k, v, start: int):
    """The decoder's attention (decoder_llm.py's scaled-dot-product step with the
    GQA head map): q [1, Hq, S, D] for positions start..start+S-1, k / v
    [1, Hkv, L, D] for positions 0..L-1; fp32 scores / sqrt(D), causal mask, fp32
    softmax, fp32 context [1, Hq, S, D] (the caller rounds it to storage)."""
    S, D = q.shape[2], q.shape[3]
    group = q.shape[1] // k.shape[1]
    kk = k.repeat_interleave(group, dim=1) if group > 1 else k
    vv = v.repeat_interleave(group, dim=1) if group > 1 else v
    scores = torch.matmul(q.float(), kk.float().transpose(-2, -1)) / math.sqrt(D)
    qpos = torch.arange(start, start + S).view(S, 1)
    kpos = torch.arange(kk.size(2)).view(1, -1)
    scores = scores.masked_fill(kpos > qpos, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, vv.float())


def spec_from_golden(meta: dict, kv_heads=None, rope_theta=10000.0) -> DecoderSpec:
    return DecoderSpec(hidden=meta["hidden_size"], heads=meta["heads"],
                       kv_heads=kv_heads or meta["heads"], intermediate=meta["intermediate_size"],
                       vocab=meta["vocabulary_size"], layers=meta["layers"],
                       capacity=meta["capacity"], epsilon=meta["epsilon"], rope_theta=rope_theta)


WEIGHT_KINDS = ("input_norm", "q", "k", "v", "o", "post_norm", "gate", "up", "down")


def weight_names(layers: int):
    names = ["embedding.weight", "final_norm.weight", "lm_head.weight"]
    for layer in range(layers):
        names += [f"layer{layer}.{k}.weight" for k in WEIGHT_KINDS]
    return names


def random_weights(spec: DecoderSpec, seed: int, std: float = 0.02) -> dict:
    """Seeded N(0, std) matrices (fp16-rounded), unit norms -- host-side small models."""
    rng = np.random.default_rng(seed)
    H, D, I, V = spec.hidden, spec.head_dim, spec.intermediate, spec.vocab

    def mat(r, c):
        return (rng.standard_normal((r, c), dtype=np.float32) * np.float32(std)).astype(np.float16)

    w = {"embedding.weight": mat(V, H), "final_norm.weight": np.ones(H, np.float16),
         "lm_head.weight": mat(V, H)}
    for layer in range(spec.layers):
        p = f"layer{layer}."
        w[p + "input_norm.weight"] = np.ones(H, np.float16)
        w[p + "post_norm.weight"] = np.ones(H, np.float16)
        w[p + "q.weight"] = mat(spec.heads * D, H)
        w[p + "k.weight"] = mat(spec.kv_heads * D, H)
        w[p + "v.weight"] = mat(spec.kv_heads * D, H)
        w[p + "o.weight"] = mat(H, spec.heads * D)
        w[p + "gate.weight"] = mat(I, H)
        w[p + "up.weight"] = mat(I, H)
        w[p + "down.weight"] = mat(H, I)
    return w


def argmax_key(values: torch.Tensor, offset: int) -> torch.Tensor:
    """Orderable int64 key per row of `values` [S, n] (fp16/fp32): the larger
    value wins, then the smaller global index (offset + column) -- the tie rule
    of emitTokenArgmax (TransformerDecodeMetalEmitter.cpp:198-257) and of
    torch.argmax on the reference's fp16 logits. A max-reduction of keys over
    vocab shards therefore equals argmax over the whole vocabulary."""
    bits = values.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    negative = (bits >> 31) == 1
    ordered = torch.where(negative, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    idx = offset + torch.arange(values.shape[-1], dtype=torch.int64)
    keys = (ordered << 31) | (0x7FFFFFFF - idx)
    return keys.max(dim=-1).values


def argmax_key_index(key: torch.Tensor) -> torch.Tensor:
    return 0x7FFFFFFF - (key & 0x7FFFFFFF)


@dataclass
class TensorParallelOracle(DecoderOracle):
    """One rank of the tensor-parallel decomposition the device decoder uses:
    column-parallel Q/K/V (whole heads per rank; the GQA group of a KV head
    stays on one rank), gate and up; row-parallel O and down whose fp32 partial
    sums are summed over ranks (`all_reduce_sum`) before the storage rounding
    and the residual add; vocab-parallel LM head whose greedy token comes from
    a max-reduction of packed (value, index) keys (`all_reduce_max`). Rank r
    owns the r-th contiguous slice of every split dimension. Not in the
    reference (it has no multi-GPU code); with world = 1 it is DecoderOracle."""

    rank: int = 0
    world: int = 1
    all_reduce_sum: object = None  # callable(torch.float32 tensor) -> summed tensor
    all_reduce_max: object = None  # callable(torch.int64 tensor) -> max tensor

    def _rows(self, w, parts):
        n = w.shape[0] // parts
        return w[self.rank * n:(self.rank + 1) * n]

    def _cols(self, w, parts):
        n = w.shape[1] // parts
        return w[:, self.rank * n:(self.rank + 1) * n]

    @torch.no_grad()
    def forward(self, seq, token_ids):
        """Returns (local logits [S, vocab / world] in storage dtype, next token)."""
        s = self.spec
        dt = s.dtype
        W = self.world
        hq, hkv, D = s.heads // W, s.kv_heads // W, s.head_dim
        ids = torch.as_tensor(np.asarray(token_ids, dtype=np.int64)).view(1, -1)
        S = ids.shape[1]
        past = self.caches.get(seq)
        start = self.length(seq)
        if start + S > s.capacity:
            raise ValueError("decoder KV cache capacity exceeded")
        positions = torch.arange(start, start + S).view(1, S)
        x = F.embedding(ids, self.w["embedding.weight"])
        group = s.heads // s.kv_heads
        new_cache = []
        for layer in range(s.layers):
            p = f"layer{layer}."
            h = _rms_norm(x, self.w[p + "input_norm.weight"], s.epsilon)
            q = F.linear(h, self._rows(self.w[p + "q.weight"], W)).view(1, S, hq, D).transpose(1, 2)
            k = F.linear(h, self._rows(self.w[p + "k.weight"], W)).view(1, S, hkv, D).transpose(1, 2)
            v = F.linear(h, self._rows(self.w[p + "v.weight"], W)).view(1, S, hkv, D).transpose(1, 2)
            q = _rope(q, self.rope_cos, self.rope_sin, positions)
            k = _rope(k, self.rope_cos, self.rope_sin, positions)
            if past is not None:
                k = torch.cat((past[layer][0].unsqueeze(0), k), dim=2)
                v = torch.cat((past[layer][1].unsqueeze(0), v), dim=2)
            new_cache.append((k[0], v[0]))
            kk = k.repeat_interleave(group, dim=1) if group > 1 else k
            vv = v.repeat_interleave(group, dim=1) if group > 1 else v
            scores = torch.matmul(q.float(), kk.float().transpose(-2, -1)) / math.sqrt(D)
            qpos = torch.arange(start, start + S).view(S, 1)
            kpos = torch.arange(kk.size(2)).view(1, -1)
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
            ctx = torch.matmul(torch.softmax(scores, dim=-1), vv.float()).to(dt)
            ctx = ctx.transpose(1, 2).contiguous().view(1, S, -1)
            partial = F.linear(ctx.float(), self._cols(self.w[p + "o.weight"], W).float())
            x = x + self.all_reduce_sum(partial).to(dt)
            h = _rms_norm(x, self.w[p + "post_norm.weight"], s.epsilon)
            gate = F.linear(h, self._rows(self.w[p + "gate.weight"], W))
            up = F.linear(h, self._rows(self.w[p + "up.weight"], W))
            act = F.silu(gate) * up
            partial = F.linear(act.float(), self._cols(self.w[p + "down.weight"], W).float())
            x = x + self.all_reduce_sum(partial).to(dt)
        logits = F.linear(_rms_norm(x, self.w["final_norm.weight"], s.epsilon),
                          self._rows(self.w["lm_head.weight"], W))
        self.caches[seq] = new_cache
        vl = s.vocab // W
        key = self.all_reduce_max(argmax_key(logits[0, -1:], self.rank * vl))
        return logits[0], int(argmax_key_index(key)[0])
