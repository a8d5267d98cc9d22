"""Tensor-parallel decomposition of one denoising forward (a single sequence over several
GPUs): the shard plan and a numpy execution of it for CPU tests (gloo ranks).

The forward is the reference graph (src/diffuse-graph.cpp:11-160): embed, per layer RMSNorm,
Q/K/V (+bias), NEOX RoPE, non-causal attention (GQA grouping of :84-95), output projection and
residual, RMSNorm, SwiGLU FFN and residual, final RMSNorm, lm_head.  Split over `world` ranks:

* column-parallel Q / K / V by heads (each rank: n_head / world query heads and the
  n_head_kv / world KV heads they read) and gate / up by FFN rows (n_ff / world);
* row-parallel output and down projections over their input (the rank's heads x head_dim, its
  FFN rows), each followed by an all-reduce (sum) of the M x n_embd partial products -- the two
  collectives per layer;
* vocab-parallel lm_head (n_vocab / world rows): the sampler never gathers logits; each rank
  reduces its slice of every row to (max, first argmax, second max, sum exp, sum exp * (z - max))
  and one all-gather of those five numbers per row gives the row's top-1 / top-2 and entropy.

A row-parallel split must fall on a quantization block boundary of the weight's input
dimension (256 for Q4_K / Q6_K, 32 for Q8_0): `plan` rejects worlds that would cut a block.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    heads: range      # query heads of this rank
    kv_heads: range   # KV heads they read
    ff: range         # FFN rows (gate / up rows, down input columns)
    vocab: range      # lm_head rows


def plan(n_head: int, n_head_kv: int, head_dim: int, n_ff: int, n_vocab: int, world: int, block: int = 256):
    """One Shard per rank, or ValueError when the model does not split `world` ways."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if n_head % world or n_head_kv % world:
        raise ValueError(f"{n_head} query / {n_head_kv} KV heads do not split {world} ways")
    if n_vocab % world:
        raise ValueError(f"vocab {n_vocab} does not split {world} ways")
    if n_ff % world:
        raise ValueError(f"FFN {n_ff} does not split {world} ways")
    if ((n_head // world) * head_dim) % block:
        raise ValueError(f"output projection input share {(n_head // world) * head_dim} cuts a {block}-element block")
    if (n_ff // world) % block:
        raise ValueError(f"down projection input share {n_ff // world} cuts a {block}-element block")
    hq, hk, f, v = n_head // world, n_head_kv // world, n_ff // world, n_vocab // world
    return [Shard(r, world, range(r * hq, (r + 1) * hq), range(r * hk, (r + 1) * hk), range(r * f, (r + 1) * f),
                  range(r * v, (r + 1) * v)) for r in range(world)]


def _rmsnorm(x, w, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _rope(x, pos, theta_base):
    """NEOX rotation of the halves of each head, angles by GGML's float recurrence."""
    hd = x.shape[-1]
    half = hd // 2
    scale = np.float32(theta_base) ** np.float32(-2.0 / hd)
    ang = np.empty((len(pos), half), np.float64)
    for j, p in enumerate(pos):
        th = np.float32(p)
        for i in range(half):
            ang[j, i] = th
            th = np.float32(th * scale)
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half], x[..., half:]
    return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)


def row_stats(z):
    """Per row of a logits slice: max, first argmax, second max (largest value at any other
    index), sum exp(z - max), sum exp(z - max) * (z - max)."""
    m = z.max(axis=1)
    am = z.argmax(axis=1)
    z2 = z.copy()
    z2[np.arange(len(z)), am] = -np.inf
    sec = z2.max(axis=1)
    e = np.exp(z - m[:, None])
    return np.stack([m, am.astype(np.float64), sec, e.sum(axis=1), (e * (z - m[:, None])).sum(axis=1)], axis=1)


def combine_stats(parts, offsets):
    """Whole-row (top-1 value, token, top-2 value, entropy) from every rank's row_stats of its
    vocab slice (offsets: first vocab id of each slice, rank order)."""
    parts = np.stack(parts)  # [ranks][rows][5]
    m = parts[:, :, 0]
    g = m.max(axis=0)
    best = np.argmax(m == g[None, :], axis=0)  # lowest rank holding the max = lowest index
    rows = np.arange(parts.shape[1])
    tok = parts[best, rows, 1] + np.asarray(offsets)[best]
    others = np.where(np.arange(parts.shape[0])[:, None] == best[None, :], parts[:, :, 2], m)
    second = others.max(axis=0)
    w = np.exp(m - g[None, :])
    S = (parts[:, :, 3] * w).sum(axis=0)
    T = ((parts[:, :, 4] + parts[:, :, 3] * (m - g[None, :])) * w).sum(axis=0)
    ent = np.log(S) - T / S
    return g, tok.astype(np.int64), second, ent


def forward_rank(W, hp, tokens, shard: Shard, allreduce):
    """This rank's part of the forward over `tokens` (all positions active).  W maps the GGUF
    tensor names to float64 arrays [rows][cols]; allreduce(a) returns the elementwise sum over
    ranks.  Returns this rank's logits slice [n][n_vocab / world]."""
    hd = hp["n_embd"] // hp["n_head"]
    n = len(tokens)
    pos = np.arange(n)
    rep = hp["n_head"] // hp["n_head_kv"]
    x = W["token_embd.weight"][tokens].copy()
    for l in range(hp["n_layer"]):
        p = f"blk.{l}."
        h = _rmsnorm(x, W[p + "attn_norm.weight"], hp["rms_norm_eps"])
        qrows = np.concatenate([np.arange(hh * hd, (hh + 1) * hd) for hh in shard.heads])
        krows = np.concatenate([np.arange(hh * hd, (hh + 1) * hd) for hh in shard.kv_heads])
        q = h @ W[p + "attn_q.weight"][qrows].T
        k = h @ W[p + "attn_k.weight"][krows].T
        v = h @ W[p + "attn_v.weight"][krows].T
        if p + "attn_q.bias" in W:
            q += W[p + "attn_q.bias"][qrows]
            k += W[p + "attn_k.bias"][krows]
            v += W[p + "attn_v.bias"][krows]
        q = _rope(q.reshape(n, len(shard.heads), hd), pos, hp["rope_theta"])
        k = _rope(k.reshape(n, len(shard.kv_heads), hd), pos, hp["rope_theta"])
        v = v.reshape(n, len(shard.kv_heads), hd)
        att = np.empty((n, len(shard.heads), hd))
        for j, hh in enumerate(shard.heads):
            kv = hh // rep - shard.kv_heads.start  # GQA: query head hh reads KV head hh / n_rep
            s = q[:, j] @ k[:, kv].T / np.sqrt(hd)
            s = np.exp(s - s.max(axis=1, keepdims=True))
            att[:, j] = (s / s.sum(axis=1, keepdims=True)) @ v[:, kv]
        # row-parallel output projection: this rank's input columns, then the first all-reduce
        x = x + allreduce(att.reshape(n, -1) @ W[p + "attn_output.weight"][:, qrows].T)
        h = _rmsnorm(x, W[p + "ffn_norm.weight"], hp["rms_norm_eps"])
        ff = np.asarray(shard.ff)
        g = h @ W[p + "ffn_gate.weight"][ff].T
        u = h @ W[p + "ffn_up.weight"][ff].T
        a = g / (1.0 + np.exp(-g)) * u
        # row-parallel down projection, second all-reduce
        x = x + allreduce(a @ W[p + "ffn_down.weight"][:, ff].T)
    h = _rmsnorm(x, W["output_norm.weight"], hp["rms_norm_eps"])
    out = W["output.weight"] if "output.weight" in W else W["token_embd.weight"]
    return h @ out[np.asarray(shard.vocab)].T
