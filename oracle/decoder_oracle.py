"""TEST INFRASTRUCTURE ONLY -- the checker for the toy MoE decoder (BASELINE
config 4).  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline
import it; the product (libmoe_b200.so, the Python binding) never does.

CPU restatement of whole-model greedy generation:
  embedding    row gather; the output head is the same matrix (tied)
  RMSNorm      y = (x * inv) * w, inv = 1 / sqrt(mean(x^2) + eps)   (config 4's
               norm; the reference's Phi model uses LayerNorm instead,
               src/tensor.cu:174-189)
  attention    multi-head, causal, softmax(q k^T / sqrt(hd)) v
  RoPE         rotate-half, as tensor_ops::apply_rope (src/tensor.cu:191-210):
               x_j' = x_j cos - x_{j+hd/2} sin, x_{j+hd/2}' = x_{j+hd/2} cos + x_j sin,
               angle = position * base^(-2j/hd)
  MoE          the C oracle (moe_oracle.c, pinned bit for bit to the
               reference's compiled PhiMoE) with the softmax / top-k /
               renormalise router, on the fp32 normalised rows
  generation   PhiTinyMoEModel::generate_decode (src/model.cu:2061-2104): the
               whole prefix is run again for every new token (no KV cache), the
               next token is the first index of the maximum logit, a sequence
               stops at EOS
Norms, projections, RoPE and attention run in float64 numpy; the MoE in the
oracle's fp32 reference arithmetic.  No reference code computes this
architecture end to end: the MoE is pinned (moe_oracle.c), and the attention
block -- projections, RoPE, causal softmax -- is checked against the
reference's own PhiAttention::forward built with plain multi-head attention
(oracle/_ref/libref_attn.so, tests/test_decoder.py); RMSNorm, the embedding
and the tied head are float64 restatements.
"""
from __future__ import annotations

import numpy as np

from oracle import POLICY_SOFTMAX, Oracle


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return (x * inv) * np.asarray(w, np.float64)


def rope_angles(positions: np.ndarray, head_dim: int, base: float):
    half = head_dim // 2
    inv = np.power(float(base), -2.0 * np.arange(half, dtype=np.float64) / head_dim)
    a = np.asarray(positions, np.float64)[:, None] * inv[None, :]
    return np.cos(a), np.sin(a)


def apply_rope(x: np.ndarray, positions: np.ndarray, head_dim: int, base: float) -> np.ndarray:
    """x [T][H][hd] (float64), row t at positions[t]; rotate-half form."""
    half = head_dim // 2
    c, s = rope_angles(positions, head_dim, base)
    c, s = c[:, None, :], s[:, None, :]
    x0, x1 = x[..., :half], x[..., half:]
    return np.concatenate([x0 * c - x1 * s, x1 * c + x0 * s], axis=-1)


def self_attention(xn: np.ndarray, wq, wk, wv, wo, B: int, S: int, H: int, hd: int,
                   base: float) -> np.ndarray:
    """Multi-head causal self-attention of B sequences of S rows each
    (xn [B*S][d], positions 0..S-1): q, k, v projections, rotate-half RoPE,
    softmax(q k^T / sqrt(hd)) over keys <= the query, the o projection.
    float64."""
    T = B * S
    xn = np.asarray(xn, np.float64)
    pos = np.tile(np.arange(S), B)
    q = (xn @ np.asarray(wq, np.float64).T).reshape(T, H, hd)
    k = (xn @ np.asarray(wk, np.float64).T).reshape(T, H, hd)
    v = (xn @ np.asarray(wv, np.float64).T).reshape(T, H, hd)
    q = apply_rope(q, pos, hd, base).reshape(B, S, H, hd)
    k = apply_rope(k, pos, hd, base).reshape(B, S, H, hd)
    v = v.reshape(B, S, H, hd)
    sc = np.einsum("bqhc,bkhc->bhqk", q, k) / np.sqrt(hd)
    mask = np.triu(np.ones((S, S), bool), 1)
    sc = np.where(mask[None, None], -np.inf, sc)
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqk,bkhc->bqhc", p, v).reshape(T, H * hd)
    return o @ np.asarray(wo, np.float64).T


class DecoderOracle:
    """The toy decoder's forward and greedy generation on the CPU.

    `weights` is the binding's DecoderWeights (numpy fp32 arrays)."""

    def __init__(self, weights, n_heads: int, head_dim: int, top_k: int = 2, eps: float = 1e-5,
                 rope_base: float = 10000.0, nthreads: int = 0):
        self.w = weights
        self.H, self.hd, self.k = n_heads, head_dim, top_k
        self.eps, self.base = eps, rope_base
        self.nthreads = nthreads
        self.orc = Oracle()
        assert weights.d == n_heads * head_dim

    def last_logits(self, tokens: np.ndarray) -> np.ndarray:
        """Logits [B][vocab] (float64) of the last position of each of the B
        equal-length sequences in tokens [B][S]."""
        w = self.w
        tok = np.asarray(tokens)
        B, S = tok.shape
        d, H, hd = w.d, self.H, self.hd
        T = B * S
        x = w.embed[tok.reshape(-1)].astype(np.float64)            # [T][d]
        for l in range(w.n_layers):
            xn = rms_norm(x, w.attn_norm[l], self.eps)
            x = x + self_attention(xn, w.wq[l], w.wk[l], w.wv[l], w.wo[l], B, S, H, hd,
                                   self.base)
            xm = rms_norm(x, w.ffn_norm[l], self.eps).astype(np.float32)
            y, *_ = self.orc.moe_forward(xm, w.moe[l], self.k, POLICY_SOFTMAX,
                                         nthreads=self.nthreads)
            x = x + y.astype(np.float64)
        last = x.reshape(B, S, d)[:, -1, :]
        h = rms_norm(last, w.final_norm, self.eps)
        return h @ w.embed.T.astype(np.float64)

    def generate(self, prompt: np.ndarray, max_new_tokens: int, eos_id: int = -1):
        """generate_decode: ids [B][n] (-1 after a sequence's EOS) and the
        logits [B][n][vocab] each token was chosen from (0 after EOS)."""
        tok = np.asarray(prompt)
        B = tok.shape[0]
        V = self.w.vocab
        ids = np.full((B, max_new_tokens), -1, np.int32)
        logits = np.zeros((B, max_new_tokens, V), np.float64)
        seqs = [list(map(int, tok[b])) for b in range(B)]
        live = [True] * B
        for step in range(max_new_tokens):
            act = [b for b in range(B) if live[b]]
            if not act:
                break
            lg = self.last_logits(np.array([seqs[b] for b in act]))
            for i, b in enumerate(act):
                nxt = int(np.argmax(lg[i]))
                logits[b, step] = lg[i]
                ids[b, step] = nxt
                if nxt == eos_id:
                    live[b] = False
                else:
                    seqs[b].append(nxt)
        return ids, logits


def top2_margin(logits: np.ndarray) -> np.ndarray:
    """Gap between the largest and second-largest logit of each row."""
    s = np.sort(np.asarray(logits, np.float64), axis=-1)
    return s[..., -1] - s[..., -2]
