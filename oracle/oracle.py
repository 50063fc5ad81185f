"""TEST INFRASTRUCTURE ONLY -- the CPU checker for the MoE layer.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference arm may import this module.  It wraps two shared libraries built by
``oracle/Makefile``:

* ``liboracle.so`` -- the C restatement of the reference MoE layer
  (``moe_oracle.c``; router src/tensor.cu:136-148, route src/layer.cu:47-70,
  expert src/layer.cu:32-45, combine src/layer.cu:80-103), plus the
  softmax/top-k/renormalise policy.
* ``_ref/libref_e<E>.so`` -- the reference's own ``PhiMoE`` compiled from its
  sources (present only where the reference tree was available at build time).
"""
from __future__ import annotations

import ctypes
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
POLICY_PHI = 0
POLICY_SOFTMAX = 1
PHI_QUANTUM = 1.0e-3   # include/config.h:22 ROUTER_SCORE_QUANTUM
PHI_TIE_EPS = 2.0e-2   # include/config.h:23 ROUTER_TIE_EPS

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)


def build(reference_dir: str | None = None) -> None:
    """Compile the checker (and the reference, when its sources exist)."""
    env = dict(os.environ)
    args = ["make", "-C", str(HERE), "-s"]
    if reference_dir:
        args.append(f"REF={reference_dir}")
    subprocess.run(args, check=True, env=env)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(_i32p)


class Oracle:
    """ctypes view of liboracle.so."""

    def __init__(self, path: Path | None = None):
        path = path or HERE / "liboracle.so"
        if not path.exists():
            build()
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.oracle_router_logits.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, _f32p, ctypes.c_int]
        L.oracle_route.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_float, _i32p, _f32p]
        L.oracle_expert_ffn.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        _f32p, _f32p, _f32p, _f32p, ctypes.c_int]
        PP = ctypes.POINTER(_f32p)
        L.oracle_moe_forward.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_float, _f32p, _f32p, PP, PP, PP, _i32p,
                                         ctypes.c_int, _f32p, _i32p, _f32p, _f32p, ctypes.c_int]
        L.oracle_moe_forward.restype = ctypes.c_int
        L.oracle_layer_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_float, ctypes.c_int,
                                        ctypes.c_int, _f32p]

    def layer_norm(self, x, w, b, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        y = np.empty_like(x)
        self.lib.oracle_layer_norm(_fp(x), _fp(np.ascontiguousarray(w, np.float32)),
                                   _fp(np.ascontiguousarray(b, np.float32)), eps, T, d, _fp(y))
        return y

    def router_logits(self, x, wg, bias=None, nthreads=0):
        x = np.ascontiguousarray(x, np.float32)
        wg = np.ascontiguousarray(wg, np.float32)
        T, d = x.shape
        E = wg.shape[0]
        out = np.empty((T, E), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.lib.oracle_router_logits(_fp(x), _fp(wg), None if b is None else _fp(b), T, d, E,
                                      _fp(out), nthreads)
        return out

    def route(self, logits, k, policy, quantum=PHI_QUANTUM, tie_eps=PHI_TIE_EPS):
        logits = np.ascontiguousarray(logits, np.float32)
        T, E = logits.shape
        idx = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        self.lib.oracle_route(_fp(logits), T, E, k, policy, quantum, tie_eps, _ip(idx), _fp(w))
        return idx, w

    def expert_ffn(self, X, w1, w3, w2, nthreads=0):
        X = np.ascontiguousarray(X, np.float32)
        rows, d = X.shape
        ff = w1.shape[0]
        out = np.empty((rows, d), np.float32)
        self.lib.oracle_expert_ffn(_fp(X), rows, d, ff, _fp(np.ascontiguousarray(w1)),
                                   _fp(np.ascontiguousarray(w3)), _fp(np.ascontiguousarray(w2)),
                                   _fp(out), nthreads)
        return out

    def moe_forward(self, x, layer, k, policy, sample=None, quantum=PHI_QUANTUM,
                    tie_eps=PHI_TIE_EPS, nthreads=0):
        """Return (y, idx, w, logits).  ``layer`` is a LayerWeights."""
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        E, ff = layer.E, layer.ff
        y = np.zeros((T, d), np.float32)
        idx = np.empty((T, k), np.int32)
        w = np.empty((T, k), np.float32)
        logits = np.empty((T, E), np.float32)
        PP = _f32p * E
        w1 = PP(*[_fp(a) for a in layer.w1])
        w3 = PP(*[_fp(a) for a in layer.w3])
        w2 = PP(*[_fp(a) for a in layer.w2])
        s = None
        ns = 0
        if sample is not None:
            s = np.ascontiguousarray(sample, np.int32)
            ns = len(s)
        bias = None if layer.router_bias is None else _fp(layer.router_bias)
        rc = self.lib.oracle_moe_forward(_fp(x), T, d, ff, E, k, policy, quantum, tie_eps,
                                         _fp(layer.wg), bias, w1, w3, w2,
                                         None if s is None else _ip(s), ns,
                                         _fp(y), _ip(idx), _fp(w), _fp(logits), nthreads)
        if rc != 0:
            raise ValueError("oracle_moe_forward rejected its arguments")
        return y, idx, w, logits

    def block_forward(self, attn, layer, k, policy, norm_w, norm_b, eps=1e-5, nthreads=0):
        """The decoder layer's MoE half (src/layer.cu:157-161): post =
        layer_norm(attn); y = moe(post) + attn.  Returns (y, idx, post)."""
        attn = np.ascontiguousarray(attn, np.float32)
        post = self.layer_norm(attn, norm_w, norm_b, eps)
        ff, idx, _, _ = self.moe_forward(post, layer, k, policy, nthreads=nthreads)
        return ff + attn, idx, post


class Reference:
    """The reference's own PhiMoE (compiled from its sources) for E experts."""

    def __init__(self, E: int):
        path = HERE / "_ref" / f"libref_e{E}.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (reference sources absent at build time)")
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.ref_moe_create.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.ref_moe_create.restype = ctypes.c_void_p
        L.ref_moe_destroy.argtypes = [ctypes.c_void_p]
        L.ref_moe_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.ref_moe_route.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, _f32p,
                                    _i32p, _f32p]
        L.ref_matmul_transposed.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int]
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_layer_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_float, ctypes.c_int,
                                     ctypes.c_int, _f32p]
        L.ref_apply_rope.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_float]
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_set_threads.restype = ctypes.c_int
        self.E = L.ref_num_experts()
        self.h = None

    @staticmethod
    def available(E: int) -> bool:
        return (HERE / "_ref" / f"libref_e{E}.so").exists()

    def set_threads(self, n: int) -> int:
        return self.lib.ref_set_threads(n)

    def load(self, model_bin: str, layer: int = 0):
        self.h = self.lib.ref_moe_create(str(model_bin).encode(), layer)
        if not self.h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return self

    def close(self):
        if self.h:
            self.lib.ref_moe_destroy(self.h)
            self.h = None

    def forward(self, x):
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        y = np.empty((T, d), np.float32)
        if self.lib.ref_moe_forward(self.h, _fp(x), T, d, _fp(y)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return y

    def route(self, x):
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        logits = np.empty((T, self.E), np.float32)
        idx = np.empty((T, 2), np.int32)
        w = np.empty((T, 2), np.float32)
        if self.lib.ref_moe_route(self.h, _fp(x), T, d, _fp(logits), _ip(idx), _fp(w)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return logits, idx, w

    def layer_norm(self, x, w, b, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        y = np.empty_like(x)
        if self.lib.ref_layer_norm(_fp(x), _fp(np.ascontiguousarray(w, np.float32)),
                                   _fp(np.ascontiguousarray(b, np.float32)), eps, T, d,
                                   _fp(y)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return y

    def apply_rope(self, q, k, heads, head_dim, theta=10000.0):
        """tensor_ops::apply_rope on copies of q [S][heads*hd] and k (same heads)."""
        q = np.array(q, np.float32, copy=True, order="C")
        k = np.array(k, np.float32, copy=True, order="C")
        if self.lib.ref_apply_rope(_fp(q), _fp(k), q.shape[0], heads, heads, head_dim,
                                   theta) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return q, k

    def matmul_transposed(self, a, b):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[0]), np.float32)
        if self.lib.ref_matmul_transposed(_fp(a), _fp(b), _fp(c), a.shape[0], a.shape[1],
                                          b.shape[0]) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return c


class ReferenceAttention:
    """The reference's own PhiAttention::forward (src/layer.cu:110-147), built
    with plain multi-head attention (2 heads of 128, no effective sliding
    window) into _ref/libref_attn.so."""

    PATH = HERE / "_ref" / "libref_attn.so"

    def __init__(self):
        if not self.PATH.exists():
            raise FileNotFoundError(f"{self.PATH} not built (reference sources absent at build time)")
        self.lib = ctypes.CDLL(str(self.PATH))
        L = self.lib
        L.ref_attention.argtypes = [ctypes.c_char_p, ctypes.c_int, _f32p, ctypes.c_int,
                                    ctypes.c_int, _f32p, ctypes.c_int]
        L.ref_attention_heads.restype = ctypes.c_int
        L.ref_decoder_layer.argtypes = [ctypes.c_char_p, ctypes.c_int, _f32p, ctypes.c_int,
                                        ctypes.c_int, _f32p]
        L.ref_apply_rope.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_float]
        L.ref_num_experts.restype = ctypes.c_int
        L.ref_last_error.restype = ctypes.c_char_p
        self.heads = L.ref_attention_heads()
        self.num_experts = L.ref_num_experts()

    @classmethod
    def available(cls) -> bool:
        return cls.PATH.exists()

    def forward(self, model_bin, layer, x, out_cols):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty((x.shape[0], out_cols), np.float32)
        if self.lib.ref_attention(str(model_bin).encode(), layer, _fp(x), x.shape[0], x.shape[1],
                                  _fp(y), out_cols) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return y

    def decoder_layer(self, model_bin, layer, x):
        """The reference's PhiDecoderLayer::forward (src/layer.cu:152-162)."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        if self.lib.ref_decoder_layer(str(model_bin).encode(), layer, _fp(x), x.shape[0],
                                      x.shape[1], _fp(y)) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return y

    def apply_rope(self, q, k, heads, kv_heads, head_dim, theta=10000.0):
        """The reference's tensor_ops::apply_rope on copies of q and k."""
        q = np.array(q, np.float32, order="C")
        k = np.array(k, np.float32, order="C")
        if self.lib.ref_apply_rope(_fp(q), _fp(k), q.shape[0], heads, kv_heads, head_dim,
                                   theta) != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return q, k
