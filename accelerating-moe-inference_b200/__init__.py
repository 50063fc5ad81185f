"""Python binding of libmoe_b200.so -- the B200 MoE FFN layer.

A thin ctypes view of the C ABI declared in ``include/moe_b200.h``; every
call goes to the CUDA kernels in that library.  There is no CPU fallback:
importing this module without the built library raises, and so does using a
layer on a machine without a B200.

Also holds the host-side data formats either side of the layer: synthetic
layer weights (seeded), and the ``model.bin`` format of the reference's
ModelLoader (src/model_loader.cu:14-50) for tensors named as PhiMoE loads
them (src/layer.cu:73-77).
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libmoe_b200.so"

MOE_OK = 0
STATUS_NAMES = {0: "MOE_OK", -1: "MOE_ERR_INVALID", -2: "MOE_ERR_UNSUPPORTED", -3: "MOE_ERR_CUDA",
                -4: "MOE_ERR_OOM", -5: "MOE_ERR_IO", -6: "MOE_ERR_TIMEOUT", -7: "MOE_ERR_NCCL"}
ROUTER_PHI_QUANTISED = 0
ROUTER_SOFTMAX_TOPK = 1
PREC_FP32 = 0
PREC_BF16 = 1
# fp32-faithful through three bf16 MMAs on bf16 hi / lo operand planes.
PREC_FP32_BF16X3 = 2
# MoeConfig.ep_transport (expert parallelism): fused NVLink peer stores, or NCCL send/recv.
EP_TRANSPORT_P2P = 0
EP_TRANSPORT_NCCL = 1
# MoeConfig.decode_max_tokens: the measured decode-kernel threshold of the precision.
DECODE_AUTO = -1
GEMM_AUTO = 0
GEMM_SINGLE_CTA = 1
GEMM_CTA_PAIR = 2

# Every symbol include/moe_b200.h declares.
EXPORTED_SYMBOLS = (
    "moe_abi_version", "moe_last_error", "moe_config_init", "moe_create", "moe_create_from_device",
    "moe_create_from_model_bin", "moe_destroy", "moe_get_config", "moe_device_bytes",
    "moe_set_decode_max_tokens", "moe_forward_device", "moe_forward_host", "moe_route_device",
    "moe_expert_counts", "moe_dispatch_layout", "moe_profile_enable", "moe_profile_read",
    "moe_dispatch_noalloc", "moe_route_host", "moe_host_alloc", "moe_host_free",
    "moe_selftest_wait_timeout", "moe_set_post_norm", "moe_block_forward_device",
    "moe_block_forward_host", "moe_layer_norm_device",
    "moe_ep_plan", "moe_ep_unique_id", "moe_ep_create", "moe_ep_create_from_device", "moe_ep_forward_device",
    "moe_ep_check",
    "moe_set_post_rms_norm", "moe_decoder_config_init", "moe_decoder_create",
    "moe_decoder_create_from_device", "moe_decoder_destroy", "moe_decoder_device_bytes",
    "moe_decoder_prefill", "moe_decoder_decode_step", "moe_decoder_generate",
    "moe_decoder_last_timing", "moe_decoder_set_fused_step", "moe_decoder_fused_step_active",
)
PROFILE_STAGES = ("router", "dispatch_scan", "dispatch_permute", "gateup_gemm", "down_gemm",
                  "ep_exchange_in", "ep_exchange_out", "ep_combine")


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class MoeConfig(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int32), ("d_ff", ctypes.c_int32),
                ("num_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("router_policy", ctypes.c_int32), ("precision", ctypes.c_int32),
                ("router_quantum", ctypes.c_float), ("router_tie_eps", ctypes.c_float),
                ("decode_max_tokens", ctypes.c_int32), ("device", ctypes.c_int32),
                ("max_tokens", ctypes.c_int32), ("gemm_variant", ctypes.c_int32),
                ("ep_transport", ctypes.c_int32), ("ep_wait_ms", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 2)]


_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)


class MoeWeightsHost(ctypes.Structure):
    _fields_ = [("router_weight", _f32p), ("router_bias", _f32p),
                ("w1", ctypes.POINTER(_f32p)), ("w3", ctypes.POINTER(_f32p)),
                ("w2", ctypes.POINTER(_f32p))]


class MoeDecoderConfig(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("d_model", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("num_experts", ctypes.c_int32),
                ("top_k", ctypes.c_int32), ("d_ff", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float),
                ("precision", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("max_seq", ctypes.c_int32), ("device", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 4)]


_f32pp = ctypes.POINTER(_f32p)


class MoeDecoderWeightsC(ctypes.Structure):
    _fields_ = [("embed", _f32p), ("final_norm", _f32p), ("attn_norm", _f32pp),
                ("wq", _f32pp), ("wk", _f32pp), ("wv", _f32pp), ("wo", _f32pp),
                ("ffn_norm", _f32pp), ("router", _f32pp), ("w1", _f32pp), ("w3", _f32pp),
                ("w2", _f32pp)]


_lib = None


def load_library(path: Optional[Path] = None) -> ctypes.CDLL:
    """Load libmoe_b200.so; raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} is not built; run accelerating-moe-inference_b200/build.py")
    L = ctypes.CDLL(str(p))
    vp = ctypes.c_void_p
    L.moe_abi_version.restype = ctypes.c_int
    L.moe_last_error.restype = ctypes.c_char_p
    L.moe_config_init.argtypes = [ctypes.POINTER(MoeConfig)]
    L.moe_create.argtypes = [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeightsHost),
                             ctypes.POINTER(vp)]
    L.moe_create_from_device.argtypes = [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeightsHost),
                                         ctypes.POINTER(vp)]
    L.moe_create_from_model_bin.argtypes = [ctypes.POINTER(MoeConfig), ctypes.c_char_p,
                                            ctypes.c_int, ctypes.POINTER(vp)]
    L.moe_destroy.argtypes = [vp]
    L.moe_get_config.argtypes = [vp, ctypes.POINTER(MoeConfig)]
    L.moe_device_bytes.argtypes = [vp]
    L.moe_device_bytes.restype = ctypes.c_size_t
    L.moe_set_decode_max_tokens.argtypes = [vp, ctypes.c_int32]
    L.moe_forward_device.argtypes = [vp, vp, vp, ctypes.c_int32, vp]
    L.moe_forward_host.argtypes = [vp, _f32p, _f32p, ctypes.c_int32]
    L.moe_route_device.argtypes = [vp, vp, ctypes.c_int32, vp, vp, vp, vp]
    L.moe_expert_counts.argtypes = [vp, _i32p]
    L.moe_dispatch_layout.argtypes = [vp, _i32p, _f32p, ctypes.c_int32, _i32p, _i32p]
    L.moe_profile_enable.argtypes = [vp, ctypes.c_int]
    L.moe_profile_read.argtypes = [vp, _f32p, ctypes.c_int32]
    L.moe_route_host.argtypes = [vp, _f32p, ctypes.c_int32, _f32p, _i32p, _f32p]
    L.moe_host_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
    L.moe_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_int32]
    L.moe_host_free.argtypes = [vp]
    L.moe_set_post_norm.argtypes = [vp, _f32p, _f32p, ctypes.c_float]
    L.moe_block_forward_device.argtypes = [vp, vp, vp, ctypes.c_int32, vp]
    L.moe_block_forward_host.argtypes = [vp, _f32p, _f32p, ctypes.c_int32]
    L.moe_layer_norm_device.argtypes = [vp, vp, vp, ctypes.c_float, ctypes.c_int32, ctypes.c_int32,
                                        vp, vp]
    i64p = ctypes.POINTER(ctypes.c_int64)
    L.moe_ep_plan.argtypes = [_i32p, _i32p, ctypes.c_int32, ctypes.c_int32, i64p, i64p, i64p, i64p]
    L.moe_ep_unique_id.argtypes = [vp]
    L.moe_ep_create.argtypes = [ctypes.POINTER(MoeConfig), ctypes.POINTER(MoeWeightsHost),
                                ctypes.c_int, ctypes.c_int, vp, ctypes.POINTER(vp)]
    L.moe_ep_create_from_device.argtypes = L.moe_ep_create.argtypes
    L.moe_ep_forward_device.argtypes = [vp, vp, vp, ctypes.c_int32, vp]
    L.moe_ep_check.argtypes = [vp]
    L.moe_dispatch_noalloc.argtypes = [vp, vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       vp, vp, ctypes.c_int32, vp, vp, vp]
    L.moe_set_post_rms_norm.argtypes = [vp, vp, ctypes.c_float]
    dcp = ctypes.POINTER(MoeDecoderConfig)
    dwp = ctypes.POINTER(MoeDecoderWeightsC)
    L.moe_decoder_config_init.argtypes = [dcp]
    L.moe_decoder_config_init.restype = None
    L.moe_decoder_create.argtypes = [dcp, dwp, ctypes.POINTER(vp)]
    L.moe_decoder_create_from_device.argtypes = [dcp, dwp, ctypes.POINTER(vp)]
    L.moe_decoder_destroy.argtypes = [vp]
    L.moe_decoder_destroy.restype = None
    L.moe_decoder_device_bytes.argtypes = [vp]
    L.moe_decoder_device_bytes.restype = ctypes.c_size_t
    L.moe_decoder_prefill.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32, _f32p, _i32p]
    L.moe_decoder_decode_step.argtypes = [vp, _i32p, _f32p, _i32p]
    L.moe_decoder_generate.argtypes = [vp, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _f32p, _i32p]
    L.moe_decoder_last_timing.argtypes = [vp, _f32p, _f32p]
    L.moe_decoder_set_fused_step.argtypes = [vp, ctypes.c_int32]
    L.moe_decoder_fused_step_active.argtypes = [vp]
    if path is None:
        _lib = L
    return L


def _check(rc: int):
    if rc != MOE_OK:
        raise MoeError(rc, load_library().moe_last_error().decode())


def ep_plan(counts: np.ndarray, counts_in: np.ndarray, world: int, e_local: int):
    """moe_ep_plan: (send_rows, send_off, recv_rows, recv_off) of one exchange."""
    c = np.ascontiguousarray(counts, np.int32)
    ci = np.ascontiguousarray(counts_in, np.int32)
    out = [np.zeros(world, np.int64), np.zeros(world + 1, np.int64),
           np.zeros(world, np.int64), np.zeros(world + 1, np.int64)]
    p64 = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))  # noqa: E731
    _check(load_library().moe_ep_plan(c.ctypes.data_as(_i32p), ci.ctypes.data_as(_i32p), world,
                                      e_local, *map(p64, out)))
    return tuple(out)


def ep_unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (rank 0 of an expert-parallel group)."""
    buf = ctypes.create_string_buffer(128)
    _check(load_library().moe_ep_unique_id(buf))
    return buf.raw


def layer_norm_device(x_ptr: int, w_ptr: int, b_ptr: int, eps: float, rows: int, cols: int,
                      y_ptr: int, stream: int = 0) -> None:
    """tensor_ops::layer_norm (src/tensor.cu:174-189) on device buffers."""
    vp = ctypes.c_void_p
    _check(load_library().moe_layer_norm_device(vp(x_ptr), vp(w_ptr), vp(b_ptr), eps, rows, cols,
                                                vp(y_ptr), vp(stream)))


def default_config(**kw) -> MoeConfig:
    cfg = MoeConfig()
    load_library().moe_config_init(ctypes.byref(cfg))
    for k, v in kw.items():
        if not hasattr(cfg, k):
            raise TypeError(f"unknown MoeConfig field {k}")
        setattr(cfg, k, v)
    return cfg


# ------------------------------------------------------------------ weights
@dataclass
class LayerWeights:
    """One MoE layer's fp32 weights in nn.Linear layout (src/layer.cu:28-30)."""
    wg: np.ndarray                      # [E][d]
    w1: list                            # E x [ff][d]   gate
    w3: list                            # E x [ff][d]   up
    w2: list                            # E x [d][ff]   down
    router_bias: Optional[np.ndarray] = None  # [E]
    # The decoder layer's post_attention_layernorm, [d] each (optional).
    norm_weight: Optional[np.ndarray] = None
    norm_bias: Optional[np.ndarray] = None

    @property
    def E(self) -> int:
        return self.wg.shape[0]

    @property
    def d(self) -> int:
        return self.wg.shape[1]

    @property
    def ff(self) -> int:
        return self.w1[0].shape[0]


def synthetic_layer(seed: int, d: int, ff: int, E: int, std: float = 0.02,
                    router_std: Optional[float] = None,
                    router_bias: Optional[np.ndarray] = None) -> LayerWeights:
    """Seeded N(0, std) weights (numpy PCG64), drawn in a fixed order:
    router, then per expert w1, w3, w2."""
    g = np.random.Generator(np.random.PCG64(seed))
    rs = std if router_std is None else router_std

    def normal(shape, s):
        return (g.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    wg = normal((E, d), rs)
    w1, w3, w2 = [], [], []
    for _ in range(E):
        w1.append(normal((ff, d), std))
        w3.append(normal((ff, d), std))
        w2.append(normal((d, ff), std))
    bias = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)
    return LayerWeights(wg, w1, w3, w2, bias)


def synthetic_tokens(seed: int, T: int, d: int) -> np.ndarray:
    """Seeded N(0, 1) activations [T][d] (numpy PCG64, stream offset by 0x5eed)."""
    g = np.random.Generator(np.random.PCG64([seed, 0x5EED]))
    return g.standard_normal((T, d), dtype=np.float32)


def zipf_router_bias(E: int) -> np.ndarray:
    """Per-expert router bias 0.5 * ln(1 / rank), rank = 1..E (Zipf-like skew)."""
    r = np.arange(1, E + 1, dtype=np.float64)
    return (0.5 * np.log(1.0 / r)).astype(np.float32)


def synthetic_post_norm(seed: int, d: int):
    """Seeded post-attention LayerNorm weight ~ 1 + N(0, 0.1) and bias ~
    N(0, 0.1), [d] each (numpy PCG64, stream offset by 0x4e4f)."""
    g = np.random.Generator(np.random.PCG64([seed, 0x4E4F]))
    w = (1.0 + 0.1 * g.standard_normal(d)).astype(np.float32)
    b = (0.1 * g.standard_normal(d)).astype(np.float32)
    return w, b


def write_tensors(path, entries) -> None:
    """Named fp32 tensors in the ModelLoader format (src/model_loader.cu:14-30):
    u32 count; per entry u32 name_len, name, u32 ndim, u32 dims[ndim],
    u64 offset, u64 bytes; then the payloads.  entries: (name, array) pairs."""
    metas = [(n.encode(), np.shape(a), np.asarray(a, np.float32).nbytes) for n, a in entries]
    hsize = 4 + sum(4 + len(nb) + 4 + 4 * len(sh) + 16 for nb, sh, _ in metas)
    header = bytearray(struct.pack("<I", len(entries)))
    off = hsize
    for (nb, sh, nbytes) in metas:
        header += struct.pack("<I", len(nb)) + nb + struct.pack("<I", len(sh))
        header += struct.pack(f"<{len(sh)}I", *sh)
        header += struct.pack("<QQ", off, nbytes)
        off += nbytes
    assert len(header) == hsize
    with open(path, "wb") as f:
        f.write(header)
        for _, arr in entries:
            f.write(np.ascontiguousarray(arr, np.float32).tobytes())


def layer_entries(L: LayerWeights, li: int = 0):
    """The (name, array) entries of one MoE layer (src/layer.cu:73-77) and
    its post_attention_layernorm when present."""
    entries = []
    if L.norm_weight is not None:
        pn = f"model.layers.{li}.post_attention_layernorm"
        entries.append((f"{pn}.weight", L.norm_weight))
        entries.append((f"{pn}.bias", L.norm_bias))
    base = f"model.layers.{li}.block_sparse_moe"
    entries.append((f"{base}.gate.weight", L.wg))
    if L.router_bias is not None:
        entries.append((f"{base}.gate.bias", L.router_bias))
    for e in range(L.E):
        entries.append((f"{base}.experts.{e}.w1.weight", L.w1[e]))
        entries.append((f"{base}.experts.{e}.w2.weight", L.w2[e]))
        entries.append((f"{base}.experts.{e}.w3.weight", L.w3[e]))
    return entries


def write_model_bin(path, layers: Sequence[LayerWeights]) -> None:
    """Write MoE layers in the ModelLoader format (write_tensors)."""
    entries = []
    for li, L in enumerate(layers):
        entries += layer_entries(L, li)
    write_tensors(path, entries)


# ------------------------------------------------------------------ layer
def _fp(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


class MoeLayer:
    """Owns one MoeHandle.  Weights are uploaded once at construction."""

    def __init__(self, weights: Optional[LayerWeights] = None, *, top_k: int = 2,
                 policy: int = ROUTER_SOFTMAX_TOPK, precision: int = PREC_FP32, device: int = 0,
                 max_tokens: int = 0, decode_max_tokens: Optional[int] = None,
                 model_bin: Optional[str] = None, layer_idx: int = 0, **cfg_kw):
        L = load_library()
        cfg = default_config(top_k=top_k, router_policy=policy, precision=precision,
                             device=device, max_tokens=max_tokens, **cfg_kw)
        if decode_max_tokens is not None:
            cfg.decode_max_tokens = decode_max_tokens
        h = ctypes.c_void_p()
        if model_bin is not None:
            cfg.d_model = cfg_kw.get("d_model", 0)
            cfg.d_ff = cfg_kw.get("d_ff", 0)
            cfg.num_experts = cfg_kw.get("num_experts", 0)
            _check(L.moe_create_from_model_bin(ctypes.byref(cfg), str(model_bin).encode(),
                                               layer_idx, ctypes.byref(h)))
        else:
            w = weights
            cfg.d_model, cfg.d_ff, cfg.num_experts = w.d, w.ff, w.E
            keep = [np.ascontiguousarray(a, np.float32) for a in (w.wg, *w.w1, *w.w3, *w.w2)]
            E = w.E
            wg, w1, w3, w2 = keep[0], keep[1:1 + E], keep[1 + E:1 + 2 * E], keep[1 + 2 * E:]
            P = _f32p * E
            pw1, pw3, pw2 = P(*map(_fp, w1)), P(*map(_fp, w3)), P(*map(_fp, w2))
            bias = None
            if w.router_bias is not None:
                bias = np.ascontiguousarray(w.router_bias, np.float32)
            hw = MoeWeightsHost(_fp(wg), None if bias is None else _fp(bias), pw1, pw3, pw2)
            _check(L.moe_create(ctypes.byref(cfg), ctypes.byref(hw), ctypes.byref(h)))
        self._h = h
        self.cfg = MoeConfig()
        _check(L.moe_get_config(h, ctypes.byref(self.cfg)))
        if weights is not None and weights.norm_weight is not None:
            self.set_post_norm(weights.norm_weight, weights.norm_bias)

    @classmethod
    def from_device_pointers(cls, d: int, ff: int, E: int, wg_ptr: int, w1_ptrs, w3_ptrs,
                             w2_ptrs, bias_ptr: Optional[int] = None, *, top_k: int = 2,
                             policy: int = ROUTER_SOFTMAX_TOPK, precision: int = PREC_FP32,
                             device: int = 0, max_tokens: int = 0,
                             decode_max_tokens: Optional[int] = None, **cfg_kw) -> "MoeLayer":
        """Build from fp32 weights already on `device` (moe_create_from_device);
        pointers are integer device addresses in the same layouts as LayerWeights."""
        L = load_library()
        cfg = default_config(d_model=d, d_ff=ff, num_experts=E, top_k=top_k,
                             router_policy=policy, precision=precision, device=device,
                             max_tokens=max_tokens, **cfg_kw)
        if decode_max_tokens is not None:
            cfg.decode_max_tokens = decode_max_tokens
        P = _f32p * E
        cast = lambda v: ctypes.cast(ctypes.c_void_p(v), _f32p)  # noqa: E731
        hw = MoeWeightsHost(cast(wg_ptr), cast(bias_ptr) if bias_ptr else None,
                            P(*map(cast, w1_ptrs)), P(*map(cast, w3_ptrs)),
                            P(*map(cast, w2_ptrs)))
        h = ctypes.c_void_p()
        _check(L.moe_create_from_device(ctypes.byref(cfg), ctypes.byref(hw), ctypes.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.cfg = MoeConfig()
        _check(L.moe_get_config(h, ctypes.byref(self.cfg)))
        return self

    @classmethod
    def expert_parallel(cls, rank: int, world: int, nccl_id: bytes, *, d: int, ff: int, E: int,
                        wg, w1, w3, w2, bias=None, device_pointers: bool = False, top_k: int = 2,
                        policy: int = ROUTER_SOFTMAX_TOPK, precision: int = PREC_FP32,
                        device: int = 0, max_tokens: int = 0, **cfg_kw) -> "MoeLayer":
        """Collective: this rank's member of an expert-parallel group
        (moe_ep_create / moe_ep_create_from_device).  Weights are numpy arrays
        (host) or integer device addresses (device_pointers=True) for all E
        experts in their own order; only this rank's experts (rank,
        rank + world, ...: round-robin placement) are read."""
        L = load_library()
        cfg = default_config(d_model=d, d_ff=ff, num_experts=E, top_k=top_k, router_policy=policy,
                             precision=precision, device=device, max_tokens=max_tokens, **cfg_kw)
        P = _f32p * E
        if device_pointers:
            cast = lambda v: ctypes.cast(ctypes.c_void_p(v), _f32p)  # noqa: E731
            keep = None
        else:
            keep = [np.ascontiguousarray(a, np.float32) for a in [wg, *w1, *w3, *w2]
                    + ([bias] if bias is not None else [])]
            wg, w1, w3, w2 = keep[0], keep[1:1 + E], keep[1 + E:1 + 2 * E], keep[1 + 2 * E:1 + 3 * E]
            if bias is not None:
                bias = keep[-1]
            cast = _fp
        hw = MoeWeightsHost(cast(wg), cast(bias) if bias is not None else None,
                            P(*map(cast, w1)), P(*map(cast, w3)), P(*map(cast, w2)))
        idbuf = ctypes.create_string_buffer(bytes(nccl_id), 128)
        h = ctypes.c_void_p()
        fn = L.moe_ep_create_from_device if device_pointers else L.moe_ep_create
        _check(fn(ctypes.byref(cfg), ctypes.byref(hw), rank, world, idbuf, ctypes.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.cfg = MoeConfig()
        _check(L.moe_get_config(h, ctypes.byref(self.cfg)))
        return self

    def ep_check(self):
        """moe_ep_check: wait for the last expert-parallel forward and raise
        MoeError (MOE_ERR_TIMEOUT) if a peer wait of this group ran out."""
        _check(load_library().moe_ep_check(self._h))

    def ep_forward_device(self, x_ptr: int, y_ptr: int, T: int, stream: int = 0):
        _check(load_library().moe_ep_forward_device(self._h, ctypes.c_void_p(x_ptr),
                                                    ctypes.c_void_p(y_ptr), T,
                                                    ctypes.c_void_p(stream)))

    # -- properties
    @property
    def d(self):
        return self.cfg.d_model

    @property
    def E(self):
        return self.cfg.num_experts

    @property
    def k(self):
        return self.cfg.top_k

    def device_bytes(self) -> int:
        return load_library().moe_device_bytes(self._h)

    def set_decode_max_tokens(self, n: int):
        _check(load_library().moe_set_decode_max_tokens(self._h, n))

    # -- compute
    def forward_host(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        if d != self.d:
            raise ValueError(f"x has {d} columns, layer expects {self.d}")
        y = np.empty_like(x)
        _check(load_library().moe_forward_host(self._h, _fp(x), _fp(y), T))
        return y

    def forward_device(self, x_ptr: int, y_ptr: int, T: int, stream: int = 0):
        _check(load_library().moe_forward_device(self._h, ctypes.c_void_p(x_ptr),
                                                 ctypes.c_void_p(y_ptr), T,
                                                 ctypes.c_void_p(stream)))

    # -- the decoder layer's MoE half: y = attn + MoE(layer_norm(attn))
    def set_post_norm(self, weight: np.ndarray, bias: np.ndarray, eps: float = 1e-5):
        w = np.ascontiguousarray(weight, np.float32)
        b = np.ascontiguousarray(bias, np.float32)
        if w.shape != (self.d,) or b.shape != (self.d,):
            raise ValueError(f"post-norm weight and bias must have shape ({self.d},)")
        _check(load_library().moe_set_post_norm(self._h, _fp(w), _fp(b), eps))

    def set_post_rms_norm(self, weight: np.ndarray, eps: float = 1e-5):
        """Attach an RMSNorm as the block's input norm (moe_set_post_rms_norm)."""
        w = np.ascontiguousarray(weight, np.float32)
        if w.shape != (self.d,):
            raise ValueError(f"rms-norm weight must have shape ({self.d},)")
        _check(load_library().moe_set_post_rms_norm(self._h, w.ctypes.data, eps))

    def block_forward_host(self, attn: np.ndarray) -> np.ndarray:
        attn = np.ascontiguousarray(attn, np.float32)
        T, d = attn.shape
        if d != self.d:
            raise ValueError(f"attn has {d} columns, layer expects {self.d}")
        y = np.empty_like(attn)
        _check(load_library().moe_block_forward_host(self._h, _fp(attn), _fp(y), T))
        return y

    def block_forward_device(self, attn_ptr: int, y_ptr: int, T: int, stream: int = 0):
        _check(load_library().moe_block_forward_device(self._h, ctypes.c_void_p(attn_ptr),
                                                       ctypes.c_void_p(y_ptr), T,
                                                       ctypes.c_void_p(stream)))

    def route_device(self, x_ptr: int, T: int, logits_ptr: int, idx_ptr: int, w_ptr: int,
                     stream: int = 0):
        _check(load_library().moe_route_device(self._h, ctypes.c_void_p(x_ptr), T,
                                               ctypes.c_void_p(logits_ptr),
                                               ctypes.c_void_p(idx_ptr), ctypes.c_void_p(w_ptr),
                                               ctypes.c_void_p(stream)))

    def route_host(self, x: np.ndarray):
        """(logits [T][E], idx [T][k], weights [T][k]) of host x."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        lg = np.empty((T, self.E), np.float32)
        idx = np.empty((T, self.k), np.int32)
        w = np.empty((T, self.k), np.float32)
        _check(load_library().moe_route_host(self._h, _fp(x), T, _fp(lg),
                                             idx.ctypes.data_as(_i32p), _fp(w)))
        return lg, idx, w

    def expert_counts(self) -> np.ndarray:
        c = np.zeros(self.E, np.int32)
        _check(load_library().moe_expert_counts(self._h, c.ctypes.data_as(_i32p)))
        return c

    def dispatch_layout(self, rows_cap: int):
        tok = np.zeros(rows_cap, np.int32)
        wt = np.zeros(rows_cap, np.float32)
        rows = ctypes.c_int32()
        eoff = np.zeros(self.E + 1, np.int32)
        _check(load_library().moe_dispatch_layout(self._h, tok.ctypes.data_as(_i32p), _fp(wt),
                                                  rows_cap, ctypes.byref(rows),
                                                  eoff.ctypes.data_as(_i32p)))
        n = rows.value
        return tok[:n], wt[:n], eoff

    def profile(self, enable: bool = True):
        _check(load_library().moe_profile_enable(self._h, int(enable)))

    def stage_ms(self) -> np.ndarray:
        """Per-stage device milliseconds of the last forward (see PROFILE_STAGES)."""
        out = np.zeros(len(PROFILE_STAGES), np.float32)
        rc = load_library().moe_profile_read(self._h, _fp(out), len(out))
        if rc < 0:
            _check(rc)
        return out

    def close(self):
        if self._h:
            load_library().moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


# ---------------------------------------------------------------------------
# Toy MoE decoder: moe_decoder_* in include/moe_b200.h.

@dataclass
class DecoderWeights:
    """fp32 weights of the toy MoE decoder, nn.Linear layout ([out][in])."""
    embed: np.ndarray                   # [vocab][d]; tied output head
    final_norm: np.ndarray              # [d]
    attn_norm: list                     # L x [d]
    wq: list                            # L x [d][d]
    wk: list
    wv: list
    wo: list
    ffn_norm: list                      # L x [d]
    moe: list                           # L x LayerWeights (router + experts)

    @property
    def n_layers(self) -> int:
        return len(self.wq)

    @property
    def d(self) -> int:
        return self.embed.shape[1]

    @property
    def vocab(self) -> int:
        return self.embed.shape[0]


def synthetic_decoder(seed: int, n_layers: int, d: int, vocab: int, E: int, ff: int,
                      std: float = 0.02, norm_jitter: float = 0.0) -> DecoderWeights:
    """Seeded N(0, std) weights (numpy PCG64), drawn in a fixed order:
    embedding, then per layer wq, wk, wv, wo and the MoE layer (router, then
    per expert w1, w3, w2, from its own seeded stream).  Norm weights are 1
    (plus N(0, norm_jitter) when norm_jitter > 0, stream offset by 0x4e4f)."""
    g = np.random.Generator(np.random.PCG64([seed, 0xDEC]))

    def normal(shape):
        return (g.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    gn = np.random.Generator(np.random.PCG64([seed, 0x4E4F]))

    def norm_w():
        w = np.ones(d, np.float32)
        if norm_jitter > 0:
            w = (w + norm_jitter * gn.standard_normal(d)).astype(np.float32)
        return w

    embed = normal((vocab, d))
    wq, wk, wv, wo, an, fn, moe = [], [], [], [], [], [], []
    for l in range(n_layers):
        wq.append(normal((d, d)))
        wk.append(normal((d, d)))
        wv.append(normal((d, d)))
        wo.append(normal((d, d)))
        an.append(norm_w())
        fn.append(norm_w())
        moe.append(synthetic_layer(seed * 1000 + 7 + l, d, ff, E, std))
    return DecoderWeights(embed, norm_w(), an, wq, wk, wv, wo, fn, moe)


def synthetic_prompt(seed: int, B: int, S: int, vocab: int) -> np.ndarray:
    """Seeded uniform token ids [B][S] (numpy PCG64, stream offset by 0x1d5)."""
    g = np.random.Generator(np.random.PCG64([seed, 0x1D5]))
    return g.integers(0, vocab, size=(B, S), dtype=np.int32)


def decoder_config(**kw) -> MoeDecoderConfig:
    c = MoeDecoderConfig()
    load_library().moe_decoder_config_init(ctypes.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


class MoeDecoder:
    """The toy MoE decoder on one GPU (moe_decoder_*): prefill, KV-cached
    decode steps and greedy generation, mirroring PhiTinyMoEModel's generate
    and generate_decode (include/model.h:8-30)."""

    def __init__(self, weights: Optional[DecoderWeights] = None, *, n_heads: int, head_dim: int,
                 top_k: int = 2, precision: int = PREC_BF16, max_batch: int = 16,
                 max_seq: int = 640, device: int = 0, rms_eps: float = 1e-5,
                 rope_base: float = 10000.0, device_pointers: Optional[dict] = None,
                 dims: Optional[dict] = None):
        """Host numpy weights, or device_pointers: a dict of integer device
        addresses with the DecoderWeights field names (per-layer entries as
        lists; 'router', 'w1', 'w3', 'w2' flattened layer-major) plus dims
        {n_layers, d, vocab, E, ff}."""
        L = load_library()
        if device_pointers is None:
            w = weights
            dm = dict(n_layers=w.n_layers, d=w.d, vocab=w.vocab, E=w.moe[0].E, ff=w.moe[0].ff)
        else:
            dm = dims
        self.cfg = decoder_config(n_layers=dm["n_layers"], d_model=dm["d"], n_heads=n_heads,
                                  head_dim=head_dim, vocab=dm["vocab"], num_experts=dm["E"],
                                  top_k=top_k, d_ff=dm["ff"], rms_eps=rms_eps,
                                  rope_base=rope_base, precision=precision,
                                  max_batch=max_batch, max_seq=max_seq, device=device)
        nl, E = dm["n_layers"], dm["E"]
        P = lambda n: _f32p * n  # noqa: E731
        if device_pointers is None:
            keep = []

            def hp(a):
                a = np.ascontiguousarray(a, np.float32)
                keep.append(a)
                return _fp(a)

            def arr(lst):
                return P(len(lst))(*[hp(a) for a in lst])
            cw = MoeDecoderWeightsC(
                hp(w.embed), hp(w.final_norm), arr(w.attn_norm), arr(w.wq), arr(w.wk), arr(w.wv),
                arr(w.wo), arr(w.ffn_norm), arr([m.wg for m in w.moe]),
                arr([a for m in w.moe for a in m.w1]), arr([a for m in w.moe for a in m.w3]),
                arr([a for m in w.moe for a in m.w2]))
            fn = L.moe_decoder_create
        else:
            dp = device_pointers
            keep = None
            cast = lambda v: ctypes.cast(ctypes.c_void_p(v), _f32p)  # noqa: E731

            def arr(lst):
                return P(len(lst))(*[cast(v) for v in lst])
            cw = MoeDecoderWeightsC(
                cast(dp["embed"]), cast(dp["final_norm"]), arr(dp["attn_norm"]), arr(dp["wq"]),
                arr(dp["wk"]), arr(dp["wv"]), arr(dp["wo"]), arr(dp["ffn_norm"]),
                arr(dp["router"]), arr(dp["w1"]), arr(dp["w3"]), arr(dp["w2"]))
            fn = L.moe_decoder_create_from_device
        h = ctypes.c_void_p()
        _check(fn(ctypes.byref(self.cfg), ctypes.byref(cw), ctypes.byref(h)))
        del keep
        self._h = h
        self.vocab = dm["vocab"]
        self.E = E
        self.n_layers = nl

    def device_bytes(self) -> int:
        return load_library().moe_decoder_device_bytes(self._h)

    def prefill(self, tokens: np.ndarray):
        """Last-position logits [B][vocab] and greedy next ids [B]."""
        tok = np.ascontiguousarray(tokens, np.int32)
        B, S = tok.shape
        logits = np.empty((B, self.vocab), np.float32)
        ids = np.empty(B, np.int32)
        self._B = 0
        _check(load_library().moe_decoder_prefill(self._h, tok.ctypes.data_as(_i32p), B, S,
                                                   _fp(logits), ids.ctypes.data_as(_i32p)))
        self._B = B
        return logits, ids

    def decode_step(self, tokens: np.ndarray):
        """tokens [B] at the next position of every sequence of the last
        prefill; logits [B][vocab] and greedy next ids [B]."""
        tok = np.ascontiguousarray(tokens, np.int32)
        B = tok.shape[0]
        if getattr(self, "_B", 0) and B != self._B:
            raise ValueError(f"decode_step needs one token per sequence ({self._B}), got {B}")
        logits = np.empty((B, self.vocab), np.float32)
        ids = np.empty(B, np.int32)
        _check(load_library().moe_decoder_decode_step(self._h, tok.ctypes.data_as(_i32p),
                                                       _fp(logits), ids.ctypes.data_as(_i32p)))
        return logits, ids

    def generate(self, prompt: np.ndarray, max_new_tokens: int, eos_id: int = -1,
                 want_logits: bool = True, logits_out: Optional[np.ndarray] = None):
        """Greedy ids [B][n] (-1 after eos) and, if wanted, logits [B][n][vocab]."""
        tok = np.ascontiguousarray(prompt, np.int32)
        B, S = tok.shape
        ids = np.empty((B, max_new_tokens), np.int32)
        logits = None
        if want_logits:
            logits = logits_out if logits_out is not None else np.empty(
                (B, max_new_tokens, self.vocab), np.float32)
        self._B = 0
        _check(load_library().moe_decoder_generate(
            self._h, tok.ctypes.data_as(_i32p), B, S, max_new_tokens, eos_id,
            _fp(logits) if logits is not None else None, ids.ctypes.data_as(_i32p)))
        self._B = B
        return ids, logits

    def set_fused_step(self, enable: bool):
        """Batch-1 decode steps as one cooperative launch (True, the default
        where the configuration allows it) or as the kernel chain (False)."""
        _check(load_library().moe_decoder_set_fused_step(self._h, 1 if enable else 0))

    @property
    def fused_step_active(self) -> bool:
        return bool(load_library().moe_decoder_fused_step_active(self._h))

    def last_timing(self):
        """(prefill_ms, decode_ms) of the last generate, CUDA events."""
        a, b = ctypes.c_float(), ctypes.c_float()
        _check(load_library().moe_decoder_last_timing(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def close(self):
        if getattr(self, "_h", None):
            load_library().moe_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
