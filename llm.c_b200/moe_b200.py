"""Python host binding of libmoe_b200.so (the B200 MoE feed-forward path).

Mirrors llm.c's MoE operator interface: `MoEWeights` holds the router and
the E SwiGLU experts in the reference's host layout (W_router [d×E],
W_gate/W_up [d×F], W_down [F×d]), and `moe_forward` returns what llm.c's
moe_forward (src/transformer.c:287-366) writes: the layer output [T×d],
cache->router_probs [T×E] and cache->expert_ids [T×k].

All arithmetic runs in the CUDA library; there is no CPU fallback.  If the
library is missing or no sm_100 device is usable the calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmoe_b200.so"

OK = 0
E_INVALID, E_CUDA, E_NOMEM, E_NCCL, E_TIMEOUT, E_NODEV, E_STATE = -1, -2, -3, -4, -5, -6, -7
PATH_AUTO, PATH_TF32, PATH_FP32, PATH_TF32X3 = 0, 1, 2, 3
STREAM_X, STREAM_ROUTER, STREAM_BIAS = 1, 2, 3


def stream_expert(e: int, which: int) -> int:
    return 0x100 + 4 * e + which


class MoEError(RuntimeError):
    def __init__(self, status: int, what: str, detail: str):
        super().__init__(f"{what}: status {status} ({detail})")
        self.status = status


_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)
_vp = C.c_void_p


class Opts(C.Structure):
    _fields_ = [("path", C.c_int), ("cta_pair", C.c_int), ("host_chunks", C.c_int),
                ("reserved", C.c_int * 5)]


_lib = None


def lib() -> C.CDLL:
    """Load libmoe_b200.so once (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(f"{LIB_PATH} missing: build it with `make -C {HERE}` "
                                "or __graft_entry__.build()")
    L = C.CDLL(str(LIB_PATH))
    L.moe_b200_version.restype = C.c_char_p
    L.moe_b200_strerror.restype = C.c_char_p
    L.moe_b200_strerror.argtypes = [C.c_int]
    L.moe_b200_last_error.restype = C.c_char_p
    L.moe_b200_init.argtypes = [C.c_int]
    L.moe_b200_shutdown.restype = None
    L.moe_b200_weights_upload.argtypes = [_fp, C.POINTER(_fp), C.POINTER(_fp), C.POINTER(_fp),
                                          C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    L.moe_b200_weights_synth.argtypes = [C.c_uint64, C.c_float, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.POINTER(_vp)]
    L.moe_b200_weights_free.argtypes = [_vp]
    L.moe_b200_weights_shape.argtypes = [_vp, _ip, _ip, _ip, _ip]
    L.moe_b200_weights_download.argtypes = [_vp, _fp, C.POINTER(_fp), C.POINTER(_fp),
                                            C.POINTER(_fp)]
    L.moe_b200_forward.argtypes = [_vp, _fp, _fp, C.c_int, _fp, _fp, _ip, C.POINTER(Opts)]
    L.moe_b200_forward_device.argtypes = [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp,
                                          C.POINTER(Opts), _vp]
    L.moe_b200_last_counts.argtypes = [_vp, _ip]
    L.moe_b200_last_launches.restype = C.c_int
    L.moe_b200_last_path.restype = C.c_int
    L.moe_b200_profile_enable.argtypes = [C.c_int]
    L.moe_b200_profile_read.argtypes = [C.POINTER(C.c_double), _ip]
    L.moe_b200_synth_fill.argtypes = [_vp, C.c_size_t, C.c_uint64, C.c_uint64, C.c_uint64,
                                      C.c_float, _vp]
    L.moe_b200_block_ffn.argtypes = [_vp, _fp, C.c_float, _fp, _fp, C.c_int, _fp, _fp, _ip,
                                     C.POINTER(Opts)]
    L.moe_b200_block_ffn_device.argtypes = [_vp, _vp, C.c_float, _vp, _vp, C.c_int, _vp, _vp,
                                            _vp, C.POINTER(Opts), _vp]
    L.moe_b200_grads_create.argtypes = [_vp, C.POINTER(_vp)]
    L.moe_b200_grads_zero.argtypes = [_vp]
    L.moe_b200_grads_download.argtypes = [_vp, _fp, _fp, C.POINTER(_fp), C.POINTER(_fp),
                                          C.POINTER(_fp)]
    L.moe_b200_grads_free.argtypes = [_vp]
    L.moe_b200_backward.argtypes = [_vp, _fp, _fp, C.c_int, _fp, C.c_float, _fp, _vp, _fp,
                                    C.POINTER(Opts)]
    L.moe_b200_backward_device.argtypes = [_vp, _vp, _vp, C.c_int, _vp, C.c_float, _vp, _vp,
                                           _vp, C.POINTER(Opts), _vp]
    L.moe_b200_checkpoint_config.argtypes = [C.c_char_p, _vp]
    L.moe_b200_checkpoint_load_experts.argtypes = [C.c_char_p, C.c_int, C.POINTER(_vp)]
    L.moe_b200_decoder_create.argtypes = [_vp, C.c_int, C.c_int, C.POINTER(_vp)]
    L.moe_b200_decoder_load.argtypes = [C.c_char_p, C.c_int, C.c_int, C.POINTER(_vp)]
    L.moe_b200_decoder_step.argtypes = [_vp, C.c_int, _fp]
    L.moe_b200_decoder_set_pos.argtypes = [_vp, C.c_int]
    L.moe_b200_decoder_pos.argtypes = [_vp]
    L.moe_b200_decoder_launches.argtypes = [_vp]
    L.moe_b200_decoder_destroy.argtypes = [_vp]
    L.moe_b200_decoder_trace.argtypes = [_vp, C.c_int, _fp, _fp]
    L.moe_b200_decoder_stage_times.argtypes = [_vp, C.POINTER(C.c_double), C.c_int]
    L.moe_b200_llmc_trace_enable.argtypes = [C.c_int]
    L.moe_b200_llmc_trace_read.argtypes = [C.c_int, _fp, _fp]
    _lib = L
    return L


def _check(rc: int, what: str):
    if rc != OK:
        L = lib()
        raise MoEError(rc, what, f"{L.moe_b200_strerror(rc).decode()}: "
                                 f"{L.moe_b200_last_error().decode()}")


def _f(a):
    if a is None:
        return None
    if not (a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]):
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data_as(_fp)


def _i(a):
    if a is None:
        return None
    if not (a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]):
        raise TypeError("expected a C-contiguous int32 array")
    return a.ctypes.data_as(_ip)


def _opts(path: int, cta_pair: bool = False, host_chunks: int = 0) -> Opts:
    o = Opts()
    o.path = path
    o.cta_pair = int(bool(cta_pair))
    o.host_chunks = int(host_chunks)
    return o


def version() -> str:
    return lib().moe_b200_version().decode()


def init(device: int = -1):
    _check(lib().moe_b200_init(device), "moe_b200_init")


def shutdown():
    lib().moe_b200_shutdown()


class MoEWeights:
    """A device-resident expert set (llm.c MoEWeights, include/transformer.h:53-58)."""

    def __init__(self, handle: int, d: int, F: int, E: int, k: int):
        self.handle, self.d, self.F, self.E, self.top_k = handle, d, F, E, k

    @classmethod
    def upload(cls, W_router, W_gate, W_up, W_down, top_k: int) -> "MoEWeights":
        W_router = np.ascontiguousarray(W_router, np.float32)
        d, E = W_router.shape
        F = np.asarray(W_gate[0]).shape[1]
        keep = [np.ascontiguousarray(a, np.float32) for a in (*W_gate, *W_up, *W_down)]
        g = (_fp * E)(*[_f(a) for a in keep[0:E]])
        u = (_fp * E)(*[_f(a) for a in keep[E:2 * E]])
        dn = (_fp * E)(*[_f(a) for a in keep[2 * E:3 * E]])
        h = _vp()
        _check(lib().moe_b200_weights_upload(_f(W_router), g, u, dn, d, F, E, top_k,
                                             C.byref(h)), "moe_b200_weights_upload")
        return cls(h.value, d, F, E, top_k)

    @classmethod
    def synth(cls, seed: int, w_std: float, d: int, F: int, E: int, top_k: int) -> "MoEWeights":
        h = _vp()
        _check(lib().moe_b200_weights_synth(seed, w_std, d, F, E, top_k, C.byref(h)),
               "moe_b200_weights_synth")
        return cls(h.value, d, F, E, top_k)

    @classmethod
    def synth_shard(cls, seed: int, w_std: float, d: int, F: int, E: int, top_k: int,
                    experts, n_slots: int) -> "MoEWeights":
        """An expert-parallel shard: the listed experts (global ids) from the
        seeded generator in the first slots, the rest spare slots."""
        ex = np.ascontiguousarray(experts, np.int32)
        L = lib()
        L.moe_b200_weights_synth_shard.argtypes = [C.c_uint64, C.c_float, C.c_int, C.c_int,
                                                   C.c_int, C.c_int, C.c_int, _ip, C.c_int,
                                                   C.POINTER(_vp)]
        h = _vp()
        _check(L.moe_b200_weights_synth_shard(seed, w_std, d, F, E, top_k, len(ex), _i(ex),
                                              n_slots, C.byref(h)), "moe_b200_weights_synth_shard")
        return cls(h.value, d, F, E, top_k)

    @classmethod
    def upload_shard(cls, W_router, W_gate, W_up, W_down, top_k: int, experts,
                     n_slots: int) -> "MoEWeights":
        """An expert-parallel shard from host matrices: W_gate[i] etc. are
        those of global expert experts[i]."""
        W_router = np.ascontiguousarray(W_router, np.float32)
        d, E = W_router.shape
        F = np.asarray(W_gate[0]).shape[1] if len(W_gate) else 1
        ex = np.ascontiguousarray(experts, np.int32)
        n = len(ex)
        keep = [np.ascontiguousarray(a, np.float32) for a in (*W_gate, *W_up, *W_down)]
        g = (_fp * max(n, 1))(*[_f(a) for a in keep[0:n]])
        u = (_fp * max(n, 1))(*[_f(a) for a in keep[n:2 * n]])
        dn = (_fp * max(n, 1))(*[_f(a) for a in keep[2 * n:3 * n]])
        L = lib()
        L.moe_b200_weights_upload_shard.argtypes = [_fp, C.POINTER(_fp), C.POINTER(_fp),
                                                    C.POINTER(_fp), C.c_int, C.c_int, C.c_int,
                                                    C.c_int, C.c_int, _ip, C.c_int,
                                                    C.POINTER(_vp)]
        h = _vp()
        _check(L.moe_b200_weights_upload_shard(_f(W_router), g, u, dn, d, F, E, top_k, n, _i(ex),
                                               n_slots, C.byref(h)),
               "moe_b200_weights_upload_shard")
        return cls(h.value, d, F, E, top_k)

    def slots(self) -> np.ndarray:
        """Global expert id in each packed slot (-1 = empty spare)."""
        L = lib()
        L.moe_b200_weights_slots.argtypes = [_vp, _ip, _ip]
        n = C.c_int()
        _check(L.moe_b200_weights_slots(self.handle, C.byref(n), None), "moe_b200_weights_slots")
        out = np.empty(n.value, np.int32)
        _check(L.moe_b200_weights_slots(self.handle, None, _i(out)), "moe_b200_weights_slots")
        return out

    @classmethod
    def from_checkpoint(cls, path, layer: int) -> "MoEWeights":
        """Block `layer`'s experts (or dense FFN, as one expert) of an llm.c
        checkpoint (model_save format), streamed straight to the device."""
        cfg = checkpoint_config(path)
        h = _vp()
        _check(lib().moe_b200_checkpoint_load_experts(_path(path), int(layer), C.byref(h)),
               "moe_b200_checkpoint_load_experts")
        moe = cfg.n_experts > 1
        return cls(h.value, cfg.d_model, cfg.ffn_hidden, cfg.n_experts if moe else 1,
                   cfg.top_k_experts if moe else 1)

    def download(self, experts: bool = True):
        d, F, E = self.d, self.F, self.E
        wr = np.empty((d, E), np.float32)
        if not experts:
            _check(lib().moe_b200_weights_download(self.handle, _f(wr), None, None, None),
                   "moe_b200_weights_download")
            return wr, None, None, None
        g = [np.empty((d, F), np.float32) for _ in range(E)]
        u = [np.empty((d, F), np.float32) for _ in range(E)]
        dn = [np.empty((F, d), np.float32) for _ in range(E)]
        _check(lib().moe_b200_weights_download(self.handle, _f(wr), (_fp * E)(*[_f(a) for a in g]),
                                                (_fp * E)(*[_f(a) for a in u]),
                                                (_fp * E)(*[_f(a) for a in dn])),
               "moe_b200_weights_download")
        return wr, g, u, dn

    def free(self):
        if self.handle:
            lib().moe_b200_weights_free(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def moe_forward(w: MoEWeights, x: np.ndarray, bias: np.ndarray | None = None,
                path: int = PATH_AUTO, cta_pair: bool = False):
    """Host-buffer forward (synchronous): returns (out [T×d], probs [T×E], ids [T×k])."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.empty((T, w.d), np.float32)
    probs = np.empty((T, w.E), np.float32)
    ids = np.empty((T, w.top_k), np.int32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    o = _opts(path, cta_pair)
    _check(lib().moe_b200_forward(w.handle, _f(b), _f(x), T, _f(out), _f(probs), _i(ids),
                                  C.byref(o)), "moe_b200_forward")
    return out, probs, ids


def moe_forward_host_ptr(w: MoEWeights, x_ptr: int, T: int, out_ptr: int, probs_ptr: int | None,
                         ids_ptr: int | None, bias_ptr: int | None = None,
                         path: int = PATH_AUTO, cta_pair: bool = False, host_chunks: int = 0):
    """Host-buffer forward from raw host pointers (e.g. pinned torch tensors);
    host_chunks: copy/compute pipeline chunks (0 auto, 1 none)."""
    o = _opts(path, cta_pair, host_chunks)
    _check(lib().moe_b200_forward(w.handle, C.cast(bias_ptr, _fp) if bias_ptr else None,
                                  C.cast(x_ptr, _fp), T, C.cast(out_ptr, _fp),
                                  C.cast(probs_ptr, _fp) if probs_ptr else None,
                                  C.cast(ids_ptr, _ip) if ids_ptr else None, C.byref(o)),
           "moe_b200_forward")


def moe_forward_device(w: MoEWeights, x_ptr: int, T: int, out_ptr: int,
                       probs_ptr: int | None = None, ids_ptr: int | None = None,
                       bias_ptr: int | None = None, path: int = PATH_AUTO,
                       stream: int | None = None, cta_pair: bool = False):
    """Device-buffer forward, asynchronous on `stream` (a cudaStream_t as int)."""
    o = _opts(path, cta_pair)
    _check(lib().moe_b200_forward_device(w.handle, bias_ptr, x_ptr, T, out_ptr, probs_ptr,
                                         ids_ptr, C.byref(o), stream), "moe_b200_forward_device")


def block_ffn(w: MoEWeights, x: np.ndarray, rms_weight: np.ndarray, eps: float = 1e-5,
              bias: np.ndarray | None = None, path: int = PATH_AUTO, cta_pair: bool = False,
              want_norm: bool = True):
    """block_forward's FFN half (src/transformer.c:752-767) on host buffers:
    returns (x + moe(rms_norm(x)) [T×d], rms_norm(x) [T×d] or None,
    probs [T×E], ids [T×k]).  `x` itself is not modified."""
    xo = np.array(x, np.float32, order="C", copy=True)
    T = xo.shape[0]
    xn = np.empty_like(xo) if want_norm else None
    probs = np.empty((T, w.E), np.float32)
    ids = np.empty((T, w.top_k), np.int32)
    rw = np.ascontiguousarray(rms_weight, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    o = _opts(path, cta_pair)
    _check(lib().moe_b200_block_ffn(w.handle, _f(rw), float(eps), _f(b), _f(xo), T, _f(xn),
                                    _f(probs), _i(ids), C.byref(o)), "moe_b200_block_ffn")
    return xo, xn, probs, ids


def block_ffn_host_ptr(w: MoEWeights, rms_ptr: int, eps: float, x_ptr: int, T: int,
                       x_norm_ptr: int | None = None, probs_ptr: int | None = None,
                       ids_ptr: int | None = None, bias_ptr: int | None = None,
                       path: int = PATH_AUTO, cta_pair: bool = False):
    """Host-buffer block FFN from raw host pointers (e.g. pinned torch tensors);
    x updated in place."""
    o = _opts(path, cta_pair)
    cf = lambda p: C.cast(p, _fp) if p else None  # noqa: E731
    _check(lib().moe_b200_block_ffn(w.handle, cf(rms_ptr), float(eps), cf(bias_ptr), cf(x_ptr),
                                    T, cf(x_norm_ptr), cf(probs_ptr),
                                    C.cast(ids_ptr, _ip) if ids_ptr else None, C.byref(o)),
           "moe_b200_block_ffn")


def block_ffn_device(w: MoEWeights, rms_ptr: int, eps: float, x_ptr: int, T: int,
                     x_norm_ptr: int | None = None, probs_ptr: int | None = None,
                     ids_ptr: int | None = None, bias_ptr: int | None = None,
                     path: int = PATH_AUTO, stream: int | None = None, cta_pair: bool = False):
    """Device-buffer block FFN, x updated in place, asynchronous on `stream`."""
    o = _opts(path, cta_pair)
    _check(lib().moe_b200_block_ffn_device(w.handle, rms_ptr, float(eps), bias_ptr, x_ptr, T,
                                           x_norm_ptr, probs_ptr, ids_ptr, C.byref(o), stream),
           "moe_b200_block_ffn_device")


class MoEGrads:
    """Accumulated gradients of an expert set (moe_b200_grads), in llm.c's
    layouts: W_router [d×E], bias [E], W_gate / W_up [d×F], W_down [F×d]."""

    def __init__(self, w: MoEWeights):
        h = _vp()
        _check(lib().moe_b200_grads_create(w.handle, C.byref(h)), "moe_b200_grads_create")
        self.handle = h.value
        self.d, self.F, self.E = w.d, w.F, w.E

    def zero(self):
        _check(lib().moe_b200_grads_zero(self.handle), "moe_b200_grads_zero")

    def download(self):
        """(dW_router, d_bias, [dW_gate], [dW_up], [dW_down])."""
        d, F, E = self.d, self.F, self.E
        wr = np.empty((d, E), np.float32)
        b = np.empty(E, np.float32)
        g = [np.empty((d, F), np.float32) for _ in range(E)]
        u = [np.empty((d, F), np.float32) for _ in range(E)]
        dn = [np.empty((F, d), np.float32) for _ in range(E)]
        _check(lib().moe_b200_grads_download(self.handle, _f(wr), _f(b),
                                              (_fp * E)(*[_f(a) for a in g]),
                                              (_fp * E)(*[_f(a) for a in u]),
                                              (_fp * E)(*[_f(a) for a in dn])),
               "moe_b200_grads_download")
        return wr, b, g, u, dn

    def free(self):
        if self.handle:
            lib().moe_b200_grads_free(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def moe_backward(w: MoEWeights, x: np.ndarray, dy: np.ndarray, grads: MoEGrads,
                 bias: np.ndarray | None = None, aux_coef: float = 0.0, path: int = PATH_FP32):
    """Backward of moe_forward at x given dy (host buffers): returns
    (dx [T×d], L_aux); weight gradients accumulate into `grads`.  path:
    PATH_FP32 (FFMA, 1e-5), PATH_TF32 (tensor cores, 2e-3) or PATH_AUTO."""
    x = np.ascontiguousarray(x, np.float32)
    dy = np.ascontiguousarray(dy, np.float32)
    T = x.shape[0]
    dx = np.empty_like(x)
    aux = np.zeros(1, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    o = _opts(path)
    _check(lib().moe_b200_backward(w.handle, _f(b), _f(x), T, _f(dy), float(aux_coef), _f(dx),
                                   grads.handle, _f(aux), C.byref(o)), "moe_b200_backward")
    return dx, float(aux[0])


def moe_backward_device(w: MoEWeights, x_ptr: int, T: int, dy_ptr: int, dx_ptr: int,
                        grads: MoEGrads, bias_ptr: int | None = None, aux_coef: float = 0.0,
                        aux_ptr: int | None = None, stream: int | None = None,
                        path: int = PATH_FP32):
    """Device-buffer backward, asynchronous on `stream`."""
    o = _opts(path)
    _check(lib().moe_b200_backward_device(w.handle, bias_ptr, x_ptr, T, dy_ptr, float(aux_coef),
                                          dx_ptr, grads.handle, aux_ptr, C.byref(o), stream),
           "moe_b200_backward_device")


def last_counts(w: MoEWeights) -> np.ndarray:
    c = np.empty(w.E, np.int32)
    _check(lib().moe_b200_last_counts(w.handle, _i(c)), "moe_b200_last_counts")
    return c


def last_path() -> int:
    """MOE_B200_PATH_* the last forward on this device ran (AUTO resolved)."""
    return int(lib().moe_b200_last_path())


def last_launches() -> int:
    return int(lib().moe_b200_last_launches())


def synth_fill(dst_ptr: int, n: int, seed: int, stream_id: int, std: float, first: int = 0,
               cuda_stream: int | None = None):
    _check(lib().moe_b200_synth_fill(dst_ptr, n, seed, stream_id, first, std, cuda_stream),
           "moe_b200_synth_fill")


# ---------------------------------------------------------------- drop-in
class LlmcMatrix(C.Structure):
    _fields_ = [("data", _fp), ("grad", _fp), ("rows", C.c_int), ("cols", C.c_int)]


class LlmcFFNWeights(C.Structure):
    _fields_ = [("W_gate", LlmcMatrix), ("W_up", LlmcMatrix), ("W_down", LlmcMatrix)]


class LlmcMoEWeights(C.Structure):
    _fields_ = [("experts", C.POINTER(LlmcFFNWeights)), ("W_router", LlmcMatrix),
                ("n_experts", C.c_int), ("top_k", C.c_int)]


class LlmcModelConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("vocab_size", "max_seq_len", "d_model", "n_layers",
                                       "n_heads", "n_kv_heads", "head_dim", "window_size",
                                       "ffn_hidden", "n_experts", "top_k_experts")] + \
               [("rms_norm_eps", C.c_float), ("rope_theta", C.c_float)]


class LlmcForwardCache(C.Structure):
    _fields_ = [(n, LlmcMatrix) for n in ("x_norm_attn", "x_norm_ffn", "attn_out", "ffn_out",
                                          "Q", "K", "V", "attn_scores", "attn_weighted",
                                          "gate_buf", "up_buf")] + \
               [("router_probs", _fp), ("expert_ids", _ip)]


def _mat(a):
    return LlmcMatrix(_f(a), None, a.shape[0], a.shape[1])


class LlmcMoE:
    """llm.c's own MoEWeights struct built over numpy arrays, for calling the
    exported drop-in `moe_forward` exactly as block_forward does
    (src/transformer.c:761-764)."""

    def __init__(self, W_router, W_gate, W_up, W_down, top_k: int, grads: bool = False):
        self._keep = [np.ascontiguousarray(a, np.float32) for a in (W_router, *W_gate, *W_up, *W_down)]
        E = len(W_gate)
        wr, g, u, dn = self._keep[0], self._keep[1:1 + E], self._keep[1 + E:1 + 2 * E], self._keep[1 + 2 * E:]
        # llm.c's .grad buffers (zeroed) when asked: [W_router, gate.., up.., down..]
        self.grads = [np.zeros_like(a) for a in self._keep] if grads else None

        def mat(i):
            a = self._keep[i]
            gr = _f(self.grads[i]) if grads else None
            return LlmcMatrix(_f(a), gr, a.shape[0], a.shape[1])

        self.experts = (LlmcFFNWeights * E)(*[LlmcFFNWeights(mat(1 + e), mat(1 + E + e), mat(1 + 2 * E + e))
                                             for e in range(E)])
        self.moe = LlmcMoEWeights(self.experts, mat(0), E, top_k)
        self.d, self.E, self.k, self.F = wr.shape[0], E, top_k, g[0].shape[1]

    def backward(self, x: np.ndarray, d_out: np.ndarray) -> np.ndarray:
        """llm.c-style moe_backward: adds into self.grads, returns d_x."""
        L = lib()
        L.moe_backward.argtypes = [C.POINTER(LlmcMatrix), C.POINTER(LlmcMoEWeights),
                                   C.POINTER(LlmcModelConfig), C.c_void_p,
                                   C.POINTER(LlmcMatrix), C.POINTER(LlmcMatrix)]
        L.moe_backward.restype = None
        x = np.ascontiguousarray(x, np.float32)
        d_out = np.ascontiguousarray(d_out, np.float32)
        d_x = np.empty_like(x)
        cfg = LlmcModelConfig()
        cfg.d_model, cfg.ffn_hidden, cfg.n_experts, cfg.top_k_experts = self.d, self.F, self.E, self.k
        L.moe_backward(C.byref(_mat(x)), C.byref(self.moe), C.byref(cfg), None,
                       C.byref(_mat(d_out)), C.byref(_mat(d_x)))
        return d_x

    def forward(self, x: np.ndarray):
        L = lib()
        L.moe_forward.argtypes = [C.POINTER(LlmcMatrix), C.POINTER(LlmcMoEWeights),
                                  C.POINTER(LlmcModelConfig), C.POINTER(LlmcForwardCache),
                                  C.POINTER(LlmcMatrix)]
        L.moe_forward.restype = None
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        out = np.empty((T, self.d), np.float32)
        probs = np.empty((T, self.E), np.float32)
        ids = np.empty((T, self.k), np.int32)
        cfg = LlmcModelConfig()
        cfg.d_model, cfg.ffn_hidden, cfg.n_experts, cfg.top_k_experts = self.d, self.F, self.E, self.k
        cache = LlmcForwardCache()
        cache.router_probs = _f(probs)
        cache.expert_ids = _i(ids)
        xm, om = _mat(x), _mat(out)
        L.moe_forward(C.byref(xm), C.byref(self.moe), C.byref(cfg), C.byref(cache), C.byref(om))
        return out, probs, ids

    def invalidate(self):
        L = lib()
        L.moe_b200_invalidate.argtypes = [_vp]
        _check(L.moe_b200_invalidate(C.addressof(self.moe)), "moe_b200_invalidate")


STAGES = ("router", "dispatch", "upgate", "down", "combine")


def profile_enable(on: bool = True):
    _check(lib().moe_b200_profile_enable(1 if on else 0), "moe_b200_profile_enable")


def device_info(device: int = -1):
    """(SM count, co-resident CTA pairs of the TF32 pair GEMM) of a device."""
    n, pairs = C.c_int(), C.c_int()
    _check(lib().moe_b200_device_info(device, C.byref(n), C.byref(pairs)), "moe_b200_device_info")
    return int(n.value), int(pairs.value)


def profile_read():
    """(dict stage -> summed device ms, number of forwards) since the last read."""
    ms = (C.c_double * len(STAGES))()
    n = C.c_int()
    _check(lib().moe_b200_profile_read(ms, C.byref(n)), "moe_b200_profile_read")
    return {k: float(ms[i]) for i, k in enumerate(STAGES)}, int(n.value)


NOALLOC_SCRATCH_BYTES = 16 << 20


def moe_forward_noalloc(w: MoEWeights, x_ptr: int, T: int, out_ptr: int,
                        probs_ptr: int | None = None, ids_ptr: int | None = None,
                        bias_ptr: int | None = None, stream: int | None = None):
    """Allocation-free forward on device buffers (FP32 expert path, synchronous).

    For callers that may not allocate device memory while they run: all
    intermediates live in a fixed 16 MiB array inside the library; shapes
    that need more are rejected (MoEError with status E_INVALID)."""
    L = lib()
    L.moe_b200_forward_noalloc.argtypes = [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp]
    _check(L.moe_b200_forward_noalloc(w.handle, bias_ptr, x_ptr, T, out_ptr, probs_ptr, ids_ptr,
                                      stream), "moe_b200_forward_noalloc")


# ---------------------------------------------------------------- expert parallel
EP_ID_BYTES = 128


def ep_unique_id() -> bytes:
    buf = C.create_string_buffer(EP_ID_BYTES)
    _check(lib().moe_b200_ep_unique_id(buf), "moe_b200_ep_unique_id")
    return buf.raw


def ep_split(counts_all: np.ndarray, place: np.ndarray, n_slots: int):
    """The per-forward split of every expert's rows among its holders, from
    the per-rank expert counts [world × E] and the placement [world × E]
    (slot of expert e on rank q, -1 = not held).  Returns a dict of numpy
    arrays: n_holders [E], holders [E × world], row_begin [E × (world+1)],
    recv_offset [E × world], recv_rows [world], cost [world]."""
    c = np.ascontiguousarray(counts_all, np.int32)
    pl = np.ascontiguousarray(place, np.int32)
    G, E = c.shape
    nh = np.empty(E, np.int32)
    hold = np.empty((E, G), np.int32)
    beg = np.empty((E, G + 1), np.int32)
    dst = np.empty((E, G), np.int32)
    rows = np.empty(G, np.int64)
    cost = np.empty(G, np.int64)
    L = lib()
    L.moe_b200_ep_split.argtypes = [_ip, C.c_int, C.c_int, _ip, C.c_int, _ip, _ip, _ip, _ip,
                                    C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]
    ll = C.POINTER(C.c_longlong)
    _check(L.moe_b200_ep_split(_i(c), G, E, _i(pl), n_slots, _i(nh), _i(hold), _i(beg), _i(dst),
                               rows.ctypes.data_as(ll), cost.ctypes.data_as(ll)),
           "moe_b200_ep_split")
    return dict(n_holders=nh, holders=hold, row_begin=beg, recv_offset=dst, recv_rows=rows,
                cost=cost)


def ep_place(counts_all: np.ndarray, base_place: np.ndarray, n_slots: int) -> np.ndarray:
    """The load-aware placement moe_b200_ep_rebalance adopts for these
    counts: the base placement plus replicas in spare slots."""
    c = np.ascontiguousarray(counts_all, np.int32)
    b = np.ascontiguousarray(base_place, np.int32)
    G, E = c.shape
    out = np.empty((G, E), np.int32)
    L = lib()
    L.moe_b200_ep_place.argtypes = [_ip, C.c_int, C.c_int, _ip, C.c_int, _ip]
    _check(L.moe_b200_ep_place(_i(c), G, E, _i(b), n_slots, _i(out)), "moe_b200_ep_place")
    return out


def ep_shard_experts(E: int, world: int, rank: int) -> list:
    """The base shard of `rank`: experts rank, rank + world, rank + 2·world, ...
    Strided, so that every rank gets a mix of popular and rare experts when
    popularity falls with the expert index (the rare ones each cost a pass
    over their weights for a handful of rows)."""
    return list(range(rank, E, world))


class EP:
    """An expert-parallel group member (collective calls on every rank)."""

    def __init__(self, uid: bytes, rank: int, world: int, max_tokens: int, w: MoEWeights):
        L = lib()
        L.moe_b200_ep_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int, _vp,
                                         C.POINTER(_vp)]
        L.moe_b200_ep_destroy.argtypes = [_vp]
        L.moe_b200_ep_forward_device.argtypes = [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp,
                                                 C.POINTER(Opts), _vp]
        L.moe_b200_ep_forward.argtypes = [_vp, _fp, _fp, C.c_int, _fp, _fp, _ip,
                                          C.POINTER(Opts)]
        L.moe_b200_ep_counts.argtypes = [_vp, _ip, _ip]
        L.moe_b200_ep_placement.argtypes = [_vp, _ip]
        L.moe_b200_ep_rebalance.argtypes = [_vp]
        L.moe_b200_ep_set_timeout.argtypes = [_vp, C.c_int]
        h = _vp()
        _check(L.moe_b200_ep_create(uid, rank, world, max_tokens, w.handle, C.byref(h)),
               "moe_b200_ep_create")
        self.handle, self.rank, self.world, self.w = h.value, rank, world, w

    def forward_device(self, x_ptr, T, out_ptr, probs_ptr=None, ids_ptr=None, bias_ptr=None,
                       path=PATH_AUTO, stream=None):
        o = _opts(path)
        _check(lib().moe_b200_ep_forward_device(self.handle, bias_ptr, x_ptr, T, out_ptr,
                                                probs_ptr, ids_ptr, C.byref(o), stream),
               "moe_b200_ep_forward_device")

    def forward(self, x: np.ndarray, bias: np.ndarray | None = None, path=PATH_AUTO,
                host_chunks: int = 0):
        """Host-buffer forward (collective); host_chunks as moe_b200_opts, the
        same on every rank."""
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        w = self.w
        out = np.empty((T, w.d), np.float32)
        probs = np.empty((T, w.E), np.float32)
        ids = np.empty((T, w.top_k), np.int32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        o = _opts(path, host_chunks=host_chunks)
        _check(lib().moe_b200_ep_forward(self.handle, _f(b), _f(x), T, _f(out), _f(probs),
                                         _i(ids), C.byref(o)), "moe_b200_ep_forward")
        return out, probs, ids

    def forward_host_ptr(self, x_ptr, T, out_ptr, probs_ptr, ids_ptr, bias_ptr=None,
                         path=PATH_AUTO):
        o = _opts(path)
        _check(lib().moe_b200_ep_forward(self.handle, C.cast(bias_ptr, _fp) if bias_ptr else None,
                                         C.cast(x_ptr, _fp), T, C.cast(out_ptr, _fp),
                                         C.cast(probs_ptr, _fp) if probs_ptr else None,
                                         C.cast(ids_ptr, _ip) if ids_ptr else None, C.byref(o)),
               "moe_b200_ep_forward")

    def counts(self):
        c = np.empty((self.world, self.w.E), np.int32)
        rows = C.c_int()
        _check(lib().moe_b200_ep_counts(self.handle, _i(c), C.byref(rows)), "moe_b200_ep_counts")
        return c, int(rows.value)

    def placement(self) -> np.ndarray:
        """[world × E]: slot of expert e on rank q, -1 = not held."""
        out = np.empty((self.world, self.w.E), np.int32)
        _check(lib().moe_b200_ep_placement(self.handle, _i(out)), "moe_b200_ep_placement")
        return out

    def rebalance(self):
        """Collective: replicate hot experts into spare slots from the last
        forward's counts."""
        _check(lib().moe_b200_ep_rebalance(self.handle), "moe_b200_ep_rebalance")

    def set_timeout(self, ms: int):
        _check(lib().moe_b200_ep_set_timeout(self.handle, int(ms)), "moe_b200_ep_set_timeout")

    def destroy(self):
        if self.handle:
            lib().moe_b200_ep_destroy(self.handle)
            self.handle = 0


def debug_fail_alloc(n: int):
    """Fail the n-th device allocation the library makes from now on (0: off)."""
    L = lib()
    L.moe_b200_debug_fail_alloc.argtypes = [C.c_int]
    _check(L.moe_b200_debug_fail_alloc(int(n)), "moe_b200_debug_fail_alloc")


def debug_wait_probe(limit_us: int, arrive: bool):
    """A bounded mbarrier wait on the device; raises MoEError(E_TIMEOUT) when
    nobody arrives."""
    L = lib()
    L.moe_b200_debug_wait_probe.argtypes = [C.c_int, C.c_int]
    _check(L.moe_b200_debug_wait_probe(int(limit_us), 1 if arrive else 0),
           "moe_b200_debug_wait_probe")


def llmc_trace_enable(on: bool = True):
    """Record each layer's (x_norm, ffn_out) in the host inference_step."""
    _check(lib().moe_b200_llmc_trace_enable(1 if on else 0), "moe_b200_llmc_trace_enable")


def llmc_trace_read(layer: int, d: int):
    xn = np.empty(d, np.float32)
    fo = np.empty(d, np.float32)
    _check(lib().moe_b200_llmc_trace_read(int(layer), _f(xn), _f(fo)), "moe_b200_llmc_trace_read")
    return xn, fo


def _path(path) -> bytes:
    return str(path).encode()


def checkpoint_config(path) -> "LlmcModelConfig":
    """The ModelConfig stored in an llm.c checkpoint (model_save format)."""
    cfg = LlmcModelConfig()
    _check(lib().moe_b200_checkpoint_config(_path(path), C.byref(cfg)),
           "moe_b200_checkpoint_config")
    return cfg


class Decoder:
    """Device-resident single-token decode of an llm.c Model (ctypes pointer
    or address of an llmc_Model, e.g. from llmc_model.LlmcDecoder or the
    reference's model_init): llm.c's inference_step on the B200."""

    STAGE_KERNELS = 1      # one kernel per stage (the default)
    PERSISTENT = 2         # the whole step as one persistent cooperative kernel

    def __init__(self, model_ptr, max_seq: int, flags: int = 0):
        L = lib()
        h = _vp()
        _check(L.moe_b200_decoder_create(model_ptr, int(max_seq), int(flags), C.byref(h)),
               "moe_b200_decoder_create")
        self.handle = h
        self._vocab = None

    @classmethod
    def from_checkpoint(cls, path, max_seq: int, flags: int = 0) -> "Decoder":
        """A device decoder straight from an llm.c checkpoint file; no llm.c
        Model is built on the host."""
        h = _vp()
        _check(lib().moe_b200_decoder_load(_path(path), int(max_seq), int(flags), C.byref(h)),
               "moe_b200_decoder_load")
        self = cls.__new__(cls)
        self.handle = h
        self._vocab = None
        return self

    def step(self, token: int, logits: np.ndarray | None = None):
        """Run one step; fills `logits` (float32, vocab) when given."""
        ptr = None if logits is None else _f(logits)
        _check(lib().moe_b200_decoder_step(self.handle, int(token), ptr), "moe_b200_decoder_step")

    def set_pos(self, pos: int):
        _check(lib().moe_b200_decoder_set_pos(self.handle, int(pos)), "moe_b200_decoder_set_pos")

    @property
    def pos(self) -> int:
        return int(lib().moe_b200_decoder_pos(self.handle))

    @property
    def launches(self) -> int:
        return int(lib().moe_b200_decoder_launches(self.handle))

    def trace(self, layer: int, d: int):
        """(x_norm, ffn_out) of `layer` in the last step: the pre-FFN
        normalised vector and the FFN/MoE output before the residual add."""
        xn = np.empty(d, np.float32)
        fo = np.empty(d, np.float32)
        _check(lib().moe_b200_decoder_trace(self.handle, int(layer), _f(xn), _f(fo)),
               "moe_b200_decoder_trace")
        return xn, fo

    def stage_times(self, n_layers: int) -> np.ndarray:
        """[5 L + 1, 4] stage timeline of the last step in microseconds
        (decoder created with MOE_B200_DECODER_STAMPS=1): earliest entry,
        earliest and latest return from the wait, latest exit."""
        ns = 5 * n_layers + 1
        out = np.empty(4 * ns, np.float64)
        rc = lib().moe_b200_decoder_stage_times(
            self.handle, out.ctypes.data_as(C.POINTER(C.c_double)), int(out.size))
        if rc < 0:
            _check(rc, "moe_b200_decoder_stage_times")
        return out.reshape(ns, 4)

    def free(self):
        if self.handle:
            lib().moe_b200_decoder_destroy(self.handle)
            self.handle = None
