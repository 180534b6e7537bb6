"""ctypes bindings for the CPU test oracle (oracle/liboracle.so) and for the
reference build (oracle/_ref/libllmref.so).

Test infrastructure only: tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent.parent
ORACLE_SO = REPO / "oracle" / "liboracle.so"
REF_SO = REPO / "oracle" / "_ref" / "libllmref.so"

_fp = C.POINTER(C.c_float)
_ip = C.POINTER(C.c_int)
_fpp = C.POINTER(_fp)


def _f(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


def _i(a):
    if a is None:
        return None
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_ip)


def _ptr_array(arrs):
    return (_fp * len(arrs))(*[_f(a) for a in arrs])


_oracle = None
_ref = None


def oracle():
    global _oracle
    if _oracle is None:
        lib = C.CDLL(str(ORACLE_SO))
        lib.oracle_synth_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64,
                                            C.c_size_t, C.c_float, _fp]
        lib.oracle_stream_x.restype = C.c_uint64
        lib.oracle_stream_router.restype = C.c_uint64
        lib.oracle_stream_bias.restype = C.c_uint64
        lib.oracle_stream_expert.restype = C.c_uint64
        lib.oracle_stream_expert.argtypes = [C.c_int, C.c_int]
        lib.oracle_exp_ref.restype = C.c_float
        lib.oracle_exp_ref.argtypes = [C.c_float]
        lib.oracle_softmax_rows.argtypes = [_fp, C.c_int, C.c_int]
        lib.oracle_swiglu.argtypes = [_fp, _fp, _fp, C.c_int]
        lib.oracle_router.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, C.c_int,
                                      C.c_int, _fp, _fp, _ip, _fp]
        lib.oracle_moe_forward.argtypes = [
            _fp, C.c_int, C.c_int, _fp, _fp, C.c_int, C.c_int,
            _fpp, _fpp, _fpp, C.c_int, _ip, C.c_int, _ip, _fp, _fp, _ip, C.c_int]
        lib.oracle_moe_forward_synth.argtypes = [
            _fp, C.c_int, C.c_int, _fp, _fp, C.c_int, C.c_int, C.c_int,
            C.c_uint64, C.c_float, _ip, C.c_int, _ip, _fp, _fp, _ip, C.c_int]
        lib.oracle_rms_norm.argtypes = [_fp, C.c_int, C.c_int, _fp, C.c_float, _fp]
        lib.oracle_rms_norm.restype = None
        lib.oracle_block_ffn.argtypes = [_fp, C.c_int, C.c_int, _fp, C.c_float, _fp, _fp,
                                         C.c_int, C.c_int, C.c_int, C.POINTER(_fp),
                                         C.POINTER(_fp), C.POINTER(_fp), _fp, _fp, _ip, C.c_int]
        lib.oracle_block_ffn.restype = None
        lib.oracle_ffn_forward.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, _fp,
                                           C.c_int, _fp]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return REF_SO.exists()


def ref():
    global _ref
    if _ref is None:
        lib = C.CDLL(str(REF_SO))
        lib.ref_set_threads.argtypes = [C.c_int]
        lib.ref_moe_forward.argtypes = [_fp, C.c_int, C.c_int, _fp, C.c_int,
                                        C.c_int, _fpp, _fpp, _fpp, C.c_int,
                                        _fp, _fp, _ip]
        lib.ref_moe_forward.restype = C.c_int
        lib.ref_softmax_rows.argtypes = [_fp, C.c_int, C.c_int]
        lib.ref_swiglu.argtypes = [_fp, _fp, _fp, C.c_int]
        lib.ref_ffn_forward.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, _fp,
                                        C.c_int, _fp]
        lib.ref_model_init.restype = C.c_void_p
        lib.ref_model_init.argtypes = [C.c_int] * 11 + [C.c_float, C.c_float, C.c_uint]
        lib.ref_model_free.argtypes = [C.c_void_p]
        lib.ref_model_forward_last.argtypes = [C.c_void_p, _ip, C.c_int, _fp]
        lib.ref_model_forward_rows.argtypes = [C.c_void_p, _ip, C.c_int, C.c_int, _fp]
        lib.ref_model_forward_rows.restype = None
        lib.ref_model_moe_forward.argtypes = [C.c_void_p, C.c_int, _fp, C.c_int, _fp, _fp, _ip]
        lib.ref_model_moe_forward.restype = C.c_int
        lib.ref_inference_init.restype = C.c_void_p
        lib.ref_inference_init.argtypes = [C.c_void_p]
        lib.ref_inference_free.argtypes = [C.c_void_p]
        lib.ref_inference_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        lib.ref_inference_logits.restype = _fp
        lib.ref_inference_logits.argtypes = [C.c_void_p]
        lib.ref_inference_pos.restype = C.c_int
        lib.ref_inference_pos.argtypes = [C.c_void_p]
        lib.ref_ffn_backward.argtypes = [_fp, C.c_int, C.c_int, _fp, _fp, _fp, C.c_int, _fp,
                                         _fp, _fp, _fp, _fp]
        lib.ref_ffn_backward.restype = None
        lib.ref_rms_norm.argtypes = [_fp, C.c_int, C.c_int, _fp, C.c_float, _fp]
        lib.ref_rms_norm.restype = None
        lib.ref_model_save.restype = C.c_int
        lib.ref_model_save.argtypes = [C.c_void_p, C.c_char_p]
        lib.ref_model_load.restype = C.c_void_p
        lib.ref_model_load.argtypes = [C.c_char_p]
        _ref = lib
    return _ref


# ---------------------------------------------------------------- generator

def synth(seed: int, stream: int, n: int, std: float, first: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    oracle().oracle_synth_normal(seed, stream, first, n, std, _f(out))
    return out


def stream_x():
    return oracle().oracle_stream_x()


def stream_router():
    return oracle().oracle_stream_router()


def stream_bias():
    return oracle().oracle_stream_bias()


def stream_expert(e, which):
    return oracle().oracle_stream_expert(e, which)


class MoEProblem:
    """Seeded synthetic MoE layer in the reference's host layout.

    x [T×d] ~ N(0, x_std); W_router [d×E], W_gate/W_up [d×F], W_down [F×d]
    ~ N(0, w_std); bias: None, "normal" (b_e ~ N(0,1)) or "zipf" (b_e =
    -s·ln(e+1), expert popularity ∝ (e+1)^-s).
    """

    def __init__(self, T, d, E, k, F, seed=0, w_std=0.02, x_std=1.0,
                 bias=None, zipf_s=1.1, with_experts=True):
        self.T, self.d, self.E, self.k, self.F = T, d, E, k, F
        self.seed, self.w_std = seed, w_std
        self.x = synth(seed, stream_x(), T * d, x_std).reshape(T, d)
        self.W_router = synth(seed, stream_router(), d * E, w_std).reshape(d, E)
        if bias is None:
            self.bias = None
        elif not isinstance(bias, str):
            self.bias = np.ascontiguousarray(bias, dtype=np.float32)
        elif bias == "normal":
            self.bias = synth(seed, stream_bias(), E, 1.0)
        elif bias == "zipf":
            self.bias = (-zipf_s * np.log(np.arange(1, E + 1, dtype=np.float64))).astype(np.float32)
        else:
            self.bias = np.ascontiguousarray(bias, dtype=np.float32)
        self.experts = None
        if with_experts:
            self.experts = []
            for e in range(E):
                g = synth(seed, stream_expert(e, 0), d * F, w_std).reshape(d, F)
                u = synth(seed, stream_expert(e, 1), d * F, w_std).reshape(d, F)
                dn = synth(seed, stream_expert(e, 2), F * d, w_std).reshape(F, d)
                self.experts.append((g, u, dn))

    # ------------------------------------------------------------ oracle
    def oracle_router(self):
        T, E, k = self.T, self.E, self.k
        logits = np.empty((T, E), np.float32)
        probs = np.empty((T, E), np.float32)
        ids = np.empty((T, k), np.int32)
        wts = np.empty((T, k), np.float32)
        oracle().oracle_router(_f(self.x), T, self.d, _f(self.W_router),
                               _f(self.bias), E, k, _f(logits), _f(probs),
                               _i(ids), _f(wts))
        return logits, probs, ids, wts

    def oracle_forward(self, rows=None, forced_ids=None, threads=0):
        T, d, E, k, F = self.T, self.d, self.E, self.k, self.F
        rows_arr = None if rows is None else np.ascontiguousarray(rows, np.int32)
        nr = T if rows is None else len(rows_arr)
        out = np.empty((nr, d), np.float32)
        probs = np.empty((T, E), np.float32)
        ids = np.empty((T, k), np.int32)
        fid = None if forced_ids is None else np.ascontiguousarray(forced_ids, np.int32)
        if self.experts is not None:
            g = _ptr_array([e[0] for e in self.experts])
            u = _ptr_array([e[1] for e in self.experts])
            dn = _ptr_array([e[2] for e in self.experts])
            oracle().oracle_moe_forward(_f(self.x), T, d, _f(self.W_router),
                                        _f(self.bias), E, k, g, u, dn, F,
                                        _i(rows_arr), nr, _i(fid), _f(out),
                                        _f(probs), _i(ids), threads)
        else:
            oracle().oracle_moe_forward_synth(_f(self.x), T, d, _f(self.W_router),
                                              _f(self.bias), E, k, F, self.seed,
                                              self.w_std, _i(rows_arr), nr,
                                              _i(fid), _f(out), _f(probs),
                                              _i(ids), threads)
        return out, probs, ids

    # ------------------------------------------------------------ reference
    def ref_forward(self, threads=0):
        assert self.bias is None, "the reference router has no bias"
        T, d, E, k, F = self.T, self.d, self.E, self.k, self.F
        out = np.empty((T, d), np.float32)
        probs = np.empty((T, E), np.float32)
        ids = np.empty((T, k), np.int32)
        lib = ref()
        if threads > 0:
            lib.ref_set_threads(threads)
        g = _ptr_array([e[0] for e in self.experts])
        u = _ptr_array([e[1] for e in self.experts])
        dn = _ptr_array([e[2] for e in self.experts])
        rc = lib.ref_moe_forward(_f(self.x), T, d, _f(self.W_router), E, k,
                                 g, u, dn, F, _f(out), _f(probs), _i(ids))
        assert rc == 0
        return out, probs, ids


def stream_rms():
    """Synthetic stream of the RMSNorm weights (clear of the expert streams,
    which start at 0x100)."""
    return 4


class BlockProblem(MoEProblem):
    """The FFN half of llm.c's block_forward (src/transformer.c:752-767) on a
    seeded synthetic MoE layer: x is the residual stream (N(0, x_std)), the
    block's rms_ffn weights are 1 + N(0, 0.1), eps as llm.c's configs."""

    def __init__(self, T, d, E, k, F, seed=0, x_std=4.0, eps=1e-5, **kw):
        super().__init__(T, d, E, k, F, seed=seed, x_std=x_std, **kw)
        self.eps = np.float32(eps)
        self.rms_w = (np.float32(1.0) + synth(seed, stream_rms(), d, 0.1)).astype(np.float32)

    def oracle_rms(self):
        xn = np.empty_like(self.x)
        oracle().oracle_rms_norm(_f(self.x), self.T, self.d, _f(self.rms_w), self.eps, _f(xn))
        return xn

    def ref_rms(self):
        xn = np.empty_like(self.x)
        ref().ref_rms_norm(_f(self.x), self.T, self.d, _f(self.rms_w), self.eps, _f(xn))
        return xn

    def moe_on(self, xn):
        """This layer's MoE problem with x_norm as its input."""
        moe = MoEProblem.__new__(MoEProblem)
        moe.__dict__.update(self.__dict__)
        moe.x = np.ascontiguousarray(xn, np.float32)
        return moe

    def oracle_block(self, threads=0):
        """(x after the block, x_norm, probs, ids) from the CPU restatement."""
        T, d, E, k, F = self.T, self.d, self.E, self.k, self.F
        x = self.x.copy()
        xn = np.empty_like(x)
        probs = np.empty((T, E), np.float32)
        ids = np.empty((T, k), np.int32)
        g = _ptr_array([e[0] for e in self.experts])
        u = _ptr_array([e[1] for e in self.experts])
        dn = _ptr_array([e[2] for e in self.experts])
        oracle().oracle_block_ffn(_f(x), T, d, _f(self.rms_w), self.eps, _f(self.W_router),
                                  _f(self.bias), E, k, F, g, u, dn, _f(xn), _f(probs), _i(ids),
                                  threads)
        return x, xn, probs, ids

    def ref_block(self, threads=0):
        """The same through the reference's own rms_norm and moe_forward, plus
        the FFN output (cache->ffn_out); the residual add is
        mat_add_inplace's plain fp32 add."""
        xn = self.ref_rms()
        out, probs, ids = self.moe_on(xn).ref_forward(threads=threads)
        return (self.x + out).astype(np.float32), xn, probs, ids, out


def routing_mismatch_allowed(logits_row: np.ndarray, ids_a, ids_b, k: int,
                             gap: float = 1e-6) -> bool:
    """True when two top-k rankings of one token differ only where the
    logits of the swapped experts lie within `gap` of each other (the
    near-tie exemption for routing parity)."""
    a, b = list(ids_a), list(ids_b)
    for r in range(k):
        if a[r] != b[r]:
            if abs(float(logits_row[a[r]]) - float(logits_row[b[r]])) >= gap:
                return False
    return True


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max|got - want| / max|want| (the layer-output tolerance measure)."""
    den = float(np.max(np.abs(want)))
    if den == 0.0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got.astype(np.float64) - want.astype(np.float64)))) / den


def release_ref_model(m_ptr):
    """Free a reference llm.c Model (from ref_model_init) after dropping the
    device copies the B200 library keeps for it: the expert sets uploaded by
    the drop-in moe_forward / inference_step (keyed by each block's
    MoEWeights pointer, or for dense blocks run through the block FFN drop-in
    by their FFNWeights pointer, the same union member) and inference_step's
    device decoder (keyed by the Model pointer).  The library's residency cache is keyed by pointer, so
    a later model allocated at the same addresses would otherwise meet the
    stale copies (its contract: invalidate before changing or freeing)."""
    import moe_b200 as M
    import llmc_model as LM
    L = M.lib()
    L.moe_b200_invalidate.argtypes = [C.c_void_p]
    model = LM.Model.from_address(m_ptr)
    ffn_off = LM.BlockWeights.u.offset        # the FFNWeights / MoEWeights union
    for l in range(model.weights.n_layers):
        L.moe_b200_invalidate(C.addressof(model.weights.blocks[l]) + ffn_off)
    L.moe_b200_invalidate(m_ptr)
    ref().ref_model_free(m_ptr)
