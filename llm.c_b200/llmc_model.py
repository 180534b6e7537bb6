"""llm.c model and inference-state structs built over numpy arrays, for
driving the drop-in `inference_step` (llm.c src/inference.c:231-358 with
the MoE branch on the B200) from Python.

The structs mirror llm.c's own layouts field for field (include/llmc_moe.h
names each one's source), so the same objects can also be handed to
llm.c's C functions.  Weights are seeded N(0, std) from numpy (configs
"weights ~N(0, 0.02)"), RMSNorm scales are ones, and the RoPE tables follow
llm.c's definition cos/sin(pos / theta^(2i/head_dim)) (include/attention.h
:66-80).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

import moe_b200 as M

_fp = C.POINTER(C.c_float)


class AttentionWeights(C.Structure):
    _fields_ = [("W_Q", M.LlmcMatrix), ("W_K", M.LlmcMatrix), ("W_V", M.LlmcMatrix),
                ("W_O", M.LlmcMatrix)]


class RoPEBuffer(C.Structure):
    _fields_ = [("cos_table", _fp), ("sin_table", _fp), ("max_seq_len", C.c_int),
                ("head_dim", C.c_int)]


class _FfnOrMoe(C.Union):
    _fields_ = [("ffn", M.LlmcFFNWeights), ("moe", M.LlmcMoEWeights)]


class BlockWeights(C.Structure):
    _anonymous_ = ("u",)
    _fields_ = [("rms_attn", _fp), ("attn", AttentionWeights), ("rms_ffn", _fp),
                ("use_moe", C.c_int), ("u", _FfnOrMoe)]


class ModelWeights(C.Structure):
    _fields_ = [("embed", M.LlmcMatrix), ("blocks", C.POINTER(BlockWeights)),
                ("n_layers", C.c_int), ("rms_final", _fp), ("lm_head", M.LlmcMatrix)]


class Model(C.Structure):
    _fields_ = [("cfg", M.LlmcModelConfig), ("weights", ModelWeights),
                ("caches", C.c_void_p), ("rope", RoPEBuffer), ("train_scratch", C.c_void_p)]


class LayerKVCache(C.Structure):
    _fields_ = [("K", _fp), ("V", _fp)]


class InferenceState(C.Structure):
    _fields_ = [("kv_cache", C.POINTER(LayerKVCache)), ("n_layers", C.c_int),
                ("seq_pos", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("kv_dim", C.c_int), ("max_seq_len", C.c_int)] + \
               [(n, _fp) for n in ("x", "x_norm", "q", "k", "v", "attn_buf", "head_out",
                                   "logits")]


@dataclass
class DecodeConfig:
    vocab: int = 4096
    d: int = 384
    n_layers: int = 6
    n_heads: int = 6
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 1536
    n_experts: int = 8
    top_k: int = 2
    max_seq: int = 640
    eps: float = 1e-5
    theta: float = 1e4
    std: float = 0.02


def _f(a):
    return a.ctypes.data_as(_fp)


def _mat(a):
    return M.LlmcMatrix(_f(a), None, a.shape[0], a.shape[1])


class LlmcDecoder:
    """An llm.c model (MoE in every block when n_experts > 1) plus its
    InferenceState; `step(token)` runs the drop-in inference_step."""

    def __init__(self, c: DecodeConfig, seed: int = 0):
        rng = np.random.default_rng(seed)
        self.c = c
        self._keep = []

        def arr(*shape, std=c.std, ones=False):
            a = (np.ones(shape, np.float32) if ones else
                 (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)))
            a = np.ascontiguousarray(a)
            self._keep.append(a)
            return a

        def zeros(*shape):
            a = np.zeros(shape, np.float32)
            self._keep.append(a)
            return a

        d, kv, nq = c.d, c.n_kv_heads * c.head_dim, c.n_heads * c.head_dim
        cfg = M.LlmcModelConfig()
        cfg.vocab_size, cfg.max_seq_len, cfg.d_model, cfg.n_layers = c.vocab, c.max_seq, d, c.n_layers
        cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.window_size = c.n_heads, c.n_kv_heads, c.head_dim, 0
        cfg.ffn_hidden, cfg.n_experts, cfg.top_k_experts = c.ffn, c.n_experts, c.top_k
        cfg.rms_norm_eps, cfg.rope_theta = c.eps, c.theta
        blocks = (BlockWeights * c.n_layers)()
        self._experts = []
        for l in range(c.n_layers):
            b = blocks[l]
            b.rms_attn = _f(arr(d, ones=True))
            b.attn = AttentionWeights(_mat(arr(d, nq)), _mat(arr(d, kv)), _mat(arr(d, kv)),
                                      _mat(arr(nq, d)))
            b.rms_ffn = _f(arr(d, ones=True))
            if c.n_experts > 1:
                b.use_moe = 1
                ex = (M.LlmcFFNWeights * c.n_experts)(*[
                    M.LlmcFFNWeights(_mat(arr(d, c.ffn)), _mat(arr(d, c.ffn)), _mat(arr(c.ffn, d)))
                    for _ in range(c.n_experts)])
                self._experts.append(ex)
                b.moe = M.LlmcMoEWeights(ex, _mat(arr(d, c.n_experts)), c.n_experts, c.top_k)
            else:
                b.use_moe = 0
                b.ffn = M.LlmcFFNWeights(_mat(arr(d, c.ffn)), _mat(arr(d, c.ffn)), _mat(arr(c.ffn, d)))
        half = c.head_dim // 2
        pos = np.arange(c.max_seq, dtype=np.float64)[:, None]
        inv = c.theta ** (-2.0 * np.arange(half, dtype=np.float64) / c.head_dim)
        cos_t = np.ascontiguousarray(np.cos(pos * inv), np.float32)
        sin_t = np.ascontiguousarray(np.sin(pos * inv), np.float32)
        self._keep += [cos_t, sin_t]
        w = ModelWeights(_mat(arr(c.vocab, d)), blocks, c.n_layers, _f(arr(d, ones=True)),
                         _mat(arr(d, c.vocab)))
        self._blocks = blocks
        self.model = Model(cfg, w, None, RoPEBuffer(_f(cos_t), _f(sin_t), c.max_seq, c.head_dim),
                           None)
        kvs = (LayerKVCache * c.n_layers)()
        for l in range(c.n_layers):
            kvs[l] = LayerKVCache(_f(zeros(c.max_seq, kv)), _f(zeros(c.max_seq, kv)))
        self._kvs = kvs
        self.state = InferenceState(kvs, c.n_layers, 0, c.n_kv_heads, c.head_dim, kv, c.max_seq,
                                    *[_f(zeros(n)) for n in (d, d, nq, kv, kv, c.max_seq, nq,
                                                              c.vocab)])
        L = M.lib()
        L.inference_step.argtypes = [C.POINTER(Model), C.POINTER(InferenceState), C.c_int]
        L.inference_step.restype = None
        self._step = L.inference_step

    def step(self, token: int):
        self._step(C.byref(self.model), C.byref(self.state), int(token))

    def logits(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.state.logits, shape=(self.c.vocab,)).copy()

    @property
    def pos(self) -> int:
        return int(self.state.seq_pos)

    def moe_weight_structs(self):
        """(layer, llmc MoEWeights struct) of every MoE block."""
        return [(l, self._blocks[l].moe) for l in range(self.c.n_layers) if self._blocks[l].use_moe]
