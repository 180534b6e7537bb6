"""Decode-site parity (configuration 2's model shape): llm.c's single-token
KV-cache forward, with the MoE branch that the reference leaves as a TODO
(src/inference.c:342-343) filled by the B200 MoE path, against the
reference's own full-sequence model_forward (src/transformer.c:774-802),
which does run MoE in every block (through its CPU moe_forward).  Both see
the same reference model (model_init with a fixed srand seed); window 0 so
the training-side attention attends to all positions like inference_step.

Tolerance: the last position's logits within 1e-4 of max|logit| and the
same argmax; the dense model (E=1) matches llm.c's own inference_step."""
import ctypes as C

import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="reference build absent")]


def _model(E, k, max_seq, seed=1, L=6):
    # d=384, 6 heads, 2 KV heads, head_dim 64, d_ff 1536, RoPE theta 1e4, vocab 4096
    return O.ref().ref_model_init(4096, max_seq, 384, L, 6, 2, 64, 0, 1536, E, k, 1e-5, 1e4, seed)


def _ours():
    L = M.lib()
    L.inference_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    L.inference_step.restype = None
    return L


def test_moe_decode_steps_match_reference_model_forward(moe):
    R = O.ref()
    n = 24
    m = _model(8, 2, max_seq=n + 4)
    s = R.ref_inference_init(m)
    toks = np.random.default_rng(5).integers(0, 4096, n).astype(np.int32)
    ours = _ours()
    for t in toks:
        ours.inference_step(m, s, int(t))
    assert R.ref_inference_pos(s) == n
    got = np.ctypeslib.as_array(R.ref_inference_logits(s), shape=(4096,)).copy()
    want = np.empty(4096, np.float32)
    R.ref_model_forward_last(m, O._i(toks), n, O._f(want))
    assert O.rel_err(got, want) < 1e-4
    assert int(np.argmax(got)) == int(np.argmax(want))
    # the MoE weights were uploaded once per layer and reused across steps
    R.ref_inference_free(s)
    O.release_ref_model(m)


def test_dense_decode_matches_reference_inference_step(moe):
    R = O.ref()
    n = 12
    m = _model(1, 1, max_seq=n + 2)
    s_ref, s_ours = R.ref_inference_init(m), R.ref_inference_init(m)
    ours = _ours()
    toks = np.random.default_rng(6).integers(0, 4096, n).astype(np.int32)
    for t in toks:
        R.ref_inference_step(m, s_ref, int(t))
        ours.inference_step(m, s_ours, int(t))
        a = np.ctypeslib.as_array(R.ref_inference_logits(s_ref), shape=(4096,))
        b = np.ctypeslib.as_array(R.ref_inference_logits(s_ours), shape=(4096,))
        assert O.rel_err(b, a) < 1e-5
    R.ref_inference_free(s_ref)
    R.ref_inference_free(s_ours)
    O.release_ref_model(m)


def test_python_model_builder_layout_matches_reference(moe):
    """llm.c_b200/llmc_model.py builds llm.c's structs from Python: two
    identical dense models stepped by llm.c's own inference_step and by the
    drop-in must agree, which checks every mirrored struct layout."""
    import llmc_model as LM
    R = O.ref()
    cfg = LM.DecodeConfig(n_experts=1, top_k=1, max_seq=16)
    a, b = LM.LlmcDecoder(cfg, seed=3), LM.LlmcDecoder(cfg, seed=3)
    R.ref_inference_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    for t in np.random.default_rng(7).integers(0, cfg.vocab, 8):
        R.ref_inference_step(C.addressof(a.model), C.addressof(a.state), int(t))
        b.step(int(t))
        assert O.rel_err(b.logits(), a.logits()) < 1e-5
    assert a.pos == b.pos == 8


def test_python_model_builder_moe_decode_runs(moe):
    import llmc_model as LM
    dec = LM.LlmcDecoder(LM.DecodeConfig(max_seq=8), seed=4)
    for t in (1, 2, 3):
        dec.step(t)
    lg = dec.logits()
    assert np.isfinite(lg).all() and dec.pos == 3
