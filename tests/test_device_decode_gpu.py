"""Device-resident decode (moe_b200_decoder_*): llm.c's single-token
KV-cache forward with MoE blocks, entirely on the B200, against the
reference built from its own sources.

  * MoE model (configuration 2's shape, E=8, top-2): after n steps the logits
    match the last row of the reference's full-sequence model_forward
    (src/transformer.c:774-802, which runs MoE through its CPU moe_forward)
    within 1e-4 of max|logit| with the same argmax, and every step matches
    the drop-in host inference_step (llm.c's arithmetic on the host, MoE on
    the B200) within 5e-5;
  * dense model (E=1): every step matches llm.c's own inference_step
    (src/inference.c:231-358) within 5e-5;
  * rewinding (set_pos) and replaying gives bit-identical logits;
  * a full KV cache and an out-of-range token are rejected.
Both device variants are checked: one kernel per stage (the default) and
the whole step as one persistent cooperative kernel.  The device sums in a
different (fixed) order than the host, so agreement is to fp32 rounding,
not bit-exact; the two device variants run the same arithmetic and agree
bit for bit."""
import ctypes as C

import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="reference build absent")]

V = 4096


def _model(E, k, max_seq, seed=1, L=6):
    # d=384, 6 heads, 2 KV heads, head_dim 64, d_ff 1536, RoPE theta 1e4, vocab 4096
    return O.ref().ref_model_init(V, max_seq, 384, L, 6, 2, 64, 0, 1536, E, k, 1e-5, 1e4, seed)


def _host_step():
    L = M.lib()
    L.inference_step.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    L.inference_step.restype = None
    return L.inference_step


def _logits(R, s):
    return np.ctypeslib.as_array(R.ref_inference_logits(s), shape=(V,)).copy()


MODES = [M.Decoder.PERSISTENT, M.Decoder.STAGE_KERNELS]
MODE_IDS = ["persistent", "stage_kernels"]


@pytest.mark.parametrize("flags", MODES, ids=MODE_IDS)
def test_moe_device_decode_matches_reference(moe, flags):
    R = O.ref()
    n = 24
    m = _model(8, 2, max_seq=n + 8)
    dec = M.Decoder(m, n + 8, flags)
    s = R.ref_inference_init(m)
    host_step = _host_step()
    toks = np.random.default_rng(5).integers(0, V, n).astype(np.int32)
    got = np.empty(V, np.float32)
    for t in toks:
        dec.step(int(t), got)
        host_step(m, s, int(t))
        assert O.rel_err(got, _logits(R, s)) < 5e-5
    assert dec.pos == n
    want = np.empty(V, np.float32)
    R.ref_model_forward_last(m, O._i(toks), n, O._f(want))
    assert O.rel_err(got, want) < 1e-4
    assert int(np.argmax(got)) == int(np.argmax(want))
    assert dec.launches == (1 if flags == M.Decoder.PERSISTENT else 6 * 5 + 1)
    dec.free()
    R.ref_inference_free(s)
    O.release_ref_model(m)


@pytest.mark.parametrize("flags", MODES, ids=MODE_IDS)
def test_dense_device_decode_matches_reference_inference_step(moe, flags):
    R = O.ref()
    n = 16
    m = _model(1, 1, max_seq=n + 2)
    dec = M.Decoder(m, n + 2, flags)
    s = R.ref_inference_init(m)
    toks = np.random.default_rng(6).integers(0, V, n).astype(np.int32)
    got = np.empty(V, np.float32)
    for t in toks:
        dec.step(int(t), got)
        R.ref_inference_step(m, s, int(t))
        assert O.rel_err(got, _logits(R, s)) < 5e-5
    dec.free()
    R.ref_inference_free(s)
    O.release_ref_model(m)


def test_device_decode_variants_agree_and_rewind_is_deterministic(moe):
    R = O.ref()
    n = 70                                   # crosses a 64-position attention chunk
    m = _model(8, 2, max_seq=n + 2, L=2)
    dec = M.Decoder(m, n + 2, M.Decoder.PERSISTENT)
    stage = M.Decoder(m, n + 2)                       # the default: one kernel per stage
    assert stage.launches == 2 * 5 + 1 and dec.launches == 1
    toks = np.random.default_rng(7).integers(0, V, n).astype(np.int32)
    first = np.empty((n, V), np.float32)
    other = np.empty(V, np.float32)
    for i, t in enumerate(toks):
        dec.step(int(t), first[i])
        stage.step(int(t), other)
        assert np.array_equal(first[i], other)
    stage.free()
    dec.set_pos(40)
    again = np.empty(V, np.float32)
    for i in range(40, n):
        dec.step(int(toks[i]), again)
        assert np.array_equal(again, first[i])
    dec.free()
    O.release_ref_model(m)


def test_device_decode_rejects_full_cache_and_bad_token(moe):
    R = O.ref()
    m = _model(8, 2, max_seq=4, L=1)
    dec = M.Decoder(m, 3)
    with pytest.raises(M.MoEError):
        dec.step(V)                          # token out of range
    for t in range(3):
        dec.step(t)
    with pytest.raises(M.MoEError):
        dec.step(0)                          # KV cache full
    with pytest.raises(M.MoEError):
        dec.set_pos(5)                       # beyond the written positions
    dec.set_pos(1)
    dec.step(0)
    assert dec.pos == 2
    dec.free()
    O.release_ref_model(m)


def test_inference_step_device_mode(moe, monkeypatch):
    """llm.c's inference_step symbol with MOE_B200_DECODE=device runs the
    whole step on the B200 and gives the reference model_forward's logits."""
    R = O.ref()
    n = 20
    m = _model(8, 2, max_seq=n + 4)
    s = R.ref_inference_init(m)
    step = _host_step()
    monkeypatch.setenv("MOE_B200_DECODE", "device")
    toks = np.random.default_rng(8).integers(0, V, n).astype(np.int32)
    for t in toks:
        step(m, s, int(t))
    assert R.ref_inference_pos(s) == n
    got = _logits(R, s)
    want = np.empty(V, np.float32)
    R.ref_model_forward_last(m, O._i(toks), n, O._f(want))
    assert O.rel_err(got, want) < 1e-4
    assert int(np.argmax(got)) == int(np.argmax(want))
    L = M.lib()
    L.moe_b200_invalidate.argtypes = [C.c_void_p]
    assert L.moe_b200_invalidate(m) == 0          # drops the model's device decoder
    R.ref_inference_free(s)
    O.release_ref_model(m)


def test_device_decode_rejects_conflicting_flags(moe):
    m = _model(8, 2, max_seq=8, L=1)
    for flags in (M.Decoder.STAGE_KERNELS | M.Decoder.PERSISTENT, 4):
        with pytest.raises(M.MoEError) as e:
            M.Decoder(m, 4, flags)
        assert e.value.status == M.E_INVALID
    O.release_ref_model(m)


def test_stage_timeline(moe, monkeypatch):
    """MOE_B200_DECODER_STAMPS=1 records every stage's entry, wait and exit
    times; the logits are the same bits as without it, the times are
    ordered within a stage, and a decoder without it refuses the read."""
    m = _model(8, 2, max_seq=16)
    plain = M.Decoder(m, 16)
    monkeypatch.setenv("MOE_B200_DECODER_STAMPS", "1")
    timed = M.Decoder(m, 16)
    a = np.empty(V, np.float32)
    b = np.empty(V, np.float32)
    for t in (3, 17, 4000, 5):
        plain.step(t, a)
        timed.step(t, b)
        assert np.array_equal(a, b)
        st = timed.stage_times(6)
        assert st.shape == (31, 4)
        assert st[0, 0] == 0.0 and np.all(st >= 0.0)
        assert np.all(st[:, 1] <= st[:, 2]) and np.all(st[:, 2] <= st[:, 3])
        assert np.all(st[:, 0] <= st[:, 3])
        assert st[-1, 3] == st[:, 3].max()
    with pytest.raises(M.MoEError):
        plain.stage_times(6)
    plain.free()
    timed.free()
