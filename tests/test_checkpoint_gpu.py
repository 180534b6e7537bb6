"""llm.c checkpoints (model_save format, src/transformer.c:573-617) streamed
straight to the B200, against the reference's own model_save / model_load.

  * every block's expert set loaded from the file equals, bit for bit, the
    reference Model's router and expert matrices (MoE), or its dense FFN as
    one expert with a zero router (dense);
  * the forward of a loaded expert set equals that of the same weights
    uploaded from host memory, bit for bit;
  * a decoder loaded from the file gives the logits of a decoder built from
    the reference's model_load of the same file (within 1e-5 of max|logit|:
    the loader builds its RoPE tables itself, the reference under
    -ffast-math), and of llm.c's model_forward (MoE) or inference_step
    (dense);
  * truncated files and a max_seq beyond the model's table are rejected,
    and a failed load leaves the library usable."""
import ctypes as C

import numpy as np
import pytest

import llmc_model as LM
import moe_b200 as M
import oracle_lib as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="reference build absent")]

V = 512


def _save(tmp_path, E, k, L=3, name="m.bin", seed=11):
    R = O.ref()
    # d=256, 4 heads, 2 KV heads, head_dim 64, d_ff 384, RoPE theta 1e4
    m = R.ref_model_init(V, 64, 256, L, 4, 2, 64, 0, 384, E, k, 1e-5, 1e4, seed)
    path = tmp_path / name
    assert R.ref_model_save(m, str(path).encode()) == 0
    return m, path


def _np(mat):
    return np.ctypeslib.as_array(mat.data, shape=(mat.rows, mat.cols)).copy()


def _host_ffn(m_ptr, layer):
    """(router [d, E], gate[], up[], down[]) of block `layer` of a reference Model."""
    bw = C.cast(m_ptr, C.POINTER(LM.Model)).contents.weights.blocks[layer]
    if not bw.use_moe:
        g, u, dn = _np(bw.ffn.W_gate), _np(bw.ffn.W_up), _np(bw.ffn.W_down)
        return np.zeros((g.shape[0], 1), np.float32), [g], [u], [dn]
    ex = [bw.moe.experts[e] for e in range(bw.moe.n_experts)]
    return (_np(bw.moe.W_router), [_np(x.W_gate) for x in ex], [_np(x.W_up) for x in ex],
            [_np(x.W_down) for x in ex])


@pytest.mark.parametrize("E,k", [(8, 2), (1, 1)], ids=["moe", "dense"])
def test_loaded_experts_equal_the_saved_model(moe, tmp_path, E, k):
    m, path = _save(tmp_path, E, k)
    for layer in range(3):
        w = M.MoEWeights.from_checkpoint(path, layer)
        assert (w.E, w.top_k) == ((E, k) if E > 1 else (1, 1))
        got = w.download()
        want = _host_ffn(m, layer)
        assert np.array_equal(got[0], want[0])
        for a, b in zip(got[1:], want[1:]):
            assert all(np.array_equal(x, y) for x, y in zip(a, b))
        w.free()
    O.release_ref_model(m)


def test_loaded_experts_forward_like_uploaded(moe, tmp_path):
    m, path = _save(tmp_path, 8, 2)
    wr, g, u, dn = _host_ffn(m, 1)
    up = M.MoEWeights.upload(wr, g, u, dn, 2)
    ld = M.MoEWeights.from_checkpoint(path, 1)
    x = np.random.default_rng(2).standard_normal((300, 256)).astype(np.float32)
    for path_id in (M.PATH_FP32, M.PATH_TF32X3):
        a = M.moe_forward(up, x, path=path_id)
        b = M.moe_forward(ld, x, path=path_id)
        for p, q in zip(a, b):
            assert np.array_equal(p, q)
    up.free()
    ld.free()
    O.release_ref_model(m)


@pytest.mark.parametrize("E,k", [(8, 2), (1, 1)], ids=["moe", "dense"])
def test_decoder_from_checkpoint_matches_model_load(moe, tmp_path, E, k):
    R = O.ref()
    m, path = _save(tmp_path, E, k)
    O.release_ref_model(m)
    loaded = R.ref_model_load(str(path).encode())
    assert loaded
    n = 20
    a = M.Decoder.from_checkpoint(path, n)
    b = M.Decoder(loaded, n)
    toks = np.random.default_rng(4).integers(0, V, n).astype(np.int32)
    la = np.empty(V, np.float32)
    lb = np.empty(V, np.float32)
    for t in toks:
        a.step(int(t), la)
        b.step(int(t), lb)
        assert O.rel_err(la, lb) < 1e-5
    if E > 1:
        want = np.empty(V, np.float32)
        R.ref_model_forward_last(loaded, O._i(toks), n, O._f(want))
    else:
        # llm.c's model_forward aborts on a dense model with seq_len <
        # max_seq_len (block_forward narrows every cache view but gate_buf /
        # up_buf, src/transformer.c:726-735, and mat_mul asserts the shape);
        # its own inference_step is the dense oracle
        s = R.ref_inference_init(loaded)
        for t in toks:
            R.ref_inference_step(loaded, s, int(t))
        want = np.ctypeslib.as_array(R.ref_inference_logits(s), shape=(V,)).copy()
        R.ref_inference_free(s)
    assert O.rel_err(la, want) < 1e-4
    assert int(np.argmax(la)) == int(np.argmax(want))
    a.free()
    b.free()
    O.release_ref_model(loaded)


def test_checkpoint_load_errors(moe, tmp_path):
    m, path = _save(tmp_path, 8, 2)
    O.release_ref_model(m)
    raw = path.read_bytes()
    cut = tmp_path / "cut.bin"
    cut.write_bytes(raw[: len(raw) * 2 // 3])          # ends inside the last block
    with pytest.raises(M.MoEError) as e:
        M.MoEWeights.from_checkpoint(cut, 2)
    assert e.value.status == M.E_INVALID
    with pytest.raises(M.MoEError) as e:
        M.Decoder.from_checkpoint(cut, 8)
    assert e.value.status == M.E_INVALID
    with pytest.raises(M.MoEError) as e:
        M.Decoder.from_checkpoint(path, 65)               # the model's max_seq_len is 64
    assert e.value.status == M.E_INVALID
    w = M.MoEWeights.from_checkpoint(path, 0)             # still usable after the failures
    assert w.E == 8
    w.free()
