"""llm.c checkpoints (model_save format, src/transformer.c:573-617) read by
the B200 library: the parts that need no GPU.

  * moe_b200_checkpoint_config returns the ModelConfig the reference wrote,
    field for field, for MoE and dense models;
  * a file without the "CLLM" magic, a truncated header, a missing file and
    an out-of-range layer are rejected with MOE_B200_E_INVALID before any
    device work."""
import numpy as np
import pytest

import moe_b200 as M
import oracle_lib as O

pytestmark = pytest.mark.skipif(not O.ref_available(), reason="reference build absent")

FIELDS = ("vocab_size", "max_seq_len", "d_model", "n_layers", "n_heads", "n_kv_heads",
          "head_dim", "window_size", "ffn_hidden", "n_experts", "top_k_experts")


def _save(tmp_path, E, k, name="m.bin", seed=3):
    R = O.ref()
    # vocab 64, max_seq 16, d 32, 2 layers, 4 heads, 2 KV heads, head_dim 8, F 48
    m = R.ref_model_init(64, 16, 32, 2, 4, 2, 8, 0, 48, E, k, 1e-5, 1e4, seed)
    path = tmp_path / name
    assert R.ref_model_save(m, str(path).encode()) == 0
    R.ref_model_free(m)
    return path


@pytest.mark.parametrize("E,k", [(4, 2), (1, 1)], ids=["moe", "dense"])
def test_checkpoint_config_matches_saved_model(tmp_path, E, k):
    cfg = M.checkpoint_config(_save(tmp_path, E, k))
    want = dict(vocab_size=64, max_seq_len=16, d_model=32, n_layers=2, n_heads=4, n_kv_heads=2,
                head_dim=8, window_size=0, ffn_hidden=48, n_experts=E, top_k_experts=k)
    assert {f: getattr(cfg, f) for f in FIELDS} == want
    assert cfg.rms_norm_eps == np.float32(1e-5)
    assert cfg.rope_theta == 1e4


def test_checkpoint_size_is_what_the_loader_walks(tmp_path):
    """The loader seeks by the layout it knows; the file the reference wrote
    is exactly that many floats after the 56-byte header."""
    for E, k in [(4, 2), (1, 1)]:
        p = _save(tmp_path, E, k, name=f"m{E}.bin")
        d, F, V, L, nq, kvd = 32, 48, 64, 2, 32, 16
        ffn = (d * E + E * 3 * d * F) if E > 1 else 3 * d * F
        floats = V * d + L * (d + d * nq + 2 * d * kvd + nq * d + d + ffn) + d + d * V
        assert p.stat().st_size == 56 + 4 * floats


def test_checkpoint_rejects_bad_files(tmp_path):
    good = _save(tmp_path, 4, 2)
    raw = good.read_bytes()
    bad_magic = tmp_path / "bad_magic.bin"
    bad_magic.write_bytes(b"XXXX" + raw[4:])
    short = tmp_path / "short.bin"
    short.write_bytes(raw[:30])
    for p in (bad_magic, short, tmp_path / "missing.bin"):
        with pytest.raises(M.MoEError) as e:
            M.checkpoint_config(p)
        assert e.value.status == M.E_INVALID
    for layer in (-1, 2):
        with pytest.raises(M.MoEError) as e:
            M.MoEWeights.from_checkpoint(good, layer)
        assert e.value.status == M.E_INVALID
