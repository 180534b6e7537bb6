"""llm.c's own programs bound to libmoe_b200.so by link order, the binding a
maintainer adds (oracle/Makefile builds oracle/link_check.c twice: against
the unmodified reference library alone, and against libmoe_b200.so first and
then the same reference library).

In the second program the reference's block_forward (src/transformer.c:
761-764) calls moe_forward through the PLT of the position-independent
reference library, and the first definition in load order, libmoe_b200.so's,
wins; the program's own call to inference_step (include/inference.h:137)
binds the same way.

  * CPU: the dynamic linker's own binding log shows both symbols bound to
    libmoe_b200.so, and without a GPU the program stops with the library's
    message and a non-zero status (no CPU fallback).
  * GPU: the B200-bound program's model_forward logits equal the pure
    reference program's within 1e-4 of max|logit| (two layers of attention
    and MoE, 48 tokens; the MoE layers run at FP32 accuracy), with the same
    argmax at every position; its inference_step logits after the 48 tokens
    equal the reference model_forward's last row the same way (the
    reference's own inference_step has no MoE, src/inference.c:342-343); and
    the library reports kernel launches, so the B200 path did run."""
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle_lib as O

REF_DIR = Path(__file__).resolve().parent.parent / "oracle" / "_ref"
LINK_REF, LINK_B200 = REF_DIR / "link_ref", REF_DIR / "link_b200"

needs_bins = pytest.mark.skipif(not (LINK_REF.exists() and LINK_B200.exists()),
                                reason="link-check programs not built (needs the reference sources)")


def _read(path):
    raw = np.fromfile(path, np.uint8)
    T, V = np.frombuffer(raw[:8].tobytes(), np.int32)
    body = np.frombuffer(raw[8:].tobytes(), np.float32)
    return body[:T * V].reshape(T, V), body[T * V:T * V + V]


def _cpu_only():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@needs_bins
@pytest.mark.skipif(not _cpu_only(), reason="checks the no-GPU failure path")
def test_binding_resolves_to_library_and_fails_loudly_without_gpu(tmp_path):
    env = dict(os.environ, LD_DEBUG="bindings")
    r = subprocess.run([str(LINK_B200), str(tmp_path / "o.bin")], env=env, capture_output=True,
                       text=True, timeout=120)
    log = r.stdout + r.stderr
    bound = {ln.split("`")[1].rstrip("'") for ln in log.splitlines()
             if "libmoe_b200.so" in ln.split(" to ")[-1] and "normal symbol `" in ln}
    assert "moe_forward" in bound
    assert r.returncode != 0 and "[moe_b200]" in log
    assert not (tmp_path / "o.bin").exists()


@needs_bins
@pytest.mark.gpu
def test_reference_program_linked_to_library_matches_reference(tmp_path):
    ref_out, b200_out = tmp_path / "ref.bin", tmp_path / "b200.bin"
    subprocess.run([str(LINK_REF), str(ref_out)], check=True, timeout=300)
    r = subprocess.run([str(LINK_B200), str(b200_out)], check=True, timeout=300,
                       capture_output=True, text=True)
    lines = dict(ln.split(":", 1) for ln in r.stdout.strip().splitlines())
    launches = {k: int(v.split("b200_launches=")[1].split()[0]) for k, v in lines.items()}
    assert launches["model_forward"] > 0 and launches["inference_step"] > 0
    want, _ = _read(ref_out)
    got, got_step = _read(b200_out)
    assert O.rel_err(got, want) < 1e-4
    assert np.array_equal(np.argmax(got, axis=1), np.argmax(want, axis=1))
    assert O.rel_err(got_step, want[-1]) < 1e-4
    assert int(np.argmax(got_step)) == int(np.argmax(want[-1]))
