"""Pins of the float64 torch reference used for the backward tests
(tests/torch_ref.py): its forward equals the oracle's restatement of
llm.c's moe_forward (same routing), its expert gradients equal llm.c's own
dense ffn_backward (src/transformer.c:181-264) for a one-expert layer, its
aux loss is 1 for perfectly balanced routing, and its gradients pass a
finite-difference check."""
import numpy as np
import pytest
import torch

import oracle_lib as O
import torch_ref


def test_reference_forward_matches_oracle():
    p = O.MoEProblem(97, 40, 6, 3, 72, seed=5, bias="normal")
    out, _, ids = p.oracle_forward()
    y, _ = torch_ref.moe_forward(p.x, p.W_router, p.bias, p.experts, ids)
    assert O.rel_err(y.astype(np.float32), out) < 2e-6


def test_aux_loss_of_balanced_routing_is_one():
    T, E, k = 64, 8, 2
    ids = np.stack([np.arange(T) % E, (np.arange(T) + 1) % E], axis=1).astype(np.int32)
    p = O.MoEProblem(T, 16, E, k, 32, seed=1)
    p.W_router[:] = 0.0                         # uniform probabilities
    _, aux = torch_ref.moe_forward(p.x, p.W_router, None, p.experts, ids)
    assert abs(aux - 1.0) < 1e-12


def test_reference_gradients_finite_difference():
    p = O.MoEProblem(6, 8, 4, 2, 12, seed=2, bias="normal")
    _, _, ids = p.oracle_forward()
    dy = np.random.default_rng(0).standard_normal((6, 8))
    tensors = torch_ref._tensors(p.x, p.W_router, p.bias, p.experts, True)
    flat = [tensors[0], tensors[1], tensors[2], *tensors[3], *tensors[4], *tensors[5]]
    E = p.E

    def f(*ts):
        y, aux = torch_ref._forward(ts[0], ts[1], ts[2], list(ts[3:3 + E]),
                                    list(ts[3 + E:3 + 2 * E]), list(ts[3 + 2 * E:]), ids)
        return (y * torch.tensor(dy)).sum() + 0.3 * aux

    assert torch.autograd.gradcheck(f, tuple(flat), eps=1e-6, atol=1e-7)


@pytest.mark.skipif(not O.ref_available(), reason="reference build absent")
def test_reference_ffn_backward_matches_autograd():
    """A one-expert MoE (zero router: p = 1, w = 1) is llm.c's dense FFN, so
    the autograd expert gradients must equal the reference's ffn_backward."""
    T, d, F = 40, 48, 72
    p = O.MoEProblem(T, d, 1, 1, F, seed=6)
    p.W_router[:] = 0.0
    dy = np.random.default_rng(1).standard_normal((T, d)).astype(np.float32)
    g, u, dn = p.experts[0]
    dWg, dWu, dWd = np.zeros_like(g), np.zeros_like(u), np.zeros_like(dn)
    dx = np.empty((T, d), np.float32)
    O.ref().ref_ffn_backward(O._f(p.x), T, d, O._f(g), O._f(u), O._f(dn), F, O._f(dy),
                             O._f(dWg), O._f(dWu), O._f(dWd), O._f(dx))
    ref = torch_ref.moe_grads(p.x, p.W_router, None, p.experts, np.zeros((T, 1), np.int32), dy, 0.0)
    assert O.rel_err(dx, ref[0]) < 1e-5
    for got, want in ((dWg, ref[3][0]), (dWu, ref[4][0]), (dWd, ref[5][0])):
        assert O.rel_err(got, want) < 1e-5
    assert not np.any(ref[1])                  # one expert: no router gradient
