"""Float64 torch autograd reference of the MoE block's gradients.

llm.c has no MoE backward, so the gradient is checked against automatic
differentiation of the forward it defines (src/transformer.c:287-366):
p = softmax(x·W_r + b), the top-k ids held fixed (given), w = p_S / Σ p_S,
y = Σ_r w_r · (silu(x·Wg_e) ⊙ x·Wu_e)·Wd_e, and the Switch load-balancing
loss L_aux = E · Σ_e f_e · P_e with f_e = n_e / (T·k) and P_e the mean
router probability.  The loss differentiated is Σ(dy ⊙ y) + aux_coef·L_aux.
Test infrastructure only."""
import numpy as np
import torch


def _forward(tx, wr, b, wg, wu, wd, ids):
    """(y, L_aux) of the MoE block on float64 tensors, routing `ids` fixed."""
    dt = torch.float64
    T, d = tx.shape
    E = wr.shape[1]
    k = ids.shape[1]
    prob = torch.softmax(tx @ wr + b, dim=-1)
    idx = torch.tensor(ids, dtype=torch.long)
    sel = prob.gather(1, idx)
    w = sel / sel.sum(dim=1, keepdim=True)
    y = torch.zeros(T, d, dtype=dt)
    for e in range(E):
        tok, r = (idx == e).nonzero(as_tuple=True)
        if len(tok) == 0:
            continue
        xe = tx[tok]
        he = torch.nn.functional.silu(xe @ wg[e]) * (xe @ wu[e])
        y = y.index_add(0, tok, w[tok, r].unsqueeze(1) * (he @ wd[e]))
    f = torch.bincount(idx.flatten(), minlength=E).to(dt) / (T * k)
    aux = E * (f * prob.mean(dim=0)).sum()
    return y, aux


def _tensors(x, W_router, bias, experts, grad):
    dt = torch.float64
    E = W_router.shape[1]
    tx = torch.tensor(x, dtype=dt, requires_grad=grad)
    wr = torch.tensor(W_router, dtype=dt, requires_grad=grad)
    b = torch.tensor(np.zeros(E) if bias is None else bias, dtype=dt, requires_grad=grad)
    wg = [torch.tensor(e[0], dtype=dt, requires_grad=grad) for e in experts]
    wu = [torch.tensor(e[1], dtype=dt, requires_grad=grad) for e in experts]
    wd = [torch.tensor(e[2], dtype=dt, requires_grad=grad) for e in experts]
    return tx, wr, b, wg, wu, wd


def moe_forward(x, W_router, bias, experts, ids):
    """(y [T×d], L_aux) as float64 numpy, routing `ids` held fixed."""
    with torch.no_grad():
        y, aux = _forward(*_tensors(x, W_router, bias, experts, False), ids)
    return y.numpy(), float(aux.item())


def moe_grads(x, W_router, bias, experts, ids, dy, aux_coef):
    """Returns (dx, dW_router, d_bias, [dW_gate], [dW_up], [dW_down], L_aux)
    as float64 numpy arrays; `ids` [T×k] is the routing to hold fixed."""
    tx, wr, b, wg, wu, wd = _tensors(x, W_router, bias, experts, True)
    y, aux = _forward(tx, wr, b, wg, wu, wd, ids)
    loss = (y * torch.tensor(dy, dtype=torch.float64)).sum() + aux_coef * aux
    loss.backward()

    def g(t):
        return t.grad.numpy() if t.grad is not None else np.zeros(tuple(t.shape))

    return (g(tx), g(wr), g(b), [g(t) for t in wg], [g(t) for t in wu], [g(t) for t in wd],
            float(aux.item()))
