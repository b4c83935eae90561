"""Float64 torch restatement of the sequence-parallel sub-span folds (the
ema_span_summary / ema_span_expand kernels): the reference the gloo tests
inject into kernels/ema_sp.py on CPU ranks and the GPU test compares the
kernels with.  ld (B, K, H) log decays, V (B K, H, P) sub-span values; with
cl_k = sum_{j<k} ld_j and tot = sum_k ld_k (see include/ema_ssd_b200.h)."""

import torch


def _mask_exp(e, keep):
    return torch.exp(torch.where(keep, e, torch.full_like(e, float("-inf"))))


def torch_fold(direction, expand, ld, V, boundary=None):
    ld = ld.to(torch.float64)
    B, K, H = ld.shape
    V = V.to(torch.float64).reshape(B, K, H, -1)
    P = V.shape[-1]
    cl = torch.cumsum(ld, dim=1) - ld
    tot = cl[:, -1] + ld[:, -1]
    k = torch.arange(K, device=ld.device)
    if not expand:
        w = torch.exp(tot[:, None] - cl - ld) if direction == 0 else torch.exp(cl)
        return (w[..., None] * V).sum(dim=1).to(torch.float32), torch.exp(tot).to(torch.float32)
    bnd = boundary.to(torch.float64)
    if direction == 0:  # exp(cl_k) S + sum_{q<k} exp(cl_k - cl_q - ld_q) V_q
        W = _mask_exp(cl[:, :, None, :] - (cl + ld)[:, None, :, :], (k[:, None] > k[None, :])[None, :, :, None])
        out = torch.exp(cl)[..., None] * bnd[:, None] + torch.einsum("bkqh,bqhp->bkhp", W, V)
    else:  # exp(tot - cl_k - ld_k) G + sum_{q>k} exp(cl_q - cl_k - ld_k) V_q
        W = _mask_exp(cl[:, None, :, :] - (cl + ld)[:, :, None, :], (k[None, :] > k[:, None])[None, :, :, None])
        out = torch.exp(tot[:, None] - cl - ld)[..., None] * bnd[:, None] + torch.einsum("bkqh,bqhp->bkhp", W, V)
    return out.reshape(B * K, H, P).to(torch.float32)
