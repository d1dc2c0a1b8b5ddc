"""Restatements of the reference's fused-op formulas (CPU, PyTorch).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  Each function returns
the same tuple as the reference extension function of the same name
(src/pymsst/training/cuda/fused_band_split.cpp:731-753) and computes in the
dtype of its inputs, so float64 inputs give a float64 reference.  The line
numbers cite src/pymsst/training/cuda/fused_band_split.cu.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

EPS = 1.0e-12


# ------------------------------------------------------------------ RMSNorm
def rms_norm_forward(x: torch.Tensor, gamma: torch.Tensor):
    """.cu:1211-1249: normed = x / max(||x||, eps) * sqrt(D); out = normed * gamma."""
    dim = x.shape[-1]
    flat = x.reshape(-1, dim)
    inv = 1.0 / torch.sqrt((flat * flat).sum(-1)).clamp_min(EPS)
    normed = flat * inv[:, None] * math.sqrt(dim)
    out = normed * gamma.to(normed.dtype)
    return out.reshape(x.shape), normed.reshape(x.shape), inv


def rms_norm_backward(grad_out, normed, inv_norm, gamma):
    """.cu:1252-1315 (input grad .cu:1263-1286, gamma grad .cu:1290-1315)."""
    dim = grad_out.shape[-1]
    scale = math.sqrt(dim)
    g = grad_out.reshape(-1, dim)
    n = normed.reshape(-1, dim).to(g.dtype)
    gn = g * gamma.to(g.dtype)
    dot = (gn * n).sum(-1, keepdim=True)
    inv = inv_norm.to(g.dtype)[:, None]
    grad_x = inv * (gn * scale - n * (dot / scale))
    grad_gamma = (g * n).sum(0)
    return grad_x.reshape(grad_out.shape), grad_gamma


# ------------------------------------------------------------------- rotary
def _interleave(even: torch.Tensor, odd: torch.Tensor) -> torch.Tensor:
    return torch.stack((even, odd), dim=-1).flatten(-2)


def rotary_forward(t, cos, sin):
    """.cu:1077-1101 on t[B,N,H,D] with cos/sin [1,N,1,D/2]."""
    e, o = t[..., 0::2], t[..., 1::2]
    return _interleave(e * cos - o * sin, o * cos + e * sin)


def rotary_backward(grad_out, cos, sin):
    """.cu:1104-1128: transpose of the rotation."""
    ge, go = grad_out[..., 0::2], grad_out[..., 1::2]
    return _interleave(ge * cos + go * sin, -ge * sin + go * cos)


# --------------------------------------------------------- BandSplit (group)
def band_split_forward(x, gamma, weight, bias=None):
    """.cu:14-71 on x[M,G,I], gamma[G,I], weight[G,O,I], bias[G,O]."""
    dim_in = x.shape[-1]
    inv = 1.0 / torch.sqrt((x * x).sum(-1)).clamp_min(EPS)  # [M, G]
    normed = x * inv[..., None] * math.sqrt(dim_in)
    out = torch.einsum("mgi,goi->mgo", normed * gamma, weight)
    if bias is not None:
        out = out + bias
    return out, normed.contiguous(), inv


def band_split_backward(grad_out, normed, inv_norm, gamma, weight, has_bias=True):
    """.cu:126-247 (v1) — v2 (.cu:315-432) and v3 (.cu:435-587) compute the same values."""
    dim_in = normed.shape[-1]
    scale = math.sqrt(dim_in)
    grad_scaled = torch.einsum("mgo,goi->mgi", grad_out, weight)
    grad_normed = grad_scaled * gamma
    dot = (grad_normed * normed).sum(-1, keepdim=True)
    grad_x = inv_norm.to(grad_out.dtype)[..., None] * (grad_normed * scale - normed * (dot / scale))
    grad_weight = torch.einsum("mgo,mgi->goi", grad_out, normed * gamma)
    grad_bias = grad_out.sum(0) if has_bias else None
    grad_gamma = (grad_scaled * normed).sum(0)
    return grad_x, grad_gamma, grad_weight, grad_bias


band_split_backward_v2 = band_split_backward
band_split_backward_v3 = band_split_backward


# -------------------------------------------------------- BandSplit (ragged)
def offsets_from_widths(dim_inputs) -> list[int]:
    offsets = [0]
    for w in dim_inputs:
        offsets.append(offsets[-1] + int(w))
    return offsets


def band_split_ragged_forward(x, gammas, weights, biases, dim_inputs, dim_offsets=None):
    """.cu:590-652 on x[M,total]; returns (out[M,nb,O], normed[M,total], inv_norm[M,nb])."""
    offs = offsets_from_widths(dim_inputs)
    outs, normeds, invs = [], [], []
    for b, w in enumerate(dim_inputs):
        xb = x[:, offs[b] : offs[b + 1]]
        inv = 1.0 / torch.sqrt((xb * xb).sum(-1)).clamp_min(EPS)
        normed = xb * inv[:, None] * math.sqrt(w)
        outs.append(F.linear(normed * gammas[b], weights[b], biases[b]))
        normeds.append(normed)
        invs.append(inv)
    return torch.stack(outs, 1), torch.cat(normeds, 1), torch.stack(invs, 1)


def band_split_ragged_backward(grad_out, normed, inv_norm, gammas, weights, dim_inputs, dim_offsets=None):
    """.cu:742-1003; returns [grad_x, *grad_gammas, *grad_weights, *grad_biases]."""
    offs = offsets_from_widths(dim_inputs)
    grad_x = torch.empty_like(normed, dtype=grad_out.dtype)
    g_gammas, g_weights, g_biases = [], [], []
    for b, w in enumerate(dim_inputs):
        nb = normed[:, offs[b] : offs[b + 1]].to(grad_out.dtype)
        dy = grad_out[:, b, :]
        gs = dy @ weights[b]
        gn = gs * gammas[b]
        dot = (gn * nb).sum(-1, keepdim=True)
        scale = math.sqrt(w)
        grad_x[:, offs[b] : offs[b + 1]] = inv_norm[:, b : b + 1].to(grad_out.dtype) * (gn * scale - nb * (dot / scale))
        g_gammas.append((gs * nb).sum(0))
        g_weights.append(dy.t() @ (nb * gammas[b]))
        g_biases.append(dy.sum(0))
    return [grad_x, *g_gammas, *g_weights, *g_biases]


# ------------------------------------------------------------ grouped linear
def grouped_linear_forward(x, weight, bias=None):
    """.cu:1006-1074: y[m,g,:] = b[g] + W[g] x[m,g,:]."""
    out = torch.einsum("mgi,goi->mgo", x, weight)
    return out + bias if bias is not None else out


# ----------------------------------------------------------- attention gate
def attention_gate_forward(attn, x, weight, bias):
    """.cu:1778-1824 and host .cu:1922-1970: returns (out, gate, attn, x)."""
    gate = torch.sigmoid(x @ weight.t() + bias)  # [M, H]
    out = (attn * gate[..., None]).reshape(attn.shape[0], -1)
    return out, gate, attn.contiguous(), x.contiguous()


def attention_gate_backward(grad_out, attn, x, weight, gate):
    """.cu:1826-1920 and host .cu:1972-2036: returns (grad_attn, grad_x, grad_weight, grad_bias)."""
    rows, heads, dim_head = attn.shape
    g = grad_out.reshape(rows, heads, dim_head)
    grad_attn = g * gate[..., None]
    grad_gate_pre = (g * attn).sum(-1) * gate * (1 - gate)  # [M, H]
    grad_x = grad_gate_pre @ weight
    grad_weight = grad_gate_pre.t() @ x
    grad_bias = grad_gate_pre.sum(0)
    return grad_attn, grad_x, grad_weight, grad_bias


# ------------------------------------------------- MaskEstimator final + GLU
def mask_estimator_final_forward(x, weights, bias, dim_inputs, dim_offsets=None):
    """.cu:2516-2553 ("direct") / .cu:2369-2420 ("grouped"): returns (out, pre, x).

    pre[m, 2*off_b : 2*off_b + 2*w_b] = x[m,b] W_b^T + bias (left half, gate half),
    out[m, off_b : off_b + w_b] = left * sigmoid(gate).
    """
    offs = offsets_from_widths(dim_inputs)
    pres, outs = [], []
    for b, w in enumerate(dim_inputs):
        pre = F.linear(x[:, b, :], weights[b], bias[2 * offs[b] : 2 * offs[b + 1]])
        left, gate_pre = pre[:, :w], pre[:, w:]
        pres.append(pre)
        outs.append(left * torch.sigmoid(gate_pre))
    return torch.cat(outs, 1), torch.cat(pres, 1), x.contiguous()


mask_estimator_final_direct_forward = mask_estimator_final_forward


def mask_estimator_final_backward(grad_out, x, pre, weights, dim_inputs, dim_offsets=None):
    """.cu:2556-2704 / .cu:2422-2513: returns [grad_x, grad_bias, *grad_weights]."""
    offs = offsets_from_widths(dim_inputs)
    grad_x = torch.empty_like(x, dtype=grad_out.dtype)
    grad_bias = torch.empty(pre.shape[1], dtype=grad_out.dtype)
    grad_weights = []
    for b, w in enumerate(dim_inputs):
        p = pre[:, 2 * offs[b] : 2 * offs[b + 1]].to(grad_out.dtype)
        left, gate = p[:, :w], torch.sigmoid(p[:, w:])
        g = grad_out[:, offs[b] : offs[b + 1]]
        grad_pre = torch.cat((g * gate, g * left * gate * (1 - gate)), 1)
        grad_bias[2 * offs[b] : 2 * offs[b + 1]] = grad_pre.sum(0)
        grad_x[:, b, :] = grad_pre @ weights[b]
        grad_weights.append(grad_pre.t() @ x[:, b, :].to(grad_out.dtype))
    return [grad_x, grad_bias, *grad_weights]


mask_estimator_final_direct_backward = mask_estimator_final_backward


# Reference names that differ only in dtype handling map to the same formulas.
rms_norm_forward_fp32_gamma = rms_norm_forward
rms_norm_backward_fp32_gamma = rms_norm_backward
rms_norm_forward_mixed = rms_norm_forward


def rms_norm_backward_mixed(grad_out, normed, inv_norm, gamma, x_meta=None):
    """.cu:1628-1691 (grad_x is cast to x_meta's dtype by the caller)."""
    return rms_norm_backward(grad_out, normed, inv_norm, gamma)
