"""fp32 attention on the GPU (TF32 off): the reference computation of full-size parity tests.

The CPU oracle (``oracle/attention.py``) states the semantics and is checked against the
reference's fixtures; at the full sizes of the benchmark workloads (8 x 32 x 4096 x 4096 prefill
scores, 256 sessions of up to 32768 tokens) it would take minutes on the host, so these
functions compute the same fp32 math with torch on the device, one unit at a time.  They are
test references: nothing in the package calls them.
"""
from __future__ import annotations

import torch

PAGE = 16


def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False


@torch.no_grad()
def prefill_unit(q, k, v, causal=True, scale=None):
    """``q [G, Sq, D]`` (the query heads of one KV head), ``k, v [Sk, D]`` -> fp32 ``o [G, Sq, D]``
    and ``lse [G, Sq]``; causal aligned bottom-right."""
    _no_tf32()
    qf, kf, vf = q.float(), k.float(), v.float()
    G, Sq, D = qf.shape
    Sk = kf.shape[0]
    scale = D ** -0.5 if scale is None else scale
    s = torch.matmul(qf, kf.t()) * scale                       # [G, Sq, Sk]
    if causal:
        qi = torch.arange(Sq, device=q.device).view(Sq, 1) + (Sk - Sq)
        kj = torch.arange(Sk, device=q.device).view(1, Sk)
        s.masked_fill_(kj > qi, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    s.sub_(lse.unsqueeze(-1)).exp_()
    return torch.matmul(s, vf), lse


@torch.no_grad()
def prefill_errors(q, k, v, o, causal=True):
    """Max / mean absolute error of ``o [B,Hq,S,D]`` over every (batch, KV head) unit."""
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    mx, tot, n = 0.0, 0.0, 0
    for b in range(B):
        for h in range(Hkv):
            ref, _ = prefill_unit(q[b, h * G:(h + 1) * G], k[b, h], v[b, h], causal)
            d = (o[b, h * G:(h + 1) * G].float() - ref).abs()
            mx = max(mx, d.max().item())
            tot += d.sum().item()
            n += d.numel()
    return mx, tot / n, B * Hkv


@torch.no_grad()
def decode_session(q, k_pages, v_pages, pages, L, scale=None):
    """One session: ``q [Hq, D]`` over its first ``L`` tokens in ``pages`` -> fp32 ``[Hq, D]``."""
    _no_tf32()
    Hq, D = q.shape
    Hkv = k_pages.shape[1]
    n = (L + PAGE - 1) // PAGE
    idx = pages[:n].long()
    kf = k_pages.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, n * PAGE, D)[:, :L].float()
    vf = v_pages.index_select(0, idx).permute(1, 0, 2, 3).reshape(Hkv, n * PAGE, D)[:, :L].float()
    scale = D ** -0.5 if scale is None else scale
    qg = q.float().view(Hkv, Hq // Hkv, D)
    p = torch.softmax(torch.bmm(qg, kf.transpose(1, 2)) * scale, dim=-1)
    return torch.bmm(p, vf).reshape(Hq, D)


@torch.no_grad()
def decode_errors(q, k_pages, v_pages, block_table, lengths, o):
    """Max / mean absolute error of ``o [N,Hq,D]`` over every session."""
    mx, tot, n = 0.0, 0.0, 0
    for i, L in enumerate(lengths):
        ref = decode_session(q[i], k_pages, v_pages, block_table[i], int(L))
        d = (o[i].float() - ref).abs()
        mx = max(mx, d.max().item())
        tot += d.sum().item()
        n += d.numel()
    return mx, tot / n, len(lengths)
