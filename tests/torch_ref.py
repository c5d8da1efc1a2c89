"""fp32 torch restatements of the reference operators, for GPU parity checks at
sizes the numpy oracle cannot reach quickly (test infrastructure only).

Each follows the reference's torch path: ``src/kadllm/ops.py:139-163``
(gated_delta), ``:215-226`` (causal_conv1d), ``:311-341`` (prefix_attention).
"""

import torch
import torch.nn.functional as F


def gated_delta(q, k, v, g, beta, s0, W, scale=None, chunk=32):
    BW, T, H, K = q.shape
    HV = v.shape[2]
    scale = K ** -0.5 if scale is None else scale
    q, k, v, g, beta = (x.float() for x in (q, k, v, g, beta))
    q = q / (q.square().sum(-1, keepdim=True) + 1e-6).sqrt() * scale
    k = k / (k.square().sum(-1, keepdim=True) + 1e-6).sqrt()
    q = q.repeat_interleave(HV // H, 2)
    k = k.repeat_interleave(HV // H, 2)
    out = torch.empty(v.shape, dtype=torch.float32, device=v.device)
    B = BW // W
    for r0 in range(0, B, chunk):
        r1 = min(B, r0 + chunk)
        sl = slice(r0 * W, r1 * W)
        st = s0[r0:r1].float().repeat_interleave(W, 0)
        for t in range(T):
            st = st * g[sl, t].exp()[..., None, None]
            kt = k[sl, t]
            corr = beta[sl, t][..., None] * (v[sl, t] - torch.einsum("nhkv,nhk->nhv", st, kt))
            st = st + kt[..., :, None] * corr[..., None, :]
            out[sl, t] = torch.einsum("nhkv,nhk->nhv", st, q[sl, t])
    return out


def causal_conv1d(x, state, w, W):
    BW, C, T = x.shape
    width = w.shape[-1]
    prefix = state[:, :, state.shape[-1] - (width - 1):].float().repeat_interleave(W, 0)
    window = torch.cat([prefix, x.float()], -1)
    return F.silu(F.conv1d(window, w.float()[:, None, :], groups=C))


def prefix_attention(q, pk, pv, sk, sv, W, mask=None, scale=None):
    """fp32 restatement of src/kadllm/ops.py:311-341 (torch path)."""
    BW, T, H, D = q.shape
    B, L, HK, _ = pk.shape
    rep = H // HK
    scale = D ** -0.5 if scale is None else scale
    query = q.float().reshape(B, W, T, H, D).permute(0, 1, 3, 2, 4)
    pkr = pk.float().repeat_interleave(rep, 2).permute(0, 2, 1, 3)
    pvr = pv.float().repeat_interleave(rep, 2).permute(0, 2, 1, 3)
    pq = query.permute(0, 2, 1, 3, 4).reshape(B, H, W * T, D)
    s = torch.matmul(pq, pkr.transpose(-1, -2)) * scale
    if mask is not None:
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))

    def part(scores, values):
        if scores.shape[-1] == 0:
            return (scores.new_zeros(*scores.shape[:-1], values.shape[-1]),
                    scores.new_full(scores.shape[:-1], float("-inf")))
        present = torch.isfinite(scores).any(-1, keepdim=True)
        safe = torch.where(present, scores, torch.zeros_like(scores))
        out = torch.matmul(torch.softmax(safe, -1) * present, values)
        lse = torch.where(present.squeeze(-1), safe.logsumexp(-1), float("-inf"))
        return out, lse

    op, lp = part(s, pvr)
    op = op.reshape(B, H, W, T, D).permute(0, 2, 1, 3, 4)
    lp = lp.reshape(B, H, W, T).permute(0, 2, 1, 3)
    skr = sk.float().repeat_interleave(rep, 2).reshape(B, W, T, H, D).permute(0, 1, 3, 2, 4)
    svr = sv.float().repeat_interleave(rep, 2).reshape(B, W, T, H, D).permute(0, 1, 3, 2, 4)
    causal = torch.ones(T, T, device=q.device, dtype=torch.bool).tril()
    s2 = (torch.matmul(query, skr.transpose(-1, -2)) * scale).masked_fill(~causal, float("-inf"))
    os_, ls = part(s2, svr)
    tot = torch.logaddexp(lp, ls)
    out = op * (lp - tot).exp()[..., None] + os_ * (ls - tot).exp()[..., None]
    return out.permute(0, 1, 3, 2, 4).reshape(BW, T, H, D)
