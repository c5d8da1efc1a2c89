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
