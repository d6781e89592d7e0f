"""Torch restatement of the expert-parallel dispatch/combine layout (test
helper): what d3_ep_dispatch_pack / d3_ep_combine compute, on any device."""
import torch


def pack(x, ids, n_ranks, epr, cap):
    """-> send_x [n_ranks*cap, H], send_eid [n_ranks*cap], src_slot [T, k]."""
    T, k = ids.shape
    H = x.shape[1]
    send_x = torch.zeros(n_ranks * cap, H, dtype=x.dtype, device=x.device)
    send_eid = torch.full((n_ranks * cap,), -1, dtype=torch.int32, device=x.device)
    src = torch.full((T, k), -1, dtype=torch.int32, device=x.device)
    fill = [0] * n_ranks
    flat = ids.reshape(-1).tolist()
    for i, e in enumerate(flat):
        if not (0 <= e < n_ranks * epr):
            continue
        d = e // epr
        j = fill[d]
        fill[d] += 1
        if j >= cap:
            continue
        row = d * cap + j
        send_eid[row] = e - d * epr
        send_x[row] = x[i // k]
        src[i // k, i % k] = row
    return send_x, send_eid, src


def combine(ret, src, weights, out=None):
    T, k = src.shape
    acc = torch.zeros(T, ret.shape[1], dtype=torch.float32, device=ret.device) if out is None \
        else out.float().clone()
    for t in range(T):
        for j in range(k):
            s = int(src[t, j])
            if s >= 0:
                acc[t] += float(weights[t, j]) * ret[s].float()
    return acc
