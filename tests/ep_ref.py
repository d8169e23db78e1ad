"""Torch restatements of the expert-parallel dispatch and combine steps (test helpers:
the CPU multi-rank test runs the host logic with them, the GPU tests check the CUDA
kernels against them)."""

import torch


def dispatch_pack_ref(rows, send, slot_of, k, E, N, ids_off):
    """Torch restatement of duplex_ep_dispatch_pack: per rank d, the rows of the tokens
    that picked one of d's experts, compacted in token order; the rest of the block
    carries an expert of rank d + 1 with weight 0."""
    T = rows.shape[0]
    ids = rows[:, ids_off:ids_off + 4 * k].contiguous().view(torch.int32)
    E_l = E // N
    for d in range(N):
        hit = ((ids >= d * E_l) & (ids < (d + 1) * E_l)).any(dim=1)
        pos = torch.cumsum(hit.to(torch.int32), 0) - 1
        slot_of[d] = torch.where(hit, pos, torch.full_like(pos, -1))
        n = int(hit.sum())
        send[d, :n] = rows[hit]
        send[d, n:] = 0
        pad = send[d, n:, ids_off:ids_off + 8 * k]
        pad[:, :4 * k] = torch.full((T - n, k), ((d + 1) % N) * E_l, dtype=torch.int32).view(torch.uint8)
        pad[:, 4 * k:] = torch.zeros((T - n, k), dtype=torch.float32).view(torch.uint8)


def combine_ref(back, slot_of, residual):
    """Torch restatement of duplex_ep_combine (fp32 out): partial rows in rank order."""
    N, T, H = back.shape
    out = torch.zeros(T, H, dtype=torch.float32)
    for d in range(N):
        for t in range(T):
            p = int(slot_of[d, t])
            if p >= 0:
                out[t] += back[d, p]
    return out + residual if residual is not None else out


