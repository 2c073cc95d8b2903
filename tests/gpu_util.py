"""Helpers for the -m gpu tests: torch provides device memory only."""
import numpy as np


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def empty(torch, shape, dtype, fill=np.nan):
    t = torch.empty(shape, dtype=dtype, device="cuda")
    t.fill_(fill)
    return t
