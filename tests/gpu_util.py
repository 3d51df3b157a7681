"""Helpers shared by the GPU parity tests."""
import numpy as np


def dev(x, dtype=None):
    import torch

    a = np.ascontiguousarray(x)
    if a.dtype == np.uint16:
        a = a.view(np.int16)  # bf16 bit patterns travel as int16 storage
    t = torch.from_numpy(a).cuda()
    return t if dtype is None else t.to(dtype)


def host(t):
    a = t.detach().cpu().numpy()
    if a.dtype == np.int16:
        a = a.view(np.uint16)
    return a


def make_ctx():
    import torch

    import qora_mixer as qm

    return qm.Ctx(0, stream=torch.cuda.current_stream())
