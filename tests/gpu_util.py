"""Device buffers for the GPU tests: numpy <-> torch CUDA tensors, bit-preserving."""
from __future__ import annotations

import numpy as np
import torch

_VIEW = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32, np.dtype(np.uint64): np.int64,
         np.dtype(np.uint8): np.uint8}


def dev(a: np.ndarray) -> torch.Tensor:
    """Copy a numpy array to cuda:0 keeping its bytes."""
    a = np.ascontiguousarray(a)
    v = a.view(_VIEW.get(a.dtype, a.dtype))
    return torch.from_numpy(v.copy()).cuda()


def host(t: torch.Tensor, dtype) -> np.ndarray:
    """Copy a device tensor back as numpy of the given dtype (bytes kept)."""
    torch.cuda.synchronize()
    a = t.detach().cpu().numpy()
    return a.view(dtype)


def empty(shape, dtype) -> torch.Tensor:
    dt = np.dtype(dtype)
    tdt = {np.dtype(np.float32): torch.float32, np.dtype(np.uint16): torch.int16, np.dtype(np.int8): torch.int8,
           np.dtype(np.uint8): torch.uint8, np.dtype(np.int32): torch.int32, np.dtype(np.uint32): torch.int32}[dt]
    return torch.empty(shape, dtype=tdt, device="cuda")


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream
