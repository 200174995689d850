"""Array plumbing between the drop-in API and the C ABI.

Inputs may be numpy arrays (host) or torch tensors; they are moved to the
current CUDA device as contiguous tensors.  Results are returned in the
caller's container: numpy in -> numpy out, torch in -> torch (on the device).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("jax_gptq_b200 needs a CUDA device (sm_100a); none is available")


def is_host(x) -> bool:
    return not isinstance(x, torch.Tensor)


def to_device(x, dtype=torch.float32) -> torch.Tensor:
    """Contiguous CUDA tensor of ``dtype`` holding ``x`` (no copy if already so)."""
    require_cuda()
    if isinstance(x, torch.Tensor):
        t = x
    else:
        arr = np.asarray(x)
        if arr.dtype == np.float64 and dtype == torch.float32:
            arr = arr.astype(np.float32)
        t = torch.from_numpy(np.ascontiguousarray(arr))
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if not t.is_cuda:
        t = t.to("cuda", non_blocking=False)
    return t.contiguous()


def like_input(t: torch.Tensor, ref):
    """Return ``t`` in the container type of ``ref``."""
    if is_host(ref):
        return t.detach().cpu().numpy()
    return t


def ptr(t) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(t.data_ptr())


def stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def empty(shape, dtype=torch.float32) -> torch.Tensor:
    return torch.empty(shape, dtype=dtype, device="cuda")


def workspace(nbytes: int) -> torch.Tensor:
    """Byte buffer, 256-byte aligned (the caching allocator guarantees 512)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device="cuda")
