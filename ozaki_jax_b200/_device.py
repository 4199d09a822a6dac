"""Array-family handling: NumPy in -> NumPy out, device tensor in -> device
tensor out (the reference's type policy, ozaki_jax/matmul.py:803-821).

Device arrays are torch CUDA tensors (the plumbing this build uses for device
memory and streams).  Staging of NumPy inputs goes through pinned host
buffers so the copies run as DMA.
"""

import numpy as np
import torch


def is_device_array(x):
    return isinstance(x, torch.Tensor)


def same_family(A, B):
    return is_device_array(A) == is_device_array(B)


def device_of(*xs):
    for x in xs:
        if is_device_array(x) and x.is_cuda:
            return x.device
    if not torch.cuda.is_available():
        raise RuntimeError("ozaki_jax_b200 needs a CUDA device; none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def ndim(x):
    return x.dim() if is_device_array(x) else np.ndim(x)


def shape(x):
    return tuple(x.shape) if is_device_array(x) else np.shape(x)


def to_device_f64(x, device):
    """A contiguous float64 CUDA tensor with the values of x (copied only when
    needed)."""
    if is_device_array(x):
        t = x.to(device=device, dtype=torch.float64)
        return t.contiguous()
    a = np.ascontiguousarray(x, dtype=np.float64)
    host = torch.from_numpy(a)
    if a.nbytes >= (1 << 20) and not host.is_pinned():
        # pageable: the library's page-locked staging with host memcpy threads
        from . import _lib as L
        out = torch.empty(a.shape, dtype=torch.float64, device=device)
        with torch.cuda.device(device):
            L.check(L.load().ozk_memcpy_staged(out.data_ptr(), a.ctypes.data, a.nbytes,
                                               stream_handle(device)))
        return out
    return host.to(device, non_blocking=True)


def host_empty_f64(shape):
    """Uninitialised float64 NumPy array; page-locked (from torch's pinned host
    pool) when large, so device-to-host copies into it run as DMA."""
    n = int(np.prod(shape)) if len(shape) else 1
    if n >= (1 << 17) and torch.cuda.is_available():
        return torch.empty(tuple(shape), dtype=torch.float64, pin_memory=True).numpy()
    return np.empty(shape, dtype=np.float64)


def to_host_f64(t):
    """NumPy float64 array with the values of the CUDA tensor t (blocking)."""
    if t.numel() >= (1 << 17):
        out = torch.empty(t.shape, dtype=torch.float64, pin_memory=True)
        out.copy_(t, non_blocking=True)
        torch.cuda.current_stream(t.device).synchronize()
        return out.numpy()
    return t.cpu().numpy()


def stream_handle(device):
    return torch.cuda.current_stream(device).cuda_stream
