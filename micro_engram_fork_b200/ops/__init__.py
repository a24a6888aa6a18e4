"""Autograd ops over the sm_100a kernels. Every op takes CUDA tensors to the native kernel
and CPU tensors to its plain PyTorch reference (which is also the numerics oracle)."""
from .. import force_reference


def use_native(*tensors):
    """True when the op should run its sm_100a kernel: any input is on CUDA."""
    if force_reference():
        return False
    return any(t is not None and t.is_cuda for t in tensors)
