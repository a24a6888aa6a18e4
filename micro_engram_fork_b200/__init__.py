"""micro_engram_fork_b200: the B200-native (sm_100a) engine under the micro_engram API.

Layout:
  ops/       autograd ops backed by the hand-written sm_100a kernels in csrc/ (engram
             hash/gather/gate/row-grad/Adam, RMSNorm, q/k/v norm + RoPE, GeGLU, softcapped
             CE, attention, tcgen05 GEMM), each with a plain PyTorch reference used on CPU
             and as the test oracle
  parallel/  symmetric peer memory over NVLink (CUDA IPC), the row store of the
             row-sharded engram tables, P2P collectives
  models/    the Gemma-4-style decoder (frozen base) built from the ops above
  utils/     per-phase CUDA-event timers with NVTX ranges (timers.py) and the benchmarks:
             kernel microbenchmarks (kernel_bench), the engram module benchmark (engram_bench),
             the peer-memory all-reduce against NCCL (p2p_bench)

The native extension is `micro_engram_fork_b200._C`, built in-tree by
``python setup.py build_ext --inplace`` for sm_100a only.
"""
import importlib
import os

_C = None
_C_ERROR = None


def _load():
    global _C, _C_ERROR
    if _C is not None or _C_ERROR is not None:
        return _C
    try:
        import torch  # noqa: F401 - loads libc10/libtorch the extension links against

        _C = importlib.import_module("micro_engram_fork_b200._C")
    except ImportError as e:  # not built (CPU-only checkout): CUDA ops raise on use
        _C_ERROR = e
    return _C


def native():
    """The compiled sm_100a extension. Raises if it is missing: CUDA tensors never fall back
    to a silent PyTorch path."""
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "micro_engram_fork_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_C_ERROR})")
    return mod


def has_native():
    return _load() is not None


def force_reference():
    """MICRO_ENGRAM_REFERENCE_OPS=1 runs the plain PyTorch ops even on CUDA (oracle runs only)."""
    return os.environ.get("MICRO_ENGRAM_REFERENCE_OPS") == "1"
