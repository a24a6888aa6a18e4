"""Python binding (ctypes) of the native engram runtime, engram_runtime/build/libengram_runtime.so:
GGUF engram metadata, the hash, token histories and the CPU / sm_100a injection. Used by the
tests and by tools that drive the runtime without llama.cpp."""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_HERE, "engram_runtime", "build", "libengram_runtime.so")
DRIVER_PATH = os.path.join(_HERE, "engram_runtime", "build", "engram_logits")
_lib = None


def build(quiet=True):
    """make -C engram_runtime (the library and the driver)."""
    import subprocess

    subprocess.run(["make", "-C", os.path.join(_HERE, "engram_runtime"), "-j4"], check=True,
                   capture_output=quiet)


def lib():
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run `make -C engram_runtime`")
        L = ctypes.CDLL(LIB_PATH)
        P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.me_rt_open.argtypes = [ctypes.c_char_p, I32, ctypes.POINTER(P)]
        L.me_rt_close.argtypes = [P]
        L.me_rt_last_error.restype = ctypes.c_char_p
        for fn in ("me_rt_n_engrams", "me_rt_max_order"):
            getattr(L, fn).argtypes = [P]
            getattr(L, fn).restype = I32
        L.me_rt_n_embd.argtypes = [P]
        L.me_rt_n_embd.restype = I64
        L.me_rt_engram_info.argtypes = [P, I32] + [ctypes.POINTER(I32)] * 4 + [ctypes.POINTER(I64)]
        L.me_rt_engram_at_layer.argtypes = [P, I32]
        L.me_rt_engram_at_layer.restype = I32
        L.me_rt_hash.argtypes = [P, I32, P, P, I64, P]
        L.me_rt_hist_new.argtypes = [ctypes.POINTER(P)]
        L.me_rt_hist_free.argtypes = [P]
        L.me_rt_hist_set.argtypes = [P, I32, I64, I32]
        L.me_rt_hist_remove.argtypes = [P, I32, I64, I64]
        L.me_rt_hist_copy.argtypes = [P, I32, I32]
        L.me_rt_hist_prev.argtypes = [P, P, P, I64, I32, P]
        L.me_rt_hist_save.argtypes = [P, I32, P, ctypes.POINTER(ctypes.c_size_t)]
        L.me_rt_hist_load.argtypes = [P, I32, P, ctypes.c_size_t]
        L.me_rt_inject_cpu.argtypes = [P, I32, P, P, P, I64]
        L.me_rt_cuda_upload.argtypes = [P, I32, I32]
        L.me_rt_cuda_inject.argtypes = [P, I32, P, P, P, I64, P]
        _lib = L
    return _lib


def _check(rc):
    if rc != 0:
        raise RuntimeError(f"engram runtime error {rc}: {lib().me_rt_last_error().decode()}")


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


class Runtime:
    """One GGUF's engrams."""

    def __init__(self, path, n_layer=-1):
        self.h = ctypes.c_void_p()
        _check(lib().me_rt_open(path.encode(), n_layer, ctypes.byref(self.h)))
        self.n_engrams = lib().me_rt_n_engrams(self.h)
        self.max_order = lib().me_rt_max_order(self.h)
        self.n_embd = lib().me_rt_n_embd(self.h)

    def info(self, e):
        v = [ctypes.c_int32() for _ in range(4)]
        rows = ctypes.c_int64()
        _check(lib().me_rt_engram_info(self.h, e, *[ctypes.byref(x) for x in v], ctypes.byref(rows)))
        layer, gate, n_tables, dim = (x.value for x in v)
        return {"layer": layer, "gate": gate, "n_tables": n_tables, "dim": dim, "total_rows": rows.value}

    def hash(self, e, tokens, prev):
        """rows [n, n_tables] int32 (absolute rows); prev [n, max_order-1] oldest first, -1 = none."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        prev = np.ascontiguousarray(prev, dtype=np.int32).reshape(len(tokens), self.max_order - 1)
        out = np.empty((len(tokens), self.info(e)["n_tables"]), dtype=np.int32)
        _check(lib().me_rt_hash(self.h, e, _ptr(tokens), _ptr(prev), len(tokens), _ptr(out)))
        return out

    def inject_cpu(self, e, hidden, rows, keep=None):
        hidden = np.ascontiguousarray(hidden, dtype=np.float32).copy()
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        keep = None if keep is None else np.ascontiguousarray(keep, dtype=np.float32)
        _check(lib().me_rt_inject_cpu(self.h, e, _ptr(hidden), _ptr(rows), _ptr(keep), hidden.shape[0]))
        return hidden

    def cuda_upload(self, e, device=0):
        _check(lib().me_rt_cuda_upload(self.h, e, device))

    def cuda_inject(self, e, d_hidden_ptr, d_rows_ptr, n, d_keep_ptr=None, stream=None):
        _check(lib().me_rt_cuda_inject(self.h, e, ctypes.c_void_p(d_hidden_ptr), ctypes.c_void_p(d_rows_ptr),
                                       ctypes.c_void_p(d_keep_ptr) if d_keep_ptr else None, n,
                                       ctypes.c_void_p(stream) if stream else None))

    def close(self):
        if self.h:
            lib().me_rt_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class History:
    """Token ids per sequence, by position (what a KV cache keeps for the engram)."""

    def __init__(self):
        self.h = ctypes.c_void_p()
        _check(lib().me_rt_hist_new(ctypes.byref(self.h)))

    def set(self, seq, pos, tok):
        _check(lib().me_rt_hist_set(self.h, seq, pos, tok))

    def remove(self, seq, p0=0, p1=-1):
        _check(lib().me_rt_hist_remove(self.h, seq, p0, p1))

    def copy(self, src, dst):
        _check(lib().me_rt_hist_copy(self.h, src, dst))

    def prev(self, seqs, poss, n_prev):
        seqs = np.ascontiguousarray(seqs, dtype=np.int32)
        poss = np.ascontiguousarray(poss, dtype=np.int64)
        out = np.empty((len(seqs), n_prev), dtype=np.int32)
        _check(lib().me_rt_hist_prev(self.h, _ptr(seqs), _ptr(poss), len(seqs), n_prev, _ptr(out)))
        return out

    def save(self, seq):
        size = ctypes.c_size_t()
        _check(lib().me_rt_hist_save(self.h, seq, None, ctypes.byref(size)))
        buf = ctypes.create_string_buffer(size.value)
        _check(lib().me_rt_hist_save(self.h, seq, buf, ctypes.byref(size)))
        return buf.raw

    def load(self, seq, blob):
        _check(lib().me_rt_hist_load(self.h, seq, blob, len(blob)))

    def __del__(self):
        try:
            if self.h:
                lib().me_rt_hist_free(self.h)
        except Exception:  # noqa: BLE001
            pass
