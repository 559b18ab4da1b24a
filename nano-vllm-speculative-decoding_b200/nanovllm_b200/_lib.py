"""ctypes binding of libspecdec_b200.so, the C-ABI library that holds every CUDA kernel of this package.

There is no CPU fallback: importing a kernel wrapper on a machine where the library is missing raises, and a
call whose tensors are not on a CUDA device raises.  PyTorch is only the owner of device memory and streams
here; every computation on the hot path is a kernel of the library.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIBRARY_PATH = Path(__file__).resolve().parent / "libspecdec_b200.so"

# dtype codes shared with csrc/common.cuh
DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}

_c_void_p = ctypes.c_void_p
_c_ll = ctypes.c_longlong
_c_ull = ctypes.c_ulonglong
_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float

# name -> (restype, argtypes); the declarations mirror include/specdec_b200.h
SIGNATURES = {
    "specdec_version": (_c_int, []),
    "specdec_last_error": (ctypes.c_char_p, []),
    "specdec_device_supported": (_c_int, []),
    "specdec_sampler_workspace_bytes": (_c_size, [_c_ll]),
    "specdec_accept_workspace_bytes": (_c_size, [_c_ll, _c_ll, _c_ll]),
    "specdec_exponential_codes": (_c_int, [_c_ull, _c_ull, _c_ll, _c_void_p, _c_void_p, _c_void_p]),
    "specdec_philox_increment": (_c_ull, [_c_ll]),
    "specdec_probs": (_c_int, [_c_void_p, _c_int, _c_ll, _c_ll, _c_ll, _c_void_p, _c_void_p, _c_void_p, _c_int,
                               _c_int, _c_void_p, _c_void_p, _c_size, _c_void_p]),
    "specdec_accept": (_c_int, [_c_void_p, _c_int, _c_int, _c_ll, _c_ll, _c_void_p, _c_void_p, _c_ll, _c_ll,
                                _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_void_p,
                                _c_ull, _c_ull, _c_ull, _c_void_p, _c_void_p, _c_void_p, _c_size, _c_void_p]),
    "specdec_accept_noalloc": (_c_int, [_c_void_p, _c_int, _c_int, _c_ll, _c_ll, _c_void_p, _c_void_p, _c_ll, _c_ll,
                                        _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p,
                                        _c_void_p, _c_ull, _c_ull, _c_ull, _c_void_p, _c_void_p, _c_void_p]),
    "specdec_accept_greedy": (_c_int, [_c_void_p, _c_int, _c_ll, _c_ll, _c_void_p, _c_ll, _c_ll, _c_void_p,
                                       _c_void_p, _c_void_p, _c_void_p, _c_size, _c_void_p]),
    "specdec_race": (_c_int, [_c_void_p, _c_ll, _c_ll, _c_void_p, _c_ull, _c_ull, _c_void_p, _c_void_p, _c_size,
                              _c_void_p]),
    "specdec_store_kvcache": (_c_int, [_c_void_p, _c_ll, _c_void_p, _c_ll, _c_void_p, _c_void_p, _c_void_p, _c_ll,
                                       _c_int, _c_int, _c_ll, _c_void_p, _c_void_p]),
    "specdec_paged_attention": (_c_int, [_c_void_p, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_void_p, _c_void_p, _c_ll,
                                         _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p, _c_int,
                                         _c_int, _c_float, _c_int, _c_void_p, _c_ll, _c_void_p, _c_ll, _c_void_p,
                                         _c_void_p]),
    "specdec_paged_attention_ex": (_c_int, [_c_void_p, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                            _c_ll, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p,
                                            _c_int, _c_int, _c_float, _c_int, _c_void_p, _c_ll, _c_void_p, _c_ll,
                                            _c_void_p, ctypes.c_uint, _c_void_p]),
    "specdec_paged_attention_multi": (_c_int, [_c_void_p, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_void_p,
                                               _c_void_p, _c_ll, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int,
                                               _c_int, _c_void_p, _c_int, _c_int, _c_float, _c_int, _c_void_p,
                                               _c_int, _c_ll, _c_void_p, _c_ll, _c_void_p, ctypes.c_uint, _c_void_p]),
    "specdec_attention_workspace_bytes": (_c_ll, [_c_int, _c_int]),
    "specdec_peer_barrier": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_ll, _c_void_p, _c_void_p]),
    "specdec_norm_rope_store": (_c_int, [_c_void_p, _c_ll, _c_ll, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                         _c_ll, _c_void_p, _c_ll, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_ll,
                                         _c_ll, _c_void_p, _c_float, _c_void_p, _c_void_p]),
    "specdec_rmsnorm": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_ll, _c_int, _c_float,
                                 _c_void_p]),
    "specdec_silu_mul": (_c_int, [_c_void_p, _c_void_p, _c_ll, _c_int, _c_void_p]),
    "specdec_markov_step": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                     _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_void_p,
                                     _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_void_p,
                                     _c_void_p, _c_void_p, _c_ll, _c_void_p, _c_void_p]),
    "specdec_markov_workspace_bytes": (_c_ll, [_c_int, _c_int, _c_int, _c_int]),
    "specdec_context_gemm_workspace_bytes": (_c_ll, [_c_int, _c_int]),
    "specdec_context_gemm": (_c_int, [_c_void_p, _c_ll, _c_void_p, _c_ll, _c_int, _c_int, _c_int, _c_void_p, _c_ll,
                                      _c_void_p, _c_ll, _c_void_p, _c_void_p]),
    "specdec_markov_bias": (_c_int, [_c_void_p, _c_ll, _c_void_p, _c_ll, _c_int, _c_int, _c_int, _c_void_p, _c_ll,
                                     _c_void_p, _c_ll, _c_void_p, _c_ll, _c_void_p, _c_void_p]),
    "specdec_context_kv_store": (_c_int, [_c_void_p, _c_ll, _c_void_p, _c_ll, _c_int, _c_int, _c_int, _c_int,
                                          _c_void_p, _c_ll, _c_void_p, _c_ll, _c_void_p, _c_void_p, _c_void_p,
                                          _c_void_p, _c_ll, _c_ll, _c_float, _c_void_p, _c_ll, _c_void_p,
                                          _c_void_p]),
}

_lib = None
_lock = threading.Lock()


class SpecdecError(RuntimeError):
    """A non-zero status from the C-ABI library, with its message."""


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Loads the library (once) and declares every entry point; raises when it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        target = Path(path) if path is not None else LIBRARY_PATH
        if not target.exists():
            raise ImportError(f"{target} is missing: build it with `python nano-vllm-speculative-decoding_b200/"
                              f"build.py` (nvcc, sm_100a); this package has no CPU fallback")
        lib = ctypes.CDLL(str(target))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load()


def check(status: int) -> None:
    if status != 0:
        message = lib().specdec_last_error().decode(errors="replace")
        raise SpecdecError(f"specdec status {status}: {message}")


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    device = None
    for tensor in tensors:
        if tensor is None:
            continue
        if tensor.device.type != "cuda":
            raise ValueError(f"the B200 kernels need CUDA tensors, got one on {tensor.device}")
        if device is None:
            device = tensor.device
        elif tensor.device != device:
            raise ValueError(f"tensors on {device} and {tensor.device}")
    if device is None:
        raise ValueError("no tensor given")
    return device


class Workspace:
    """A zero-initialised device byte buffer per (device, name), grown on demand.  The library keeps its tickets
    and argmax keys self-cleaning at fixed offsets, so the buffer is zeroed once per allocation only.  A grown
    buffer's predecessor is kept alive: a CUDA graph captured with the old address keeps replaying into valid
    memory (its own, since later calls outside the graph use the new buffer)."""

    _buffers: dict[tuple[int, str], torch.Tensor] = {}
    _retired: list[torch.Tensor] = []

    @classmethod
    def get(cls, device: torch.device, nbytes: int, name: str = "sampler") -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), name)
        buf = cls._buffers.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None:
                cls._retired.append(buf)
            size = max(nbytes, 1 << 20)
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            cls._buffers[key] = buf
        return buf


def device_status(device: torch.device, name: str = "sampler") -> int:
    """The device-side input-check word of the last sampler call on this device (synchronises): 0 ok,
    1 verified lengths outside 1..k+1 or not summing to T, 2 a draft id outside [0, V), 3 a top_k above the cap."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), name)
    buf = Workspace._buffers.get(key)
    return 0 if buf is None else int(buf[:4].view(torch.int32).item())
