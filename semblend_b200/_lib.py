"""ctypes binding of the semblend_b200 C ABI (``include/semblend_b200.h``).

The native library is the only compute path: if it is missing or cannot be
loaded, every entry point raises :class:`NativeLibraryError` rather than
falling back to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_native" / "libsemblend_b200.so"

# Status codes (semblend_b200.h)
SB_OK = 0
SB_ERR_INVALID_ARGUMENT = -1
SB_ERR_UNSUPPORTED = -2
SB_ERR_CUDA = -3
SB_ERR_WORKSPACE_TOO_SMALL = -4
SB_ERR_TOO_LARGE = -5

SB_DTYPE_F32, SB_DTYPE_F16, SB_DTYPE_BF16 = 0, 1, 2
SB_INDEX_I32, SB_INDEX_I64 = 0, 1
SB_ROTARY_INTERLEAVED, SB_ROTARY_NEOX = 0, 1
SB_ANGLE_NONE, SB_ANGLE_DELTA, SB_ANGLE_NOPE, SB_ANGLE_CONST = 0, 1, 2, 3
SB_ROW_AT_SRC_POS, SB_ROW_AT_DST_POS, SB_ROW_AT_PAIR = 0, 1, 2
SB_KV_K, SB_KV_V, SB_KV_BOTH = 1, 2, 3
SB_MAX_INJECT_DESC = 64
SB_PERMUTE_NOALLOC_SCRATCH_BYTES = 32 << 20
SB_DESC_CHECK_SRC_IN_DST = 1
SB_INJECT_BULK_STAGED = 1

_DTYPES = {torch.float32: SB_DTYPE_F32, torch.float16: SB_DTYPE_F16, torch.bfloat16: SB_DTYPE_BF16}
_INDEX_DTYPES = {torch.int32: SB_INDEX_I32, torch.int64: SB_INDEX_I64}


class NativeLibraryError(RuntimeError):
    """The CUDA extension is missing, failed to load, or rejected a call."""


class SbRows(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_void_p),
        ("layer_ptrs", ctypes.c_void_p),
        ("stride_layer", ctypes.c_int64),
        ("stride_block", ctypes.c_int64),
        ("stride_kv", ctypes.c_int64),
        ("stride_head", ctypes.c_int64),
        ("stride_pos", ctypes.c_int64),
        ("stride_dim", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("n_logical", ctypes.c_int64),
        ("n_physical", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("block_table_dtype", ctypes.c_int32),
    ]


class SbInjectDesc(ctypes.Structure):
    _fields_ = [
        ("src", SbRows),
        ("dst", SbRows),
        ("src_pos", ctypes.c_void_p),
        ("dst_pos", ctypes.c_void_p),
        ("n_pairs", ctypes.c_int64),
        ("pos_dtype", ctypes.c_int32),
        ("src_row", ctypes.c_int32),
        ("dst_row", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class SbInjectParams(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32),
        ("n_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("rotary_style", ctypes.c_int32),
        ("k_angle", ctypes.c_int32),
        ("kv_select", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("const_delta", ctypes.c_int64),
        ("inv_freq", ctypes.c_void_p),
    ]


class SbAttnTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("stride_batch", ctypes.c_int64),
        ("stride_head", ctypes.c_int64),
        ("stride_seq", ctypes.c_int64),
    ]


_P = ctypes.POINTER
_SIGNATURES: dict[str, tuple] = {
    "sb_inject": (ctypes.c_int, [_P(SbInjectDesc), ctypes.c_int32, _P(SbInjectParams), ctypes.c_void_p, ctypes.c_void_p]),
    "sb_inject_table_bytes": (ctypes.c_int64, [ctypes.c_int32]),
    "sb_inject_many": (
        ctypes.c_int,
        [_P(SbInjectDesc), ctypes.c_int32, _P(SbInjectParams), ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
         ctypes.c_void_p],
    ),
    "sb_permute_workspace_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "sb_permute_paged": (
        ctypes.c_int,
        [_P(SbRows), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, _P(SbInjectParams),
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_permute_paged_noalloc": (
        ctypes.c_int,
        [_P(SbRows), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, _P(SbInjectParams),
         ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_search_prepare_rows": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_cosine_topk_workspace_bytes": (
        ctypes.c_int64, [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "sb_cosine_topk": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
         ctypes.c_int64,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_float, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_cosine_screen": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_float, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_cosine_rescore": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_float, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_chunk_digests": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_chunk_align": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_chunk_align_batch": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_token_overlap_workspace_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64]),
    "sb_token_overlap": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_topk_merge": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_mask_to_rows": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_partial_attention": (
        ctypes.c_int,
        [SbAttnTensor, SbAttnTensor, SbAttnTensor, SbAttnTensor, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
         ctypes.c_float, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_masked_linear_workspace_bytes": (ctypes.c_int64, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "sb_masked_linear": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "sb_profile_start": (ctypes.c_int, [ctypes.c_int32]),
    "sb_profile_stop": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "sb_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "sb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "sb_version": (ctypes.c_int, []),
    "sb_last_cuda_error": (ctypes.c_int, []),
}

_lib = None
_lib_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the native library once (raises NativeLibraryError if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("SEMBLEND_B200_LIB", LIB_PATH))
        if not path.exists():
            raise NativeLibraryError(
                f"semblend_b200 native library not found at {path}; build it with "
                "`python -m semblend_b200.build` (needs nvcc with sm_100a support)"
            )
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as exc:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"cannot load {path}: {exc}") from exc
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                raise NativeLibraryError(f"{path} does not export {name}")
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == SB_OK:
        return
    lib = load()
    msg = lib.sb_status_string(status).decode()
    if status == SB_ERR_CUDA:
        msg += f" (cudaError {lib.sb_last_cuda_error()})"
    if status in (SB_ERR_INVALID_ARGUMENT, SB_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise NativeLibraryError(f"{what}: {msg}")


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise NativeLibraryError(
            f"{name} is on {t.device}; the semblend_b200 kernels run on CUDA devices only "
            "(there is no CPU implementation)"
        )


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported KV dtype {dt}; expected float32, float16 or bfloat16") from None


def index_code(dt: torch.dtype) -> int:
    try:
        return _INDEX_DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported index dtype {dt}; expected int32 or int64") from None


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# Per-device state: the skipped-pair counter and RoPE frequency tables.
# ---------------------------------------------------------------------------
_state_lock = threading.Lock()
_err_counters: dict[int, torch.Tensor] = {}
_inv_freq_cache: dict[tuple, torch.Tensor] = {}


def err_counter(device: torch.device) -> torch.Tensor:
    """Device counter of pairs skipped as out of range (int64, one element)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _err_counters.get(idx)
    if t is None:
        with _state_lock:
            t = _err_counters.get(idx)
            if t is None:
                t = torch.zeros(1, dtype=torch.int64, device=torch.device("cuda", idx))
                _err_counters[idx] = t
    return t


def skipped_pairs(device: torch.device | int | None = None, reset: bool = False) -> int:
    """Number of pairs the kernels skipped as out of range on ``device``.

    Reading synchronises with the device.  The reference's GPU kernels skip
    such pairs silently (semblend_core/rope_correction.py:117-129); this counter
    makes the skips observable.
    """
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    t = err_counter(device)
    n = int(t.item())
    if reset:
        t.zero_()
    return n


def inv_freq(rope_base: float, head_dim: int, device: torch.device) -> torch.Tensor:
    """RoPE inverse frequencies ``1 / base**(2i/D)`` on ``device``.

    Built on the host with the reference's own fp32 torch expression
    (semblend_core/rope_correction.py:235-238) and uploaded once per
    (base, head_dim, device), so device results use the exact same table as
    the reference's CPU path.
    """
    key = (float(rope_base), int(head_dim), device.index)
    t = _inv_freq_cache.get(key)
    if t is None:
        host = 1.0 / (rope_base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        t = host.to(device)
        with _state_lock:
            _inv_freq_cache[key] = t
    return t


class KernelTimer:
    """Times the dominant kernel of the C-ABI calls made inside the ``with``
    block (CUDA events on the launch stream, recorded by the library)."""

    def __init__(self, max_launches: int = 4096):
        self.max_launches = max_launches
        self.total_ms = 0.0
        self.launches = 0

    def __enter__(self):
        check(load().sb_profile_start(self.max_launches), "sb_profile_start")
        return self

    def __exit__(self, *exc):
        ms = ctypes.c_float()
        n = ctypes.c_int32()
        check(load().sb_profile_stop(ctypes.byref(ms), ctypes.byref(n)), "sb_profile_stop")
        self.total_ms, self.launches = float(ms.value), int(n.value)
        return False

    @property
    def mean_ms(self) -> float:
        return self.total_ms / self.launches if self.launches else float("nan")
