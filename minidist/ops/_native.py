"""ctypes binding to the native sm_100a library (``minidist/_lib/libminidist_cuda.so``).

The library exposes plain ``extern "C"`` entry points that take device
pointers, sizes and a ``cudaStream_t``; this module turns torch tensors into
those arguments.  Allocation stays with PyTorch's caching allocator, streams are
PyTorch's current streams, and every kernel runs in the same primary context.

On a CUDA machine the library is mandatory: :func:`lib` raises if it is missing
rather than silently falling back to eager PyTorch, so a test that passes on a
GPU is known to have run the hand-written kernels.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# MINIDIST_BOUNDS_CHECK=1 loads the checking build (python -m minidist._build --bounds-check).
_LIB_PATH = Path(__file__).resolve().parent.parent / "_lib" / (
    "libminidist_cuda_checked.so" if os.environ.get("MINIDIST_BOUNDS_CHECK", "0") not in ("0", "", "false", "no")
    else "libminidist_cuda.so")
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A native entry point rejected its arguments or a kernel reported a fault."""


class CommTimeoutError(NativeError):
    """A bounded wait on a peer GPU (or an intra-kernel pipeline) expired."""


def library_path() -> Path:
    return _LIB_PATH


def bounds_checked() -> bool:
    """True when the bounds-checking build is the one loaded (``MINIDIST_BOUNDS_CHECK=1``)."""
    return _LIB_PATH.name == "libminidist_cuda_checked.so"


def available() -> bool:
    return torch.cuda.is_available() and _LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise NativeError(
                f"native library {_LIB_PATH} is missing; build it with "
                "`python -m minidist._build` (needs nvcc)"
            )
        handle = ctypes.CDLL(str(_LIB_PATH), mode=ctypes.RTLD_GLOBAL)
        _declare(handle)
        _lib = handle
    return _lib


def _declare(h: ctypes.CDLL) -> None:
    vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float
    h.md_gemm.argtypes = [ctypes.POINTER(GemmParams), vp]
    h.md_gemm.restype = i32
    h.md_gemm_ce_slab.argtypes = []
    h.md_gemm_ce_slab.restype = i32
    for name, args in _EXTRA_DECLS.items():
        fn = getattr(h, name, None)
        if fn is None:
            continue
        fn.argtypes = [_TYPES[a] for a in args[1:]]
        fn.restype = _TYPES[args[0]]
    del vp, i32, i64, f32


_TYPES = {
    "p": ctypes.c_void_p,
    "i": ctypes.c_int,
    "l": ctypes.c_longlong,
    "f": ctypes.c_float,
    "d": ctypes.c_double,
}

# name -> (restype, argtypes...) using the single-letter codes above.  Kernels
# register themselves here from their Python wrappers.
_EXTRA_DECLS: dict[str, tuple[str, ...]] = {}


def declare(name: str, signature: str) -> None:
    """Register an entry point signature, e.g. ``declare("md_ln_fwd", "i:pppplliip")``."""
    ret, args = signature.split(":")
    _EXTRA_DECLS[name] = (ret, *args)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.argtypes = [_TYPES[a] for a in args]
        fn.restype = _TYPES[ret]


class GemmParams(ctypes.Structure):
    """Mirror of ``struct MdGemmParams`` in csrc/gemm_sm100.cu."""

    _fields_ = [
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("D", ctypes.c_void_p),
        ("lda", ctypes.c_longlong),
        ("ldb", ctypes.c_longlong),
        ("ldd", ctypes.c_longlong),
        ("M", ctypes.c_int),
        ("N", ctypes.c_int),
        ("K", ctypes.c_int),
        ("a_mn_major", ctypes.c_int),
        ("b_mn_major", ctypes.c_int),
        ("epi", ctypes.c_int),
        ("alpha", ctypes.c_float),
        ("beta", ctypes.c_int),
        ("gelu", ctypes.c_int),
        ("bias", ctypes.c_void_p),
        ("aux", ctypes.c_void_p),
        ("ldaux", ctypes.c_longlong),
        ("resid", ctypes.c_void_p),
        ("ldres", ctypes.c_longlong),
        ("workspace", ctypes.c_void_p),
        ("ldws", ctypes.c_longlong),
        ("k_splits", ctypes.c_int),
        ("ce_target", ctypes.c_void_p),
        ("ce_max", ctypes.c_void_p),
        ("ce_sum", ctypes.c_void_p),
        ("ce_tgt", ctypes.c_void_p),
        ("ce_col_offset", ctypes.c_longlong),
        ("num_sms", ctypes.c_int),
        ("status", ctypes.c_void_p),
        ("cta_group", ctypes.c_int),
        ("epi_warps", ctypes.c_int),
        ("colsum", ctypes.c_void_p),
        ("dot_in", ctypes.c_void_p),
        ("lddot", ctypes.c_longlong),
        ("dot_out", ctypes.c_void_p),
        ("dot_group", ctypes.c_int),
        ("dot_seq", ctypes.c_int),
    ]


# ---------------------------------------------------------------------------
# Per-device status word (md::Status in csrc/md_sm100.cuh)
# ---------------------------------------------------------------------------

_status: dict[int, torch.Tensor] = {}

_STATUS_NAMES = {1: "pipeline wait timed out", 2: "peer wait timed out", 3: "bad kernel argument"}


def status_buffer(device: torch.device | int | None = None) -> torch.Tensor:
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        idx = device.index if device.index is not None else torch.cuda.current_device()
    else:
        idx = int(device)
    buf = _status.get(idx)
    if buf is None:
        buf = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = buf
    return buf


def status_ptr(device=None) -> int:
    return status_buffer(device).data_ptr()


def check_status(device=None, reset: bool = True) -> None:
    """Raise if any kernel on ``device`` reported a fault since the last check.

    Synchronises the device (the status word is written by kernels).
    """
    buf = status_buffer(device)
    torch.cuda.synchronize(buf.device)
    code, where, block, detail = (int(v) for v in buf.tolist())
    if code == 0 and bounds_checked():
        # The checking build's kernels without a status argument report into per-file words.
        for reader in ("md_check_status_embedding", "md_check_status_cross_entropy"):
            word = (ctypes.c_uint32 * 4)()
            check(getattr(lib(), reader)(ctypes.cast(word, ctypes.c_void_p), int(reset)), reader)
            if word[0]:
                code, where, block, detail = (int(v) for v in word)
                break
    if code == 0:
        return
    if reset:
        buf.zero_()
    msg = (
        f"native kernel reported '{_STATUS_NAMES.get(code, code)}' at site {where} "
        f"(block {block}, detail {detail})"
    )
    if code in (1, 2):
        raise CommTimeoutError(msg)
    raise NativeError(msg)


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise NativeError(f"{what} failed with code {rc}")


def num_sms(device=None) -> int:
    props = torch.cuda.get_device_properties(device if device is not None else torch.cuda.current_device())
    return props.multi_processor_count


def env_flag(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v not in ("0", "", "false", "False", "no")


declare("md_peer_wait_enable", "i:ii")
declare("md_peer_wait_read", "i:p")
declare("md_gemm_ar_wait_enable", "i:ii")
declare("md_gemm_ar_wait_read", "i:p")

# Channel of each peer-memory kernel family (minidist.parallel.collectives).
_PEER_WAIT_FAMILIES = {0: "md_ar_bucket", 1: "md_ar_bucket", 2: "md_ar_bucket", 3: "md_ar_bucket",
                       4: "md_rs_shard", 5: "md_ag_shards", 6: "md_ce_tp", 7: "md_embed_tp"}


def peer_wait_counters(enable: bool, reset: bool = False) -> dict[str, dict[str, float]]:
    """Turn the fused kernels' device-side wait counters on or off for the current device and
    return what they hold: ``{family: {"run_ms", "wait_ms", "wait_frac", "launches"}}`` with
    times summed over CTAs (``wait`` = time in cross-rank barriers / peer-flag polls).  Host-
    synchronous; for analysis runs (``minidist.profiling.PeerWaitCounters``), not inside a
    CUDA-graph capture."""
    h = lib()
    raw = (ctypes.c_ulonglong * 24)()
    check(h.md_peer_wait_read(ctypes.cast(raw, ctypes.c_void_p)), "md_peer_wait_read")
    gar = (ctypes.c_ulonglong * 3)()
    check(h.md_gemm_ar_wait_read(ctypes.cast(gar, ctypes.c_void_p)), "md_gemm_ar_wait_read")
    check(h.md_peer_wait_enable(int(enable), int(reset)), "md_peer_wait_enable")
    check(h.md_gemm_ar_wait_enable(int(enable), int(reset)), "md_gemm_ar_wait_enable")
    acc: dict[str, list[float]] = {}
    for ch, fam in _PEER_WAIT_FAMILIES.items():
        run, wait, n = raw[3 * ch], raw[3 * ch + 1], raw[3 * ch + 2]
        if run or n:
            a = acc.setdefault(fam, [0.0, 0.0, 0.0])
            a[0] += run
            a[1] += wait
            a[2] += n
    if gar[0] or gar[2]:
        acc["md_gemm_ar"] = [float(gar[0]), float(gar[1]), float(gar[2])]
    return {fam: {"run_ms": a[0] / 1e6, "wait_ms": a[1] / 1e6, "wait_frac": a[1] / a[0] if a[0] else 0.0,
                  "launches": a[2]} for fam, a in acc.items()}


declare("md_check_status_embedding", "i:pi")
declare("md_check_status_cross_entropy", "i:pi")
