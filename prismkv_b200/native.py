"""ctypes binding of libprismkv_b200.so (the C ABI of include/prismkv_b200.h).

The same calling convention as the reference's bindings
(src/prismkv/native8b.py:46-80, kernels/cuda_sm90/native.py:16-35): raw device
addresses, the current CUDA stream last, and a nonzero return raised as
RuntimeError.  There is no fallback: if the library is missing or cannot be
loaded, every operation raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libprismkv_b200.so"

PK_F32, PK_BF16 = 0, 1
PK_TERM_COUNT, PK_TERM_MEAN, PK_TERM_VARIANCE = 1, 2, 4
STATUS_BUCKET_FULL, STATUS_BOUNDARY_FULL, STATUS_MEMBERS_FULL = 1, 2, 4
STATUS_BUCKET_TOO_BIG, STATUS_OUT_FULL, STATUS_HISTORY_TOO_LONG = 8, 16, 32
STATUS_NEEDS_EXACT = 64
STATUS_EXCHANGE_TIMEOUT = 128
STATUS_BITS = {
    1: "bucket region full (append)",
    2: "boundary buffer full (build)",
    4: "member buffer full (build)",
    8: "bucket larger than the sort limit (build)",
    16: "union output row too short",
    32: "history longer than the union bitmap",
    64: "bounds could not bracket the threshold: exact build needed",
    128: "peer exchange timed out: a rank did not publish its buffer",
}

# name: (argument codes including the trailing stream, restype).
# P = device address / size_t, i = int, l = int64, f = float.
SIGNATURES = {
    "pk_version": ("", ctypes.c_int),
    "pk_supported_head_dim": ("i", ctypes.c_int),
    "pk_route_qact_workspace_bytes": ("iiii", ctypes.c_size_t),
    "pk_route_qact": ("PiPiPPPPfPiiiiiPPPPiPPP", ctypes.c_int),
    "pk_route_qact_shard_workspace_bytes": ("iiii", ctypes.c_size_t),
    "pk_route_qact_shard": ("PiPPPPfiiiiiiiPPPP", ctypes.c_int),
    "pk_route_qact_merge_workspace_bytes": ("iii", ctypes.c_size_t),
    "pk_route_qact_merge": ("PiPiiiiPPPPiPP", ctypes.c_int),
    "pk_sae_prepare": ("PiiPPP", ctypes.c_int),
    "pk_sae_prepare_half": ("PiiPP", ctypes.c_int),
    "pk_route_moments_workspace_bytes": ("iii", ctypes.c_size_t),
    "pk_route_moments": ("PiPPPiiiiiiPPPPPiP", ctypes.c_int),
    "pk_union": ("PPPlPPiPPiiiPlPPPPPP", ctypes.c_int),
    "pk_sparse_av_workspace_bytes": ("iiii", ctypes.c_size_t),
    "pk_sparse_av": ("PPPiilllPlPPPiiiiPPPPP", ctypes.c_int),
    "pk_sparse_av_append": ("PPPiilllPlPPPiiiiPPPPPPP", ctypes.c_int),
    "pk_lse_merge": ("PiiiPiP", ctypes.c_int),
    "pk_p2p_region_bytes": ("il", ctypes.c_size_t),
    "pk_p2p_alloc": ("PP", ctypes.c_int),
    "pk_p2p_free": ("P", ctypes.c_int),
    "pk_p2p_handle": ("PP", ctypes.c_int),
    "pk_p2p_open": ("PP", ctypes.c_int),
    "pk_p2p_close": ("P", ctypes.c_int),
    "pk_p2p_allgather": ("PliiPPPPlP", ctypes.c_int),
    "pk_gather_kv": ("PPiilllPlPPPiilPPPP", ctypes.c_int),
    "pk_kv_append": ("PPPPiilllPiiiP", ctypes.c_int),
    "pk_sparse_av_noalloc": ("PPPiilllPlPPPiiiiPP", ctypes.c_int),
    "pk_key_center": ("PilliliPP", ctypes.c_int),
    "pk_build_ids_capacity": ("liifi", ctypes.c_int64),
    "pk_build_workspace_bytes": ("iliil", ctypes.c_size_t),
    "pk_build_index": ("PillPfPPPPiliiilfiPPPllPPPP", ctypes.c_int),
    "pk_summarize": ("PillPPPliiiPPP", ctypes.c_int),
    "pk_merge_moments": ("PPPPPPiiiP", ctypes.c_int),
    "pk_append_workspace_bytes": ("iliiil", ctypes.c_size_t),
    "pk_append_index": ("PilllPfPPPPiiiilPPPlPPlPPPP", ctypes.c_int),
    "pk_build_shard_layout": ("ilillP", ctypes.c_int),
    "pk_build_shard_workspace_bytes": ("ilill", ctypes.c_size_t),
    "pk_build_shard_phase": ("iPillPfPPPPiliiillPPldlPPPllfiPPilPPPP", ctypes.c_int),
    "pk_key_center_chunks": ("PillililPP", ctypes.c_int),
    "pk_key_center_chunk_rows": ("l", ctypes.c_int64),
}
_CT = {"P": ctypes.c_uint64, "i": ctypes.c_int, "l": ctypes.c_int64, "f": ctypes.c_float, "d": ctypes.c_double}
# Entry points that take the stream as their last argument.
_ASYNC = {n for n, (c, r) in SIGNATURES.items() if r is ctypes.c_int and c.endswith("P") and n not in
          ("pk_version", "pk_supported_head_dim", "pk_build_shard_layout", "pk_p2p_alloc", "pk_p2p_free",
           "pk_p2p_handle", "pk_p2p_open", "pk_p2p_close")}

_lib = None


class NativeError(RuntimeError):
    pass


HEAD_DIM = 128   # the one head dimension the kernels are compiled for


def require_head_dim(d: int) -> None:
    """Refuse, before any launch, a head dimension the kernels do not
    implement (the library returns PK_ERR_UNSUPPORTED for it)."""
    if int(d) != HEAD_DIM:
        raise ValueError(f"head_dim {int(d)} is not supported: the CUDA kernels are built for head_dim {HEAD_DIM} only")


def lib():
    """Load the library once; raise if it is absent (no CPU fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise NativeError(f"{LIB_PATH} is missing: build it with `python -m prismkv_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (codes, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = [_CT[c] for c in codes]
            fn.restype = res
        _lib = L
    return _lib


def addr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, torch.Tensor):
        if x.numel() and not x.is_cuda:
            raise ValueError("device tensor required")
        return x.data_ptr()
    return int(x)


def stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def call(name: str, *args) -> None:
    """Calls an asynchronous entry point; tensor arguments pass their
    data_ptr and the current stream is appended.  Nonzero return ->
    RuntimeError (as native8b.py:79)."""
    fn = getattr(lib(), name)
    codes = SIGNATURES[name][0]
    if len(args) != len(codes) - 1:
        raise TypeError(f"{name} takes {len(codes) - 1} arguments, got {len(args)}")
    conv = []
    for a, c in zip(args, codes):
        if c == "P":
            conv.append(addr(a))
        elif c in ("f", "d"):
            conv.append(float(a))
        else:
            conv.append(int(a))
    conv.append(stream_handle())
    rc = fn(*conv)
    if rc:
        raise RuntimeError(f"{name}: {'argument error' if rc < 0 else 'CUDA error'} {rc}")


def query(name: str, *args):
    """Calls a host-only entry point (sizes, capacities, facts)."""
    return getattr(lib(), name)(*args)


def check_status(status: torch.Tensor, what: str) -> None:
    """Raise if a kernel flagged a condition in the device status word."""
    v = int(status.item())
    if v:
        msgs = [m for b, m in STATUS_BITS.items() if v & b]
        raise RuntimeError(f"{what}: " + "; ".join(msgs))


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return PK_F32
    if t.dtype == torch.bfloat16:
        return PK_BF16
    raise ValueError(f"unsupported dtype {t.dtype}: float32 or bfloat16 required")


class Workspace:
    """Zero-initialised device scratch buffers, kept across calls.  The kernels
    leave their counters zeroed, so a buffer is cleared only when created; the
    key names the call and its shape, because counter positions inside a
    workspace depend on the shape."""

    def __init__(self, device=None):
        self.device = torch.device(device or "cuda")
        self.buffers: dict = {}

    def get(self, name, nbytes: int) -> torch.Tensor:
        nbytes = max(int(nbytes), 256)
        buf = self.buffers.get(name)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self.buffers[name] = buf
        return buf

    def bytes(self) -> int:
        return sum(b.numel() for b in self.buffers.values())
