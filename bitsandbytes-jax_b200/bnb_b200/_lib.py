"""ctypes binding of libbnbq.so (include/bnbq.h) for torch CUDA tensors.

The library is built in-tree by ``bitsandbytes-jax_b200/build.py`` and loaded
from this directory; there is no other implementation behind these calls. A
missing library, a missing GPU or a non-sm_100 device raises -- nothing falls
back to another code path.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libbnbq.so"

F32, F16, BF16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_MISALIGNED, ERR_CUDA, ERR_DEVICE, ERR_TOO_LARGE = 0, -1, -2, -3, -4, -5, -6
GEMV_MAX_M = 20
GEMV8_MAX_M = 4  # BNBQ_GEMV8_MAX_M

DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

# argument kinds: p = pointer, i = int32, l = int64
_SIGNATURES = {
    "bnbq_quantize_nf4": "ipliPPP",
    "bnbq_quantize_blockwise": "ipliPPPPP",
    "bnbq_absmax_mean": "PlPP",
    "bnbq_quantize_nf4_dq": "ipliPiPPPPPPlP",
    "bnbq_quantize_nf4_dq_workspace_bytes": "",
    "bnbq_dequantize_nf4": "iPPliPP",
    "bnbq_dequantize_blockwise": "iPPPliPPP",
    "bnbq_dequantize_nf4_nested": "iPPPPPliiPP",
    "bnbq_dequantize_blockwise_nested": "iPPPPPPliiPP",
    "bnbq_gemv_nf4": "iPiiPliPPPPPilPlP",
    "bnbq_matmul_nf4": "iPiiPliPPPPPilPlP",
    "bnbq_gemv_nf4_ws": "iPiiPliPPPPPilPlPlP",
    "bnbq_matmul_nf4_ws": "iPiiPliPPPPPilPlPlP",
    "bnbq_matmul_nf4_allgather": "iPiiPliPPPPPilPlllPlPiiPlP",
    "bnbq_gemv_workspace_bytes": "iilP",
    "bnbq_gemv_blockwise_ws": "iPiiPliPPPPPPilPlPlP",
    "bnbq_gemv_blockwise_workspace_bytes": "iilP",
    "bnbq_gemv_t_nf4_ws": "iPillipiPPPPPilPlPlP",
    "bnbq_gemv_t_nf4_workspace_bytes": "iilP",
    "bnbq_gemv_route": "iiliPiPlP",
    "bnbq_set_gemv_policy": "i",
    "bnbq_rcp_approx_ftz": "PPlP",
    "bnbq_version": "",
    "bnbq_wait_timeouts": "P",
    "bnbq_peer_allgather_rows": "iPilllPllPlPiiP",
    "bnbq_peer_allgather_rows_noalloc": "iPilllPllPliiiP",
    "bnbq_peer_allgather_noalloc_setup": "",
    "bnbq_peer_allgather_noalloc_reset": "iP",
    "bnbq_set_wait_limit_ns": "u",
    "bnbq_enable_peer_access": "i",
    "bnbq_ipc_handle": "PPP",
    "bnbq_ipc_open": "PP",
    "bnbq_ipc_close": "P",
}
_KIND = {"i": C.c_int32, "l": C.c_int64, "u": C.c_uint64, "P": C.c_void_p, "p": C.c_void_p}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def exported_symbols() -> list[str]:
    return [*_SIGNATURES, "bnbq_error_string"]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python bitsandbytes-jax_b200/build.py`")
                L = C.CDLL(str(LIB_PATH))
                for name, sig in _SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.argtypes = [_KIND[c] for c in sig]
                    fn.restype = C.c_int32
                L.bnbq_quantize_nf4_dq_workspace_bytes.restype = C.c_int64
                L.bnbq_error_string.argtypes = [C.c_int32]
                L.bnbq_error_string.restype = C.c_char_p
                _lib = L
    return _lib


class BnbqError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = f"{what}: {lib().bnbq_error_string(status).decode()} (status {status})"
    if status in (ERR_INVALID, ERR_TOO_LARGE):
        raise ValueError(msg)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise BnbqError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError(f"expected a CUDA tensor, got one on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("no CUDA tensor given")
    return dev


def aligned(t: torch.Tensor, a: int = 16) -> torch.Tensor:
    """Contiguous and `a`-byte aligned (slices may start mid-allocation)."""
    t = t.contiguous()
    if t.numel() and t.data_ptr() % a:
        t = t.clone()
    return t


def wait_timeouts() -> int:
    """Device-side bounded waits that expired so far (0 in normal operation)."""
    n = C.c_uint32(0)
    check(lib().bnbq_wait_timeouts(C.byref(n)), "bnbq_wait_timeouts")
    return int(n.value)


def set_wait_limit_ns(ns: int) -> None:
    """Time limit of the current device's bounded device-side waits (a test
    hook: shorten it to make a wait expire on purpose); 0 restores the defaults."""
    check(lib().bnbq_set_wait_limit_ns(int(ns)), "bnbq_set_wait_limit_ns")


_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """A device buffer of at least `nbytes` for the kernels that split K
    across SMs (their partial sums; no initial contents needed), one per
    (device, stream) so that the calls sharing one are ordered. Allocated on
    first use and kept for the life of the process."""
    key = (device.index, stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def gemv_workspace_bytes(m: int, k: int, n_rows: int) -> int:
    n = C.c_int64(0)
    check(lib().bnbq_gemv_workspace_bytes(m, k, n_rows, C.byref(n)), "bnbq_gemv_workspace_bytes")
    return int(n.value)


def gemv8_workspace_bytes(m: int, k: int, n_rows: int) -> int:
    n = C.c_int64(0)
    check(lib().bnbq_gemv_blockwise_workspace_bytes(m, k, n_rows, C.byref(n)), "bnbq_gemv_blockwise_workspace_bytes")
    return int(n.value)


def gemv_t_workspace_bytes(m: int, k: int, n_rows: int) -> int:
    n = C.c_int64(0)
    check(lib().bnbq_gemv_t_nf4_workspace_bytes(m, k, n_rows, C.byref(n)), "bnbq_gemv_t_nf4_workspace_bytes")
    return int(n.value)


ROUTE_TABLE_GEMV, ROUTE_GEMV, ROUTE_GEMM = 1, 2, 3
POLICY_AUTO, POLICY_TABLE, POLICY_NO_TABLE = 0, 1, 2


def set_gemv_policy(policy: int) -> None:
    """Which GEMV the workspace entry points use where both apply (POLICY_*)."""
    check(lib().bnbq_set_gemv_policy(int(policy)), "bnbq_set_gemv_policy")


def gemv_route(m: int, k: int, n_rows: int, blocksize: int, absmax_q_ptr, blocksize2: int, ws_ptr, ws_bytes: int) -> int:
    """Which kernels bnbq_matmul_nf4_ws runs for such a call (ROUTE_*)."""
    r = C.c_int32(0)
    check(lib().bnbq_gemv_route(m, k, n_rows, blocksize, absmax_q_ptr, blocksize2, ws_ptr, ws_bytes, C.byref(r)),
          "bnbq_gemv_route")
    return int(r.value)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
