"""ctypes binding of libfkb200.so, the C ABI declared in include/fkb200.h.

The library is loaded on first use.  If it has not been built, every op raises
RuntimeError: there is no CPU fallback for any op in this package.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libfkb200.so"

FK_F32, FK_F16, FK_BF16 = 0, 1, 2
_DTYPE_CODES = {torch.float32: FK_F32, torch.float16: FK_F16, torch.bfloat16: FK_BF16}

_vp, _i64, _i32, _f32, _sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> argtypes (restype is int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "fk_version": [],
    "fk_status_string": [_i32],
    "fk_last_error": [],
    "fk_swiglu_fwd": [_vp, _vp, _vp, _i64, _i32, _vp],
    "fk_swiglu_bwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _vp],
    "fk_rmsnorm_fwd": [_vp, _i64, _vp, _i32, _vp, _i64, _vp, _i64, _i64, _f32, _i32, _vp],
    "fk_rmsnorm_bwd_workspace_size": [_i64, _i64, C.POINTER(_sz)],
    "fk_rmsnorm_bwd": [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp, _sz, _i64, _i64, _i32, _vp],
    "fk_rmsnorm_bwd_noalloc": [_vp, _vp, _vp, _i32, _vp, _vp, _vp, _i64, _i64, _i32, _vp],
    "fk_router_fwd": [_vp, _i64, _i32, _i64, _i32, _i32, _vp, _vp, _vp],
    "fk_router_bwd": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp],
    "fk_ce_fwd": [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _f32, _i32, _vp, _vp, _vp, _vp,
                  _vp],
    "fk_ce_bwd_scale": [_vp, _i64, _i64, _i64, _vp, _i32, _vp],
    "fk_moe_capacity": [_i64, _i32, _i32, C.POINTER(_i64), C.POINTER(_sz)],
    "fk_moe_route_meta": [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64,
                          _vp, _sz, _vp, _vp],
    "fk_moe_gather": [_vp, _i32, _vp, _i32, _vp, _i64, _vp, _i32, _vp],
    "fk_moe_gather_by_token": [_vp, _i32, _vp, _i64, _i32, _vp, _vp, _i64, _vp, _i32, _vp],
    "fk_moe_combine": [_vp, _i32, _vp, _vp, _i64, _i32, _vp, _i32, _vp],
    "fk_moe_combine_bwd": [_vp, _vp, _i32, _vp, _vp, _i32, _vp, _i64, _vp, _vp, _i32, _vp],
    "fk_moe_gemm_up": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _vp],
    "fk_moe_gemm_down": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _vp],
    "fk_moe_gemm_down_dgrad": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _vp,
                               _vp],
    "fk_moe_gemm_up_dgrad": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _vp],
    "fk_moe_gemm_wgrad": [_vp, _i32, _vp, _i32, _i64, _vp, _i32, _vp, _i32, _vp, _vp],
    "fk_moe_gemm_up_weighted": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                _i32, _vp, _vp],
    "fk_moe_gemm_down_dgrad_weighted": [_vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _i32, _vp, _vp],
    "fk_moe_dw_from_parts": [_vp, _i32, _vp, _vp, _i64, _vp, _vp],
    "fk_tf32_split": [_vp, _i64, _vp, _vp, _vp],
    "fk_moe_gemm_up_typed": [_vp, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp,
                             _i32, _vp, _vp],
    "fk_moe_gemm_down_typed": [_vp, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _i32,
                               _vp, _vp],
    "fk_moe_gemm_down_dgrad_typed": [_vp, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp,
                                     _vp, _i32, _vp, _vp],
    "fk_moe_gemm_up_dgrad_typed": [_vp, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp,
                                   _i32, _vp, _vp],
    "fk_moe_gemm_wgrad_typed": [_vp, _vp, _i32, _vp, _vp, _i32, _i64, _vp, _i32, _vp, _i32, _vp,
                                _vp],
    "fk_moe_route_meta_skip": [_vp, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                               _i64, _vp, _sz, _vp, _vp],
    "fk_ep_plan_workspace_size": [_i64, _i32, C.POINTER(_sz)],
    "fk_ep_plan": [_vp, _vp, _i64, _i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                   _vp, _vp],
    "fk_ep_pack": [_vp, _i32, _vp, _i64, _vp, _i32, _vp],
    "fk_ep_unpack_sum": [_vp, _i32, _vp, _i64, _i32, _vp, _i32, _vp],
    "fk_ep_unpack_dw": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp],
    "fk_ipc_alloc": [_sz, C.POINTER(_vp), _vp],
    "fk_ipc_open": [_vp, C.POINTER(_vp)],
    "fk_ipc_close": [_vp],
    "fk_ipc_free": [_vp],
    "fk_ep_peer_put_rows": [_vp, _i32, _vp, _i64, _i32, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp,
                            _i32, _vp, _i32, _vp],
    "fk_ep_peer_combine_put": [_vp, _i32, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                               _i32, _vp, _i32, _vp],
    "fk_ep_peer_wait": [_vp, _i32, _i32, _vp, _i32, _vp, _vp],
    "fk_bitonic_sort_i32": [_vp, _i64, _i32, _i64, _vp, _i64, _vp],
    "fk_bitonic_sort_bounded_i32": [_vp, _i64, _i32, _i64, _i32, _vp, _vp],
    "fk_bitonic_merge_topk_i32": [_vp, _vp, _i64, _i32, _vp, _vp],
}
_RESTYPES = {"fk_status_string": C.c_char_p, "fk_last_error": C.c_char_p}

_lib = None
_lock = threading.Lock()


def load() -> C.CDLL:
    """Load libfkb200.so (once) and attach the declared signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is not built; run `python -m fusedkernels_b200._build` "
                    "(fusedkernels_b200 has no CPU fallback)")
            lib = C.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = lib
    return _lib


def check(status: int, name: str) -> None:
    if status != 0:
        lib = load()
        msg = lib.fk_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({lib.fk_status_string(status).decode()}): {msg}")


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise RuntimeError on failure."""
    check(getattr(load(), name)(*args), name)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16")


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_ws_cache: dict = {}


def rmsnorm_bwd_workspace_bytes(rows: int, cols: int, device: torch.device) -> int:
    key = (rows, cols, device.index)
    v = _ws_cache.get(key)
    if v is None:
        out = C.c_size_t(0)
        with torch.cuda.device(device):
            check(load().fk_rmsnorm_bwd_workspace_size(rows, cols, C.byref(out)),
                  "fk_rmsnorm_bwd_workspace_size")
        v = _ws_cache[key] = out.value
    return v


def ep_plan_workspace_bytes(n_tokens: int, n_ranks: int) -> int:
    out = C.c_size_t(0)
    check(load().fk_ep_plan_workspace_size(n_tokens, n_ranks, C.byref(out)),
          "fk_ep_plan_workspace_size")
    return out.value


_cap_cache: dict = {}


def moe_capacity(n_tokens: int, k: int, n_experts: int) -> tuple[int, int]:
    """(max sorted rows, metadata workspace bytes) for a routing of this size."""
    key = (n_tokens, k, n_experts)
    v = _cap_cache.get(key)
    if v is None:
        rows = C.c_int64(0)
        ws = C.c_size_t(0)
        check(load().fk_moe_capacity(n_tokens, k, n_experts, C.byref(rows), C.byref(ws)),
              "fk_moe_capacity")
        v = _cap_cache[key] = (rows.value, ws.value)
    return v


def num_sms(device: torch.device | None = None) -> int:
    """Streaming multiprocessors of the current (or given) CUDA device: the grid of the
    persistent kernels, one CTA per SM."""
    dev = torch.cuda.current_device() if device is None else device
    return torch.cuda.get_device_properties(dev).multi_processor_count
