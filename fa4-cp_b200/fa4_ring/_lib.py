"""ctypes binding of ``libfa4cp_b200.so`` (the C ABI declared in ``include/fa4cp_b200.h``).

There is no fallback: every public op of this package runs the CUDA library, and
loading fails loudly if the library has not been built
(``make -C fa4-cp_b200/csrc``).  Status codes map back to the exception types the
reference raises (AssertionError / ValueError for bad arguments,
``fa4_ring/config.py:24-33``, ``fa4_ring/merge.py:94``; RuntimeError for a missing or
failing backend, ``fa4_ring/fa4_backend.py:83-87``).
"""

import ctypes
import os
import threading

import torch

LIB_NAME = "libfa4cp_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_DEVICE = -4

DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_E4M3 = 0, 1, 2, 3
PATTERN_VARLEN, PATTERN_FRONT_KV, PATTERN_BACK_Q = 0, 1, 2

_TORCH_DTYPES = {
    torch.float16: DTYPE_F16,
    torch.bfloat16: DTYPE_BF16,
    torch.float32: DTYPE_F32,
    torch.float8_e4m3fn: DTYPE_E4M3,
}

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> argtypes (all return int32 status unless listed in _RESTYPE)
_SIGNATURES = {
    "fa4cp_version": [],
    "fa4cp_last_error": [],
    "fa4cp_device_status": [ctypes.POINTER(_i32), _i32],
    "fa4cp_selftest_wait_expiry": [_vp, _vp, _vp, _vp, _vp, _vp, _i32, ctypes.POINTER(_i32), _vp],
    "fa4cp_attn_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i64, _i64, _i32, _i32,
                       _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _i32, _vp],
    "fa4cp_attn_fwd_kv8": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i64, _i64, _i32,
                           _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _vp, _i64, _vp],
    "fa4cp_attn_fwd_kv8_noalloc": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i64, _i64,
                                   _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _vp],
    "fa4cp_attn_kv8_workspace_bytes": [_i64, _i32, _i32],
    "fa4cp_attn_fwd_paged": [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _i32,
                             _i64, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp],
    "fa4cp_dequant_e4m3": [_vp, _vp, _vp, _i64, _i32, _i32, _vp],
    "fa4cp_quantize_e4m3": [_vp, _i32, _i64, _vp, _vp, _vp],
    "fa4cp_merge_state_inplace": [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp],
    "fa4cp_merge_states": [ctypes.POINTER(_vp), ctypes.POINTER(_vp), _i32, _vp, _vp, _i64, _i32,
                           _i32, _i32, _vp],
    "fa4cp_fill_f32": [_vp, _i64, _f32, _vp],
    "fa4cp_zigzag_shard": [_vp, _vp, _vp, _i32, _i64, _i32, _i32, _i64, _vp],
    "fa4cp_zigzag_unshard": [ctypes.POINTER(_vp), _vp, _vp, _i32, _i64, _i32, _i64, _vp],
    "fa4cp_half_index": [_vp, _i32, _i64, _i32, _vp, _vp],
    "fa4cp_local_cu": [_vp, _i32, _i32, _vp, _vp],
    "fa4cp_gdn_cp_indices": [_vp, _i32, _i32, _i32, _i64, _vp, _vp, _vp],
    "fa4cp_ring_ipc_alloc": [_i64, _i64, _vp],
    "fa4cp_ring_ipc_open": [_i64, _vp, _vp],
    "fa4cp_ring_ipc_close": [_i64],
    "fa4cp_ring_ce_plan": [_i32, _i32, _i64, _i32, _vp, _i32],
    "fa4cp_ring_ce_direct_plan": [_i32, _i32, _i64, _i32, _vp, _i32],
    "fa4cp_ring_set_direct": [_i64, _i32],
    "fa4cp_ring_ipc_open_all": [_i64, _vp],
    "fa4cp_ring_attn_fused": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i64,
                              _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _i32, _i32, _vp,
                              ctypes.c_uint32, _vp],
    "fa4cp_ring_attn_fused_mixed": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _i32,
                                    _i64, _i32, _i32, _i32, _f32, _vp, _vp, _i32, _i32, _vp,
                                    ctypes.c_uint32, _vp],
    "fa4cp_ring_attn_fused_remote": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _i32,
                                     _i64, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _vp,
                                     ctypes.c_uint32, _vp],
    "fa4cp_ring_unique_id": [_vp],
    "fa4cp_ring_comm_init": [_vp, _i32, _i32, ctypes.POINTER(_i64)],
    "fa4cp_ring_comm_destroy": [_i64],
    "fa4cp_ring_set_sm_reserve": [_i64, _i32],
    "fa4cp_ring_set_fused": [_i64, _i32],
    "fa4cp_ring_set_wait_timeout_ms": [_i32],
    "fa4cp_ring_timing": [_i64, _i32],
    "fa4cp_ring_timeline": [_i64, _vp, _i32, _vp, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32)],
    "fa4cp_ring_timing_read": [_i64, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i32)],
    "fa4cp_ring_attn_fwd": [_i64, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i32, _i32, _i64, _i32,
                            _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp, _i64, _vp],
    "fa4cp_attn_bwd_preprocess": [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp],
    "fa4cp_attn_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i64,
                       _i64, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp],
    "fa4cp_convert_f32": [_vp, _vp, _i64, _i32, _vp],
    "fa4cp_add_f32": [_vp, _vp, _i64, _vp],
}
_RESTYPE = {"fa4cp_last_error": ctypes.c_char_p, "fa4cp_attn_kv8_workspace_bytes": _i64}

EXPORTED = tuple(_SIGNATURES)


def load():
    """Load the CUDA library once; raise RuntimeError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"fa4_ring B200 backend not built: {LIB_NAME} is missing next to "
                    f"{os.path.dirname(LIB_PATH)}; build it with `make -C fa4-cp_b200/csrc` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPE.get(name, ctypes.c_int32)
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().fa4cp_last_error()
    return msg.decode() if msg else ""


# Number of kernel launches made through this binding (successful calls of the
# launching entry points), for the benchmark's launch count.
launch_count = 0


def count_launches(n: int = 1) -> None:
    global launch_count
    launch_count += n


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == ERR_INVALID:
        raise ValueError(msg)
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def device_status(clear: bool = True) -> int:
    """Synchronise and return (and by default clear) the device status word."""
    st = _i32(0)
    check(load().fa4cp_device_status(ctypes.byref(st), 1 if clear else 0), "device_status")
    return int(st.value)


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _TORCH_DTYPES[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(
                "fa4_ring (B200) runs on CUDA tensors only; got "
                f"{'a CPU tensor' if isinstance(t, torch.Tensor) else type(t).__name__} "
                "(there is no CPU fallback)")


def ptr_array(tensors):
    arr = (_vp * len(tensors))()
    for i, t in enumerate(tensors):
        arr[i] = t.data_ptr()
    return arr
