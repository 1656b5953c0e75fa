"""ctypes binding of libdsv41q.so (include/dsv41q.h).

The library is loaded on first use.  Loading needs no GPU; every compute call
checks that its tensors live on a CUDA device and maps a non-zero status to
``DSV41Error`` (a ``RuntimeError``) or ``ValueError`` for shape / dtype /
alignment problems, as the reference raises ValueError on layout mismatches
(deepseek_v41_mlx/engram.py:140-152).
"""

from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libdsv41q.so"
_lock = threading.Lock()
_lib = None

OK, BAD_SHAPE, BAD_DTYPE, MISALIGNED, CUDA_ERR, NCCL_ERR, TIMEOUT, BAD_ARG, UNSUPPORTED, \
    WORKSPACE = range(10)
F32, BF16, F16, U8 = 0, 1, 2, 3
SCORE_FUNCS = {"sqrtsoftplus": 0, "sigmoid": 1, "softmax": 2}
MOE_ROUND_BF16, MOE_NO_SHARED, MOE_SHARED_ONLY, MOE_PACKED_SCALES, MOE_NO_ROWPAIR = 1, 2, 4, 8, 16


class DSV41Error(RuntimeError):
    """A CUDA-side failure reported by libdsv41q."""


def lib_path() -> str:
    return os.path.join(_HERE, _LIB_NAME)


class MoeWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "gate_w", "gate_bias", "w1", "s1", "w3", "s3", "w2", "s2",
        "sw1", "ss1", "sw3", "ss3", "sw2", "ss2")]


class MoeConfig(C.Structure):
    _fields_ = [("dim", C.c_int64), ("inter", C.c_int64), ("n_experts", C.c_int64),
                ("topk", C.c_int), ("score_func", C.c_int), ("gate_temp", C.c_float),
                ("norm_topk_prob", C.c_int), ("route_scale", C.c_float),
                ("swiglu_limit", C.c_float), ("flags", C.c_int)]


_P, _I64, _I, _F, _SZ, _U32P = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t, \
    C.POINTER(C.c_uint32)

# name -> (restype, argtypes); must list every function of include/dsv41q.h
PROTOTYPES = {
    "dsv41_get_last_error": (C.c_char_p, []),
    "dsv41_abi_version": (_I, []),
    "dsv41_device_status": (_I, [_P, _U32P]),
    "dsv41_set_wait_limit_ns": (_I, [C.c_uint64]),
    "dsv41_prof_enable": (_I, [_I]),
    "dsv41_prof_reset": (_I, []),
    "dsv41_prof_report": (_I, [C.c_char_p, _SZ]),
    "dsv41_prof_select": (_I, [C.c_char_p]),
    "dsv41_prof_launches": (C.c_longlong, []),
    "dsv41_e8m0_to_float": (_I, [_P, _I64, _P, _P]),
    "dsv41_dequant_fp8_block": (_I, [_P, _P, _I64, _I64, _I, _P, _P]),
    "dsv41_unpack_fp4": (_I, [_P, _I64, _I64, _P, _P]),
    "dsv41_dequant_fp4": (_I, [_P, _P, _I64, _I64, _I, _P, _P]),
    "dsv41_dequant_fp8_rows": (_I, [_P, _P, _I64, _I64, _I64, _P, _P]),
    "dsv41_dequant_affine": (_I, [_P, _P, _P, _I, _I64, _I64, _I, _I, _I, _P, _P]),
    "dsv41_quantize_affine": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "dsv41_act_quant_fp8": (_I, [_P, _I64, _I64, _I, _I, _P, _P, _I, _P, _P]),
    "dsv41_gemv_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "dsv41_gemv_fp8_block": (_I, [_P, _I64, _I64, _P, _P, _I64, _I, _P, _P, _SZ, _P]),
    "dsv41_gemv_fp8_block_noalloc": (_I, [_P, _I64, _I64, _P, _P, _I64, _I, _P, _P]),
    "dsv41_gemv_fp4": (_I, [_P, _I64, _I64, _P, _P, _I64, _I, _P, _P, _SZ, _P]),
    "dsv41_gemv_affine": (_I, [_P, _I64, _I64, _P, _P, _P, _I, _I64, _I, _P, _P, _SZ, _P]),
    "dsv41_moe_route_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "dsv41_moe_route": (_I, [_P, _I64, _I64, _P, _P, _I64, _I, _I, _F, _I, _F, _P, _P, _P, _SZ,
                             _P]),
    "dsv41_moe_decode_workspace_size": (_SZ, [C.POINTER(MoeConfig), _I64]),
    "dsv41_moe_decode_pack_size": (_SZ, [C.POINTER(MoeConfig)]),
    "dsv41_ep_create": (_I, [_I, _I, _I64, _I, _I64, C.POINTER(_P)]),
    "dsv41_ep_handle_bytes": (_SZ, []),
    "dsv41_ep_handle": (_I, [_P, _P]),
    "dsv41_ep_connect": (_I, [_P, _P]),
    "dsv41_ep_destroy": (_I, [_P]),
    "dsv41_ep_wait": (_I, [_P, _I, _P]),
    "dsv41_moe_ep_decode_workspace_size": (_SZ, [C.POINTER(MoeConfig), _P, _I64]),
    "dsv41_moe_ep_decode": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _P, _I64, _I,
                                 _P, _P, _P, _P, _SZ, _P]),
    "dsv41_moe_decode_pack": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _SZ, _P]),
    "dsv41_moe_experts": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _I64, _P, _P, _P,
                               _SZ, _P]),
    "dsv41_moe_decode": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _I64, _I, _P, _P,
                              _P, _P, _SZ, _P]),
    "dsv41_qmm_affine": (_I, [_P, _I64, _I64, _P, _P, _P, _I, _I64, _I, _P, _P]),
    "dsv41_fp8_gemm": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _I, _P]),
    "dsv41_fp4_gemm": (_I, [_P, _P, _P, _P, _I64, _I64, _I64, _I, _P, _I, _P]),
    "dsv41_moe_prefill_pack_size": (_SZ, [C.POINTER(MoeConfig)]),
    "dsv41_moe_prefill_pack": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _SZ, _P]),
    "dsv41_moe_prefill_workspace_size": (_SZ, [C.POINTER(MoeConfig), _I64, _I, _I]),
    "dsv41_moe_prefill": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _P, _I64, _P, _P,
                               _I, _P, _P, _SZ, _P]),
    "dsv41_moe_prefill_a16_workspace_size": (_SZ, [C.POINTER(MoeConfig), _I64, _I]),
    "dsv41_moe_prefill_a16": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _I64, _P,
                                   _P, _I, _P, _P, _SZ, _P]),
    "dsv41_moe_ep_row_bytes": (_SZ, [_I64]),
    "dsv41_moe_ep_pack_workspace_size": (_SZ, [C.POINTER(MoeConfig), _I64]),
    "dsv41_moe_ep_pack": (_I, [C.POINTER(MoeConfig), _P, _I64, _P, _P, _I, _P, _P, _P, _P, _SZ,
                               _P]),
    "dsv41_moe_ep_experts_workspace_size": (_SZ, [C.POINTER(MoeConfig), _I64, _I]),
    "dsv41_moe_ep_experts": (_I, [C.POINTER(MoeConfig), C.POINTER(MoeWeights), _P, _P, _I64, _P,
                                  _P, _SZ, _P]),
    "dsv41_moe_ep_combine": (_I, [_P, _P, _P, _P, _I64, _I, _I64, _I, _P, _P]),
    "dsv41_engram_hash": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _I, _I, _I,
                               _I64, _P, _P]),
    "dsv41_engram_lookup_sum": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P, _P, _I,
                                     _I, _I, _I, _I64, _P, _I64, _I64, _I64, _I64, _I, _P, _P]),
    "dsv41_engram_lookup_sum_peers": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P, _P, _P,
                                           _P, _I, _I, _I, _I, _I64, _P, _P, _I, _I64, _I64,
                                           _I64, _I64, _I, _P, _P]),
    "dsv41_engram_gather_rows": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I, _P, _P]),
    "dsv41_engram_gather_sum": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I, _I, _P, _P]),
    "dsv41_engram_row_bytes": (_SZ, [_I64, _I64]),
    "dsv41_engram_gate": (_I, [_P, _I, _P, _I, _P, _P, _P, _I64, _I, _I64, _F, _F, _P, _P]),
    "dsv41_ipc_export": (_I, [_P, _P, C.POINTER(_I64)]),
    "dsv41_ipc_import": (_I, [_P, C.POINTER(_P)]),
    "dsv41_ipc_close": (_I, [_P]),
    "dsv41_engram_gather_sum_peers": (_I, [_P, _P, _I, _I64, _I64, _I64, _I64, _P, _I64, _I, _I, _P,
                                           _P]),
    "dsv41_engram_pack_rows": (_I, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "dsv41_engram_sum_rows": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I, _I, _P, _P]),
    "dsv41_engram_dequant_rows": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I, _P, _P]),
}


def load():
    """Load libdsv41q.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            p = lib_path()
            if not os.path.exists(p):
                raise DSV41Error(f"{p} is missing: build it with "
                                 f"`python deepseek-v41-mlx_b200/build.py` (no CPU fallback)")
            lib = C.CDLL(p)
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().dsv41_get_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str):
    if status == OK:
        return
    msg = f"{what}: {last_error()} (status {status})"
    if status in (BAD_SHAPE, BAD_DTYPE, MISALIGNED, BAD_ARG, WORKSPACE):
        raise ValueError(msg)
    raise DSV41Error(msg)


def call(name: str, *args):
    check(getattr(load(), name)(*args), name)


# ---------------------------------------------------------------- torch glue --

def torch():
    import torch as _t
    return _t


def as_tensor(a):
    """DLPack-capable array -> torch tensor (no copy)."""
    t = torch()
    if isinstance(a, t.Tensor):
        return a
    if hasattr(a, "__dlpack__"):
        return t.from_dlpack(a)
    raise TypeError(f"expected a torch tensor or a DLPack array, got {type(a)!r}")


def cuda_tensor(a, name="array"):
    t = as_tensor(a)
    if not t.is_cuda:
        raise DSV41Error(f"{name} must be a CUDA tensor (this library has no CPU path)")
    return t.contiguous()


def ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def stream_of(t) -> int:
    return torch().cuda.current_stream(t.device).cuda_stream


def dtype_code(dt) -> int:
    t = torch()
    return {t.float32: F32, t.bfloat16: BF16, t.float16: F16, t.uint8: U8}[dt]


def u8(t):
    """Accept uint8 / int8 / float8 / float4x2 / e8m0 byte storage as uint8."""
    tt = torch()
    if t.dtype == tt.uint8:
        return t
    if t.element_size() == 1:
        return t.view(tt.uint8)
    raise ValueError(f"expected a 1-byte dtype, got {t.dtype}")


def prof_enable(on: bool = True):
    load().dsv41_prof_enable(1 if on else 0)
    load().dsv41_prof_reset()


def prof_select(names=None):
    """Time only the named kernels (an iterable of names; None = all of them)."""
    load().dsv41_prof_select(",".join(names).encode() if names else None)


def prof_launches() -> int:
    """Kernel launches counted since prof_enable, timed or not."""
    return int(load().dsv41_prof_launches())


def prof_report() -> dict:
    """{kernel name: (launches, total_ms)} for launches since prof_enable."""
    buf = C.create_string_buffer(1 << 16)
    call("dsv41_prof_report", buf, len(buf))
    out = {}
    for line in buf.value.decode().splitlines():
        name, n, ms = line.split()
        out[name] = (int(n), float(ms))
    return out


def workspace(nbytes: int, device):
    t = torch()
    return t.empty(max(int(nbytes), 1), dtype=t.uint8, device=device)
