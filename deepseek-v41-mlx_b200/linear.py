"""Quantized linear layers with the weight decode fused into the product.

``linear_fp8`` / ``linear_fp4`` are the a16 form of upstream ``linear()``
(docs/reference/model.py:181-207) on the release's fp8 32x32 / fp4 weights;
``linear_affine`` is ``mx.quantized_matmul`` behind ``nn.QuantizedLinear``
(deepseek_v41_mlx/load.py:124-131) for the MLX affine 4/8-bit group-64 layout.
Inputs are bf16 activations [..., K]; outputs are bf16 (default) or fp32.
Tokens are processed 32 at a time per weight pass (decode-time GEMV).
"""

from __future__ import annotations

from . import _lib as L

_WS = {}


def _ws(nbytes, device):
    key = (device.type, device.index)
    w = _WS.get(key)
    if w is None or w.numel() < nbytes:
        w = L.workspace(nbytes, device)
        _WS[key] = w
    return w


def _prep(x, out_dtype):
    t = L.torch()
    xt = L.cuda_tensor(x, "x")
    if xt.dtype != t.bfloat16:
        xt = xt.to(t.bfloat16)
    K = xt.shape[-1]
    xf = xt.reshape(-1, K)
    odt = out_dtype or t.bfloat16
    return xt, xf, K, odt


def linear_fp8(x, weight, scale, out_dtype=None):
    t = L.torch()
    xt, xf, K, odt = _prep(x, out_dtype)
    w = L.u8(L.cuda_tensor(weight, "weight"))
    s = L.u8(L.cuda_tensor(scale, "scale"))
    N = w.shape[0]
    if w.shape[1] != K or tuple(s.shape) != ((N + 31) // 32, (K + 31) // 32):
        raise ValueError("fp8 weight must be [N, K] with scale [ceil(N/32), ceil(K/32)]")
    M = xf.shape[0]
    y = t.empty((M, N), dtype=odt, device=xf.device)
    ws = _ws(L.load().dsv41_gemv_workspace_size(M, N, K), xf.device)
    L.call("dsv41_gemv_fp8_block", L.ptr(xf), M, K, L.ptr(w), L.ptr(s), N, L.dtype_code(odt),
           L.ptr(y), L.ptr(ws), ws.numel(), L.stream_of(xf))
    return y.reshape(tuple(xt.shape[:-1]) + (N,))


def linear_fp4(x, weight, scale, out_dtype=None):
    t = L.torch()
    xt, xf, K, odt = _prep(x, out_dtype)
    w = L.u8(L.cuda_tensor(weight, "weight"))
    s = L.u8(L.cuda_tensor(scale, "scale"))
    N = w.shape[0]
    if w.shape[1] * 2 != K or tuple(s.shape) != (N, K // 32):
        raise ValueError("fp4 weight must be [N, K/2] with scale [N, K/32]")
    M = xf.shape[0]
    y = t.empty((M, N), dtype=odt, device=xf.device)
    ws = _ws(L.load().dsv41_gemv_workspace_size(M, N, K), xf.device)
    L.call("dsv41_gemv_fp4", L.ptr(xf), M, K, L.ptr(w), L.ptr(s), N, L.dtype_code(odt), L.ptr(y),
           L.ptr(ws), ws.numel(), L.stream_of(xf))
    return y.reshape(tuple(xt.shape[:-1]) + (N,))


# Above this many activation rows the affine product runs on the tensor cores.
QMM_MIN_ROWS = 64


def linear_affine(x, wq, scales, biases, bits=4, group_size=64, out_dtype=None):
    t = L.torch()
    if group_size != 64:
        raise ValueError("linear_affine supports group_size 64")
    xt, xf, K, odt = _prep(x, out_dtype)
    w = L.cuda_tensor(wq, "wq")
    s = L.cuda_tensor(scales, "scales")
    b = L.cuda_tensor(biases, "biases")
    if s.dtype != t.bfloat16 or b.dtype != t.bfloat16:
        raise ValueError("scales and biases must be bfloat16")
    N = w.shape[0]
    if w.shape[1] * 32 // bits != K or tuple(s.shape) != (N, K // 64):
        raise ValueError("affine weight must be [N, K*bits/32] u32 with scales [N, K/64]")
    M = xf.shape[0]
    y = t.empty((M, N), dtype=odt, device=xf.device)
    if M > QMM_MIN_ROWS and N % 128 == 0 and bits in (4, 8):
        # prefill sizes: tensor-core GEMM on weights dequantized to bf16 (MLX's qmm form)
        L.call("dsv41_qmm_affine", L.ptr(xf), M, K, L.ptr(w), L.ptr(s), L.ptr(b), bits, N,
               L.dtype_code(odt), L.ptr(y), L.stream_of(xf))
    else:
        ws = _ws(L.load().dsv41_gemv_workspace_size(M, N, K), xf.device)
        L.call("dsv41_gemv_affine", L.ptr(xf), M, K, L.ptr(w), L.ptr(s), L.ptr(b), bits, N,
               L.dtype_code(odt), L.ptr(y), L.ptr(ws), ws.numel(), L.stream_of(xf))
    return y.reshape(tuple(xt.shape[:-1]) + (N,))


class FP8Linear:
    """Release fp8 linear: weight e4m3 [out, in], scale ue8m0 [ceil(out/32), ceil(in/32)]."""

    def __init__(self, weight, scale):
        self.weight, self.scale = weight, scale

    def __call__(self, x, out_dtype=None):
        return linear_fp8(x, self.weight, self.scale, out_dtype)


class FP4Linear:
    """Release fp4 linear: weight e2m1 pairs [out, in/2], scale ue8m0 [out, in/32]."""

    def __init__(self, weight, scale):
        self.weight, self.scale = weight, scale

    def __call__(self, x, out_dtype=None):
        return linear_fp4(x, self.weight, self.scale, out_dtype)


class QuantizedLinear:
    """MLX nn.QuantizedLinear layout (weight u32, scales, biases bf16)."""

    def __init__(self, weight, scales, biases, group_size=64, bits=4):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits

    def __call__(self, x, out_dtype=None):
        return linear_affine(x, self.weight, self.scales, self.biases, self.bits,
                             self.group_size, out_dtype)
