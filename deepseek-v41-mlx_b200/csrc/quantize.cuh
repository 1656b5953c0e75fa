// quantize.cuh -- MLX affine group quantization on the GPU (the mx.quantize step of
// deepseek_v41_mlx/convert.py:156-175 quantize_tree and :178-196 quantize_engram_table).
//
// MLX is not in the reference tree (mlx>=0.32.0).  Its published affine scheme, as restated
// here (parity unpinned: no reference test checks these numerics), per group of `group`
// consecutive values of a row, in fp32 (bf16 inputs widened exactly):
//   n      = 2^bits - 1
//   scale  = max((w_max - w_min) / n, 1e-7)
//   edge   = w_min if |w_min| > |w_max| else w_max;  scale = -scale when edge is w_max
//   q0     = round(edge / scale)                      (round half away from zero)
//   q0 != 0: scale = edge / q0, bias = edge;   q0 == 0: bias = 0
//   code   = clamp(round((w - bias) / scale), 0, n)   (with the fp32 scale and bias)
// scale and bias are stored in the input's dtype (bf16 rounded to nearest even); codes are
// packed little-endian into uint32 words (element j of a row at bit bits*j), the layout that
// dsv41_dequant_affine and dsv41_gemv_affine read.
#pragma once
#include "common.cuh"

namespace dsv41 {

template <typename T> __device__ __forceinline__ float qa_load(const T *p);
template <> __device__ __forceinline__ float qa_load<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float qa_load<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void qa_store(T *p, float v);
template <> __device__ __forceinline__ void qa_store<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void qa_store<__nv_bfloat16>(__nv_bfloat16 *p, float v) {
  *p = __float2bfloat16_rn(v);
}

// One warp per group; lane l holds the V = group / 32 values l*V .. l*V + V - 1 of its group
// (V * bits divides 32, so a lane's codes never straddle a word); the lanes sharing a word
// OR their pieces together and the first of them stores it.
template <typename T, int V>
__global__ void __launch_bounds__(256) k_quantize_affine(const T *__restrict__ w, int64_t rows,
                                                         int64_t cols, int bits,
                                                         uint32_t *__restrict__ wq,
                                                         T *__restrict__ scales,
                                                         T *__restrict__ biases) {
  constexpr int G = 32 * V;
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t gpr = cols / G;
  if (gw >= rows * gpr) return;
  const int64_t row = gw / gpr, g = gw % gpr;
  const T *src = w + row * cols + g * G + lane * V;
  float x[V];
  float hi = -INFINITY, lo = INFINITY;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    x[i] = qa_load<T>(src + i);
    hi = fmaxf(hi, x[i]);
    lo = fminf(lo, x[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
  }
  const float nb = float((1 << bits) - 1);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), nb), 1e-7f);
  const bool side = fabsf(lo) > fabsf(hi);
  scale = side ? scale : -scale;
  const float edge = side ? lo : hi;
  const float q0 = roundf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  uint32_t piece = 0;
  const int e0 = lane * V;
  const int off = (e0 * bits) & 31;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float q = fminf(fmaxf(roundf(__fdiv_rn(__fsub_rn(x[i], bias), scale)), 0.0f), nb);
    piece |= uint32_t(q) << (off + i * bits);
  }
  const int lpw = 32 / (V * bits);                 // lanes sharing a word (a power of two)
  for (int o = 1; o < lpw; o <<= 1) piece |= __shfl_xor_sync(0xffffffffu, piece, o);
  const int64_t wpr = cols * bits / 32;            // words a row
  if (lane % lpw == 0) wq[row * wpr + g * (G * bits / 32) + (e0 * bits) / 32] = piece;
  if (lane == 0) {
    qa_store<T>(scales + row * gpr + g, scale);
    qa_store<T>(biases + row * gpr + g, bias);
  }
}

}  // namespace dsv41
