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

// The group's parameters from its range (the steps of the header comment).
__device__ __forceinline__ void qa_params(float hi, float lo, float nb, float &scale,
                                          float &bias) {
  scale = fmaxf(__fdiv_rn(__fsub_rn(hi, lo), nb), 1e-7f);
  const bool side = fabsf(lo) > fabsf(hi);
  scale = side ? scale : -scale;
  const float edge = side ? lo : hi;
  const float q0 = roundf(__fdiv_rn(edge, scale));
  bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
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
  float scale, bias;
  qa_params(hi, lo, nb, scale, bias);
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

// round(RN(a / s)) (a correctly rounded divide, then round half away from zero) from the
// product y = RN(a * rs), rs = RN(1 / s): y is within 1.2e-7 |y| of a / s and RN(a / s) within
// 6e-8 |y| of it, so when y lies farther than m = 4e-7 |y| + 1e-6 (which also covers the
// error of computing y - floor(y)) from every half-integer, both round to the same integer;
// otherwise -- near a half-integer, or |y| above about 2^20 where m reaches 0.5 -- the divide
// itself decides.
__device__ __forceinline__ float qa_round_div(float a, float s, float rs) {
  const float y = __fmul_rn(a, rs);
  const float d = fabsf(__fsub_rn(__fsub_rn(y, floorf(y)), 0.5f));
  const float m = __fmaf_rn(fabsf(y), 4e-7f, 1e-6f);
  return d > m ? roundf(y) : roundf(__fdiv_rn(a, s));
}

// 16 bytes of T as floats (8 bf16 or 4 fp32)
__device__ __forceinline__ void qa_load16(const __nv_bfloat16 *p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4 *>(p);
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void qa_load16(const float *p, float (&f)[4]) {
  const float4 v = *reinterpret_cast<const float4 *>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}

// One thread per group: 16-byte loads of the group (all of a thread's loads in flight at
// once), its range, then a second read of the same bytes (from L1) to quantize, and the
// group's G * BITS / 32 words stored together.  Needs w and every row 16-byte aligned and wq
// 16-byte aligned (the host checks; otherwise k_quantize_affine runs).  The same results as
// k_quantize_affine: the per-element divide is qa_round_div, which rounds identically.
template <typename T, int G, int BITS>
__global__ void __launch_bounds__(256) k_quantize_affine_t(const T *__restrict__ w, int64_t rows,
                                                           int64_t cols,
                                                           uint32_t *__restrict__ wq,
                                                           T *__restrict__ scales,
                                                           T *__restrict__ biases) {
  constexpr int EPV = 16 / int(sizeof(T));         // elements a 16-byte load
  constexpr int NV = G / EPV;
  constexpr int WORDS = G * BITS / 32, PER = 32 / BITS;
  const int64_t gpr = cols / G;
  const int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gi >= rows * gpr) return;
  const int64_t row = gi / gpr, g = gi % gpr;
  const T *src = w + row * cols + g * G;
  float hi = -INFINITY, lo = INFINITY;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float f[EPV];
    qa_load16(src + k * EPV, f);
#pragma unroll
    for (int j = 0; j < EPV; ++j) {
      hi = fmaxf(hi, f[j]);
      lo = fminf(lo, f[j]);
    }
  }
  const float nb = float((1 << BITS) - 1);
  float scale, bias;
  qa_params(hi, lo, nb, scale, bias);
  const float rs = __frcp_rn(scale);
  uint32_t word[WORDS];
#pragma unroll
  for (int i = 0; i < WORDS; ++i) word[i] = 0u;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    float f[EPV];
    qa_load16(src + k * EPV, f);
#pragma unroll
    for (int j = 0; j < EPV; ++j) {
      const int e = k * EPV + j;
      const float q = fminf(fmaxf(qa_round_div(__fsub_rn(f[j], bias), scale, rs), 0.0f), nb);
      word[e / PER] |= uint32_t(q) << ((e % PER) * BITS);
    }
  }
  uint32_t *dst = wq + row * (cols * BITS / 32) + g * WORDS;
  if constexpr (WORDS % 4 == 0) {
#pragma unroll
    for (int i = 0; i < WORDS; i += 4)
      *reinterpret_cast<uint4 *>(dst + i) = make_uint4(word[i], word[i + 1], word[i + 2], word[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < WORDS; i += 2)
      *reinterpret_cast<uint2 *>(dst + i) = make_uint2(word[i], word[i + 1]);
  }
  qa_store<T>(scales + row * gpr + g, scale);
  qa_store<T>(biases + row * gpr + g, bias);
}

}  // namespace dsv41
