// dequant.cuh -- bit-exact release-format decode kernels.
//
// Mirrors deepseek_v41_mlx/dequant.py:33-79 (e8m0_to_float, dequant_fp8 with
// the ceil-cropped 32x32 scale grid, unpack_fp4 / dequant_fp4 with low nibble =
// even index and code 8 -> +0.0, dequant_fp8_rows) and the MLX affine group
// decode used by QuantizedEngramEmbedding (deepseek_v41_mlx/engram.py:219-223).
// Every value is an exact fp8/fp4 code times a power of two, so fp32 results
// are exact and bf16 results are exact roundings.
#pragma once
#include "common.cuh"

namespace dsv41 {

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__global__ void k_e8m0_to_float(const uint8_t *__restrict__ s, int64_t n, float *__restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = e8m0f(s[i]);
}

// decode 8 consecutive e4m3 codes (a u64) to 8 exact floats
__device__ __forceinline__ void e4m3x8_to_f32(uint64_t v, float (&f)[8]) {
  uint32_t h[4];
  e4m3x4_to_f16x4(uint32_t(v), h[0], h[1]);
  e4m3x4_to_f16x4(uint32_t(v >> 32), h[2], h[3]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p = h2f2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

// decode 8 consecutive e2m1 nibbles (a u32, low nibble first) to 8 floats; code 8
// gives -0 from the hardware conversion and is normalised to +0 by adding +0.
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t v, float (&f)[8]) {
  uint32_t h[4];
  e2m1x8_to_f16x8(v, h[0], h[1], h[2], h[3]);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p = h2f2(h[i]);
    f[2 * i] = __fadd_rn(p.x, 0.0f);
    f[2 * i + 1] = __fadd_rn(p.y, 0.0f);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T *dst, const float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = from_f32<T>(f[i]);
}

// fp8 e4m3 [rows, cols] * ue8m0 [ceil(rows/32), ceil(cols/32)]; chunk of 8 columns
// per thread when cols % 8 == 0, else one element per thread.
template <typename T, bool VEC>
__global__ void k_dequant_fp8_block(const uint8_t *__restrict__ w, const uint8_t *__restrict__ s,
                                    int64_t rows, int64_t cols, T *__restrict__ out) {
  const int64_t scols = (cols + 31) / 32;
  if (VEC) {
    const int64_t cpr = cols / 8, n = rows * cpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / cpr, c = (i % cpr) * 8;
      uint64_t v = *reinterpret_cast<const uint64_t *>(w + r * cols + c);
      float f[8];
      e4m3x8_to_f32(v, f);
      const float sc = e8m0f(s[(r / 32) * scols + c / 32]);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = __fmul_rn(f[j], sc);
      store8(out + r * cols + c, f);
    }
  } else {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / cols, c = i % cols;
      const uint8_t b = w[i];
      float2 p = h2f2(e4m3x2_to_f16x2(b));
      out[i] = from_f32<T>(__fmul_rn(p.x, e8m0f(s[(r / 32) * scols + c / 32])));
    }
  }
}

// fp4 e2m1 packed [rows, cols/2] (* ue8m0 [rows, ceil(cols/32)] when s != null)
template <typename T, bool VEC>
__global__ void k_dequant_fp4(const uint8_t *__restrict__ p, const uint8_t *__restrict__ s,
                              int64_t rows, int64_t cols, T *__restrict__ out) {
  const int64_t scols = (cols + 31) / 32, half = cols / 2;
  if (VEC) {
    const int64_t cpr = cols / 8, n = rows * cpr;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / cpr, c = (i % cpr) * 8;
      uint32_t v = *reinterpret_cast<const uint32_t *>(p + r * half + c / 2);
      float f[8];
      e2m1x8_to_f32(v, f);
      if (s) {
        const float sc = e8m0f(s[r * scols + c / 32]);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = __fadd_rn(__fmul_rn(f[j], sc), 0.0f);
      }
      store8(out + r * cols + c, f);
    }
  } else {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t r = i / cols, c = i % cols;
      const uint32_t b = p[r * half + c / 2];
      const uint32_t nib = (c & 1) ? (b >> 4) : (b & 0xF);
      uint32_t h0, h1, h2, h3;
      e2m1x8_to_f16x8(nib, h0, h1, h2, h3);
      float v = __fadd_rn(h2f2(h0).x, 0.0f);
      if (s) v = __fadd_rn(__fmul_rn(v, e8m0f(s[r * scols + c / 32])), 0.0f);
      out[i] = from_f32<T>(v);
    }
  }
}

// engram rows: e4m3 [rows, d] * ue8m0 [rows, d/block] -> f32
__global__ void k_dequant_fp8_rows(const uint8_t *__restrict__ w, const uint8_t *__restrict__ s,
                                   int64_t rows, int64_t d, int64_t block, float *__restrict__ out) {
  const int64_t n = rows * d, sb = d / block;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / d, c = i % d;
    float2 p = h2f2(e4m3x2_to_f16x2(w[i]));
    out[i] = __fmul_rn(p.x, e8m0f(s[r * sb + c / block]));
  }
}

template <int SB>  // 0 f32, 1 bf16, 2 f16
__device__ __forceinline__ float load_sb(const void *p, int64_t i) {
  if (SB == 0) return reinterpret_cast<const float *>(p)[i];
  if (SB == 1) return bf_bits2f(reinterpret_cast<const uint16_t *>(p)[i]);
  return __half2float(reinterpret_cast<const __half *>(p)[i]);
}

// MLX affine: q = bits-wide code at bit bits*j of the row's little-endian stream
template <typename T, int SB>
__global__ void k_dequant_affine(const uint32_t *__restrict__ wq, const void *__restrict__ sc,
                                 const void *__restrict__ bi, int64_t rows, int64_t cols, int bits,
                                 int group, T *__restrict__ out) {
  const int64_t wpr = cols * bits / 32, gpr = cols / group, n = rows * cols;
  const uint32_t mask = (bits == 32) ? 0xFFFFFFFFu : ((1u << bits) - 1u);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, j = i % cols;
    const int64_t bit = (int64_t)bits * j;
    const int64_t wi = bit >> 5;
    const int off = int(bit & 31);
    const uint32_t *row = wq + r * wpr;
    uint64_t v = row[wi];
    if (off + bits > 32) v |= uint64_t(row[wi + 1]) << 32;
    const float q = float(uint32_t(v >> off) & mask);
    const int64_t g = r * gpr + j / group;
    out[i] = from_f32<T>(__fmaf_rn(load_sb<SB>(sc, g), q, load_sb<SB>(bi, g)));
  }
}

static inline unsigned grid_for(int64_t n, int threads = 256) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = (int64_t)num_sms() * 16;
  if (b > cap) b = cap;
  return unsigned(b < 1 ? 1 : b);
}

}  // namespace dsv41
