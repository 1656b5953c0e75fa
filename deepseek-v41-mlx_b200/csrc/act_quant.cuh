// act_quant.cuh -- upstream block-wise fp8 activation quantization (a12).
//
// Semantics of docs/reference/kernel.py:40-124 (act_quant_kernel) as pinned by
// the reference's CPU transcription tests/kernel_stub.py:26-63:
//   amax = max(|x| over the block, 1e-4)
//   s    = 2^ceil(log2(amax * f32(1/448)))   (round_scale; fast_round_scale via IEEE bits)
//        = amax / 448                        (otherwise)
//   q    = e4m3_rn(clamp(x / s, -448, 448))
// One warp per (row, block); block is 32, 64 or 128 along K.
#pragma once
#include "common.cuh"

namespace dsv41 {

__device__ __forceinline__ float pow2_ceil_log2(float r) {
  const uint32_t b = __float_as_uint(r);
  const int e = int((b >> 23) & 0xFF) - 127 + ((b & 0x7FFFFF) != 0 ? 1 : 0);
  return __uint_as_float(uint32_t(e + 127) << 23);
}

__device__ __forceinline__ uint8_t f32_to_e4m3_sat(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return uint8_t(r & 0xFF);
}

template <int PER_LANE>
__global__ void k_act_quant(const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K,
                            int round_scale, uint8_t *__restrict__ q, void *__restrict__ s,
                            int s_u8, __nv_bfloat16 *__restrict__ deq) {
  constexpr int BLOCK = 32 * PER_LANE;
  const int64_t nblk = K / BLOCK;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M * nblk) return;
  const int64_t m = warp / nblk, kb = warp % nblk;
  const int64_t base = m * K + kb * BLOCK + lane * PER_LANE;
  float v[PER_LANE];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    v[i] = __bfloat162float(x[base + i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-4f);
  const float sc = round_scale ? pow2_ceil_log2(__fmul_rn(amax, 1.0f / 448.0f))
                               : __fdiv_rn(amax, 448.0f);
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const float r = __fdiv_rn(v[i], sc);
    const float y = isnan(r) ? r : fminf(fmaxf(r, -448.0f), 448.0f);  // torch clamp keeps NaN
    const uint8_t code = f32_to_e4m3_sat(y);
    q[base + i] = code;
    if (deq) {
      const float back = h2f2(e4m3x2_to_f16x2(code)).x;
      deq[base + i] = __float2bfloat16_rn(__fmul_rn(back, sc));
    }
  }
  if (lane == 0) {
    if (s_u8)
      reinterpret_cast<uint8_t *>(s)[m * nblk + kb] = uint8_t((__float_as_uint(sc) >> 23) & 0xFF);
    else
      reinterpret_cast<float *>(s)[m * nblk + kb] = sc;
  }
}

// Vectorized form of k_act_quant (same arithmetic): 8 elements per thread from one 16-byte
// load; a block of 8*G elements is G adjacent lanes combining their amax by shuffles.
// When s_atoms is set (G == 4, ue8m0 bytes) the scales are also written as tcgen05.cp atoms
// of 224-row tiles (row m -> tile m / 224), the layout the block-scaled GEMM bulk-copies.
template <int G>
__global__ void k_act_quant_v8(const __nv_bfloat16 *__restrict__ x, int64_t M, int64_t K,
                               int round_scale, uint8_t *__restrict__ q, void *__restrict__ s,
                               int s_u8, __nv_bfloat16 *__restrict__ deq,
                               uint8_t *__restrict__ s_atoms, int tile_rows) {
  const int64_t nthr = M * (K / 8);
  const int64_t tid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if ((tid & ~int64_t(31)) >= nthr) return;   // whole warps only: the shuffles below
  const bool valid = tid < nthr;
  float v[8];
  float amax = 0.0f;
  if (valid) {
    const uint4 raw = *reinterpret_cast<const uint4 *>(x + tid * 8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bf_bits2f(uint16_t(w[i] & 0xFFFF));
      v[2 * i + 1] = bf_bits2f(uint16_t(w[i] >> 16));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 1; o < G; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (!valid) return;
  amax = fmaxf(amax, 1e-4f);
  const float sc = round_scale ? pow2_ceil_log2(__fmul_rn(amax, 1.0f / 448.0f))
                               : __fdiv_rn(amax, 448.0f);
  uint32_t c[2] = {0u, 0u};
  uint32_t dq[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float r = __fdiv_rn(v[i], sc);
    const float y = isnan(r) ? r : fminf(fmaxf(r, -448.0f), 448.0f);   // torch clamp keeps NaN
    const uint8_t code = f32_to_e4m3_sat(y);
    c[i >> 2] |= uint32_t(code) << (8 * (i & 3));
    if (deq) {
      const float back = h2f2(e4m3x2_to_f16x2(code)).x;
      dq[i >> 1] |= uint32_t(f2bf_bits(__fmul_rn(back, sc))) << (16 * (i & 1));
    }
  }
  *reinterpret_cast<uint2 *>(q + tid * 8) = make_uint2(c[0], c[1]);
  if (deq) *reinterpret_cast<uint4 *>(deq + tid * 8) = make_uint4(dq[0], dq[1], dq[2], dq[3]);
  if ((tid % G) == 0) {
    const int64_t e0 = tid * 8, m = e0 / K, blk = (e0 % K) / (8 * G), nblk = K / (8 * G);
    if (s_u8) {
      const uint8_t e8 = uint8_t((__float_as_uint(sc) >> 23) & 0xFF);
      reinterpret_cast<uint8_t *>(s)[m * nblk + blk] = e8;
      if (s_atoms)
        s_atoms[(m / tile_rows) * (K / 128) * 1024 +
                (int64_t(blk) >> 2) * 1024 + ((m % tile_rows) >> 7) * 512 +
                ((m % tile_rows) & 31) * 16 + (((m % tile_rows) >> 5) & 3) * 4 + (blk & 3)] = e8;
    } else {
      reinterpret_cast<float *>(s)[m * nblk + blk] = sc;
    }
  }
}

}  // namespace dsv41
