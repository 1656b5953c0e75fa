// gemv_m1.cuh -- one activation row times a quantized weight on the CUDA cores: MLX affine
// 4-bit and 8-bit (mx.quantized_matmul at M = 1) and fp8 e4m3 with 32 x 32 block scales (the
// dense fp8 linear at M = 1).
//
// Affine:
// y[n] = sum_g ( s[n,g] * sum_{k in g} q[n,k] x[k]  +  b[n,g] * sum_{k in g} x[k] ), the form
// mx.quantized_matmul evaluates (deepseek_v41_mlx/load.py:124-131): per 64-code group the
// scale times the codes' dot product with x, plus the bias times the sum of x.  With a single
// activation row the tensor-core engine (qgemv.cuh) computes 8 columns for every useful one and
// needs a separate activation-prep launch; here the CUDA cores do it in one launch:
//   * every CTA copies x (bf16) into shared memory once, in an order that matches how the codes
//     are unpacked (see below), together with the fp32 sum of each 32-code chunk of x;
//   * a warp takes one weight row at a time, each lane 16-byte streaming loads of 32 codes
//     (lane l: chunks l, l + 32, ... of the row -- coalesced 512-byte spans), all of the
//     lane's loads in flight before the first is used;
//   * codes become exact bf16 through the 0x4300 exponent (bf16 128 + q, minus 128 in one
//     bf16x2 subtract), two codes a word k and k + 4 of each 8-code word;
//   * sm_100's mixed-precision `fma.rn.f32.bf16` multiplies a bf16 code by a bf16 activation
//     exactly and adds the product to an fp32 sum with one rounding;
//   * the lane folds scale and bias per chunk in fp32, the warp sums its lanes in a fixed
//     butterfly order, lane 0 stores.
// Deterministic: every order is fixed by the shapes alone.
#pragma once
#include "common.cuh"

namespace dsv41 {

constexpr int GM1_THREADS = 256;
constexpr int GM1_U = 8;              // 16-byte chunks a lane keeps in flight per row

// a0 += q.lo * x.lo, a1 += q.hi * x.hi (bf16 halves; exact products, fp32 sums)
__device__ __forceinline__ void gm1_fma2(uint32_t q2, uint32_t x2, float &a0, float &a1) {
  asm("{\n\t.reg .b16 q0, q1, x0, x1;\n\tmov.b32 {q0, q1}, %2;\n\tmov.b32 {x0, x1}, %3;\n\t"
      "fma.rn.f32.bf16 %0, q0, x0, %0;\n\tfma.rn.f32.bf16 %1, q1, x1, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(q2), "r"(x2));
}

// codes of nibbles j and j + 4 of w (MLX packs code 8i + j at bits 4j of word i) as exact
// bf16x2: (0x4300 | q) is bf16 128 + q, minus 128
__device__ __forceinline__ uint32_t gm1_pair(uint32_t w, int j) {
  const uint32_t t = ((w >> (4 * j)) & 0x000F000Fu) | 0x43004300u;
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(0x43004300u));
  return r;
}

// x: [K] bf16 (16-byte aligned); wq: [N, K/8] u32 rows (16-byte aligned); scales, biases:
// [N, K/64] bf16; K % 64 == 0, K <= 16384.  Dynamic shared memory: 2K + 4(K/32) bytes.
template <typename TO>
__global__ void __launch_bounds__(GM1_THREADS, 4) k_gemv_affine4_m1(
    const uint16_t *__restrict__ x, int64_t K, const uint32_t *__restrict__ wq,
    const uint16_t *__restrict__ scales, const uint16_t *__restrict__ biases, int64_t N,
    TO *__restrict__ y) {
  extern __shared__ __align__(16) uint8_t gm1_smem[];
  const int nch = int(K / 32);                     // 16-byte code chunks a row
  // x as 16-byte segments: the 8 activations of word i of chunk c (x[32c + 8i ..]) at
  // xt[i * nch + c], as words (x0, x4), (x1, x5), (x2, x6), (x3, x7) -- the code pairs that
  // gm1_pair produces; a warp's lanes then read consecutive segments
  uint4 *xt = reinterpret_cast<uint4 *>(gm1_smem);
  float *xsum = reinterpret_cast<float *>(gm1_smem + size_t(K) * 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = int(K / 64);
  const int64_t row0 = int64_t(blockIdx.x) * (GM1_THREADS / 32) + warp;
  const int64_t rstride = int64_t(gridDim.x) * (GM1_THREADS / 32);
  // the first row's loads go out before the set-up below: the lane's GM1_U code chunks, and
  // the scale and bias of groups c0/2 + 32j + lane (j < GM1_U/2), which the chunks' lanes take
  // by shuffle (chunk c belongs to group c/2)
  uint4 v[GM1_U];
  uint32_t sbv[GM1_U / 2];                         // scale bits << 16 | bias bits
  auto load_row = [&](int64_t r, int c0) {
    const uint4 *wr = reinterpret_cast<const uint4 *>(wq + r * (K / 8));
#pragma unroll
    for (int u = 0; u < GM1_U; ++u) {
      const int c = c0 + u * 32 + lane;
      v[u] = (r < N && c < nch) ? __ldcs(wr + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < GM1_U / 2; ++j) {
      const int g = c0 / 2 + 32 * j + lane;
      sbv[j] = (r < N && g < G) ? (uint32_t(__ldcs(scales + r * G + g)) << 16) |
                                      uint32_t(__ldcs(biases + r * G + g))
                                : 0u;
    }
  };
  load_row(row0, 0);
  for (int s = threadIdx.x; s < 4 * nch; s += GM1_THREADS) {
    const int c = s >> 2, i = s & 3;
    const uint4 in = __ldg(reinterpret_cast<const uint4 *>(x) + (c * 4 + i));
    uint4 o;
    o.x = __byte_perm(in.x, in.z, 0x5410);
    o.y = __byte_perm(in.x, in.z, 0x7632);
    o.z = __byte_perm(in.y, in.w, 0x5410);
    o.w = __byte_perm(in.y, in.w, 0x7632);
    xt[i * nch + c] = o;
  }
  __syncthreads();
  // chunk sums of x in the segments' order (word by word, lo halves then hi halves)
  for (int c = threadIdx.x; c < nch; c += GM1_THREADS) {
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 xv = xt[i * nch + c];
      const uint32_t wv[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) sum += __uint_as_float(wv[j] << 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) sum += __uint_as_float(wv[j] & 0xFFFF0000u);
    }
    xsum[c] = sum;
  }
  __syncthreads();
  for (int64_t r = row0; r < N; r += rstride) {
    float acc = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 32 * GM1_U) {
      if (c0 > 0) load_row(r, c0);
#pragma unroll
      for (int u = 0; u < GM1_U; ++u) {
        if (c0 + u * 32 >= nch) break;                 // warp-uniform
        const int c = c0 + u * 32 + lane;
        // group c/2 - c0/2 = 16u + lane/2: word u/2 of lane (16(u&1) + lane/2)
        const uint32_t sb = __shfl_sync(0xffffffffu, sbv[u >> 1], 16 * (u & 1) + (lane >> 1));
        if (c >= nch) continue;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 xv = xt[i * nch + c];
          gm1_fma2(gm1_pair(w[i], 0), xv.x, a0, a1);
          gm1_fma2(gm1_pair(w[i], 1), xv.y, a0, a1);
          gm1_fma2(gm1_pair(w[i], 2), xv.z, a0, a1);
          gm1_fma2(gm1_pair(w[i], 3), xv.w, a0, a1);
        }
        const float s = __uint_as_float(sb & 0xFFFF0000u);
        const float b = __uint_as_float(sb << 16);
        acc = __fmaf_rn(s, a0 + a1, acc);
        acc = __fmaf_rn(b, xsum[c], acc);
      }
    }
    // the next row's loads go out before this row's reduction
    if (r + rstride < N) load_row(r + rstride, 0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if constexpr (sizeof(TO) == 4)
        y[r] = acc;
      else
        y[r] = __float2bfloat16_rn(acc);
    }
  }
}

// a0 += h.lo * xh.lo, a1 += h.hi * xh.hi (f16 halves; exact products, fp32 sums)
__device__ __forceinline__ void gm1_fma2_f16(uint32_t h, uint32_t xh, float &a0, float &a1) {
  asm("{\n\t.reg .b16 q0, q1, x0, x1;\n\tmov.b32 {q0, q1}, %2;\n\tmov.b32 {x0, x1}, %3;\n\t"
      "fma.rn.f32.f16 %0, q0, x0, %0;\n\tfma.rn.f32.f16 %1, q1, x1, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(h), "r"(xh));
}

// k_gemv_byte_m1<false>: one activation row times an fp8 e4m3 weight with ue8m0 scales per
// 32 x 32 block (upstream `weight_dequant` then the product; the dense linear at decode).  The
// same arithmetic as
// the tensor-core engine's single-row case, without its activation-prep launch: every CTA
// finds the row's max |x|, keeps x * 2^-E as f16 in shared memory (E = exponent(max) - 14, the
// engine's per-row multiplier: exact for bf16 values within 2^29 of the max), and per 32-code
// block sums code x activation products (`cvt.rn.f16x2.e4m3x2`, then the mixed-precision
// `fma.rn.f32.f16`: exact products, fp32 sums), folds the block scale (byte 0 applied as 0, as
// the engine does) and finally 2^E.  A warp takes a row at a time, lane l the 16-code chunks
// l, l + 32, ...; its 16 chunk slots (a whole row at K <= 8192) are refilled one step ahead (the
// same slot of the next 512 chunks of the row, or of its next row) as soon as they are
// consumed, so up to 8 KB of codes per warp stay in flight.  x: [K] bf16, w: [N, K] (both
// 16-byte aligned), s: [ceil(N/32), sld]; K % 32 == 0, K <= 16384.  Dynamic shared memory: 2K
// bytes (AFF: 2K + K/2).
//
// AFF: the same kernel for MLX affine 8-bit codes ([N, K/4] u32 words, bf16
// scales and biases per 64-code group): codes become exact f16 through the 0x6400 exponent
// (1024 + q, minus 1024), bytes 0 and 2 of a word together, then 1 and 3, with x kept in that
// order; the lane sums scale x (codes . x * 2^-E) and, apart, bias x (sum of x) per 16-code
// chunk, the first scaled by 2^E at the end.  s: scales, b: biases (AFF); s: ue8m0 (fp8).
constexpr int GF8_U = 16;             // 16-byte chunk slots a lane (fp8)
template <bool AFF, typename TO>
__global__ void __launch_bounds__(GM1_THREADS, 2) k_gemv_byte_m1(
    const uint16_t *__restrict__ x, int64_t K, const uint8_t *__restrict__ w,
    const void *__restrict__ sv, const uint16_t *__restrict__ bv, int64_t sld, int64_t N,
    TO *__restrict__ y) {
  extern __shared__ __align__(16) uint8_t gm1_smem[];
  // x * 2^-E as f16, 16-byte segment i of 16-code chunk c (x[16c + 8i ..]) at xt[i*nch + c]
  // (AFF: pairs (x0, x2), (x1, x3) of every 4); AFF: then the fp32 sum of each segment of x
  uint4 *xt = reinterpret_cast<uint4 *>(gm1_smem);
  float *xsum8 = reinterpret_cast<float *>(gm1_smem + size_t(K) * 2);
  __shared__ float red[GM1_THREADS / 32];
  __shared__ int s_e;
  const int nch = int(K / 16);
  const int npass = (nch + 32 * GF8_U - 1) / (32 * GF8_U);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = int64_t(blockIdx.x) * (GM1_THREADS / 32) + warp;
  const int64_t rstride = int64_t(gridDim.x) * (GM1_THREADS / 32);
  uint4 v[GF8_U];
  uint32_t sc[GF8_U];
  // step t of this warp: row row0 + (t / npass) * rstride, chunks from 512 (t % npass)
  auto load_slot = [&](int64_t t, int u) {
    const int64_t r = row0 + (t / npass) * rstride;
    const int c = int(t % npass) * (32 * GF8_U) + u * 32 + lane;
    const bool in = r < N && c < nch;
    v[u] = in ? __ldcs(reinterpret_cast<const uint4 *>(w + r * K) + c) : make_uint4(0u, 0u, 0u, 0u);
    if constexpr (AFF) {
      const int64_t gi = r * sld + (c >> 2);
      sc[u] = in ? (uint32_t(__ldg(static_cast<const uint16_t *>(sv) + gi)) << 16) |
                       uint32_t(__ldg(bv + gi))
                 : 0u;
    } else {
      sc[u] = in ? uint32_t(__ldg(static_cast<const uint8_t *>(sv) + (r >> 5) * sld + (c >> 1)))
                 : 0u;
    }
  };
#pragma unroll
  for (int u = 0; u < GF8_U; ++u) load_slot(0, u);
  // the row's max |x| and the f16 copy: x's first 4 x 256 segments read once into registers,
  // any further ones (K > 8192) read again for the copy
  constexpr int XR = 4;
  const int nseg = int(K / 8);
  uint4 xr[XR];
  float amax = 0.0f;
  for (int i = threadIdx.x + XR * GM1_THREADS; i < nseg; i += GM1_THREADS) {
    const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(x) + i);
    const uint32_t wv[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(wv[j] << 16)),
                               fabsf(__uint_as_float(wv[j] & 0xFFFF0000u))));
  }
#pragma unroll
  for (int k = 0; k < XR; ++k) {
    const int i = threadIdx.x + k * GM1_THREADS;
    xr[k] = i < nseg ? __ldg(reinterpret_cast<const uint4 *>(x) + i) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t wv[4] = {xr[k].x, xr[k].y, xr[k].z, xr[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(wv[j] << 16)),
                               fabsf(__uint_as_float(wv[j] & 0xFFFF0000u))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int i = 0; i < GM1_THREADS / 32; ++i) m = fmaxf(m, red[i]);
    int E = 0;
    if (m > 0.0f && m < INFINITY) E = int((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14;
    s_e = E < -126 ? -126 : E;
  }
  __syncthreads();
  const int E = s_e;
  const float inv = ldexpf(1.0f, -E);
  auto put = [&](const uint4 &xv, int i) {
    uint32_t wv[4] = {xv.x, xv.y, xv.z, xv.w};
    if constexpr (AFF) {
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        sum += __uint_as_float(wv[j] << 16) + __uint_as_float(wv[j] & 0xFFFF0000u);
      xsum8[i] = sum;
      const uint32_t a = wv[0], b = wv[1], c = wv[2], d = wv[3];
      wv[0] = __byte_perm(a, b, 0x5410);        // (x0, x2)
      wv[1] = __byte_perm(a, b, 0x7632);        // (x1, x3)
      wv[2] = __byte_perm(c, d, 0x5410);        // (x4, x6)
      wv[3] = __byte_perm(c, d, 0x7632);        // (x5, x7)
    }
    uint32_t hv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2 h = __floats2half2_rn(__uint_as_float(wv[j] << 16) * inv,
                                          __uint_as_float(wv[j] & 0xFFFF0000u) * inv);
      hv[j] = *reinterpret_cast<const uint32_t *>(&h);
    }
    xt[(i & 1) * nch + (i >> 1)] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  };
#pragma unroll
  for (int k = 0; k < XR; ++k) {
    const int i = threadIdx.x + k * GM1_THREADS;
    if (i < nseg) put(xr[k], i);
  }
  for (int i = threadIdx.x + XR * GM1_THREADS; i < nseg; i += GM1_THREADS)
    put(__ldg(reinterpret_cast<const uint4 *>(x) + i), i);
  __syncthreads();
  const float out_scale = ldexpf(1.0f, E);
  int64_t t = 0;
  for (int64_t r = row0; r < N; r += rstride) {
    float acc = 0.0f, accb = 0.0f;                   // AFF: accb = the bias terms
    for (int pass = 0; pass < npass; ++pass, ++t) {
      const int c0 = pass * (32 * GF8_U);
#pragma unroll
      for (int u = 0; u < GF8_U; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < nch) {
          const uint4 xa = xt[c], xb = xt[nch + c];
          const uint32_t wv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
          const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
          float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t h0, h1;
            if constexpr (AFF) {
              // (0x6400 | q) is f16 1024 + q: bytes 0, 2 and then 1, 3 of the word
              const __half2 m = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
              uint32_t t0 = (wv[j] & 0x00FF00FFu) | 0x64006400u;
              uint32_t t1 = ((wv[j] >> 8) & 0x00FF00FFu) | 0x64006400u;
              const __half2 q0 = __hsub2(*reinterpret_cast<const __half2 *>(&t0), m);
              const __half2 q1 = __hsub2(*reinterpret_cast<const __half2 *>(&t1), m);
              h0 = *reinterpret_cast<const uint32_t *>(&q0);
              h1 = *reinterpret_cast<const uint32_t *>(&q1);
            } else {
              e4m3x4_to_f16x4(wv[j], h0, h1);
            }
            gm1_fma2_f16(h0, xw[2 * j], a0, a1);
            gm1_fma2_f16(h1, xw[2 * j + 1], a0, a1);
          }
          if constexpr (AFF) {
            acc = __fmaf_rn(__uint_as_float(sc[u] & 0xFFFF0000u), a0 + a1, acc);
            accb = __fmaf_rn(__uint_as_float(sc[u] << 16), xsum8[2 * c] + xsum8[2 * c + 1], accb);
          } else {
            acc = __fmaf_rn(__uint_as_float(sc[u] << 23), a0 + a1, acc);
          }
        }
        load_slot(t + 1, u);                        // this slot's next step
      }
    }
    acc = acc * out_scale + accb;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      if constexpr (sizeof(TO) == 4)
        y[r] = acc;
      else
        y[r] = __float2bfloat16_rn(acc);
    }
  }
}

}  // namespace dsv41
