// aqgemm.cuh -- MLX affine quantized matmul at prefill sizes on the 5th-generation tensor
// cores (tcgen05.mma kind::f16, bf16 x bf16 -> fp32 in TMEM).
//
// y[m, n] = sum_k x[m, k] * w[n, k], w[n, k] = bf16(scale[n, k/64] * q[n, k] + bias[n, k/64])
// (8-bit codes: fp32 fma then bf16; 4-bit codes: one fused bf16x2 fma, i.e. a single
// rounding) with q the 4- or 8-bit code of the little-endian row bit stream
// (mx.quantized_matmul behind nn.QuantizedLinear, deepseek_v41_mlx/load.py:124-131; the
// layout written by deepseek_v41_mlx/convert.py:156-175).  The weights are dequantized to
// bf16 once per tile in shared memory -- the form MLX's own quantized matmul computes for
// bf16 activations -- and multiplied by the bf16 activations as they are, no conversion.
//
// One persistent CTA per SM, 448 threads:
//   warp 0     TMA producer: packed codes (128 rows x 64 k, no swizzle) and activations
//              (256 rows x 64 k bf16, 128-byte swizzle) into a 3-stage ring;
//   warp 1     TMEM allocator + MMA issuer: 4 MMAs of K=16 per stage, M=128, N=256;
//   warps 2-5  epilogue: tcgen05.ld, transpose through shared memory, 16-byte stores;
//   warps 6-13 decoders: two threads per weight row of the tile, each expanding 32 of the
//              row's 64 codes with the group's scale and bias into half of one 128-byte row
//              of the swizzled bf16 A tile (the layout TMA's 128-byte swizzle would give),
//              then fencing the async proxy; the MMA waits for all eight warps (two decoder
//              warps per SM sub-partition, so one hides the other's latency).
// Accumulators are double-buffered (2 x 256 TMEM columns).  Every wait is bounded.
#pragma once
#include "bsgemm.cuh"

namespace dsv41 {

constexpr int AQ_BM = 128, AQ_BN = 256, AQ_BK = 64, AQ_STAGES = 3;
constexpr int AQ_THREADS = 448;
constexpr int AQ_DEC_WARPS = 8;
constexpr int AQ_A_BYTES = AQ_BM * AQ_BK * 2;          // bf16 weights, 16 KB
constexpr int AQ_B_BYTES = AQ_BN * AQ_BK * 2;          // bf16 activations, 32 KB
constexpr int AQ_RAW_BYTES = AQ_BM * AQ_BK;            // codes (8-bit; 4-bit uses half)
constexpr int AQ_OFF_A = 0;
constexpr int AQ_OFF_B = AQ_OFF_A + AQ_STAGES * AQ_A_BYTES;
constexpr int AQ_OFF_RAW = AQ_OFF_B + AQ_STAGES * AQ_B_BYTES;
constexpr int AQ_OFF_EPI = AQ_OFF_RAW + AQ_STAGES * AQ_RAW_BYTES;
constexpr int AQ_OFF_BAR = AQ_OFF_EPI + 4 * BS_EPI_BYTES;
constexpr int AQ_SMEM = AQ_OFF_BAR + 256 + 1024;
constexpr uint32_t AQ_TMEM_COLS = 512;
static_assert(AQ_SMEM <= 232448, "aqgemm shared memory");

struct AqArgs {
  int nkb;                 // K / 64
  int64_t M, N;
  const uint16_t *scale;   // bf16 [N, K/64]
  const uint16_t *bias;    // bf16 [N, K/64]
  int tiles, nt;           // tiles = (N / 128) * nt, nt = ceil(M / 256)
  void *out;               // [M, ldo]
  int64_t ldo;
};

struct AqMaps {
  CUtensorMap w;           // codes as bytes [N, K*bits/8], box {64*bits/8, 128}, no swizzle
  CUtensorMap x;           // bf16 [M, K], box {64, 256}, 128-byte swizzle
};

// kind::f16 instruction descriptor: fp32 accumulator, A and B bf16, both K-major,
// N>>3 at bits 17-22, M>>4 = 8 at bits 24-28.
__device__ __forceinline__ uint32_t idesc_bf16(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (8u << 24);
}
__device__ __forceinline__ void tc_mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                            uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

// tcgen05.mma issued by one elect.sync lane of a converged warp (the whole
// warp runs the issuing loop with warp-uniform operands): back-to-back M=128 N=224 K=16 MMAs
// then run at the tensor pipe's rate, where a single-lane branch issuing them was measured
// ~40% slower on B200.
__device__ __forceinline__ void tc_mma_bf16_el(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                               uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

template <int BITS, int EPI>
__global__ void __launch_bounds__(AQ_THREADS, 1)
    k_aqgemm(const __grid_constant__ AqMaps maps, const AqArgs args) {
  constexpr int S = AQ_STAGES;
  constexpr uint32_t RAW_ROW = AQ_BK * BITS / 8;       // code bytes per row per stage
  extern __shared__ uint8_t aq_raw[];
  const uint32_t raw_s = smem_u32(aq_raw);
  uint8_t *smem = aq_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + AQ_OFF_BAR);
  uint64_t *full = bars;                 // [S] count 1 (+ tx): codes and activations landed
  uint64_t *afull = bars + S;            // [S] count 8: decoded A tile written
  uint64_t *empty = bars + 2 * S;        // [S] count 1 (tcgen05.commit)
  uint64_t *acc_full = bars + 3 * S;     // [2] count 1
  uint64_t *acc_empty = acc_full + 2;    // [2] count 4
  uint64_t *mma_done = acc_full + 4;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&afull[s], AQ_DEC_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, AQ_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = args.nkb;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (whole warp; one
    // elected lane issues)
    {
      if (lane == 0) {
        prefetch_tmap(&maps.w);
        prefetch_tmap(&maps.x);
      }
      const uint64_t pol_w = l2_policy_evict_normal();
      const uint64_t pol_x = l2_policy_evict_normal();
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.tiles && ok; t += gridDim.x) {
        const int mt = t / args.nt, nt = t % args.nt;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (!warp_wait(&empty[s], (uint32_t(it / S) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx_el(&full[s], AQ_BM * RAW_ROW + AQ_B_BYTES);
          tma_load_2d_el(smem + AQ_OFF_RAW + s * AQ_RAW_BYTES, &maps.w, &full[s],
                         int32_t(kb * RAW_ROW), mt * AQ_BM, pol_w);
          tma_load_2d_el(smem + AQ_OFF_B + s * AQ_B_BYTES, &maps.x, &full[s], kb * AQ_BK,
                         nt * AQ_BN, pol_x);
        }
      }
      for (int j = it - S < 0 ? 0 : it - S; j < it; ++j)
        warp_wait(&full[j % S], uint32_t(j / S) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp; one
    // elected lane issues)
    {
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.tiles && ok; t += gridDim.x, ++tc) {
        const int ab = tc & 1;
        if (!warp_wait(&acc_empty[ab], (uint32_t(tc >> 1) & 1u) ^ 1u)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + uint32_t(ab) * AQ_BN;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = uint32_t(it / S) & 1u;
          if (!warp_wait(&full[s], ph) || !warp_wait(&afull[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_sw128(sbase + AQ_OFF_A + s * AQ_A_BYTES);
          const uint64_t db = sdesc_sw128(sbase + AQ_OFF_B + s * AQ_B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k)   // K = 16 bf16 = 32 bytes per MMA
            tc_mma_bf16_el(tacc, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc_bf16(AQ_BN),
                           (kb | k) != 0 ? 1u : 0u);
          tc_commit_el(&empty[s]);
        }
        if (!ok) break;
        tc_commit_el(&acc_full[ab]);
      }
      tc_commit_el(mma_done);
      warp_wait(mma_done, 0);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    float *tp = reinterpret_cast<float *>(smem + AQ_OFF_EPI + q * BS_EPI_BYTES);
    int tc = 0;
    for (int t = blockIdx.x; t < args.tiles; t += gridDim.x, ++tc) {
      const int mt = t / args.nt, nt = t % args.nt;
      const int ab = tc & 1;
      if (!warp_wait(&acc_full[ab], uint32_t(tc >> 1) & 1u)) break;
      tc_fence_after();
      const uint32_t tq = tmem + (uint32_t(32 * q) << 16) + uint32_t(ab) * AQ_BN;
      const int64_t n0 = int64_t(mt) * AQ_BM + 32 * q;
      for (int cc = 0; cc < AQ_BN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tq + uint32_t(cc * 32), r);
#pragma unroll
        for (int j = 0; j < 32; ++j) tp[j * BS_EPI_LD + lane] = __uint_as_float(r[j]);
        __syncwarp();
        const int64_t m = int64_t(nt) * AQ_BN + cc * 32 + lane;
        if (m < args.M) {
          const float4 *src = reinterpret_cast<const float4 *>(tp + lane * BS_EPI_LD);
          if constexpr (EPI == BS_EPI_F32) {
            float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(args.out) +
                                                     m * args.ldo + n0);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = src[i];
          } else {
            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(args.out) +
                                                   m * args.ldo + n0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 a = src[2 * i], b = src[2 * i + 1];
              uint4 o;
              o.x = uint32_t(f2bf_bits(a.x)) | (uint32_t(f2bf_bits(a.y)) << 16);
              o.y = uint32_t(f2bf_bits(a.z)) | (uint32_t(f2bf_bits(a.w)) << 16);
              o.z = uint32_t(f2bf_bits(b.x)) | (uint32_t(f2bf_bits(b.y)) << 16);
              o.w = uint32_t(f2bf_bits(b.z)) | (uint32_t(f2bf_bits(b.w)) << 16);
              dst[i] = o;
            }
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  } else {
    // ------------------------------------------------------------ decoders
    const int dt = (warp - 6) * 32 + lane;             // 0 .. 255
    const int row = dt >> 1, half = dt & 1;             // tile row, k half (32 codes)
    constexpr uint32_t HALF_BYTES = RAW_ROW / 2;        // 16 (4-bit) or 32 (8-bit)
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < args.tiles && ok; t += gridDim.x) {
      const int mt = t / args.nt;
      const int64_t grow = int64_t(mt) * AQ_BM + row;   // weight row (N % 128 == 0)
      const uint16_t *sp = args.scale + grow * nkb;
      const uint16_t *bp = args.bias + grow * nkb;
      uint16_t sc_b = __ldg(sp), bi_b = __ldg(bp);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        // next group's scale and bias while this one decodes
        const uint16_t sc_nb = kb + 1 < nkb ? __ldg(sp + kb + 1) : uint16_t(0);
        const uint16_t bi_nb = kb + 1 < nkb ? __ldg(bp + kb + 1) : uint16_t(0);
        const float sc = bf_bits2f(sc_b), bi = bf_bits2f(bi_b);
        if (!warp_wait(&full[s], uint32_t(it / S) & 1u)) {
          ok = false;
          break;
        }
        const uint4 *src = reinterpret_cast<const uint4 *>(
            smem + AQ_OFF_RAW + s * AQ_RAW_BYTES + row * RAW_ROW + half * HALF_BYTES);
        uint32_t code[HALF_BYTES / 4];
#pragma unroll
        for (int i = 0; i < int(HALF_BYTES / 16); ++i) {
          const uint4 v = src[i];
          code[4 * i] = v.x;
          code[4 * i + 1] = v.y;
          code[4 * i + 2] = v.z;
          code[4 * i + 3] = v.w;
        }
        uint8_t *arow = smem + AQ_OFF_A + s * AQ_A_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
        // bf16x2 forms of the scale and bias, and 128 (the code magic's offset)
        const uint32_t s2u = uint32_t(sc_b) | (uint32_t(sc_b) << 16);
        const uint32_t b2u = uint32_t(bi_b) | (uint32_t(bi_b) << 16);
        const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162 *>(&s2u);
        const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162 *>(&b2u);
        const uint32_t m2u = 0x43004300u;
        const __nv_bfloat162 m2 = *reinterpret_cast<const __nv_bfloat162 *>(&m2u);
#pragma unroll
        for (int cl = 0; cl < 4; ++cl) {    // local chunk: k 8cl .. 8cl+7 of this half
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k0 = 8 * cl + 2 * e;
            if (BITS == 4) {
              // codes k0, k0+1 are the two nibbles of one byte: bf16 pair (128 + q) exactly,
              // minus 128, then one fused fma.rn.bf16x2 -- round(s*q + b) to bf16 once
              const uint32_t t = code[k0 >> 3] >> (4 * (k0 & 7));
              const uint32_t pu = (t & 0xFu) | ((t << 12) & 0xF0000u) | 0x43004300u;
              const __nv_bfloat162 q2 = __hsub2(*reinterpret_cast<const __nv_bfloat162 *>(&pu), m2);
              const __nv_bfloat162 h2 = __hfma2(s2, q2, b2);
              wv[e] = *reinterpret_cast<const uint32_t *>(&h2);
            } else {
              const uint32_t q0 = (code[k0 >> 2] >> (8 * (k0 & 3))) & 0xFFu;
              const uint32_t q1 = (code[k0 >> 2] >> (8 * ((k0 + 1) & 3))) & 0xFFu;
              // exact integer -> float (2^23 + q - 2^23), the affine fma in fp32, then bf16
              const float f0 = __uint_as_float(0x4B000000u | q0) - 8388608.0f;
              const float f1 = __uint_as_float(0x4B000000u | q1) - 8388608.0f;
              const __nv_bfloat162 h2 = __floats2bfloat162_rn(__fmaf_rn(sc, f0, bi),
                                                              __fmaf_rn(sc, f1, bi));
              wv[e] = *reinterpret_cast<const uint32_t *>(&h2);
            }
          }
          const int c = 4 * half + cl;      // chunk of the 128-byte row
          *reinterpret_cast<uint4 *>(arow + ((c ^ (row & 7)) << 4)) =
              make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[s]);
        sc_b = sc_nb;
        bi_b = bi_nb;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, AQ_TMEM_COLS);
  }
}

}  // namespace dsv41
