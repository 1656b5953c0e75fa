// a16gemm.cuh -- the MoE layer at prefill sizes in the port's numerics ("a16": bf16
// activations, never quantized) on the 5th-generation tensor cores.
//
// deepseek_v41_mlx/moe.py:101-112 runs the routed experts as SwitchGLU over weights
// decoded by dequant.py:63-68 (fp4 e2m1 x ue8m0 per 32, exact in bf16) and multiplies them
// by the bf16 activations with fp32 accumulation; ClampedSwiGLU (moe.py:30-43) works in fp32
// and the down projection takes that fp32 h; the expert outputs are weighted and summed in
// top-k order after the down projection.  The shared expert (moe.py:77-93, fp8 32x32
// weights) rounds its intermediates to bf16.  Here:
//
//   D[p, n] = sum_k X[p, k] * bf16(W[n, k])     tcgen05.mma.cta_group::1.kind::f16, bf16 x
//                                               bf16 -> fp32 in TMEM; M = 128 weight rows,
//                                               N = up to 224 activation rows, K = 64 a stage
//
// The weights arrive as codes by TMA (no swizzle) and eight decoder warps expand them -- fp4
// through cvt.rn.f16x2.e2m1x2, fp8 through cvt.rn.f16x2.e4m3x2, times the ue8m0 scale in
// fp32 (exact), then bf16 (exact: at most 4 significant bits) -- into the 128-byte-swizzled
// A tile the MMA reads.  When an operand holds an fp32 value (the routed down projection's
// input h, or every intermediate in the exact mode) it is split into bf16 halves hi = bf16(h)
// and lo = bf16(h - hi) and the stage runs the MMAs for both (HILO): the product then carries
// ~16 significant bits of h, a relative error of ~2^-18 per element.
//
// One persistent CTA per SM, 704 threads: warp 0 TMA producer, warp 1 TMEM allocator + MMA
// issuer (each a whole warp whose elect.sync lane issues), warps 2-5 epilogue, warps 6-21
// decoders (a tile row quarter, 16 codes, each).  Tiles are taken in a fixed stride
// (tile blockIdx.x + i * gridDim.x) by every role from the prefill's grouped tile lists
// (expert, m-tile, first row, rows) or, dense, over all rows.  Accumulators are
// double-buffered (2 x 224 TMEM columns).  Epilogues: SwiGLU (the tile's 128 weight rows are
// 64 gate rows then the matching 64 up rows; warps q and q + 2 pair up through shared memory)
// writing h as bf16 hi (+ lo) rows, or fp32 rows.  Every wait is bounded; no multicast.
#pragma once
#include "aqgemm.cuh"
#include "engram.cuh"   // store8

namespace dsv41 {

constexpr int A16_BM = 128, A16_BK = 64, A16_BN = 224;
constexpr int A16_DEC_WARPS = 16;
constexpr int A16_PF = 16;   // k-blocks of weight codes prefetched into L2 ahead of their load
constexpr int A16_THREADS = 32 * (6 + A16_DEC_WARPS);

enum { A16_EPI_SWIGLU = 0, A16_EPI_F32 = 1 };

template <int WFMT, bool HILO>
struct A16Cfg {
  static constexpr int RB = WFMT == BS_W_FP4 ? A16_BK / 2 : A16_BK;   // code bytes a row a stage
  static constexpr int RAW = A16_BM * RB;
  static constexpr int A_BYTES = A16_BM * A16_BK * 2;                 // bf16 weights, 16 KB
  static constexpr int B_BYTES = A16_BN * A16_BK * 2;                 // bf16 rows, 28 KB
  static constexpr int NB = HILO ? 2 : 1;
  static constexpr int STAGE = A_BYTES + NB * B_BYTES + RAW;
  static constexpr int EPI = 4 * BS_EPI_BYTES;
  static constexpr int FIT = (232448 - 1024 - 512 - EPI) / STAGE;
  static constexpr int STAGES = FIT > 4 ? 4 : FIT;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_RAW = OFF_B + STAGES * NB * B_BYTES;
  static constexpr int OFF_EPI = OFF_RAW + STAGES * RAW;
  static constexpr int OFF_BAR = OFF_EPI + EPI;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;
  static_assert(STAGES >= 2, "a16 stages");
  static_assert(SMEM <= 232448, "a16 shared memory");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0 && RAW % 1024 == 0, "alignment");
};

struct A16Args {
  int nkb;                   // K / 64
  int a_rows;                // weight rows of one group (moe_inter_dim for SwiGLU, dim for down)
  const uint8_t *s, *s2;     // ue8m0 weight scales (s2: the up projection's, SwiGLU)
  int64_t sld;               // scale bytes a scale row (K / 32)
  int sshift;                // scale row of weight row r: r >> sshift (0 fp4; 5 fp8 32x32)
  int svec;                  // scale rows 16-byte aligned and sld % 16 == 0 (vector loads)
  const int4 *tiles;         // grouped tiles {group, m-tile, first row, rows | row tile << 8}
  const int *ntiles;         //   and their count (device); null tiles = dense
  int dense_nt, dense_rows, dense_tiles;   // dense: m-tiles x ceil(rows / 224) tiles
  float *out;                // F32: out[p * ldo + n]
  int64_t ldo;
  int round_out;             // F32: values rounded to bf16 (stored as fp32)
  __nv_bfloat16 *hhi, *hlo;  // SwiGLU: h = bf16 hi (+ lo when hlo) rows of ldh
  int64_t ldh;
  int round_gu;              // SwiGLU: gate and up outputs rounded to bf16 first
  float limit;               // SwiGLU clamp (<= 0: none)
};

struct A16Maps {
  CUtensorMap w, w2;         // codes as bytes, box {RB, 64 (SwiGLU) or 128 rows}, no swizzle
  CUtensorMap x[4], xlo[4];  // bf16 rows, box {64, 32 / 64 / 128 / 224 rows}, 128-byte swizzle
};

__device__ __forceinline__ int4 a16_tile(const A16Args &a, int t) {
  if (a.tiles) return a.tiles[t];
  const int nt = t % a.dense_nt, mt = t / a.dense_nt;
  const int row0 = nt * A16_BN;
  return make_int4(0, mt, row0, min(A16_BN, a.dense_rows - row0) | (nt << 8));
}

template <int WFMT, int EPI, bool HILO>
__global__ void __launch_bounds__(A16_THREADS, 1)
    k_a16gemm(const __grid_constant__ A16Maps maps, const A16Args args) {
  using Cfg = A16Cfg<WFMT, HILO>;
  constexpr int S = Cfg::STAGES;
  constexpr bool SWI = EPI == A16_EPI_SWIGLU;
  extern __shared__ uint8_t a16_raw[];
  const uint32_t raw_s = smem_u32(a16_raw);
  uint8_t *smem = a16_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::OFF_BAR);
  uint64_t *full = bars;                 // [S] count 1 (+ tx): codes and activations landed
  uint64_t *afull = bars + S;            // [S] count 8: decoded A tile written
  uint64_t *empty = bars + 2 * S;        // [S] count 1 (tcgen05.commit)
  uint64_t *acc_full = bars + 3 * S;     // [2] count 1
  uint64_t *acc_empty = acc_full + 2;    // [2] count 4
  uint64_t *xfull = acc_full + 4;        // [2] count 64 (SwiGLU pair exchange)
  uint64_t *xempty = acc_full + 6;       // [2] count 64
  uint64_t *mma_done = acc_full + 8;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&afull[s], A16_DEC_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
      mbar_init(&xfull[i], 64);
      mbar_init(&xempty[i], 64);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = args.nkb;
  const int ntiles = args.tiles ? *args.ntiles : args.dense_tiles;
  constexpr int WROWS = SWI ? 64 : A16_BM;            // weight rows a TMA box covers

  if (warp == 0) {
    // ------------------------------------------------------------ producer (whole warp; one
    // elected lane issues)
    {
      if (lane == 0) {
        prefetch_tmap(&maps.w);
        if (SWI) prefetch_tmap(&maps.w2);
      }
      // an expert's m-tile is read by its consecutive row tiles (neighbouring CTAs): keep it
      const uint64_t pol_w = l2_policy_evict_normal();
      const uint64_t pol_x = l2_policy_evict_normal();
      // The weight codes come from HBM as 32- or 64-byte pieces of 128 rows, the slowest
      // copies of a stage: the producer prefetches them into L2 A16_PF k-blocks ahead (into
      // the CTA's next tile), so the stage ring waits on L2 rather than HBM latency.
      auto wrow_of = [&](int t) {
        const int4 tl = a16_tile(args, t);
        return int32_t(int64_t(tl.x) * args.a_rows + int64_t(tl.y) * WROWS);
      };
      auto prefetch_w = [&](int32_t wrow, int kb) {
        tma_prefetch_2d_el(&maps.w, kb * Cfg::RB, wrow);
        if (SWI) tma_prefetch_2d_el(&maps.w2, kb * Cfg::RB, wrow);
      };
      if (blockIdx.x < ntiles) {
        const int32_t w0 = wrow_of(blockIdx.x);
        for (int kb = 0; kb < A16_PF && kb < nkb; ++kb) prefetch_w(w0, kb);
      }
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const int4 tl = a16_tile(args, t);
        const int nmma = bs_nmma<A16_BN>(tl.w & 0xFF), bi = bs_box(nmma);
        const uint32_t xbytes = bs_box_rows(bi) * A16_BK * 2;
        const int32_t wrow0 = int32_t(int64_t(tl.x) * args.a_rows + int64_t(tl.y) * WROWS);
        const int tn = t + int(gridDim.x);
        const int32_t wnext = tn < ntiles ? wrow_of(tn) : 0;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          const int kp = kb + A16_PF;
          if (kp < nkb) prefetch_w(wrow0, kp);
          else if (tn < ntiles && kp - nkb < nkb) prefetch_w(wnext, kp - nkb);
          if (!warp_wait(&empty[s], (uint32_t(it / S) & 1u) ^ 1u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx_el(&full[s], uint32_t(Cfg::RAW) + uint32_t(Cfg::NB) * xbytes);
          uint8_t *raw = smem + Cfg::OFF_RAW + s * Cfg::RAW;
          tma_load_2d_el(raw, &maps.w, &full[s], kb * Cfg::RB, wrow0, pol_w);
          if (SWI) tma_load_2d_el(raw + 64 * Cfg::RB, &maps.w2, &full[s], kb * Cfg::RB, wrow0, pol_w);
          uint8_t *b = smem + Cfg::OFF_B + s * Cfg::NB * Cfg::B_BYTES;
          tma_load_2d_el(b, &maps.x[bi], &full[s], kb * A16_BK, tl.z, pol_x);
          if (HILO) tma_load_2d_el(b + Cfg::B_BYTES, &maps.xlo[bi], &full[s], kb * A16_BK, tl.z, pol_x);
        }
      }
      // every copy issued has landed before the CTA can finish
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
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
        const int4 tl = a16_tile(args, t);
        const int nmma = bs_nmma<A16_BN>(tl.w & 0xFF);
        const int ab = tc & 1;
        if (!warp_wait(&acc_empty[ab], (uint32_t(tc >> 1) & 1u) ^ 1u)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + uint32_t(ab) * A16_BN;
        const uint32_t idesc = idesc_bf16(uint32_t(nmma));
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = uint32_t(it / S) & 1u;
          if (!warp_wait(&full[s], ph) || !warp_wait(&afull[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sdesc_sw128(sbase + Cfg::OFF_A + s * Cfg::A_BYTES);
          const uint32_t b0 = sbase + Cfg::OFF_B + s * Cfg::NB * Cfg::B_BYTES;
          const uint64_t db = sdesc_sw128(b0);
#pragma unroll
          for (int k = 0; k < 4; ++k)   // K = 16 bf16 = 32 bytes an MMA
            tc_mma_bf16_el(tacc, da + uint64_t(2 * k), db + uint64_t(2 * k), idesc,
                           (kb | k) != 0 ? 1u : 0u);
          if (HILO) {
            const uint64_t dl = sdesc_sw128(b0 + Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              tc_mma_bf16_el(tacc, da + uint64_t(2 * k), dl + uint64_t(2 * k), idesc, 1u);
          }
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
    float *tp = reinterpret_cast<float *>(smem + Cfg::OFF_EPI + q * BS_EPI_BYTES);
    int tc = 0, xc = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
      const int4 tl = a16_tile(args, t);
      const int nrows = tl.w & 0xFF;
      const int nmma = bs_nmma<A16_BN>(nrows);
      const int ab = tc & 1;
      if (!warp_wait(&acc_full[ab], uint32_t(tc >> 1) & 1u)) break;
      tc_fence_after();
      const uint32_t tq = tmem + (uint32_t(32 * q) << 16) + uint32_t(ab) * A16_BN;
      for (int cc = 0; cc * 32 < nmma && ok; ++cc) {
        uint32_t r[32];
        tmem_ld32(tq + uint32_t(cc * 32), r);
        if constexpr (!SWI) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float v = __uint_as_float(r[j]);
            tp[j * BS_EPI_LD + lane] = args.round_out ? round_bf16f(v) : v;
          }
          __syncwarp();
          if (cc * 32 + lane < nrows) {
            const int64_t p = int64_t(tl.z) + cc * 32 + lane;
            const int64_t n0 = int64_t(tl.y) * A16_BM + 32 * q;
            const float4 *src = reinterpret_cast<const float4 *>(tp + lane * BS_EPI_LD);
            float4 *dst = reinterpret_cast<float4 *>(args.out + p * args.ldo + n0);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = src[i];
          }
          __syncwarp();
        } else {
          // warp q (gate rows 32q..) and warp q + 2 (the same features' up rows) park their
          // chunk transposed, then each finishes 16 of the 32 activation rows: lane l takes
          // row 16 * half + l / 2 and features (l & 1) * 16 .. + 15 of the pair's 32
          const int pr = q & 1, half = q >> 1;
          const uint32_t xph = uint32_t(xc) & 1u;
          const float L = args.limit;
          if (!warp_wait(&xempty[pr], xph ^ 1u)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = __uint_as_float(r[j]);
            if (args.round_gu) v = round_bf16f(v);
            if (L > 0.0f) v = half ? fminf(fmaxf(v, -L), L) : fminf(v, L);
            tp[j * BS_EPI_LD + lane] = v;
          }
          mbar_arrive(&xfull[pr]);
          if (!warp_wait(&xfull[pr], xph)) {
            ok = false;
            break;
          }
          const int jt = 16 * half + (lane >> 1), fh = lane & 1;
          const float *tg = reinterpret_cast<const float *>(smem + Cfg::OFF_EPI + pr * BS_EPI_BYTES) +
                            jt * BS_EPI_LD + fh * 16;
          const float *tu = reinterpret_cast<const float *>(smem + Cfg::OFF_EPI +
                                                            (pr + 2) * BS_EPI_BYTES) +
                            jt * BS_EPI_LD + fh * 16;
          float h[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 g4 = reinterpret_cast<const float4 *>(tg)[i];
            const float4 u4 = reinterpret_cast<const float4 *>(tu)[i];
            const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int b = 0; b < 4; ++b)
              h[4 * i + b] = __fmul_rn(__fdividef(gg[b], 1.0f + __expf(-gg[b])), uu[b]);
          }
          mbar_arrive(&xempty[pr]);
          if (cc * 32 + jt < nrows) {
            const int64_t p = int64_t(tl.z) + cc * 32 + jt;
            const int64_t f0 = int64_t(tl.y) * 64 + 32 * pr + fh * 16;
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint16_t a = f2bf_bits(h[2 * i]), b = f2bf_bits(h[2 * i + 1]);
              hi[i] = uint32_t(a) | (uint32_t(b) << 16);
              const uint16_t la = f2bf_bits(__fsub_rn(h[2 * i], bf_bits2f(a)));
              const uint16_t lb = f2bf_bits(__fsub_rn(h[2 * i + 1], bf_bits2f(b)));
              lo[i] = uint32_t(la) | (uint32_t(lb) << 16);
            }
            uint4 *dh = reinterpret_cast<uint4 *>(args.hhi + p * args.ldh + f0);
            dh[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            dh[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
            if (args.hlo) {
              uint4 *dl = reinterpret_cast<uint4 *>(args.hlo + p * args.ldh + f0);
              dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
              dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            }
          }
          ++xc;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  } else {
    // ------------------------------------------------------------ decoders
    // thread dt: tile row dt / 4, K quarter dt % 4 (16 codes) of every stage
    const int dt = (warp - 6) * 32 + lane;             // 0 .. 511
    const int row = dt >> 2, q = dt & 3, half = q >> 1;  // half: the quarter's 32-wide scale block
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int4 tl = a16_tile(args, t);
      // this row's scales: gate rows from s, up rows from s2 (SwiGLU), K block 2 kb + half
      const uint8_t *sv = (SWI && row >= 64) ? args.s2 : args.s;
      const int64_t wr = int64_t(tl.x) * args.a_rows + int64_t(tl.y) * WROWS + (SWI ? (row & 63) : row);
      const uint8_t *srow = sv + (wr >> args.sshift) * args.sld;   // the row's K/32 scale bytes
      // The row's scales 16 bytes (8 stages) a load, the next block fetched 8 stages ahead,
      // so no stage waits on a global load (rows 16-byte aligned: args.svec); else a byte a
      // stage, one stage ahead.
      uint4 blk = make_uint4(0, 0, 0, 0), nxt = make_uint4(0, 0, 0, 0);
      uint32_t sb = 0;
      if (args.svec) {
        blk = __ldg(reinterpret_cast<const uint4 *>(srow));
        if (nkb > 8) nxt = __ldg(reinterpret_cast<const uint4 *>(srow) + 1);
      } else {
        sb = __ldg(srow + half);
      }
      uint8_t *arow = smem + Cfg::OFF_A + (row >> 3) * 1024 + (row & 7) * 128;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        uint32_t sb_next = 0;
        if (args.svec) {
          if (kb > 0 && (kb & 7) == 0) {
            blk = nxt;
            if (kb + 8 < nkb) nxt = __ldg(reinterpret_cast<const uint4 *>(srow) + (kb >> 3) + 1);
          }
          const uint32_t wsel = (kb & 7) >> 1;             // word of the block
          const uint32_t wv = wsel == 0 ? blk.x : wsel == 1 ? blk.y : wsel == 2 ? blk.z : blk.w;
          sb = (wv >> (8 * (2 * (kb & 1) + half))) & 0xFFu;
        } else {
          sb_next = kb + 1 < nkb ? uint32_t(__ldg(srow + 2 * (kb + 1) + half)) : 0u;
        }
        if (!warp_wait(&full[s], uint32_t(it / S) & 1u)) {
          ok = false;
          break;
        }
        const float sc = e8m0f(sb);
        const uint8_t *src = smem + Cfg::OFF_RAW + s * Cfg::RAW + row * Cfg::RB + q * (Cfg::RB / 4);
        uint32_t wv[8];                                  // 16 bf16 of this row's quarter
        if constexpr (WFMT == BS_W_FP4) {
          const uint2 c = *reinterpret_cast<const uint2 *>(src);   // 16 codes, low nibble first
          const uint32_t cw[2] = {c.x, c.y};
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            uint32_t h4[4];
            e2m1x8_to_f16x8(cw[i], h4[0], h4[1], h4[2], h4[3]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = h2f2(h4[j]);
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc));
              wv[4 * i + j] = *reinterpret_cast<const uint32_t *>(&b2);
            }
          }
        } else {
          const uint4 c = *reinterpret_cast<const uint4 *>(src);
          const uint32_t cw[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t h2[2];
            e4m3x4_to_f16x4(cw[i], h2[0], h2[1]);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const float2 f = h2f2(h2[j]);
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(__fmul_rn(f.x, sc), __fmul_rn(f.y, sc));
              wv[2 * i + j] = *reinterpret_cast<const uint32_t *>(&b2);
            }
          }
        }
        uint8_t *a = arow + s * Cfg::A_BYTES;
#pragma unroll
        for (int cl = 0; cl < 2; ++cl) {               // 16-byte chunks 2 q, 2 q + 1
          const int c = 2 * q + cl;
          *reinterpret_cast<uint4 *>(a + ((c ^ (row & 7)) << 4)) =
              make_uint4(wv[4 * cl], wv[4 * cl + 1], wv[4 * cl + 2], wv[4 * cl + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[s]);
        if (!args.svec) sb = sb_next;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The bf16 activation rows of the sorted pairs: dst row r = x row tok[r] (T rows; a slot past
// the placed pairs, left by out-of-range expert ids, is never read by a tile and is skipped
// here unless it holds a token index).  One warp a row.
__global__ void k_a16_gather(const __nv_bfloat16 *__restrict__ x, const int *__restrict__ tok,
                             int64_t T, int64_t R, int64_t K, __nv_bfloat16 *__restrict__ dst) {
  const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const int64_t t = tok[r];
  if (t < 0 || t >= T) return;
  const uint4 *src = reinterpret_cast<const uint4 *>(x + t * K);
  uint4 *d = reinterpret_cast<uint4 *>(dst + r * K);
  for (int64_t i = lane; i < K / 8; i += 32) d[i] = __ldg(src + i);
}

// The port's combine (moe.py:105-112): out[t] = sum_j w[t, j] * Y[slot_pos[t*k + j]] in top-k
// order, fp32, then + Ys[t] (may be null).  8 columns a thread.
template <typename TO>
__global__ void k_a16_combine(const float *__restrict__ Y, const float *__restrict__ Ys,
                              const float *__restrict__ w, const int *__restrict__ slot_pos,
                              int64_t T, int topk, int64_t D, TO *__restrict__ out) {
  const int64_t groups = D / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * groups) return;
  const int64_t t = i / groups, c0 = (i % groups) * 8;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
  for (int j = 0; j < topk; ++j) {
    const int pos = slot_pos[t * topk + j];
    if (pos < 0) continue;
    const float wj = w[t * topk + j];
    const float4 *src = reinterpret_cast<const float4 *>(Y + int64_t(pos) * D + c0);
    const float4 a = src[0], b = src[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = __fadd_rn(acc[c], __fmul_rn(v[c], wj));
  }
  if (Ys) {
    const float4 *src = reinterpret_cast<const float4 *>(Ys + t * D + c0);
    const float4 a = src[0], b = src[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = __fadd_rn(acc[c], v[c]);
  }
  store8(out + t * D + c0, acc);
}

}  // namespace dsv41
