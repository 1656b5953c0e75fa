// qgemv.cuh -- weight-decode fused into skinny matrix products (decode-time GEMV).
//
// y[m, n] = sum_k x[m, k] * W[n, k] for a few tokens m (<= 32 per pass) and a
// weight W stored in one of the reference's quantized formats:
//   WF_FP4  : e2m1 nibbles [N, K/2] + ue8m0 per (row, 32 k)      (dequant.py:53-68)
//   WF_FP8B : e4m3 bytes [N, K] + ue8m0 per (32 rows, 32 k)      (dequant.py:45-50)
//   WF_AFF4 / WF_AFF8 : MLX affine codes, bf16 scale/bias per (row, 64 k)
// The weight bytes are the HBM stream this kernel is bounded by.
//
// Structure (one CTA = 4 consumer warps + 1 producer warp, persistent, 3 CTAs/SM):
//   * producer lane 0 streams 64-row x 128-byte weight tiles and the matching
//     activation tiles into a shared-memory ring with 2D TMA (128-byte swizzle,
//     no multicast), signalling mbarriers with tx counts; every producer lane
//     copies its share of the stage's raw ue8m0 / bf16 scale bytes with cp.async,
//     whose completion arrives on the same mbarrier (no wait in the producer);
//   * each consumer warp owns 16 weight rows; it reads its rows' raw scale words once
//     per stage and, per 32/64-k scale group, turns the group's byte into fp32 and decodes
//     its share of the tile in registers straight to exact f16 (cvt.rn.f16x2.
//     e2m1x2 / e4m3x2, or the 0x6400 magic for affine codes), runs
//     mma.sync m16n8k16 f16 x f16 -> f32 against the activations, and folds the
//     group's scale into an fp32 accumulator (scale * partial [+ bias * sum x]);
//   * activations arrive as f16 with a per-row power-of-two scale applied by the
//     producer of x (exact for bf16 inputs, see qx_prep), so every product is
//     exact and accumulation is fp32.
// The k order inside a group is permuted per thread (any permutation applied to
// both operands leaves the dot product unchanged) so that each thread's slice of
// a group is contiguous in shared memory.
//
// Work = chunks (a group of <= NT*8 x rows bound to one weight matrix, e.g. one
// expert's tokens) x 64-row tiles x K splits.  K splits write fp32 fragments to a
// workspace and the last CTA of a tile (atomic ticket) sums them in split order,
// so results are deterministic.
//
// A ue8m0 scale byte of 0 (2^-127) is applied as 0 here: the group's decoded
// weights are then below 6 * 2^-127 in magnitude.
#pragma once
#include "common.cuh"

namespace dsv41 {

enum : int { WF_FP4 = 0, WF_FP8B = 1, WF_AFF4 = 2, WF_AFF8 = 3 };
enum : int { EPI_STORE_F32 = 0, EPI_STORE_BF16 = 1, EPI_SWIGLU = 2, EPI_DOWN = 3 };

template <int WF> struct Fmt;
template <> struct Fmt<WF_FP4> { static constexpr int KS = 256, GK = 32, NG = 8; };
template <> struct Fmt<WF_FP8B> { static constexpr int KS = 128, GK = 32, NG = 4; };
template <> struct Fmt<WF_AFF4> { static constexpr int KS = 256, GK = 64, NG = 4; };
template <> struct Fmt<WF_AFF8> { static constexpr int KS = 128, GK = 64, NG = 2; };

constexpr int QG_CW = 4;                   // consumer warps
constexpr int QG_ROWS = 16 * QG_CW;        // weight rows per tile
constexpr int QG_THREADS = 32 * (QG_CW + 1);
constexpr int QG_MIN_CTAS = 3;             // CTAs per SM the shared memory is sized for
constexpr int QG_SMEM_BUDGET = 72 * 1024;  // stage ring bytes per CTA

// x-row chunk descriptor (device list for MoE, implicit for dense)
struct QChunk {
  int32_t mat;   // weight matrix index (expert); row base = mat * N
  int32_t xrow;  // first x row
  int32_t ntok;  // valid x rows
  int32_t orow;  // output row / pair base
};

struct QParams {
  const uint8_t *scale[2];     // FP4 / FP8B scale bytes per matrix
  const uint16_t *aff_s;       // affine bf16 scales [N, K/64]
  const uint16_t *aff_b;       // affine bf16 biases
  int64_t N, K;
  int64_t sld;                 // scale row stride in elements
  int svec;                    // scale rows are NG-aligned and K % KS == 0: vector loads
  int spack;                   // FP4: scales in the decode-packed layout (k_pack_decode_sf):
                               // one 512-byte block [64 rows][8 groups] per (row tile, stage)
  int tiles;                   // ceil(N / QG_ROWS); ceil(N / (2 * QG_ROWS)) with rowpair
  int rowpair;                 // NMAT = 2 over ONE matrix: "matrix" m of tile t is the 64-row
                               // tile 2t + m (wmap1 = wmap0, scale[1] = scale[0]); needs
                               // spack, N % (2 * QG_ROWS) == 0 and EPI_DOWN
  int nsplit;
  int kstages;                 // ceil(K / KS)
  const float *xscale;         // per x row multiplier (power of two), or null
  const float *xsum;           // affine: [xrows, K/64] sums of the f16 x values
  const QChunk *chunks;        // null -> dense
  const int *nchunks_dev;
  int nchunks_host;            // dense: number of chunks
  int dense_m;                 // dense: total x rows (tokens for dense_down)
  int dense_rows;              // dense: x rows per chunk (NT*8)
  int dense_down;              // dense: x rows are hi/lo H rows of dense_rows/2 tokens
  int epi;
  void *out;
  int64_t ldo;
  const int32_t *pair_row;     // EPI_DOWN: pair -> output row (null = identity below npairs)
  int npairs;
  float limit;
  int round_gu;                // SWIGLU: round gate/up to bf16 first
  int round_h;                 // SWIGLU: round h to bf16 (shared expert, port)
  int round_out;               // DOWN: round output to bf16 (stored as f32)
  float *partial;              // split-K fragments
  int *counters;               // split-K tickets, zero on entry
  int pdl_early;               // dense: launched as a programmatic dependent of the activation
                               // prep, the producer issues its first item's weight copies (and
                               // scale copies) before waiting for that kernel; only the
                               // activation copies wait
};

__device__ __forceinline__ int rhoA(int g) { return ((g & 3) << 1) | (g >> 2); }  // 0,2,4,6,1,3,5,7
__device__ __forceinline__ int rhoB(int g) { return ((g & 1) << 2) | (g >> 1); }  // 0,4,1,5,2,6,3,7

// Which smem row (mod 8) an mma row g reads, per format: chosen so that the
// warp's shared-memory loads of one group hit distinct banks (LDS.32 for fp4,
// LDS.64 pairs of 16-byte chunks for fp8/aff4, LDS.128 chunks for aff8).
template <int WF> __device__ __forceinline__ int wrow_perm(int g) {
  return WF == WF_AFF8 ? rhoB(g) : rhoA(g);
}
// Which x row (within an n8 tile) mma column c reads.  fp4/fp8 use rhoB (one
// LDS.128 per group; columns 2t / 2t+1 then hold slots t / 4+t, which the
// down-projection epilogue relies on), affine uses the identity (two LDS.128).
template <int WF> __device__ __forceinline__ int xcol_perm(int c) {
  return (WF == WF_AFF4 || WF == WF_AFF8) ? c : rhoB(c);
}

// Shared-memory reads of the stage data as plain C++ loads from the dynamic shared array
// (every extern __shared__ array names its base), so the compiler may overlap one scale
// group's loads with the previous group's MMAs; the mbarrier wait before a stage and the
// arrive after it carry "memory" clobbers, so no load crosses either.
extern __shared__ __align__(1024) uint8_t qg_dyn_smem[];
__device__ __forceinline__ const uint8_t *qg_sptr(uint32_t a) {
  return qg_dyn_smem + (a - static_cast<uint32_t>(__cvta_generic_to_shared(qg_dyn_smem)));
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  return *reinterpret_cast<const uint32_t *>(qg_sptr(a));
}
__device__ __forceinline__ uint2 lds64(uint32_t a) { return *reinterpret_cast<const uint2 *>(qg_sptr(a)); }
__device__ __forceinline__ uint4 lds128(uint32_t a) { return *reinterpret_cast<const uint4 *>(qg_sptr(a)); }
__device__ __forceinline__ float4 lds128f(uint32_t a) {
  return *reinterpret_cast<const float4 *>(qg_sptr(a));
}
__device__ __forceinline__ float2 lds64f(uint32_t a) {
  return *reinterpret_cast<const float2 *>(qg_sptr(a));
}
__device__ __forceinline__ void sts128f(uint32_t a, float x, float y, float z, float w) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w)
               : "memory");
}
__device__ __forceinline__ void sts64f(uint32_t a, float x, float y) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(x), "f"(y) : "memory");
}

// affine magic decode: f16x2 (1024 + q) - 1024 = exact q
__device__ __forceinline__ uint32_t aff_pair(uint32_t bits) {
  uint32_t v = bits | 0x64006400u;
  __half2 h = __hsub2(*reinterpret_cast<__half2 *>(&v), __halves2half2(__ushort_as_half(0x6400),
                                                                         __ushort_as_half(0x6400)));
  return *reinterpret_cast<uint32_t *>(&h);
}

// ue8m0 byte (in the low 8 bits) -> 2^(b-127), with b = 0 applied as 0
__device__ __forceinline__ float e8m0_fast(uint32_t b) { return __uint_as_float((b & 0xFFu) << 23); }

template <int WF, int NMAT, int NT>
struct QCfg {
  static constexpr int KS = Fmt<WF>::KS;
  static constexpr int NG = Fmt<WF>::NG;
  static constexpr bool AFF = (WF == WF_AFF4 || WF == WF_AFF8);
  static constexpr int NBOX = KS / 64;                       // x boxes per stage
  static constexpr int W_BYTES = QG_ROWS * 128;              // per matrix per stage
  static constexpr int XBOX_BYTES = NT * 8 * 128;            // max rows
  static constexpr int TILE_BYTES = NMAT * W_BYTES + NBOX * XBOX_BYTES;   // 1024-multiple
  // raw scale operands per stage, as stored in memory:
  //   FP4  u8 [NMAT * 64 rows][NG]            FP8B u8 [NMAT * 2 row blocks][NG]
  //   AFF  bf16 s [64][NG] at 0, bf16 b [64][NG] at B_OFF, fp32 x sums [NT * 8][NG] at X_OFF
  static constexpr int B_OFF = QG_ROWS * NG * 2;
  static constexpr int X_OFF = 2 * QG_ROWS * NG * 2;
  static constexpr int SC_RAW =
      WF == WF_FP4 ? NMAT * QG_ROWS * NG : (WF == WF_FP8B ? NMAT * 2 * NG : X_OFF + NT * 8 * NG * 4);
  static constexpr int SC_BYTES = (SC_RAW + 127) / 128 * 128;
  static constexpr int STAGES_RAW = QG_SMEM_BUDGET / (TILE_BYTES + SC_BYTES);
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
  static constexpr int SMEM = STAGES * (TILE_BYTES + SC_BYTES) + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int FRAG = NMAT * NT * 4;                 // fp32 per consumer thread
  // scale rows each producer lane converts per stage
  static constexpr int PRODUCER_ITEMS =
      WF == WF_FP4 ? NMAT * QG_ROWS / 32 : (WF == WF_FP8B ? 1 : 3);
};

// Work item -> (chunk, row tile, K split) and the chunk's descriptor.  In list form the
// descriptor comes from `pre`, which the caller loaded one item ahead (chunk_prefetch), so
// no item waits on a dependent global load before its first stage.
__device__ __forceinline__ void decode_chunk(const QParams &p, int item, int &chunk, int &tile,
                                             int &split, QChunk &c, const QChunk &pre) {
  const int per_chunk = p.tiles * p.nsplit;
  chunk = item / per_chunk;
  const int rem = item % per_chunk;
  tile = rem / p.nsplit;
  split = rem % p.nsplit;
  if (p.chunks) {
    c = pre;
  } else if (!p.dense_down) {
    c.mat = 0;
    c.xrow = chunk * p.dense_rows;
    c.ntok = min(p.dense_rows, p.dense_m - c.xrow);
    c.orow = c.xrow;
  } else {
    // H rows of tokens q0 .. q0 + dense_rows/2: hi/lo halves in blocks of 4 tokens
    const int per = p.dense_rows / 2;
    const int q0 = chunk * per;
    const int nt = min(per, p.dense_m - q0);
    c.mat = 0;
    c.xrow = 2 * q0;
    c.ntok = 8 * ((nt + 3) / 4);
    c.orow = q0;
  }
}

__device__ __forceinline__ void chunk_prefetch(const QParams &p, int item, int nitems, QChunk &pre) {
  if (p.chunks && item < nitems) pre = p.chunks[item / (p.tiles * p.nsplit)];
}

// ------------------------------------------------------------------ producer scale staging
// Raw scale words one producer lane fetches for one stage (registers), then
// converts to fp32 into the stage's scale area.
template <int WF, int NMAT, int NT>
struct ScaleRaw {
  using C = QCfg<WF, NMAT, NT>;
  uint32_t w[C::PRODUCER_ITEMS][C::AFF ? 4 : (C::NG / 4 > 0 ? C::NG / 4 : 1)];
};

template <int WF, int NMAT, int NT>
__device__ __forceinline__ void scales_fetch(const QParams &p, const QChunk &c, int64_t nbase, int ks,
                                             int lane, ScaleRaw<WF, NMAT, NT> &r) {
  using C = QCfg<WF, NMAT, NT>;
  constexpr int NG = C::NG;
  constexpr int GK = Fmt<WF>::GK;
  if constexpr (WF == WF_FP4) {
    // lane handles (mat, row) = items j: idx = lane + 32 j over NMAT x 64 rows
#pragma unroll
    for (int j = 0; j < C::PRODUCER_ITEMS; ++j) {
      const int idx = lane + 32 * j, m = idx / QG_ROWS, row = idx % QG_ROWS;
      const bool ok = nbase + row < p.N;
      const uint8_t *sp = p.scale[m] + ((int64_t)c.mat * p.N + nbase + row) * p.sld + (int64_t)ks * NG;
      if (p.svec) {
        const uint2 v = ok ? __ldg(reinterpret_cast<const uint2 *>(sp)) : make_uint2(0, 0);
        r.w[j][0] = v.x;
        r.w[j][1] = v.y;
      } else {
        uint32_t v0 = 0, v1 = 0;
#pragma unroll
        for (int q = 0; q < NG; ++q) {
          const bool in = ok && (int64_t)(ks * NG + q) * GK < p.K;
          const uint32_t b = in ? __ldg(sp + q) : 0u;
          if (q < 4) v0 |= b << (8 * q);
          else v1 |= b << (8 * (q - 4));
        }
        r.w[j][0] = v0;
        r.w[j][1] = v1;
      }
    }
  } else if constexpr (WF == WF_FP8B) {
    // lanes 0 .. 2*NMAT-1: (mat, row block) -> NG = 4 bytes
    if (lane < 2 * NMAT) {
      const int m = lane >> 1, rbl = lane & 1;
      const int64_t rb = (int64_t)c.mat * ((p.N + 31) / 32) + ((nbase >> 5) + rbl);
      const bool ok = nbase + 32 * rbl < p.N;
      const uint8_t *sp = p.scale[m] + rb * p.sld + (int64_t)ks * NG;
      uint32_t v = 0;
      if (ok && p.svec) {
        v = __ldg(reinterpret_cast<const uint32_t *>(sp));
      } else if (ok) {
#pragma unroll
        for (int q = 0; q < NG; ++q)
          if ((int64_t)(ks * NG + q) * GK < p.K) v |= uint32_t(__ldg(sp + q)) << (8 * q);
      }
      r.w[0][0] = v;
    }
  } else {
    // rows lane, lane + 32: NG bf16 scales and biases; item 2: x sums for x row `lane`
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = lane + 32 * j;
      const bool ok = nbase + row < p.N;
      const int64_t o = ((int64_t)c.mat * p.N + nbase + row) * p.sld + (int64_t)ks * NG;
#pragma unroll
      for (int q = 0; q < 4; ++q) r.w[j][q] = 0;
      if (ok) {
        // NG bf16 -> NG/2 words each for s and b (NG = 4: 2 + 2 words, NG = 2: 1 + 1)
        if (p.svec) {
          if (NG == 4) {
            const uint2 s = __ldg(reinterpret_cast<const uint2 *>(p.aff_s + o));
            const uint2 b = __ldg(reinterpret_cast<const uint2 *>(p.aff_b + o));
            r.w[j][0] = s.x; r.w[j][1] = s.y; r.w[j][2] = b.x; r.w[j][3] = b.y;
          } else {
            r.w[j][0] = __ldg(reinterpret_cast<const uint32_t *>(p.aff_s + o));
            r.w[j][2] = __ldg(reinterpret_cast<const uint32_t *>(p.aff_b + o));
          }
        } else {
#pragma unroll
          for (int q = 0; q < NG; ++q) {
            if ((int64_t)(ks * NG + q) * GK >= p.K) continue;
            r.w[j][q >> 1] |= uint32_t(__ldg(p.aff_s + o + q)) << (16 * (q & 1));
            r.w[j][2 + (q >> 1)] |= uint32_t(__ldg(p.aff_b + o + q)) << (16 * (q & 1));
          }
        }
      }
    }
    // x sums: x row slot `lane` (< NT*8), NG floats kept as raw bits
#pragma unroll
    for (int q = 0; q < 4; ++q) r.w[2][q] = 0;
    if (lane < NT * 8 && lane < c.ntok) {
      const float *xp = p.xsum + (int64_t)(c.xrow + lane) * (p.K / 64) + (int64_t)ks * NG;
#pragma unroll
      for (int q = 0; q < NG; ++q)
        if ((int64_t)(ks * NG + q) * GK < p.K) r.w[2][q] = __float_as_uint(__ldg(xp + q));
    }
  }
}

__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void sts64(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
// cp.async of N (4, 8 or 16) bytes; ok = false fills zeros and reads nothing
template <int N>
__device__ __forceinline__ void qg_cp_async(uint32_t dst, const void *src, bool ok) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(dst), "l"(src), "n"(N),
               "r"(ok ? N : 0)
               : "memory");
}
// arrive on `bar` once every cp.async this thread issued so far has landed
__device__ __forceinline__ void qg_cp_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void qg_cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Producer exit: its scale copies and the last ST stages' TMA copies have landed (bounded
// waits on the stages' full barriers), so no copy can arrive after the CTA has exited even
// when the consumers gave up early.  On the normal path those phases completed already.
template <int ST>
__device__ __forceinline__ void qg_drain(uint64_t *full, uint32_t issued, int lane) {
  qg_cp_wait_all();
  if (lane == 0)
    for (uint32_t i = issued > uint32_t(ST) ? issued - ST : 0u; i < issued; ++i)
      mbar_wait(&full[i % ST], (i / ST) & 1);
  __syncwarp();
}
// bulk copy global -> shared (16-byte aligned, size a multiple of 16), completes on `bar`
__device__ __forceinline__ void qg_bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                             uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Ragged shapes: store the synchronously fetched words in the raw layout.
template <int WF, int NMAT, int NT>
__device__ __forceinline__ void scales_raw_store(uint32_t scb, int lane, const ScaleRaw<WF, NMAT, NT> &r) {
  using C = QCfg<WF, NMAT, NT>;
  constexpr int NG = C::NG;
  if constexpr (WF == WF_FP4) {
#pragma unroll
    for (int j = 0; j < C::PRODUCER_ITEMS; ++j) sts64(scb + (lane + 32 * j) * 8, r.w[j][0], r.w[j][1]);
  } else if constexpr (WF == WF_FP8B) {
    if (lane < 2 * NMAT) sts32(scb + lane * 4, r.w[0][0]);
  } else {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = lane + 32 * j;
      if (NG == 4) {
        sts64(scb + row * 8, r.w[j][0], r.w[j][1]);
        sts64(scb + C::B_OFF + row * 8, r.w[j][2], r.w[j][3]);
      } else {
        sts32(scb + row * 4, r.w[j][0]);
        sts32(scb + C::B_OFF + row * 4, r.w[j][2]);
      }
    }
    if (lane < NT * 8) {
      if (NG == 4) sts128(scb + C::X_OFF + lane * 16, r.w[2][0], r.w[2][1], r.w[2][2], r.w[2][3]);
      else sts64(scb + C::X_OFF + lane * 8, r.w[2][0], r.w[2][1]);
    }
  }
}

// Vector shapes: the same bytes by cp.async (rows past N and x rows past the chunk are
// zero-filled); the caller then arrives on the stage's full barrier through qg_cp_arrive.
template <int WF, int NMAT, int NT>
__device__ __forceinline__ void scales_issue(const QParams &p, const QChunk &c, int64_t nbase, int ks,
                                             int lane, uint32_t scb) {
  using C = QCfg<WF, NMAT, NT>;
  constexpr int NG = C::NG;
  if constexpr (WF == WF_FP4) {
#pragma unroll
    for (int j = 0; j < C::PRODUCER_ITEMS; ++j) {
      const int idx = lane + 32 * j, m = idx / QG_ROWS, row = idx % QG_ROWS;
      const bool ok = nbase + row < p.N;
      const uint8_t *sp =
          p.scale[m] + (ok ? ((int64_t)c.mat * p.N + nbase + row) * p.sld + (int64_t)ks * NG : 0);
      qg_cp_async<8>(scb + idx * 8, sp, ok);
    }
  } else if constexpr (WF == WF_FP8B) {
    if (lane < 2 * NMAT) {
      const int m = lane >> 1, rbl = lane & 1;
      const bool ok = nbase + 32 * rbl < p.N;
      const int64_t rb = (int64_t)c.mat * ((p.N + 31) / 32) + ((nbase >> 5) + rbl);
      qg_cp_async<4>(scb + lane * 4, p.scale[m] + (ok ? rb * p.sld + (int64_t)ks * NG : 0), ok);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int row = lane + 32 * j;
      const bool ok = nbase + row < p.N;
      const int64_t o = ok ? ((int64_t)c.mat * p.N + nbase + row) * p.sld + (int64_t)ks * NG : 0;
      qg_cp_async<NG * 2>(scb + row * NG * 2, p.aff_s + o, ok);
      qg_cp_async<NG * 2>(scb + C::B_OFF + row * NG * 2, p.aff_b + o, ok);
    }
    if (lane < NT * 8) {
      const bool ok = lane < c.ntok;
      const float *xp = p.xsum + (ok ? (int64_t)(c.xrow + lane) * (p.K / 64) + (int64_t)ks * NG : 0);
      qg_cp_async<NG * 4>(scb + C::X_OFF + lane * NG * 4, xp, ok);
    }
  }
}

// ue8m0 byte j of a raw word -> fp32 (2^(b-127); b = 0 gives 0)
__device__ __forceinline__ float e8m0_byte(uint32_t w, int j) {
  return __uint_as_float(((w >> (8 * j)) & 0xFFu) << 23);
}
// bf16 half j of a raw word -> fp32
__device__ __forceinline__ float bf16_half(uint32_t w, int j) {
  return __uint_as_float(j ? (w & 0xFFFF0000u) : (w << 16));
}

// ------------------------------------------------------------------ the kernel
template <int WF, int NMAT, int NT>
__global__ void __launch_bounds__(QG_THREADS, QG_MIN_CTAS)
    k_qgemv(const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
            const __grid_constant__ CUtensorMap xmap8, const __grid_constant__ CUtensorMap xmap16,
            const __grid_constant__ CUtensorMap xmap32, const QParams p) {
  using C = QCfg<WF, NMAT, NT>;
  constexpr int KS = C::KS, NG = C::NG, ST = C::STAGES;
  constexpr bool AFF = C::AFF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  uint8_t *sc_ring = smem + ST * C::TILE_BYTES;                      // ST x SC_BYTES
  uint64_t *full = reinterpret_cast<uint64_t *>(sc_ring + ST * C::SC_BYTES);
  uint64_t *empty = full + ST;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // set by the first warp whose bounded wait ran out: the others then give up at their
  // next wait, and consumer warps that gave up keep taking part in the split-K barriers, so
  // no warp is left at a barrier that another warp never reaches
  __shared__ volatile int s_abort;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 33);     // TMA tx arrival + one scale-store arrival per producer lane
      mbar_init(&empty[s], QG_CW);
    }
    fence_barrier_init();
    prefetch_tmap(&wmap0);
    if (NMAT == 2) prefetch_tmap(&wmap1);
  }
  __syncthreads();
  // Dense lists launched with pdl_early: the producer issues its first item's weight copies
  // before waiting for the previous kernel (the weights are not written by it); everything
  // else waits first -- the plan, activations and split-K state come from earlier kernels.
  // Not for the affine formats: their stage copies carry the activations' group sums too.
  const bool early = p.pdl_early && !p.chunks && !AFF;
  if (!early || warp != QG_CW) pdl_wait();
  pdl_trigger();
  const int nchunks = p.chunks ? *p.nchunks_dev : p.nchunks_host;
  const int nitems = nchunks * p.tiles * p.nsplit;

  if (warp == QG_CW) {
    // ---------------------------------------------------------------- producer warp
    if (lane == 0) {
      prefetch_tmap(&wmap0);
      if (NMAT == 2) prefetch_tmap(&wmap1);
    }
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    uint32_t it = 0;
    const uint32_t sc0 = smem_u32(sc_ring);
    const bool packed = WF == WF_FP4 && p.spack;
    // a stage's weight side: the barrier's byte count (weights, scales, activations), the weight
    // tiles and the scale copies (whose arrivals complete the barrier's count)
    auto issue_w = [&](int slot, int ks, const QChunk &c, int64_t nbase, int32_t wrow,
                       int32_t wrow1, int64_t sblk, uint32_t bytes) {
      uint8_t *st = smem + slot * C::TILE_BYTES;
      const uint32_t scb = sc0 + slot * C::SC_BYTES;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[slot], bytes + (packed ? NMAT * QG_ROWS * 8 : 0));
        if (WF == WF_FP4 && packed) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const int64_t blk = p.rowpair ? 2 * sblk + m : sblk;
            qg_bulk_load(scb + m * QG_ROWS * 8, p.scale[m] + (blk * p.kstages + ks) * (QG_ROWS * 8),
                         QG_ROWS * 8, &full[slot]);
          }
        }
        tma_load_2d(st, &wmap0, &full[slot], ks * 128, wrow, pol_w);
        if (NMAT == 2) tma_load_2d(st + C::W_BYTES, &wmap1, &full[slot], ks * 128, wrow1, pol_w);
      }
      if (packed) {
        mbar_arrive(&full[slot]);        // the scales came with the stage's bulk copies
      } else if (p.svec) {
        scales_issue<WF, NMAT, NT>(p, c, nbase, ks, lane, scb);
        qg_cp_arrive(&full[slot]);       // every lane: arrives when its copies land
      } else {
        ScaleRaw<WF, NMAT, NT> raw;
        scales_fetch<WF, NMAT, NT>(p, c, nbase, ks, lane, raw);
        scales_raw_store<WF, NMAT, NT>(scb, lane, raw);
        mbar_arrive(&full[slot]);        // every lane: its scale stores are in
      }
    };
    auto issue_x = [&](int slot, int ks, const QChunk &c, const CUtensorMap *xm) {
      if (lane == 0) {
        uint8_t *st = smem + slot * C::TILE_BYTES;
#pragma unroll
        for (int b = 0; b < C::NBOX; ++b)
          tma_load_2d(st + NMAT * C::W_BYTES + b * C::XBOX_BYTES, xm, &full[slot],
                      ks * KS + b * 64, c.xrow, pol_x);
      }
    };
    QChunk pre{};
    chunk_prefetch(p, blockIdx.x, nitems, pre);
    uint32_t npre = 0;                 // stages of the first item whose weight side is issued
    bool first = true;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
      int chunk, tile, split;
      QChunk c;
      decode_chunk(p, item, chunk, tile, split, c, pre);
      chunk_prefetch(p, item + gridDim.x, nitems, pre);      // used by the next item
      const int kb = int((int64_t)p.kstages * split / p.nsplit);
      const int ke = int((int64_t)p.kstages * (split + 1) / p.nsplit);
      const int xr = c.ntok <= 8 ? 8 : (c.ntok <= 16 ? 16 : 32);
      const CUtensorMap *xm = xr == 8 ? &xmap8 : (xr == 16 ? &xmap16 : &xmap32);
      const uint32_t bytes = NMAT * C::W_BYTES + C::NBOX * xr * 128;
      const int64_t nbase = (int64_t)tile * QG_ROWS * (p.rowpair ? 2 : 1);
      const int32_t wrow = int32_t(c.mat * p.N + nbase);
      const int32_t wrow1 = wrow + (p.rowpair ? QG_ROWS : 0);     // matrix 1's first row
      // packed scale blocks are per 64-row tile: rowpair tile t holds tiles 2t and 2t + 1
      const int64_t sblk = (int64_t)c.mat * p.tiles + tile;
      if (first && early) {
        // the first ST stages' slots are free: their weight side goes out now, the
        // activations after the previous kernel has finished
        npre = uint32_t(min(ST, ke - kb));
        for (uint32_t i = 0; i < npre; ++i)
          issue_w(int(i), kb + int(i), c, nbase, wrow, wrow1, sblk, bytes);
        pdl_wait();
      }
      first = false;
      for (int ks = kb; ks < ke; ++ks, ++it) {
        const int slot = it % ST;
        const uint32_t ph = (it / ST) & 1;
        if (it >= npre) {
          bool ok = true;
          if (lane == 0) ok = mbar_wait_or_abort(&empty[slot], ph ^ 1, &s_abort);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            s_abort = 1;
            qg_drain<ST>(full, it, lane);   // no copy may land after the CTA is gone
            return;
          }
          issue_w(slot, ks, c, nbase, wrow, wrow1, sblk, bytes);
        }
        issue_x(slot, ks, c, xm);
      }
    }
    if (early && first) pdl_wait();      // a CTA without items still waits (no early exit race)
    qg_drain<ST>(full, it, lane);
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int g = lane >> 2, t = lane & 3;
  const int ra = wrow_perm<WF>(g);                // smem row (mod 8) of mma rows g, g+8
  const int rowA = warp * 16 + ra;                // tile rows rowA, rowA + 8
  const int xb = xcol_perm<WF>(g);                // x smem row (mod 8) for mma column g
  const int cs[2] = {xcol_perm<WF>(2 * t), xcol_perm<WF>(2 * t + 1)};  // slots of my columns
  uint32_t it = 0;
  bool dead = false;                // this warp's wait ran out (warp-uniform)

  QChunk pre{};
  chunk_prefetch(p, blockIdx.x, nitems, pre);
  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    int chunk, tile, split;
    QChunk c;
    decode_chunk(p, item, chunk, tile, split, c, pre);
    chunk_prefetch(p, item + gridDim.x, nitems, pre);        // used by the next item
    const int kb = int((int64_t)p.kstages * split / p.nsplit);
    const int ke = int((int64_t)p.kstages * (split + 1) / p.nsplit);
    const int64_t nbase = (int64_t)tile * QG_ROWS * (p.rowpair ? 2 : 1);   // row in the matrix
    const int ntiles_x = (c.ntok + 7) / 8;                      // active n8 tiles
    float acc[NMAT][NT][4];
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][n][i] = 0.0f;

    for (int ks = kb; ks < ke; ++ks, ++it) {
      const int slot = it % ST;
      const uint32_t ph = (it / ST) & 1;
      if (!dead) {
        bool ok = mbar_wait_or_abort(&full[slot], ph, &s_abort);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          dead = true;
          s_abort = 1;
        }
      }
      if (dead) continue;           // no data, no compute; barriers below are still met
      const uint32_t st = smem_u32(smem + slot * C::TILE_BYTES);
      const uint32_t xst = st + NMAT * C::W_BYTES;
      const uint32_t scb = smem_u32(sc_ring + slot * C::SC_BYTES);

      // this stage's raw scale words for my rows (one vector load per row)
      uint32_t rs[NMAT][2][2];        // FP4: [mat][h] 8 bytes; FP8B: [mat] 4 bytes; AFF: s [h]
      uint32_t rb[2][2];              // AFF: biases [h]
      if constexpr (WF == WF_FP4) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint2 v = lds64(scb + (m * QG_ROWS + rowA + 8 * h) * 8);
            rs[m][h][0] = v.x;
            rs[m][h][1] = v.y;
          }
      } else if constexpr (WF == WF_FP8B) {
#pragma unroll
        for (int m = 0; m < NMAT; ++m) rs[m][0][0] = lds32(scb + (m * 2 + (warp >> 1)) * 4);
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t r = rowA + 8 * h;
          if (NG == 4) {
            const uint2 sv = lds64(scb + r * 8), bv = lds64(scb + C::B_OFF + r * 8);
            rs[0][h][0] = sv.x; rs[0][h][1] = sv.y;
            rb[h][0] = bv.x; rb[h][1] = bv.y;
          } else {
            rs[0][h][0] = lds32(scb + r * 4);
            rb[h][0] = lds32(scb + C::B_OFF + r * 4);
            rs[0][h][1] = 0u;
            rb[h][1] = 0u;
          }
        }
      }
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) {
        constexpr int STEPS = Fmt<WF>::GK / 16;
        // ---- this group's scale operands ----
        float sc[NMAT][2];
        float bi[2];
        float xs[NT][2];
        if constexpr (WF == WF_FP4) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) sc[m][h] = e8m0_byte(rs[m][h][grp >> 2], grp & 3);
        } else if constexpr (WF == WF_FP8B) {
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            const float v = e8m0_byte(rs[m][0][0], grp);
            sc[m][0] = v;
            sc[m][1] = v;
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            sc[0][h] = bf16_half(rs[0][h][grp >> 1], grp & 1);
            bi[h] = bf16_half(rb[h][grp >> 1], grp & 1);
          }
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int j = 0; j < 2; ++j)
              xs[n][j] = __uint_as_float(lds32(scb + C::X_OFF + ((n * 8 + cs[j]) * NG + grp) * 4));
        }
        // ---- A fragments: [mat][step][4 regs] ----
        uint32_t a[NMAT][STEPS][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          const uint32_t wb = st + m * C::W_BYTES;
          const uint32_t r0 = wb + rowA * 128, r1 = wb + (rowA + 8) * 128;
          if constexpr (WF == WF_FP4) {
            const uint32_t off = (uint32_t(grp ^ ra) << 4) + 4 * t;
            const uint32_t w0 = lds32(r0 + off), w1 = lds32(r1 + off);
            uint32_t h0[4], h1[4];
            e2m1x8_to_f16x8(w0, h0[0], h0[1], h0[2], h0[3]);
            e2m1x8_to_f16x8(w1, h1[0], h1[1], h1[2], h1[3]);
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              a[m][s2][0] = h0[2 * s2];
              a[m][s2][1] = h1[2 * s2];
              a[m][s2][2] = h0[2 * s2 + 1];
              a[m][s2][3] = h1[2 * s2 + 1];
            }
          } else if constexpr (WF == WF_FP8B) {
            const uint32_t off = (uint32_t((2 * grp + (t >> 1)) ^ ra) << 4) + 8 * (t & 1);
            const uint2 w0 = lds64(r0 + off), w1 = lds64(r1 + off);
            uint32_t h0[4], h1[4];
            e4m3x4_to_f16x4(w0.x, h0[0], h0[1]);
            e4m3x4_to_f16x4(w0.y, h0[2], h0[3]);
            e4m3x4_to_f16x4(w1.x, h1[0], h1[1]);
            e4m3x4_to_f16x4(w1.y, h1[2], h1[3]);
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              a[m][s2][0] = h0[2 * s2];
              a[m][s2][1] = h1[2 * s2];
              a[m][s2][2] = h0[2 * s2 + 1];
              a[m][s2][3] = h1[2 * s2 + 1];
            }
          } else if constexpr (WF == WF_AFF4) {
            const uint32_t off = (uint32_t((2 * grp + (t >> 1)) ^ ra) << 4) + 8 * (t & 1);
            const uint2 w0 = lds64(r0 + off), w1 = lds64(r1 + off);
            const uint32_t wr0[2] = {w0.x, w0.y}, wr1[2] = {w1.x, w1.y};
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2) {
              const uint32_t u0 = wr0[s2 >> 1] >> (8 * (s2 & 1));
              const uint32_t u1 = wr1[s2 >> 1] >> (8 * (s2 & 1));
              a[m][s2][0] = aff_pair(u0 & 0x000F000Fu);
              a[m][s2][1] = aff_pair(u1 & 0x000F000Fu);
              a[m][s2][2] = aff_pair((u0 >> 4) & 0x000F000Fu);
              a[m][s2][3] = aff_pair((u1 >> 4) & 0x000F000Fu);
            }
          } else {  // WF_AFF8
            const uint32_t off = (uint32_t((4 * grp + t) ^ ra) << 4);
            const uint4 w0 = lds128(r0 + off), w1 = lds128(r1 + off);
            const uint32_t wr0[4] = {w0.x, w0.y, w0.z, w0.w}, wr1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int s2 = 0; s2 < 4; ++s2) {
              a[m][s2][0] = aff_pair(wr0[s2] & 0x00FF00FFu);
              a[m][s2][1] = aff_pair(wr1[s2] & 0x00FF00FFu);
              a[m][s2][2] = aff_pair((wr0[s2] >> 8) & 0x00FF00FFu);
              a[m][s2][3] = aff_pair((wr1[s2] >> 8) & 0x00FF00FFu);
            }
          }
        }
        // ---- B fragments and MMA per n8 tile ----
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (n >= ntiles_x) break;
          const int xr = n * 8 + xb;                 // x smem row
          uint32_t b[STEPS][2];
          if constexpr (Fmt<WF>::GK == 32) {
            const uint32_t box = xst + (grp >> 1) * C::XBOX_BYTES;
            const uint32_t off = (uint32_t(((grp & 1) * 4 + t) ^ (xr & 7)) << 4);
            const uint4 v = lds128(box + xr * 128 + off);
            b[0][0] = v.x; b[0][1] = v.y; b[1][0] = v.z; b[1][1] = v.w;
          } else {
            const uint32_t box = xst + grp * C::XBOX_BYTES;
            const uint4 v0 = lds128(box + xr * 128 + (uint32_t((2 * t) ^ (xr & 7)) << 4));
            const uint4 v1 = lds128(box + xr * 128 + (uint32_t((2 * t + 1) ^ (xr & 7)) << 4));
            b[0][0] = v0.x; b[0][1] = v0.y; b[1][0] = v0.z; b[1][1] = v0.w;
            b[2][0] = v1.x; b[2][1] = v1.y; b[3][0] = v1.z; b[3][1] = v1.w;
          }
#pragma unroll
          for (int m = 0; m < NMAT; ++m) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s2 = 0; s2 < STEPS; ++s2)
              mma_f16(d, a[m][s2][0], a[m][s2][1], a[m][s2][2], a[m][s2][3], b[s2][0], b[s2][1]);
            // fold the group scale (and the affine bias times the group's x sum)
            acc[m][n][0] = __fmaf_rn(d[0], sc[m][0], acc[m][n][0]);
            acc[m][n][1] = __fmaf_rn(d[1], sc[m][0], acc[m][n][1]);
            acc[m][n][2] = __fmaf_rn(d[2], sc[m][1], acc[m][n][2]);
            acc[m][n][3] = __fmaf_rn(d[3], sc[m][1], acc[m][n][3]);
            if constexpr (AFF) {
              acc[m][n][0] = __fmaf_rn(bi[0], xs[n][0], acc[m][n][0]);
              acc[m][n][1] = __fmaf_rn(bi[0], xs[n][1], acc[m][n][1]);
              acc[m][n][2] = __fmaf_rn(bi[1], xs[n][0], acc[m][n][2]);
              acc[m][n][3] = __fmaf_rn(bi[1], xs[n][1], acc[m][n][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---------------------------------------------------------------- split-K fixup
    // Each split stores its fragment as float4s ([tile][split][thread][FRAG]); after the
    // CTA barrier one thread's acq_rel ticket both publishes the CTA's stores (release is
    // cumulative over the barrier) and, for the last split, acquires every other split's.
    // The last split then sums the fragments in split order, all of a split's vectors in
    // flight at once -- the same fp32 additions, in the same order, for every launch.
    if (p.nsplit > 1) {
      const int tile_id = chunk * p.tiles + tile;
      const int ctid = threadIdx.x;                        // 0 .. 32*QG_CW-1
      constexpr int CT = 32 * QG_CW;
      constexpr int NV = NMAT * NT;                        // float4s per thread
      float4 *base = reinterpret_cast<float4 *>(p.partial) + (int64_t)tile_id * p.nsplit * (CT * NV);
      float4 *mine = base + (int64_t)split * (CT * NV) + ctid * NV;
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n)
          __stcg(mine + m * NT + n, make_float4(acc[m][n][0], acc[m][n][1], acc[m][n][2], acc[m][n][3]));
      asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
      __shared__ int s_last;
      if (ctid == 0) {
        int prev;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(p.counters + tile_id)
                     : "memory");
        s_last = (prev == p.nsplit - 1);
        if (s_last) p.counters[tile_id] = 0;               // ready for the next call
      }
      asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
      const int last = s_last;
      asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");  // s_last reused next item
      if (!last) continue;
      float4 v[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 *src = base + ctid * NV;
#pragma unroll 4
      for (int sp = 0; sp < p.nsplit; ++sp) {
        float4 t[NV];
#pragma unroll
        for (int k = 0; k < NV; ++k) t[k] = __ldcg(src + (int64_t)sp * (CT * NV) + k);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          v[k].x += t[k].x;
          v[k].y += t[k].y;
          v[k].z += t[k].z;
          v[k].w += t[k].w;
        }
      }
#pragma unroll
      for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          acc[m][n][0] = v[m * NT + n].x;
          acc[m][n][1] = v[m * NT + n].y;
          acc[m][n][2] = v[m * NT + n].z;
          acc[m][n][3] = v[m * NT + n].w;
        }
    }

    // ---------------------------------------------------------------- epilogue
    // acc[m][n][2h + j] is (tile row rowA + 8h, x slot n*8 + cs[j]).
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      if (n >= ntiles_x) break;
      if (p.epi == EPI_DOWN) {
        // H rows of pair q: hi at 8*(q/4) + q%4, lo 4 rows later, so slots t and
        // 4+t of tile n (columns 2t, 2t+1 under rhoB) are the two halves of pair
        // c.orow + 4n + t.
        const int q = c.orow + n * 4 + t;
        const int orow = p.pair_row ? p.pair_row[q] : (q < p.npairs ? q : -1);
        if (orow < 0) continue;
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
          if (m > 0 && !p.rowpair) break;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int64_t nn = nbase + m * QG_ROWS + rowA + 8 * h;
            if (nn >= p.N) continue;
            float v = acc[m][n][2 * h] + acc[m][n][2 * h + 1];
            if (p.round_out) v = round_bf16f(v);
            reinterpret_cast<float *>(p.out)[(int64_t)orow * p.ldo + nn] = v;
          }
        }
        continue;
      }
      if (p.epi == EPI_SWIGLU) {
        // the four outputs (j, h) of this thread are computed together, branch-free, so
        // their exp / divide chains overlap; only the stores are predicated.  silu uses
        // the fast exp and divide (a few ulp; for g below about -88 the quotient is -0).
        float hv[2][2];
        bool ok[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int i = 2 * h + j;
            ok[j][h] = (n * 8 + cs[j] < c.ntok) && (nbase + rowA + 8 * h < p.N);
            const float xsc = (p.xscale && n * 8 + cs[j] < c.ntok) ? p.xscale[c.xrow + n * 8 + cs[j]] : 1.0f;
            float gv = acc[0][n][i] * xsc, uv = acc[NMAT - 1][n][i] * xsc;
            if (p.round_gu) {
              gv = round_bf16f(gv);
              uv = round_bf16f(uv);
            }
            if (p.limit > 0.0f) {
              uv = fminf(fmaxf(uv, -p.limit), p.limit);
              gv = fminf(gv, p.limit);
            }
            float v = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
            if (p.round_h) v = round_bf16f(v);
            hv[j][h] = v;
          }
        __half *H = reinterpret_cast<__half *>(p.out);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int q = c.xrow + n * 8 + cs[j];               // pair (or token) index
          const int64_t hr = 8 * (q >> 2) + (q & 3);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!ok[j][h]) continue;
            const int64_t nn = nbase + rowA + 8 * h;
            const __half hi = __float2half_rn(hv[j][h]);
            const __half lo = __float2half_rn(hv[j][h] - __half2float(hi));
            H[hr * p.ldo + nn] = hi;
            H[(hr + 4) * p.ldo + nn] = lo;
          }
        }
        continue;
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int slotx = n * 8 + cs[j];
        if (slotx >= c.ntok) continue;
        const float xsc = p.xscale ? p.xscale[c.xrow + slotx] : 1.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t nn = nbase + rowA + 8 * h;
          if (nn >= p.N) continue;
          const float v = acc[0][n][2 * h + j] * xsc;
          const int64_t o = (int64_t)(c.orow + slotx) * p.ldo + nn;
          if (p.epi == EPI_STORE_F32)
            reinterpret_cast<float *>(p.out)[o] = v;
          else
            reinterpret_cast<__nv_bfloat16 *>(p.out)[o] = __float2bfloat16_rn(v);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ activation prep
// x bf16 [M, K] -> f16 [M, K] scaled by 2^-E per row (E = floor(log2 amax) - 14,
// so |x| * 2^-E < 2^15), the multiplier 2^E per row, and (affine) per-64 sums
// of the scaled values.  bf16 values are exact in f16 within 2^29 of the row max;
// smaller ones keep an absolute error below 2^-39 of the max.  perm selects the
// per-16 k order the affine decode expects (0 none, 4 aff4, 8 aff8).
// One CTA (256 threads) per row, 16-byte vectors (K % 8 == 0); optional gather:
// row r reads x[gather[r]] (-1 = zero row).
__global__ void __launch_bounds__(256) k_qx_prep(const __nv_bfloat16 *__restrict__ x, int64_t M,
                                                 int64_t K, const int32_t *__restrict__ gather,
                                                 const int *__restrict__ nrows_dev,
                                                 __half *__restrict__ xq, float *__restrict__ xscale,
                                                 float *__restrict__ xsum, int perm,
                                                 int *__restrict__ zero_ctr, int64_t nzero) {
  pdl_wait();
  pdl_trigger();
  const int64_t r = blockIdx.x;
  // the dense GEMV's split-K tickets, zeroed here so that no separate memset precedes it
  if (zero_ctr && r == 0)
    for (int64_t i = threadIdx.x; i < nzero; i += blockDim.x) zero_ctr[i] = 0;
  const int64_t nrows = nrows_dev ? *nrows_dev : M;
  if (r >= nrows) return;
  const int64_t src = gather ? gather[r] : r;
  __shared__ float red[8];
  __shared__ float s_inv;
  const int64_t nv = K / 8;
  const uint4 *xv = reinterpret_cast<const uint4 *>(x + (src >= 0 ? src : 0) * K);
  // the row is read once: a thread's first QXP_R vectors stay in registers for the conversion
  // (all of it for K <= QXP_R * 8 * blockDim.x), any further ones are read again
  constexpr int QXP_R = 4;
  uint4 xr[QXP_R];
  float amax = 0.0f;
  auto absmax = [&](const uint4 &v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      amax = fmaxf(amax, fmaxf(fabsf(bf_bits2f(uint16_t(w[j]))), fabsf(bf_bits2f(uint16_t(w[j] >> 16)))));
  };
#pragma unroll
  for (int k = 0; k < QXP_R; ++k) {
    const int64_t i = threadIdx.x + int64_t(k) * blockDim.x;
    xr[k] = (src >= 0 && i < nv) ? __ldg(xv + i) : make_uint4(0u, 0u, 0u, 0u);
    absmax(xr[k]);
  }
  if (src >= 0)
    for (int64_t i = threadIdx.x + int64_t(QXP_R) * blockDim.x; i < nv; i += blockDim.x)
      absmax(__ldg(xv + i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    int E = 0;
    if (m > 0.0f && m < INFINITY) E = int((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14;
    if (E < -126) E = -126;
    xscale[r] = ldexpf(1.0f, E);
    s_inv = ldexpf(1.0f, -E);                      // exact power of two
  }
  __syncthreads();
  const float inv = s_inv;
  uint4 *qv = reinterpret_cast<uint4 *>(xq + r * K);
  // vector i of the row (zeros for a padding row) -> f16 * 2^-E, in the format's k order
  auto emit = [&](const uint4 &v, int64_t i) {
    float f[8];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = bf_bits2f(uint16_t(w[j])) * inv;
      f[2 * j + 1] = bf_bits2f(uint16_t(w[j] >> 16)) * inv;
    }
    __half h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // destination position inside the 8-vector for the affine k orders:
      // aff4: [0,4,1,5,2,6,3,7] per 8 (the 16-k block order is per half), aff8: [0,2,1,3] per 4
      int dj = j;
      if (perm == 4) dj = ((j & 3) << 1) | (j >> 2);
      else if (perm == 8) dj = (j & 4) | ((j & 1) << 1) | ((j >> 1) & 1);
      h[dj] = __float2half_rn(f[j]);
    }
    qv[i] = *reinterpret_cast<uint4 *>(h);
    if (xsum) {
      // per-64 sums of the f16 values: vectors 8g .. 8g+7 form group g (8 lanes)
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += __half2float(h[j]);
      // the 8 lanes of a group are active together (K % 64 == 0); a warp may be partial
      const unsigned gmask = 0xFFu << (threadIdx.x & 24);
      s += __shfl_xor_sync(gmask, s, 1);
      s += __shfl_xor_sync(gmask, s, 2);
      s += __shfl_xor_sync(gmask, s, 4);
      if ((threadIdx.x & 7) == 0) xsum[r * (K / 64) + i / 8] = s;
    }
  };
#pragma unroll
  for (int k = 0; k < QXP_R; ++k) {
    const int64_t i = threadIdx.x + int64_t(k) * blockDim.x;
    if (i < nv) emit(xr[k], i);
  }
  for (int64_t i = threadIdx.x + int64_t(QXP_R) * blockDim.x; i < nv; i += blockDim.x)
    emit(src >= 0 ? __ldg(xv + i) : make_uint4(0u, 0u, 0u, 0u), i);
}

// ------------------------------------------------------------------ decode scale pack
// FP4 expert scales u8 [rows, G] (G = K / 32 groups per row, rows % 64 == 0, G % 8 == 0) ->
// [rows / 64 tiles][G / 8 stages][64 rows][8 groups]: the scales one decode stage of one
// 64-row tile needs are one contiguous 512-byte block (one bulk copy, whole lines), where the
// row-major layout costs a separate 8-byte request per row and stage.  One thread per block
// row (8 bytes).
__global__ void __launch_bounds__(256) k_pack_decode_sf(const uint8_t *__restrict__ src, int64_t rows,
                                                        int64_t G, uint8_t *__restrict__ dst) {
  const int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;   // (tile, stage, r)
  const int64_t nst = G / 8;
  if (u >= rows * nst) return;
  const int64_t r = u % QG_ROWS, ts = u / QG_ROWS;
  const int64_t tile = ts / nst, stg = ts % nst;
  const uint2 v = __ldg(reinterpret_cast<const uint2 *>(src + (tile * QG_ROWS + r) * G + stg * 8));
  reinterpret_cast<uint2 *>(dst)[u] = v;
}

}  // namespace dsv41
