// bsgemm.cuh -- block-scaled GEMM on the 5th-generation tensor cores (prefill, "a8" mode).
//
// Computes D[n, p] = sum_k W[n, k] * X[p, k] with ue8m0 scales per 32 (or 128) along K on
// both operands, i.e. upstream fp8_gemm / fp4_gemm (docs/reference/kernel.py:207-307,
// :478-591) with the weights as the MMA's A operand (M = 128 weight rows per tile) and the
// fp8 activations as the B operand (N = up to 256 activation rows per tile):
//
//   tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale, scale_vec 1X (one ue8m0 per 32 K)
//   A = fp4 e2m1 (TMA 16U4_ALIGN16B: 16 codes + 8 pad bytes per 16-byte smem chunk) or
//       fp8 e4m3; B = fp8 e4m3; fp32 accumulator in TMEM (256 columns).
//
// One persistent CTA per SM walks a tile list (grouped: one tile = (group, 128 weight rows,
// <= 256 activation rows); the MMA's N shrinks to the tile's rows rounded up to 16, so
// ragged expert groups cost what they use).  Warp roles, 192 threads:
//   warp 0     TMA producer: A/B tiles (128B swizzle) into a 4-stage ring; its 32 lanes
//              stage the scale words into the 32x16-byte layout tcgen05.cp wants
//              (byte l*16 + c*4 + b = scale of row 32c+l, K-block b), fence the async proxy
//              and arrive (full barrier count 33 = expect_tx arrive + 32 lanes);
//   warp 1     TMEM allocator + MMA issuer (lane 0): per stage copy SFA/SFB smem -> TMEM,
//              4 MMAs of K=32 (sf_id = K-block), commit -> empty[stage];
//              after a tile, commit -> acc_full;
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns, transpose through shared memory,
//              vector stores.  Store mode writes fp32/bf16 rows; SwiGLU mode pairs the gate
//              and up halves of the tile (A = 64 gate rows + 64 up rows), applies the clamped
//              SwiGLU, the routing weight and bf16 rounding, then act_quant's per-32 fp8
//              quantization of h (the down projection's input) -- upstream Expert.forward
//              (docs/reference/model.py:841-851) with linear() in a8 form (:181-207).
//
// Every wait is bounded (2 s); on expiry the device status flag is raised and the CTA
// drains its own copies and MMAs before freeing TMEM.  No multicast anywhere.
#pragma once
#include "act_quant.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int BS_BM = 128, BS_BN = 256, BS_BK = 128, BS_STAGES = 4;
constexpr int BS_A_BYTES = BS_BM * BS_BK;      // 16 KB: fp8, or fp4 padded to one byte/code
constexpr int BS_B_BYTES = BS_BN * BS_BK;      // 32 KB
constexpr int BS_SFA_BYTES = 512, BS_SFB_BYTES = 1024;
constexpr int BS_EPI_LD = 36;                  // floats per row of a transposition tile
constexpr int BS_EPI_BYTES = 32 * BS_EPI_LD * 4;
constexpr int BS_OFF_A = 0;
constexpr int BS_OFF_B = BS_OFF_A + BS_STAGES * BS_A_BYTES;
constexpr int BS_OFF_SFA = BS_OFF_B + BS_STAGES * BS_B_BYTES;
constexpr int BS_OFF_SFB = BS_OFF_SFA + BS_STAGES * BS_SFA_BYTES;
constexpr int BS_OFF_EPI = BS_OFF_SFB + BS_STAGES * BS_SFB_BYTES;
constexpr int BS_OFF_BAR = BS_OFF_EPI + 4 * BS_EPI_BYTES;
constexpr int BS_SMEM_BYTES = BS_OFF_BAR + 256 + 1024;   // + barriers + alignment slack
constexpr int BS_THREADS = 192;
constexpr uint32_t BS_TMEM_COLS = 512;
constexpr uint32_t BS_SF_COL0 = 256;           // SF slot s: SFA at 256+16s (4), SFB at +4 (8)
static_assert(BS_SMEM_BYTES <= 232448, "bsgemm shared memory");

enum { BS_W_FP4 = 0, BS_W_FP8 = 1 };
enum { BS_EPI_F32 = 0, BS_EPI_BF16 = 1, BS_EPI_SWIGLU = 2 };

// Scale addressing for one operand: byte (row >> rshift) * ld + (k / kblk), where kblk is 32
// (kshift 0: a u32 word holds the 4 per-32 scales of one 128-wide K stage) or 128 (kshift 2:
// one byte, replicated to the 4 per-32 slots).
struct BsScale {
  const uint8_t *p;
  int64_t ld;
  int rshift;
  int kshift;
  int64_t rows;    // rows of the operand (loads of rows >= rows are skipped)
};

struct BsArgs {
  int nkb;             // K / 128
  int a_rows;          // weight rows of one group (N; I in SwiGLU mode)
  BsScale sw, sw2;     // weight scales (sw2: up projection in SwiGLU mode)
  BsScale sx;          // activation scales
  const int4 *tiles;   // grouped: {group, m-tile, first activation row, rows}; null = dense
  const int *ntiles;   // grouped tile count (device)
  int dense_tiles, dense_nt, dense_rows;
  void *out;           // store mode: out[p * ldo + n]
  int64_t ldo;
  const float *pw;     // SwiGLU: per-row routing weight (null = none)
  uint8_t *hq;         // SwiGLU: fp8 h [rows, ldh]
  uint8_t *hs;         // SwiGLU: ue8m0 scales of h [rows, ldh / 32]
  int64_t ldh;
  float limit;         // SwiGLU clamp (<= 0: none)
};

struct BsMaps {
  CUtensorMap w;       // weights, box {128 K, 128 rows} (64 rows in SwiGLU mode)
  CUtensorMap w2;      // up-projection weights (SwiGLU mode)
  CUtensorMap x[4];    // activations, box {128 K, 32 << i rows}
};

// ------------------------------------------------------------------ tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 rows x 16 bytes of shared memory -> 4 TMEM columns of lanes 0-31, broadcast to all
// four lane quadrants.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
__device__ __forceinline__ void tc_mma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t sfa, uint32_t sfb, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 bytes, 8-row
// groups 1024 bytes apart (SBO), version 1, layout type 2.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// K-major, no swizzle: 16-byte rows, 8-row core matrices 128 bytes apart (the 32x128b
// source of tcgen05.cp).
__device__ __forceinline__ uint64_t sdesc_sf(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t(128 >> 4) << 32) | (uint64_t(1) << 46);
}
// Instruction descriptor of kind::mxf8f6f4: A format (e4m3 0, e2m1 5) bits 7-9, B e4m3,
// K-major both, N>>3 bits 17-22, ue8m0 scales bit 23, M>>4 = 8 bits 24-28, scale-factor id
// of A bits 29-30 and of B bits 4-5.
__device__ __forceinline__ uint32_t idesc_mx(uint32_t a_fmt, uint32_t n, uint32_t sf_id) {
  return (a_fmt << 7) | ((n >> 3) << 17) | (1u << 23) | (8u << 24) | (sf_id << 29) | (sf_id << 4);
}

__device__ __forceinline__ uint32_t bs_scale_word(const BsScale &s, int64_t row, int kb) {
  if (row >= s.rows) return 0x7F7F7F7Fu;   // 1.0: rows past the operand feed discarded columns
  const uint8_t *p = s.p + (row >> s.rshift) * s.ld;
  if (s.kshift == 0) return __ldg(reinterpret_cast<const uint32_t *>(p + 4 * kb));
  return uint32_t(__ldg(p + kb)) * 0x01010101u;
}

__device__ __forceinline__ int4 bs_tile(const BsArgs &a, int t) {
  if (a.tiles) return a.tiles[t];
  const int nt = t % a.dense_nt, mt = t / a.dense_nt;
  const int row0 = nt * BS_BN;
  return make_int4(0, mt, row0, min(BS_BN, a.dense_rows - row0));
}

__device__ __forceinline__ int bs_nmma(int nrows) {
  const int n = (nrows + 15) & ~15;
  return n < 16 ? 16 : (n > BS_BN ? BS_BN : n);
}
__device__ __forceinline__ int bs_box(int nmma) {   // activation box index: 32 << i rows
  return nmma <= 32 ? 0 : nmma <= 64 ? 1 : nmma <= 128 ? 2 : 3;
}

// Bounded wait taken by all 32 lanes; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

template <int WFMT, int EPI>
__global__ void __launch_bounds__(BS_THREADS, 1)
    k_bsgemm(const __grid_constant__ BsMaps maps, const BsArgs args) {
  extern __shared__ uint8_t bs_raw[];
  const uint32_t raw_s = smem_u32(bs_raw);
  uint8_t *smem = bs_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + BS_OFF_BAR);
  uint64_t *full = bars;                    // [4] count 33
  uint64_t *empty = bars + 4;               // [4] count 1 (tcgen05.commit)
  uint64_t *acc_full = bars + 8;            // count 1 (tcgen05.commit)
  uint64_t *acc_empty = bars + 9;           // count 4 (epilogue warps)
  uint64_t *xfull = bars + 10;              // [2] count 32 (SwiGLU pair exchange)
  uint64_t *xempty = bars + 12;             // [2] count 32
  uint64_t *mma_done = bars + 14;           // count 1
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < BS_STAGES; ++s) {
      mbar_init(&full[s], 33);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&xfull[i], 32);
      mbar_init(&xempty[i], 32);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BS_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = args.tiles ? *args.ntiles : args.dense_tiles;
  const int nkb = args.nkb;
  constexpr uint32_t W_TX = WFMT == BS_W_FP4 ? BS_BM * BS_BK / 2 : BS_BM * BS_BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&maps.w);
      if (EPI == BS_EPI_SWIGLU) prefetch_tmap(&maps.w2);
      for (int i = 0; i < 4; ++i) prefetch_tmap(&maps.x[i]);
    }
    const uint64_t pol_w = l2_policy_evict_normal();
    const uint64_t pol_x = l2_policy_evict_last();
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
      const int4 tl = bs_tile(args, t);
      const int nmma = bs_nmma(tl.w), bi = bs_box(nmma);
      const uint32_t x_tx = uint32_t(32 << bi) * BS_BK;
      const int64_t wrow0 = int64_t(tl.x) * args.a_rows +
                            int64_t(tl.y) * (EPI == BS_EPI_SWIGLU ? 64 : BS_BM);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % BS_STAGES;
        const uint32_t ph = uint32_t(it / BS_STAGES) & 1u;
        if (!warp_wait(&empty[s], ph ^ 1u)) {
          ok = false;
          break;
        }
        uint8_t *sa = smem + BS_OFF_A + s * BS_A_BYTES;
        uint8_t *sb = smem + BS_OFF_B + s * BS_B_BYTES;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], W_TX + x_tx);
          if (EPI == BS_EPI_SWIGLU) {
            tma_load_2d(sa, &maps.w, &full[s], kb * BS_BK, int32_t(wrow0), pol_w);
            tma_load_2d(sa + BS_A_BYTES / 2, &maps.w2, &full[s], kb * BS_BK, int32_t(wrow0), pol_w);
          } else {
            tma_load_2d(sa, &maps.w, &full[s], kb * BS_BK, int32_t(wrow0), pol_w);
          }
          tma_load_2d(sb, &maps.x[bi], &full[s], kb * BS_BK, tl.z, pol_x);
        }
        // scale words -> tcgen05.cp layout (row 32c + l at byte l*16 + c*4)
        uint4 va;
        uint32_t *vw = reinterpret_cast<uint32_t *>(&va);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (EPI == BS_EPI_SWIGLU)
            vw[c] = c < 2 ? bs_scale_word(args.sw, wrow0 + 32 * c + lane, kb)
                          : bs_scale_word(args.sw2, wrow0 + 32 * (c - 2) + lane, kb);
          else
            vw[c] = bs_scale_word(args.sw, wrow0 + 32 * c + lane, kb);
        }
        *reinterpret_cast<uint4 *>(smem + BS_OFF_SFA + s * BS_SFA_BYTES + lane * 16) = va;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 vb;
          uint32_t *bw = reinterpret_cast<uint32_t *>(&vb);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            bw[c] = bs_scale_word(args.sx, int64_t(tl.z) + 32 * (4 * h + c) + lane, kb);
          *reinterpret_cast<uint4 *>(smem + BS_OFF_SFB + s * BS_SFB_BYTES + h * 512 + lane * 16) = vb;
        }
        fence_proxy_async_smem();
        mbar_arrive(&full[s]);
      }
    }
    // every copy this warp issued has landed before the CTA can finish
    for (int j = it - BS_STAGES < 0 ? 0 : it - BS_STAGES; j < it; ++j)
      mbar_wait(&full[j % BS_STAGES], uint32_t(j / BS_STAGES) & 1u);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tc) {
        const int4 tl = bs_tile(args, t);
        const int nmma = bs_nmma(tl.w);
        if (!mbar_wait(acc_empty, (uint32_t(tc) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % BS_STAGES;
          const uint32_t ph = uint32_t(it / BS_STAGES) & 1u;
          if (!mbar_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t t_sfa = tmem + BS_SF_COL0 + 16u * s;
          const uint32_t t_sfb = t_sfa + 4u;
          const uint32_t s_sfa = sbase + BS_OFF_SFA + s * BS_SFA_BYTES;
          const uint32_t s_sfb = sbase + BS_OFF_SFB + s * BS_SFB_BYTES;
          tc_cp_sf(t_sfa, sdesc_sf(s_sfa));
          tc_cp_sf(t_sfb, sdesc_sf(s_sfb));
          if (nmma > 128) tc_cp_sf(t_sfb + 4u, sdesc_sf(s_sfb + 512u));
          const uint64_t da = sdesc_sw128(sbase + BS_OFF_A + s * BS_A_BYTES);
          const uint64_t db = sdesc_sw128(sbase + BS_OFF_B + s * BS_B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // +32 bytes along K inside the swizzle atom = +2 in the descriptor's address field
            tc_mma_mx(tmem, da + uint64_t(2 * k), db + uint64_t(2 * k),
                      idesc_mx(WFMT == BS_W_FP4 ? 5u : 0u, uint32_t(nmma), uint32_t(k)),
                      t_sfa | (uint32_t(k) << 30), t_sfb | (uint32_t(k) << 30),
                      (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(acc_full);
      }
      tc_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    float *tp = reinterpret_cast<float *>(smem + BS_OFF_EPI + q * BS_EPI_BYTES);
    int tc = 0, xc = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const int4 tl = bs_tile(args, t);
      const int nmma = bs_nmma(tl.w);
      if (!warp_wait(acc_full, uint32_t(tc) & 1u)) break;
      tc_fence_after();
      const uint32_t tq = tmem + (uint32_t(32 * q) << 16);
      bool ok = true;
      for (int cc = 0; cc * 32 < nmma && ok; ++cc) {
        uint32_t r[32];
        tmem_ld32(tq + uint32_t(cc * 32), r);
        const int64_t p_lane = int64_t(tl.z) + cc * 32 + lane;   // this lane's row after transpose
        const bool live = cc * 32 + lane < tl.w;
        if constexpr (EPI != BS_EPI_SWIGLU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) tp[j * BS_EPI_LD + lane] = __uint_as_float(r[j]);
          __syncwarp();
          if (live) {
            const float4 *src = reinterpret_cast<const float4 *>(tp + lane * BS_EPI_LD);
            const int64_t n0 = int64_t(tl.y) * BS_BM + 32 * q;
            if constexpr (EPI == BS_EPI_F32) {
              float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(args.out) +
                                                       p_lane * args.ldo + n0);
#pragma unroll
              for (int i = 0; i < 8; ++i) dst[i] = src[i];
            } else {
              uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(args.out) +
                                                     p_lane * args.ldo + n0);
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
        } else {
          const int pr = q & 1;
          const uint32_t xph = uint32_t(xc) & 1u;
          const float L = args.limit;
          if (q >= 2) {
            // up half: bf16-round, clamp, hand to the gate warp of the same rows
            if (!warp_wait(&xempty[pr], xph ^ 1u)) {
              ok = false;
              break;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float u = round_bf16f(__uint_as_float(r[j]));
              if (L > 0.0f) u = fminf(fmaxf(u, -L), L);
              tp[j * BS_EPI_LD + lane] = u;
            }
            mbar_arrive(&xfull[pr]);
          } else {
            if (!warp_wait(&xfull[pr], xph)) {
              ok = false;
              break;
            }
            const float *ub = reinterpret_cast<const float *>(smem + BS_OFF_EPI +
                                                              (q + 2) * BS_EPI_BYTES);
            const float wl = (args.pw && live) ? args.pw[p_lane] : 1.0f;
            float h[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float g = round_bf16f(__uint_as_float(r[j]));
              if (L > 0.0f) g = fminf(g, L);
              const float u = ub[j * BS_EPI_LD + lane];
              const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
              float v = __fmul_rn(sg, u);
              if (args.pw) v = __fmul_rn(v, __shfl_sync(0xffffffffu, wl, j));
              h[j] = round_bf16f(v);
            }
            mbar_arrive(&xempty[pr]);
#pragma unroll
            for (int j = 0; j < 32; ++j) tp[j * BS_EPI_LD + lane] = h[j];
            __syncwarp();
            if (live) {
              // act_quant of 32 features of row p_lane (docs/reference/kernel.py:40-95)
              const float *row = tp + lane * BS_EPI_LD;
              float amax = 0.0f;
#pragma unroll
              for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(row[i]));
              amax = fmaxf(amax, 1e-4f);
              const float sc = pow2_ceil_log2(__fmul_rn(amax, 1.0f / 448.0f));
              uint32_t wq[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                uint32_t w = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                  const float y = fminf(fmaxf(__fdiv_rn(row[4 * i + b], sc), -448.0f), 448.0f);
                  w |= uint32_t(f32_to_e4m3_sat(y)) << (8 * b);
                }
                wq[i] = w;
              }
              const int64_t f0 = int64_t(tl.y) * 64 + 32 * q;
              uint4 *dst = reinterpret_cast<uint4 *>(args.hq + p_lane * args.ldh + f0);
              dst[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
              dst[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
              args.hs[p_lane * (args.ldh / 32) + f0 / 32] =
                  uint8_t((__float_as_uint(sc) >> 23) & 0xFF);
            }
            __syncwarp();
          }
          ++xc;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (!ok) break;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BS_TMEM_COLS);
  }
}

}  // namespace dsv41
