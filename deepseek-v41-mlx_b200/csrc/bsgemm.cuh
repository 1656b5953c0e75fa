// bsgemm.cuh -- block-scaled GEMM on the 5th-generation tensor cores (prefill, "a8" mode).
//
// Computes D[n, p] = sum_k W[n, k] * X[p, k] with ue8m0 scales per 32 (or 128) along K on
// both operands, i.e. upstream fp8_gemm / fp4_gemm (docs/reference/kernel.py:207-307,
// :478-591) with the weights as the MMA's A operand (M = 128 weight rows per tile) and the
// fp8 activations as the B operand (N = up to 224 activation rows per tile):
//
//   tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale, scale_vec 1X (one ue8m0 per 32 K)
//   A = fp4 e2m1 (TMA 16U4_ALIGN16B: 16 codes + 8 pad bytes per 16-byte smem chunk) or
//       fp8 e4m3; B = fp8 e4m3; fp32 accumulators in TMEM, double-buffered (2 x 224
//       columns) so that a tile's epilogue overlaps the next tile's MMAs.
//
// One persistent CTA per SM walks a tile list (grouped: one tile = (group, 128 weight rows,
// <= 224 activation rows); the MMA's N shrinks to the tile's rows rounded up to 16, so
// ragged expert groups cost what they use).  Warp roles, 192 threads:
//   warp 0     TMA producer: A/B tiles (128B swizzle) into a 4-stage ring; its 32 lanes
//              copy the scale words (4-byte cp.async, completion tracked by the stage's
//              mbarrier) into the 32x16-byte layout tcgen05.cp wants (byte l*16 + c*4 + b =
//              scale of row 32c+l, K-block b); full barrier count 33 = expect_tx arrive +
//              32 lane arrivals;
//   warp 1     TMEM allocator + MMA issuer (lane 0): per stage copy SFA/SFB smem -> TMEM,
//              4 MMAs of K=32 (sf_id = K-block), commit -> empty[stage];
//              after a tile, commit -> acc_full[buffer];
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns, transpose through shared memory,
//              vector stores.  Store mode writes fp32/bf16 rows; SwiGLU mode pairs the gate
//              and up halves of the tile (A = 64 gate rows + 64 up rows; warps q and q+2
//              hold the same features), applies the clamped SwiGLU (CUDA's __expf and
//              __fdividef), the routing weight and bf16 rounding, then act_quant's per-32
//              fp8 quantization of h (the down projection's input) -- upstream
//              Expert.forward (docs/reference/model.py:841-851) with linear() in a8 form
//              (:181-207).
//
// 2-CTA form (PAIR, wide tiles of grouped lists): clusters of 2 CTAs take m-tiles 2i, 2i + 1
// of one token tile; each CTA loads its weights and half of the activation rows, rank 0
// issues tcgen05.mma.cta_group::2 (M = 256) for both, so each activation byte is read from L2
// once per two m-tiles.
//
// Every wait is bounded (2 s); on expiry the device status flag is raised and the CTA
// drains its own copies and MMAs before freeing TMEM.  No copy is multicast (in the 2-CTA
// form only MMA-completion arrivals reach both CTAs).
#pragma once
#include "act_quant.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int BS_BM = 128, BS_BK = 128, BS_BN = 224, BS_BN_NARROW = 64;
constexpr int BS_THREADS = 192;
constexpr int BS_EPI_LD = 36;                  // floats per row of a transposition tile
constexpr int BS_EPI_BYTES = 32 * BS_EPI_LD * 4;
constexpr int BS_RING = 4;                     // tile-ring slots (producer -> MMA, epilogue)

// Two shapes of the same pipeline.  Wide: up to 224 activation rows per tile, 4 stages of
// 128 K (16 KB of weights + 28 KB of activations) -- the compute-bound shape.  Narrow: up to
// 64 rows, 4 stages of 256 K (32 + 16 KB): the tiles of lightly routed experts only stream
// weights, and a stage that carries two 128-wide K blocks halves the waits and commits the
// single MMA-issuing thread spends per weight byte.
template <bool NARROW, bool PAIR = false>
struct BsCfg {
  static constexpr int BN = NARROW ? BS_BN_NARROW : BS_BN;
  // PAIR (2-CTA MMA): each CTA of the pair holds half of the activation rows, at most 128
  static constexpr int B_ROWS = PAIR ? 128 : BN;
  static constexpr int STAGES = 4;
  static constexpr int KSUB = NARROW ? 2 : 1;            // 128-wide K blocks per stage
  static constexpr int NBOX = NARROW ? 2 : 4;            // activation boxes 32/64(/128/224)
  static constexpr int SFB_CHUNKS = NARROW ? 4 : 8;      // 32-row scale chunks staged
  static constexpr int A_SUB = BS_BM * BS_BK;            // fp8, or fp4 padded to a byte/code
  static constexpr int B_SUB = B_ROWS * BS_BK;
  static constexpr int SFB_SUB = SFB_CHUNKS * 128;
  static constexpr int A_BYTES = KSUB * A_SUB;
  static constexpr int B_BYTES = KSUB * B_SUB;
  static constexpr int SFA_BYTES = KSUB * 512;
  static constexpr int SFB_BYTES = KSUB * SFB_SUB;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_SFB = OFF_SFA + STAGES * SFA_BYTES;
  static constexpr int OFF_EPI = OFF_SFB + STAGES * SFB_BYTES;
  static constexpr int OFF_RING = OFF_EPI + 4 * BS_EPI_BYTES;
  static constexpr int OFF_BAR = OFF_RING + BS_RING * 16;
  static constexpr int SMEM = OFF_BAR + 512 + 1024;     // + barriers + alignment slack
  static constexpr uint32_t TMEM_COLS = NARROW ? 256 : 512;
  static constexpr uint32_t ACC_COLS = BN;               // accumulator b at column b * BN
  static constexpr uint32_t SF_COL0 = 2 * BN;            // SF slot s at SF_COL0 + 16 s
  static constexpr uint32_t SFA_COLS = 4 * KSUB;         // then SFB: 4 columns per atom
  static constexpr uint32_t SFB_ATOMS = SFB_CHUNKS / 4;
  static_assert(SFA_COLS + 4 * KSUB * SFB_ATOMS <= 16, "SF slot");
  static_assert(SF_COL0 + 16 * STAGES <= TMEM_COLS, "TMEM columns");
  static_assert(B_SUB % 1024 == 0 && A_SUB % 1024 == 0, "swizzle atoms");
  static_assert(SMEM <= 232448, "shared memory");
};

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
  int nkb;             // K / 128 (the launcher divides by the stage's K blocks)
  int a_rows;          // weight rows of one group (N; I in SwiGLU mode)
  BsScale sw, sw2;     // weight scales (sw2: up projection in SwiGLU mode)
  BsScale sx;          // activation scales
  const int4 *tiles;   // grouped: {group, m-tile, first activation row, rows | row tile << 8};
                       // null = dense
  const int *ntiles;   // grouped tile count (device)
  int *next_tile;      // grouped: work counter (zeroed before the launch), tiles taken in order
  int dense_tiles, dense_nt, dense_bn, dense_rows;
  void *out;           // store mode: out[p * ldo + n]
  int64_t ldo;
  int sf_async;        // 1: every staged scale operand is per-32 (cp.async staging)
  int nkq;             // K / 128 (scale-atom addressing)
  int mtiles;          // m-tiles per group (weight-atom addressing)
  const uint8_t *sfa_atoms;  // weight scales as tcgen05.cp atoms [group][m-tile][K/128][512]
                             // (null: staged from sw / sw2)
  const uint8_t *sfb_atoms;  // activation scales as atoms [row tile][K/128][2][512]
                             // (null: staged from sx)
  uint8_t *hs_atoms;   // SwiGLU: write h's scales as atoms [row tile][ldh/128][2][512]
  const float *pw;     // SwiGLU: per-row routing weight (null = none)
  uint8_t *hq;         // SwiGLU: fp8 h [rows, ldh]
  uint8_t *hs;         // SwiGLU: ue8m0 scales of h [rows, ldh / 32]
  int64_t ldh;
  float limit;         // SwiGLU clamp (<= 0: none)
};

struct BsMaps {
  CUtensorMap w;       // weights, box {128 K, 128 rows} (64 rows in SwiGLU mode)
  CUtensorMap w2;      // up-projection weights (SwiGLU mode)
  CUtensorMap x[4];    // activations, box {128 K, bs_box_rows(i)}
  CUtensorMap sfa;     // PAIR: weight scale atoms as 256-byte rows, box {256, 2} (one atom)
  CUtensorMap sfb;     // PAIR: activation scale atoms as 256-byte rows, box {256, 4} (two)
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
// The same three issued by one elect.sync lane of a converged warp that runs the issuing
// loop as a whole (warp-uniform operands): measured on B200, back-to-back MMAs of N = 224
// then run at the tensor pipe's rate instead of ~40% slower from a single-lane branch.
__device__ __forceinline__ void tc_cp_sf_el(uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc)
      : "memory");
}
__device__ __forceinline__ void tc_mma_mx_el(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t sfa, uint32_t sfb, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
      : "memory");
}
__device__ __forceinline__ void tc_commit_el(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load_el(uint32_t dst, const void *src, uint32_t bytes,
                                             uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n\t}" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
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
// 4-byte asynchronous copy global -> shared; src_bytes 0 fills zeros.
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
// Bulk copy global -> shared (16-byte aligned, size a multiple of 16), completes on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Byte offset of row r (of a <= 256-row tile), 32-wide K block j, in a tile's scale atoms
// [K/128][2][512]: atom (r / 128) of K stage j / 4, lane r % 32, column (r / 32) % 4, byte j % 4.
__host__ __device__ __forceinline__ int64_t sf_atom_off(int r, int j) {
  return int64_t(j >> 2) * 1024 + (r >> 7) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (j & 3);
}
// Arrive on `bar` (counted in its expected arrivals) once this thread's cp.asyncs landed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
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
__device__ __forceinline__ uint32_t idesc_mx(uint32_t a_fmt, uint32_t n, uint32_t sf_id,
                                             uint32_t m = 128) {
  return (a_fmt << 7) | ((n >> 3) << 17) | (1u << 23) | ((m >> 4) << 24) | (sf_id << 29) |
         (sf_id << 4);
}

// ------------------------------------------------------------------ 2-CTA (CTA pair) helpers
// A pair is a cluster of 2 CTAs; rank 0 issues the M = 256 MMAs for both.  Each CTA loads its
// own operands (no multicast copies); its copies complete on rank 0's stage barrier, rank 0's
// MMA commits arrive on both CTAs' barriers, and rank 1's epilogue releases an accumulator on
// rank 0's barrier by a remote arrival (mapa).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t ncluster_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// the shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_rank(const void *p, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
  return d;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// every thread of both CTAs (a hardware barrier: both CTAs are resident together)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// 2D TMA load into this CTA's shared memory that completes on the barrier at `bar_cluster`
// (rank 0's full barrier), one elected lane
__device__ __forceinline__ void tma_load_2d_pair_el(void *dst, const CUtensorMap *map,
                                                    uint32_t bar_cluster, int32_t x, int32_t y,
                                                    uint64_t policy) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tc_cp_sf_pair_el(uint32_t taddr, uint64_t sdesc) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;\n\t}" ::"r"(taddr),
      "l"(sdesc)
      : "memory");
}
__device__ __forceinline__ void tc_mma_mx_pair_el(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                                  uint32_t sfa, uint32_t sfb, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
      : "memory");
}
// commit of the pair's MMAs to a barrier of this (rank 0) CTA
__device__ __forceinline__ void tc_commit_pair_el(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
// the same commit arriving on the barrier at this offset in both CTAs of the pair (an
// arrival signal, not a copy: no data moves)
__device__ __forceinline__ void tc_commit_pair_both_el(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}

// cp.async of the 4 per-32 scales of (row, K stage kb) to shared address dst.
__device__ __forceinline__ void bs_scale_copy(const BsScale &s, int64_t row, int kb, uint32_t dst) {
  const bool ok = row < s.rows;
  const uint8_t *p = ok ? s.p + (row >> s.rshift) * s.ld + 4 * kb : s.p;
  cp_async4(dst, p, ok ? 4u : 0u);
}

__device__ __forceinline__ uint32_t bs_scale_word(const BsScale &s, int64_t row, int kb) {
  if (row >= s.rows) return 0x7F7F7F7Fu;   // 1.0: rows past the operand feed discarded columns
  const uint8_t *p = s.p + (row >> s.rshift) * s.ld;
  if (s.kshift == 0) return __ldg(reinterpret_cast<const uint32_t *>(p + 4 * kb));
  return uint32_t(__ldg(p + kb)) * 0x01010101u;
}

__device__ __forceinline__ int4 bs_dense_tile(const BsArgs &a, int t) {
  const int nt = t % a.dense_nt, mt = t / a.dense_nt;
  const int row0 = nt * a.dense_bn;
  return make_int4(0, mt, row0, min(a.dense_bn, a.dense_rows - row0) | (nt << 8));
}

template <int BN>
__device__ __forceinline__ int bs_nmma(int nrows) {
  const int n = (nrows + 15) & ~15;
  return n < 16 ? 16 : (n > BN ? BN : n);
}
__device__ __forceinline__ int bs_box(int nmma) {   // activation box index
  return nmma <= 32 ? 0 : nmma <= 64 ? 1 : nmma <= 128 ? 2 : 3;
}
__host__ __device__ constexpr uint32_t bs_box_rows(int i) { return i < 3 ? 32u << i : uint32_t(BS_BN); }

// Bounded wait taken by all 32 lanes; the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

template <int WFMT, int EPI, bool NARROW, bool PAIR = false>
__global__ void __launch_bounds__(BS_THREADS, 1)
    k_bsgemm(const __grid_constant__ BsMaps maps, const BsArgs args) {
  static_assert(!(PAIR && NARROW), "the 2-CTA form is the wide shape");
  using Cfg = BsCfg<NARROW, PAIR>;
  constexpr int S = Cfg::STAGES;
  extern __shared__ uint8_t bs_raw[];
  const uint32_t raw_s = smem_u32(bs_raw);
  uint8_t *smem = bs_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  int4 *ring = reinterpret_cast<int4 *>(smem + Cfg::OFF_RING);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::OFF_BAR);
  uint64_t *full = bars;                    // [S] count 33 (1 when all scales are atoms)
  uint64_t *empty = bars + S;               // [S] count 1 (tcgen05.commit)
  uint64_t *acc_full = bars + 2 * S;        // [2] count 1 (tcgen05.commit)
  uint64_t *acc_empty = acc_full + 2;       // [2] count 4 (epilogue warps; 8: both CTAs' in PAIR)
  uint64_t *xfull = acc_full + 4;           // [2] count 64 (SwiGLU pair exchange)
  uint64_t *xempty = acc_full + 6;          // [2] count 64
  uint64_t *tfull = acc_full + 8;           // [BS_RING] count 1 (producer)
  uint64_t *tempty = tfull + BS_RING;       // [BS_RING] count 5 (MMA + 4 epilogue warps)
  uint64_t *mma_done = tempty + BS_RING;    // count 1
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: rank 0 of the CTA pair issues the MMAs; rank 1 only loads its operands and drains
  // its half of the accumulators
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  if (threadIdx.x == 0) {
    const bool lanes = !(args.sfa_atoms && args.sfb_atoms);   // some scales staged by lanes
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], lanes ? 33 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], PAIR ? 8 : 4);
      mbar_init(&xfull[i], 64);
      mbar_init(&xempty[i], 64);
    }
    for (int i = 0; i < BS_RING; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 5);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
    if (PAIR) fence_mbar_init_cluster();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();   // both CTAs' barriers exist before either reaches them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = args.nkb;
  constexpr uint32_t W_TX = WFMT == BS_W_FP4 ? BS_BM * BS_BK / 2 : BS_BM * BS_BK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&maps.w);
      if (EPI == BS_EPI_SWIGLU) prefetch_tmap(&maps.w2);
      for (int i = 0; i < Cfg::NBOX; ++i) prefetch_tmap(&maps.x[i]);
      if (PAIR) {
        prefetch_tmap(&maps.sfa);
        prefetch_tmap(&maps.sfb);
      }
    }
    // narrow tiles read their weights once; activation rows are reused by the m-tiles of
    // their expert, which the tile order keeps close together in time
    const uint64_t pol_w = NARROW ? l2_policy_evict_first() : l2_policy_evict_normal();
    const uint64_t pol_x = l2_policy_evict_normal();
    const int ntiles = args.tiles ? *args.ntiles : args.dense_tiles;
    int it = 0;
    bool ok = true;
    for (int ti = 0; ok; ++ti) {
      // next tile -> ring slot (an end marker when the work runs out)
      const int slot = ti % BS_RING;
      if (!warp_wait(&tempty[slot], (uint32_t(ti / BS_RING) & 1u) ^ 1u)) break;
      int4 tl = make_int4(-1, 0, 0, 0);
      if (lane == 0) {
        if constexpr (PAIR) {
          // pairs of consecutive list entries (m-tiles 2i, 2i + 1 of one token tile) in a
          // fixed stride over the clusters; rank r takes entry 2i + r
          const int pi = int(cluster_id_x()) + ti * int(ncluster_x());
          if (2 * pi + 1 < ntiles) tl = args.tiles[2 * pi + int(rank)];
        } else {
          const int t = args.tiles ? atomicAdd(args.next_tile, 1) : int(blockIdx.x) + ti * int(gridDim.x);
          if (t < ntiles) tl = args.tiles ? args.tiles[t] : bs_dense_tile(args, t);
        }
        ring[slot] = tl;
        mbar_arrive(&tfull[slot]);
      }
      tl.x = __shfl_sync(0xffffffffu, tl.x, 0);
      tl.y = __shfl_sync(0xffffffffu, tl.y, 0);
      tl.z = __shfl_sync(0xffffffffu, tl.z, 0);
      tl.w = __shfl_sync(0xffffffffu, tl.w, 0);
      if (tl.x < 0) break;
      const int nrows = tl.w & 0xFF, rtile = tl.w >> 8;
      const int nmma = bs_nmma<Cfg::BN>(nrows), bi = bs_box(nmma);
      const uint32_t x_tx = bs_box_rows(bi) * BS_BK;
      const uint32_t sfb_ks = (NARROW || nmma <= 128) ? 512u : 1024u;   // atom bytes per K stage
      const uint32_t sf_tx = (args.sfa_atoms ? 512u * Cfg::KSUB : 0u) +
                             (args.sfb_atoms ? sfb_ks * Cfg::KSUB : 0u);
      const int64_t wrow0 = int64_t(tl.x) * args.a_rows +
                            int64_t(tl.y) * (EPI == BS_EPI_SWIGLU ? 64 : BS_BM);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = uint32_t(it / S) & 1u;
        if (!warp_wait(&empty[s], ph ^ 1u)) {
          ok = false;
          break;
        }
        uint8_t *sa = smem + Cfg::OFF_A + s * Cfg::A_BYTES;
        uint8_t *sb = smem + Cfg::OFF_B + s * Cfg::B_BYTES;
        if constexpr (PAIR) {
          // this CTA's weight rows (its m-tile), its half of the activation rows, its m-tile's
          // weight scale atom and the whole tile's activation scale atoms, all completing on
          // rank 0's barrier, which expects both CTAs' bytes
          const int half = nmma >> 1, bih = bs_box(half);
          const uint32_t xh_tx = bs_box_rows(bih) * BS_BK;
          const uint32_t fb = mapa_rank(&full[s], 0);
          if (rank == 0) mbar_arrive_expect_tx_el(&full[s], 2u * (W_TX + xh_tx + 512u + 1024u));
          const int kx = kb * BS_BK;
          tma_load_2d_pair_el(sa, &maps.w, fb, kx, int32_t(wrow0), pol_w);
          if (EPI == BS_EPI_SWIGLU)
            tma_load_2d_pair_el(sa + Cfg::A_SUB / 2, &maps.w2, fb, kx, int32_t(wrow0), pol_w);
          tma_load_2d_pair_el(sb, &maps.x[bih], fb, kx, tl.z + int(rank) * half, pol_x);
          tma_load_2d_pair_el(smem + Cfg::OFF_SFA + s * Cfg::SFA_BYTES, &maps.sfa, fb, 0,
                              int32_t(((int64_t(tl.x) * args.mtiles + tl.y) * args.nkq + kb) * 2),
                              pol_x);
          tma_load_2d_pair_el(smem + Cfg::OFF_SFB + s * Cfg::SFB_BYTES, &maps.sfb, fb, 0,
                              int32_t((int64_t(rtile) * args.nkq + kb) * 4), pol_x);
          continue;
        }
        {   // one elected lane of the converged warp issues (warp-uniform operands)
          mbar_arrive_expect_tx_el(&full[s], uint32_t(Cfg::KSUB) * (W_TX + x_tx) + sf_tx);
          if (args.sfa_atoms)
            bulk_load_el(sbase + Cfg::OFF_SFA + s * Cfg::SFA_BYTES,
                         args.sfa_atoms + ((int64_t(tl.x) * args.mtiles + tl.y) * args.nkq +
                                           kb * Cfg::KSUB) * 512,
                         512u * Cfg::KSUB, &full[s]);
          if (args.sfb_atoms) {
#pragma unroll
            for (int ks = 0; ks < Cfg::KSUB; ++ks)
              bulk_load_el(sbase + Cfg::OFF_SFB + s * Cfg::SFB_BYTES + ks * Cfg::SFB_SUB,
                           args.sfb_atoms + (int64_t(rtile) * args.nkq + kb * Cfg::KSUB + ks) * 1024,
                           sfb_ks, &full[s]);
          }
#pragma unroll
          for (int ks = 0; ks < Cfg::KSUB; ++ks) {
            const int kx = (kb * Cfg::KSUB + ks) * BS_BK;
            uint8_t *a = sa + ks * Cfg::A_SUB;
            tma_load_2d_el(a, &maps.w, &full[s], kx, int32_t(wrow0), pol_w);
            if (EPI == BS_EPI_SWIGLU)
              tma_load_2d_el(a + Cfg::A_SUB / 2, &maps.w2, &full[s], kx, int32_t(wrow0), pol_w);
            tma_load_2d_el(sb + ks * Cfg::B_SUB, &maps.x[bi], &full[s], kx, tl.z, pol_x);
          }
        }
        // scale words -> tcgen05.cp layout (row 32c + l at byte l*16 + c*4)
#pragma unroll
        for (int ks = 0; ks < Cfg::KSUB; ++ks) {
          const int kq = kb * Cfg::KSUB + ks;
          const uint32_t sfa = sbase + Cfg::OFF_SFA + s * Cfg::SFA_BYTES + ks * 512 + lane * 16;
          const uint32_t sfb = sbase + Cfg::OFF_SFB + s * Cfg::SFB_BYTES + ks * Cfg::SFB_SUB +
                               lane * 16;
          if (args.sf_async) {
            if (!args.sfa_atoms) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                if (EPI == BS_EPI_SWIGLU && c >= 2)
                  bs_scale_copy(args.sw2, wrow0 + 32 * (c - 2) + lane, kq, sfa + 4 * c);
                else
                  bs_scale_copy(args.sw, wrow0 + 32 * c + lane, kq, sfa + 4 * c);
              }
            }
            if (!args.sfb_atoms) {
#pragma unroll
              for (int c = 0; c < Cfg::SFB_CHUNKS; ++c)
                bs_scale_copy(args.sx, int64_t(tl.z) + 32 * c + lane, kq,
                              sfb + (c >> 2) * 512 + 4 * (c & 3));
            }
          } else {
            uint4 va;
            uint32_t *vw = reinterpret_cast<uint32_t *>(&va);
            if (!args.sfa_atoms) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                if (EPI == BS_EPI_SWIGLU && c >= 2)
                  vw[c] = bs_scale_word(args.sw2, wrow0 + 32 * (c - 2) + lane, kq);
                else
                  vw[c] = bs_scale_word(args.sw, wrow0 + 32 * c + lane, kq);
              }
              *reinterpret_cast<uint4 *>(smem + (sfa - sbase)) = va;
            }
#pragma unroll
            for (int h = 0; h < (args.sfb_atoms ? 0 : Cfg::SFB_ATOMS); ++h) {
              uint4 vb;
              uint32_t *bw = reinterpret_cast<uint32_t *>(&vb);
#pragma unroll
              for (int c = 0; c < 4; ++c)
                bw[c] = bs_scale_word(args.sx, int64_t(tl.z) + 32 * (4 * h + c) + lane, kq);
              *reinterpret_cast<uint4 *>(smem + (sfb - sbase) + h * 512) = vb;
            }
          }
        }
        if (args.sfa_atoms && args.sfb_atoms) {
          // every scale arrives by bulk copy: lane 0's expect_tx is the only arrival
        } else if (args.sf_async) {
          cp_async_arrive_noinc(&full[s]);
        } else {
          fence_proxy_async_smem();
          mbar_arrive(&full[s]);
        }
      }
    }
    // every copy this warp issued has landed before the CTA can finish (in a pair, rank 1's
    // copies complete on rank 0's barriers, which rank 0 drains before the final cluster
    // barrier)
    if (!PAIR || rank == 0)
      for (int j = it - S < 0 ? 0 : it - S; j < it; ++j)
        mbar_wait(&full[j % S], uint32_t(j / S) & 1u);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer: the whole warp
    // runs the loop, one elect.sync lane issues
    if (PAIR && rank != 0) {
      // rank 1 of a pair issues nothing: it only releases its tile-ring slots
      for (int ti = 0;; ++ti) {
        const int slot = ti % BS_RING;
        if (!warp_wait(&tfull[slot], uint32_t(ti / BS_RING) & 1u)) break;
        const int4 tl = ring[slot];
        if (tl.x < 0) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
      }
    } else {
      int it = 0;
      for (int ti = 0;; ++ti) {
        const int slot = ti % BS_RING;
        if (!warp_wait(&tfull[slot], uint32_t(ti / BS_RING) & 1u)) break;
        const int4 tl = ring[slot];
        if (tl.x < 0) break;
        const int nmma = bs_nmma<Cfg::BN>(tl.w & 0xFF);
        const int ab = ti & 1;
        if (!warp_wait(&acc_empty[ab], (uint32_t(ti >> 1) & 1u) ^ 1u)) break;
        tc_fence_after();
        const uint32_t tacc = tmem + uint32_t(ab) * Cfg::ACC_COLS;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = uint32_t(it / S) & 1u;
          if (!warp_wait(&full[s], ph)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();   // scale words written by cp.async -> tcgen05.cp reads
          tc_fence_after();
          const uint32_t t_sfa = tmem + Cfg::SF_COL0 + 16u * s;
          const uint32_t t_sfb = t_sfa + Cfg::SFA_COLS;
#pragma unroll
          for (int ks = 0; ks < Cfg::KSUB; ++ks) {
            const uint32_t ta = t_sfa + 4u * ks, tb = t_sfb + 4u * Cfg::SFB_ATOMS * ks;
            const uint32_t s_sfa = sbase + Cfg::OFF_SFA + s * Cfg::SFA_BYTES + ks * 512;
            const uint32_t s_sfb = sbase + Cfg::OFF_SFB + s * Cfg::SFB_BYTES + ks * Cfg::SFB_SUB;
            const uint64_t da = sdesc_sw128(sbase + Cfg::OFF_A + s * Cfg::A_BYTES + ks * Cfg::A_SUB);
            const uint64_t db = sdesc_sw128(sbase + Cfg::OFF_B + s * Cfg::B_BYTES + ks * Cfg::B_SUB);
            if constexpr (PAIR) {
              // both CTAs' scale atoms into both TMEMs, then M = 256 MMAs over both CTAs'
              // weight rows and activation halves
              tc_cp_sf_pair_el(ta, sdesc_sf(s_sfa));
              tc_cp_sf_pair_el(tb, sdesc_sf(s_sfb));
              if (nmma > 128) tc_cp_sf_pair_el(tb + 4u, sdesc_sf(s_sfb + 512u));
#pragma unroll
              for (int k = 0; k < 4; ++k)
                tc_mma_mx_pair_el(tacc, da + uint64_t(2 * k), db + uint64_t(2 * k),
                                  idesc_mx(WFMT == BS_W_FP4 ? 5u : 0u, uint32_t(nmma), uint32_t(k), 256u),
                                  ta | (uint32_t(k) << 30), tb | (uint32_t(k) << 30),
                                  (kb | ks | k) != 0 ? 1u : 0u);
            } else {
              tc_cp_sf_el(ta, sdesc_sf(s_sfa));
              tc_cp_sf_el(tb, sdesc_sf(s_sfb));
              if (Cfg::SFB_ATOMS > 1 && nmma > 128) tc_cp_sf_el(tb + 4u, sdesc_sf(s_sfb + 512u));
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                // +32 bytes along K inside the swizzle atom = +2 in the descriptor's address field
                tc_mma_mx_el(tacc, da + uint64_t(2 * k), db + uint64_t(2 * k),
                             idesc_mx(WFMT == BS_W_FP4 ? 5u : 0u, uint32_t(nmma), uint32_t(k)),
                             ta | (uint32_t(k) << 30), tb | (uint32_t(k) << 30),
                             (kb | ks | k) != 0 ? 1u : 0u);
              }
            }
          }
          if constexpr (PAIR) tc_commit_pair_both_el(&empty[s]);   // both CTAs refill
          else tc_commit_el(&empty[s]);
        }
        if (!ok) break;
        if constexpr (PAIR) tc_commit_pair_both_el(&acc_full[ab]);   // both CTAs drain
        else tc_commit_el(&acc_full[ab]);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
      }
      if constexpr (PAIR) tc_commit_pair_el(mma_done);
      else tc_commit_el(mma_done);
      warp_wait(mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quadrant of this warp
    float *tp = reinterpret_cast<float *>(smem + Cfg::OFF_EPI + q * BS_EPI_BYTES);
    int xc = 0;
    for (int ti = 0;; ++ti) {
      const int slot = ti % BS_RING;
      if (!warp_wait(&tfull[slot], uint32_t(ti / BS_RING) & 1u)) break;
      const int4 tl = ring[slot];
      if (tl.x < 0) break;
      const int nrows = tl.w & 0xFF, rtile = tl.w >> 8;
      const int nmma = bs_nmma<Cfg::BN>(nrows);
      const int ab = ti & 1;
      if (!warp_wait(&acc_full[ab], uint32_t(ti >> 1) & 1u)) break;
      tc_fence_after();
      const uint32_t tq = tmem + (uint32_t(32 * q) << 16) + uint32_t(ab) * Cfg::ACC_COLS;
      bool ok = true;
      for (int cc = 0; cc * 32 < nmma && ok; ++cc) {
        uint32_t r[32];
        tmem_ld32(tq + uint32_t(cc * 32), r);
        const int64_t p_lane = int64_t(tl.z) + cc * 32 + lane;   // this lane's row after transpose
        const bool live = cc * 32 + lane < nrows;
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
          // SwiGLU pair: warp q (gate rows 32q..) and warp q+2 (the same up rows) both park
          // their chunk transposed in shared memory, then each finishes 16 of the 32 rows:
          // lane l takes row 16*half + l/2 and features (l&1)*16 .. +15 of the pair's 32.
          const int pr = q & 1, half = q >> 1;
          const uint32_t xph = uint32_t(xc) & 1u;
          const float L = args.limit;
          if (!warp_wait(&xempty[pr], xph ^ 1u)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float v = round_bf16f(__uint_as_float(r[j]));
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
          const bool jlive = cc * 32 + jt < nrows;
          const int64_t pj = int64_t(tl.z) + cc * 32 + jt;
          const float w = (args.pw && jlive) ? args.pw[pj] : 1.0f;
          float h[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 g4 = reinterpret_cast<const float4 *>(tg)[i];
            const float4 u4 = reinterpret_cast<const float4 *>(tu)[i];
            const float gg[4] = {g4.x, g4.y, g4.z, g4.w}, uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const float sg = __fdividef(gg[b], 1.0f + __expf(-gg[b]));
              float v = sg * uu[b];
              if (args.pw) v = v * w;
              h[4 * i + b] = round_bf16f(v);
            }
          }
          mbar_arrive(&xempty[pr]);
          // act_quant of the 32 features of row pj (docs/reference/kernel.py:40-95): the two
          // lanes of a row combine their amax; the scale is a power of two, so x / s is the
          // exact product x * (1 / s)
          float amax = 0.0f;
#pragma unroll
          for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(h[i]));
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
          amax = fmaxf(amax, 1e-4f);
          const float sc = pow2_ceil_log2(__fmul_rn(amax, 1.0f / 448.0f));
          const float inv = __uint_as_float((254u << 23) - __float_as_uint(sc));
          uint32_t wq[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t wv = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const float y = fminf(fmaxf(__fmul_rn(h[4 * i + b], inv), -448.0f), 448.0f);
              wv |= uint32_t(f32_to_e4m3_sat(y)) << (8 * b);
            }
            wq[i] = wv;
          }
          if (jlive) {
            const int64_t f0 = int64_t(tl.y) * 64 + 32 * pr;
            *reinterpret_cast<uint4 *>(args.hq + pj * args.ldh + f0 + fh * 16) =
                make_uint4(wq[0], wq[1], wq[2], wq[3]);
            if (fh == 0) {
              const uint8_t e8 = uint8_t((__float_as_uint(sc) >> 23) & 0xFF);
              if (args.hs_atoms)
                args.hs_atoms[int64_t(rtile) * (args.ldh / 128) * 1024 +
                              sf_atom_off(cc * 32 + jt, int(f0 / 32))] = e8;
              else
                args.hs[pj * (args.ldh / 32) + f0 / 32] = e8;
            }
          }
          ++xc;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR && rank != 0) mbar_arrive_cluster(mapa_rank(&acc_empty[ab], 0));
        else mbar_arrive(&acc_empty[ab]);
        mbar_arrive(&tempty[slot]);
      }
      if (!ok) break;
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync();   // no CTA leaves while the other may still reach its barriers or TMEM
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
  }
}

}  // namespace dsv41
