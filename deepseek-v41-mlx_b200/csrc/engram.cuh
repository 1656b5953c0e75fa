// engram.cuh -- n-gram hashing and fp8 row gather (a15, a16).
//
// Hash: deepseek_v41_mlx/engram.py:154-180 (and upstream NgramHashState.forward,
// docs/reference/engram.py).  Per position: compressed ids of the token and its
// G-1 predecessors (pad once the lookback passes the sequence start), int64
// products with the per-(layer, lookback) odd multipliers, running XOR; after
// step i the value is the (i+1)-gram hash, taken % prime[layer][i-1][head] and
// offset into the layer's flat table.  All operands are non-negative int64.
//
// Gather: EngramEmbedding.__call__ (engram.py:197-203) / upstream
// ParallelEngramEmbedding.forward (docs/reference/model.py:312-325): rows of an
// e4m3 table times their ue8m0 block scales, fp32; ids outside this shard's
// [row_lo, row_lo + rows) contribute zero rows.  The gather-sum form adds the
// n_per_tok rows of a token in column order in fp32.
#pragma once
#include "common.cuh"

namespace dsv41 {

// Hash (engram.py:163-180): compressed ids (engram.py:163-164) and the n-gram hashes in one
// launch, one thread per (b, l, layer, column): column c = (shift - 1) * H + head hashes the
// (shift + 1)-gram ending at its position, reading the compressed ids of
// positions pos - s (s <= shift) from input_ids through token_map inside this call's
// positions and from the cache before them (pad_id before position 0), as the hasher does;
// the (layer 0, column 0) thread of each position writes that position's compressed id into
// the cache.  The cache is read only below start and written only from start on.  x % p by
// Barrett reduction: with m = floor((2^64 - 1) / p), q = hi64(x * m) is floor(x / p) or one
// less, so one conditional subtraction gives the exact remainder (x < 2^63, p < 2^63); each
// block computes the m of every prime once into shared memory.
__global__ void k_engram_hash_cols(const int64_t *__restrict__ ids, int64_t B, int64_t L,
                                   int64_t start, const int64_t *__restrict__ token_map,
                                   int64_t vocab, int64_t *__restrict__ cache, int64_t max_seq,
                                   const int64_t *__restrict__ mult,
                                   const int64_t *__restrict__ primes,
                                   const int64_t *__restrict__ offsets, int nL, int G, int H,
                                   int64_t pad_id, int64_t *__restrict__ out) {
  extern __shared__ uint64_t s_recip[];   // [nL * (G - 1) * H]
  const int cols = (G - 1) * H;
  const int np = nL * cols;
  for (int k = threadIdx.x; k < np; k += blockDim.x) {
    const uint64_t pk = uint64_t(primes[k]);
    s_recip[k] = pk > 1 ? ~0ull / pk : 0ull;
  }
  __syncthreads();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= B * L * np) return;
  const int k = int(i % np);                            // layer * cols + column
  const int64_t bl = i / np, b = bl / L, l = bl % L;
  const int layer = k / cols, c = k % cols, shift = c / H + 1;
  const int64_t pos = start + l;
  const int64_t *bids = ids + b * L;
  int64_t *bcache = cache + b * max_seq;
  auto compressed = [&](int64_t q) -> int64_t {       // position q's compressed id, q <= pos
    if (q < start) return bcache[q];
    int64_t id = bids[q - start];
    if (id < 0 || id >= vocab) {
      dev_flag(DSV41_DEVST_BAD_INDEX);
      id = 0;
    }
    return token_map[id];
  };
  const int64_t *mrow = mult + (int64_t)layer * G;
  int64_t rolling = 0;
  for (int sh = 0; sh <= shift; ++sh) {
    const int64_t tok = pos < sh ? pad_id : compressed(pos - sh);
    const int64_t prod = tok * mrow[sh];
    rolling = sh == 0 ? prod : (rolling ^ prod);
  }
  const uint64_t x = uint64_t(rolling), pr = uint64_t(primes[k]);
  uint64_t r = 0;
  if (pr > 1) {
    r = x - __umul64hi(x, s_recip[k]) * pr;
    if (r >= pr) r -= pr;
  }
  out[bl * np + k] = int64_t(r) + offsets[k];
  if (k == 0) bcache[pos] = compressed(pos);
}

// 8 consecutive outputs from one 16-byte (bf16) or 32-byte (fp32) store.
__device__ __forceinline__ void store8(float *p, const float *v) {
  reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16 *p, const float *v) {
  uint4 o;
  o.x = uint32_t(f2bf_bits(v[0])) | (uint32_t(f2bf_bits(v[1])) << 16);
  o.y = uint32_t(f2bf_bits(v[2])) | (uint32_t(f2bf_bits(v[3])) << 16);
  o.z = uint32_t(f2bf_bits(v[4])) | (uint32_t(f2bf_bits(v[5])) << 16);
  o.w = uint32_t(f2bf_bits(v[6])) | (uint32_t(f2bf_bits(v[7])) << 16);
  *reinterpret_cast<uint4 *>(p) = o;
}

template <typename T> __device__ __forceinline__ void store_out(T *p, float v);
template <> __device__ __forceinline__ void store_out<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16 *p, float v) {
  *p = __float2bfloat16_rn(v);
}

// One warp per gathered row; each lane decodes 8-byte chunks.  d % 8 == 0.  tld / sld:
// table / scale row strides in bytes (d and d / block for a plain table; the packed row
// size for rows received from their owners, whose scale bytes follow the codes).
template <typename T>
__global__ void k_engram_gather_rows(const uint8_t *__restrict__ table,
                                     const uint8_t *__restrict__ scale, int64_t rows,
                                     int64_t row_lo, int64_t d, int64_t block, int64_t tld,
                                     int64_t sld, const int64_t *__restrict__ idx, int64_t n_idx,
                                     T *__restrict__ out) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_idx) return;
  const int64_t local = idx[warp] - row_lo;
  const bool in = local >= 0 && local < rows;
  const int blk = int(block);                 // <= d, so 32-bit index arithmetic
  T *o = out + warp * d;
  for (int64_t c = lane * 8; c < d; c += 256) {
    float f[8];
    if (in) {
      const uint64_t v = __ldg(reinterpret_cast<const unsigned long long *>(table + local * tld + c));
      uint32_t h[4];
      e4m3x4_to_f16x4(uint32_t(v), h[0], h[1]);
      e4m3x4_to_f16x4(uint32_t(v >> 32), h[2], h[3]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sc = e8m0f(scale[local * sld + (int(c) + j) / blk]);
        const float2 p = h2f2(h[j >> 1]);
        f[j] = __fmul_rn((j & 1) ? p.y : p.x, sc);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) store_out<T>(o + c + j, f[j]);
  }
}

// Lane l's row (id `mine`): its codes and scale bytes, and whether it lies in the table.
// PEERS: shard id / rows of the pointer arrays, ids at or past `total` out; otherwise the
// rows [row_lo, row_lo + rows) of `table` / `scale`.
template <bool PEERS>
__device__ __forceinline__ bool gs_row(int64_t id, const uint8_t *&rt, const uint8_t *&rs,
                                       const uint8_t *__restrict__ table,
                                       const uint8_t *__restrict__ scale, int64_t rows,
                                       int64_t row_lo, int64_t tld, int64_t sld,
                                       const uint8_t *const *__restrict__ tabs,
                                       const uint8_t *const *__restrict__ scs, int nsh,
                                       int64_t total) {
  if (PEERS) {
    const int64_t sh = id >= 0 ? id / rows : -1, local = id - sh * rows;
    const bool in = id >= 0 && id < total && sh < nsh;   // the last shard may be shorter
    rt = in ? tabs[sh] + local * tld : nullptr;
    rs = in ? scs[sh] + local * sld : nullptr;
    return in;
  }
  const int64_t local = id - row_lo;
  const bool in = id >= 0 && local >= 0 && local < rows;
  rt = in ? table + local * tld : nullptr;
  rs = in ? scale + local * sld : nullptr;
  return in;
}

__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// The row scale 2^(sb - 127) as the accumulation takes it: the f16 bits of the scale when it
// is an f16 (sb in [103, 142], the scales real tables use), else 0x10000 | sb.
constexpr uint32_t GS_SV_ONE = 0x3C00u;               // 1.0: the scale of a skipped row
__device__ __forceinline__ uint32_t gs_sv(uint32_t sb) {
  return sb - 103u <= 39u ? (sb >= 113u ? (sb - 112u) << 10 : 1u << (sb - 103u))
                          : (0x10000u | sb);
}

// a[j] += code j of the row (NW 32-bit words w) x its scale sv (gs_sv), in fp32 with the
// reference's roundings: its product, rounded, then its sum, rounded.
// f16 scale: the codes stay f16 and the mixed-precision fused multiply-add
// (`fma.rn.f32.f16`, sm_100) forms the exact product of code and scale and adds it to the
// fp32 sum with one rounding -- the same bits, since that product is exact.  Other scales:
// e4m3 x a power of two is exact in fp32 whenever the scale byte is below 240 (no overflow;
// the smallest product, 2^-9 x 2^-127, is still a whole multiple of 2^-149), so there one
// fp32 fused multiply-add gives the same bits.  From 240 on a product can overflow to
// infinity, and the reference's sum then sees that infinity (inf + -inf = NaN, inf + finite =
// inf): those rows take __fmul_rn / __fadd_rn, which are never contracted into a fused
// multiply-add.  A skipped row (codes 0, scale 1) adds +0.0, which leaves every sum as it was
// (a sum that starts at +0.0 is never -0.0).
template <int NW>
__device__ __forceinline__ void gs_accum(float (&a)[4 * NW], const uint32_t (&w)[NW],
                                         uint32_t sv) {
  if (sv < 0x10000u) {
    const uint16_t s16 = uint16_t(sv);
#pragma unroll
    for (int k = 0; k < NW; ++k) {
      uint32_t hq[2];
      e4m3x4_to_f16x4(w[k], hq[0], hq[1]);
#pragma unroll
      for (int j = 0; j < 2; ++j)
        asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\t"
            "fma.rn.f32.f16 %0, a, %3, %0;\n\tfma.rn.f32.f16 %1, b, %3, %1;\n\t}"
            : "+f"(a[4 * k + 2 * j]), "+f"(a[4 * k + 2 * j + 1])
            : "r"(hq[j]), "h"(s16));
    }
    return;
  }
  const uint32_t sb = sv & 0xFFu;
  const float s = e8m0f(sb);
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    uint32_t hq[2];
    e4m3x4_to_f16x4(w[k], hq[0], hq[1]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 p = h2f2(hq[j]);
      float &lo = a[4 * k + 2 * j], &hi = a[4 * k + 2 * j + 1];
      if (sb < 240u) {
        lo = __fmaf_rn(p.x, s, lo);
        hi = __fmaf_rn(p.y, s, hi);
      } else {
        lo = __fadd_rn(lo, __fmul_rn(p.x, s));
        hi = __fadd_rn(hi, __fmul_rn(p.y, s));
      }
    }
  }
}

// Sums into acc (the 8 columns of this lane) the nh <= 32 rows whose ids lane l holds in
// `mine` (-1 past the token's ids), in lane order: each lane resolves its own row once
// (pointers and range, and its scale when the warp's columns share one scale block,
// `uscale`), then the rows are read 8 at a time, the pointers broadcast by shuffle, 8-byte
// streaming loads a lane.  Rows outside the table add nothing (codes 0, scale 1).
// (16-byte loads, two warps a 1 KB row, measured slower: 0.072 against 0.066 ms for 8192
// tokens of 24 rows.)
template <bool PEERS>
__device__ __forceinline__ void gs_rows(float (&acc)[8], int64_t mine, int nh,
                                        int64_t col, int soff, bool uscale,
                                        const uint8_t *__restrict__ table,
                                        const uint8_t *__restrict__ scale, int64_t rows,
                                        int64_t row_lo, int64_t tld, int64_t sld,
                                        const uint8_t *const *__restrict__ tabs,
                                        const uint8_t *const *__restrict__ scs, int nsh,
                                        int64_t total) {
  constexpr int NW = 2;                           // 32-bit words a lane reads of a row
  const uint8_t *rt_m, *rs_m;
  const bool in_m = gs_row<PEERS>(mine, rt_m, rs_m, table, scale, rows, row_lo, tld, sld, tabs,
                                  scs, nsh, total);
  const unsigned inmask = __ballot_sync(0xffffffffu, in_m);
  const uint32_t sv_m = (uscale && in_m) ? gs_sv(uint32_t(rs_m[soff])) : GS_SV_ONE;
  const uint64_t pt_m = reinterpret_cast<uint64_t>(rt_m), ps_m = reinterpret_cast<uint64_t>(rs_m);
  for (int h = 0; h < nh; h += 8) {               // h + u <= 31: every source lane exists
    uint32_t w[8][NW];
    uint32_t sv[8];
    // the batch's row loads first: nothing in front of them waits on a load
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int src = h + u;
      const bool in = (inmask >> src) & 1u;                              // warp-uniform
      const uint8_t *rt = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, pt_m, src));
      const uint64_t v = in ? __ldcs(reinterpret_cast<const unsigned long long *>(rt + col)) : 0ull;
      w[u][0] = uint32_t(v);
      w[u][1] = uint32_t(v >> 32);
    }
    // then the scales: broadcast from the row's own lane, or loaded per lane when the warp's
    // columns span several scale blocks
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int src = h + u;
      if (uscale) {
        sv[u] = __shfl_sync(0xffffffffu, sv_m, src);
      } else {
        const bool in = (inmask >> src) & 1u;
        const uint8_t *rs = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, ps_m, src));
        sv[u] = in ? gs_sv(uint32_t(rs[soff])) : GS_SV_ONE;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) gs_accum<NW>(acc, w[u], sv[u]);
  }
}

// Warps per token = d / 256: a warp covers 256 columns, its lanes 8-column chunks at
// lane*8 (coalesced 256-byte spans); rows summed in column order, fp32, 8 rows in flight per
// warp, table rows streamed (read once, not kept in L1/L2).  The token's ids are read once,
// one per lane; each lane resolves its own row's address (and its scale byte, when the warp
// shares one scale block) and the batch's loads take them by shuffle, so no row load waits
// on an index computation.  64 registers: 4 CTAs (32 warps) an SM.
// PEERS: the table is sharded over ranks by rows (rank r holds rows [r*rows, (r+1)*rows),
// `rows` = the shard size); row id's codes and scales are read from shard id / rows through
// the pointer arrays tabs / scs (other ranks' shards mapped into this process: peer loads
// over NVLink); ids at or past `total` (the table's rows) read as zero rows; table / scale /
// row_lo unused.
template <typename T, bool PEERS = false>
__global__ void __launch_bounds__(256, 4) k_engram_gather_sum(
    const uint8_t *__restrict__ table, const uint8_t *__restrict__ scale, int64_t rows,
    int64_t row_lo, int64_t D, int64_t block, int64_t tld, int64_t sld,
    const int64_t *__restrict__ idx, int64_t n_tok, int n_per_tok, T *__restrict__ out,
    const uint8_t *const *__restrict__ tabs = nullptr,
    const uint8_t *const *__restrict__ scs = nullptr, int nsh = 0, int64_t total = 0) {
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int wpt = int(D / 256);
  const int64_t tok = gw / wpt;
  if (tok >= n_tok) return;
  const int64_t col = (gw % wpt) * 256 + lane * 8;
  const int soff = int(col / block);            // 8 | block keeps a chunk in one scale block
  const bool uscale = block % 256 == 0;         // the warp's columns share one scale block
  float acc[8] = {};
  const int64_t *ti = idx + tok * n_per_tok;
  for (int h0 = 0; h0 < n_per_tok; h0 += 32) {
    // lane l holds id h0 + l (-1 past the token's ids)
    const int64_t mine = h0 + lane < n_per_tok ? ti[h0 + lane] : -1;
    gs_rows<PEERS>(acc, mine, min(32, n_per_tok - h0), col, soff, uscale, table, scale, rows,
                   row_lo, tld, sld, tabs, scs, nsh, total);
  }
  store8(out + tok * D + col, acc);
}

// a15 + a16 in one pass: the (G-1)*H <= 32 row ids of each position of one hash layer
// (k_engram_hash_cols, same arithmetic) computed by the lanes that would have
// loaded them, summed as rows of a packed table (codes then scale bytes, rb bytes a row).
// Lane c < (G-1)*H hashes column c = (shift-1)*H + head: the compressed ids of positions
// pos - s (s <= shift) come from input_ids through token_map inside this call's positions and
// from the id cache before them (pad_id before position 0); the first warp of each position
// writes that position's compressed id into the cache, as the hasher does.  The cache is read
// only below start and written only from start on, so no position is both read and written.
// recips[c] = floor((2^64 - 1) / prime[c]) (0 for prime <= 1) when given; otherwise each lane
// divides for its own prime.  No shared memory and no barrier: a warp's hash loads (its
// lookback unrolled, G <= ENGRAM_MAX_G) issue together and its row loads follow at once.
// PEERS: the rows come from row shards as in k_engram_gather_sum's PEERS mode (tabs / scs,
// shard size `rows`, `total` rows in all); table / scale / row_lo unused.
constexpr int ENGRAM_MAX_G = 8;
template <typename T, bool PEERS = false>
__global__ void __launch_bounds__(256, 4) k_engram_lookup_sum(
    const int64_t *__restrict__ ids, int64_t B, int64_t L, int64_t start,
    const int64_t *__restrict__ token_map, int64_t vocab, int64_t *__restrict__ cache,
    int64_t max_seq, const int64_t *__restrict__ mult, const int64_t *__restrict__ primes,
    const int64_t *__restrict__ offsets, const uint64_t *__restrict__ recips, int G, int H,
    int64_t pad_id, const uint8_t *__restrict__ table, const uint8_t *__restrict__ scale,
    int64_t rows, int64_t row_lo, int64_t D, int64_t block, int64_t tld, int64_t sld,
    T *__restrict__ out, const uint8_t *const *__restrict__ tabs = nullptr,
    const uint8_t *const *__restrict__ scs = nullptr, int nsh = 0, int64_t total = 0) {
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int wpt = int(D / 256);
  const int64_t tok = gw / wpt;
  if (tok >= B * L) return;
  const int cols = (G - 1) * H;
  const int64_t b = tok / L, l = tok % L, pos = start + l;
  const int64_t *bids = ids + b * L;
  int64_t *bcache = cache + b * max_seq;
  auto compressed = [&](int64_t q) -> int64_t {      // position q's compressed id, q <= pos
    if (q < start) return bcache[q];
    int64_t id = bids[q - start];
    if (id < 0 || id >= vocab) {
      dev_flag(DSV41_DEVST_BAD_INDEX);
      id = 0;
    }
    return token_map[id];
  };
  int64_t mine = -1;
  if (lane < cols) {
    const int shift = lane / H + 1;
    const uint64_t p = uint64_t(primes[lane]);
    const int64_t off = offsets[lane];
    int64_t tk[ENGRAM_MAX_G], mu[ENGRAM_MAX_G];
#pragma unroll
    for (int s = 0; s < ENGRAM_MAX_G; ++s) {
      if (s <= shift) {
        tk[s] = pos < s ? pad_id : compressed(pos - s);
        mu[s] = mult[s];
      }
    }
    int64_t rolling = 0;
#pragma unroll
    for (int s = 0; s < ENGRAM_MAX_G; ++s) {
      if (s <= shift) {
        const int64_t prod = tk[s] * mu[s];
        rolling = s == 0 ? prod : (rolling ^ prod);
      }
    }
    const uint64_t x = uint64_t(rolling);
    uint64_t r = 0;
    if (p > 1) {
      const uint64_t m = recips ? recips[lane] : ~0ull / p;
      r = x - __umul64hi(x, m) * p;
      if (r >= p) r -= p;
    }
    mine = int64_t(r) + off;
  }
  if (gw % wpt == 0 && lane == 0) bcache[pos] = compressed(pos);
  const int64_t col = (gw % wpt) * 256 + lane * 8;
  const int soff = int(col / block);
  const bool uscale = block % 256 == 0;
  float acc[8] = {};
  gs_rows<PEERS>(acc, mine, cols, col, soff, uscale, table, scale, rows, row_lo, tld, sld, tabs,
                 scs, nsh, total);
  store8(out + tok * D + col, acc);
}

// Row-sharded tables: the owner of rows [row_lo, row_lo + rows) copies the raw rows
// idx[i] (global ids, all owned) into packed rows of rb bytes -- D code bytes, then the
// D / block scale bytes, zero padding to rb (a multiple of 16) -- for the ranks whose
// tokens need them.  One warp per row, 16-byte copies; rows not owned are zero.  Without
// idx, rows 0 .. n-1 of the table in order: a whole table repacked so that a lookup reads
// one contiguous row (codes and scales) instead of two places.
__global__ void __launch_bounds__(256) k_engram_pack_rows(
    const uint8_t *__restrict__ table, const uint8_t *__restrict__ scale, int64_t rows,
    int64_t row_lo, int64_t D, int64_t block, const int64_t *__restrict__ idx, int64_t n,
    uint8_t *__restrict__ out, int64_t rb) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  const int64_t local = idx ? idx[i] - row_lo : i;   // no list: the table's rows in order
  const bool in = local >= 0 && local < rows;
  uint8_t *o = out + i * rb;
  for (int64_t c = lane * 16; c < D; c += 512) {
    const uint4 v = in ? __ldcs(reinterpret_cast<const uint4 *>(table + local * D + c))
                       : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4 *>(o + c) = v;
  }
  const int64_t sb = D / block;
  for (int64_t b = lane; b < rb - D; b += 32) o[D + b] = (in && b < sb) ? scale[local * sb + b] : 0;
}

// ---- Engram gate (deepseek_v41_mlx/engram.py:245-264; upstream Engram.forward,
// docs/reference/model.py:344-365), after kv = wkv(rows).  One CTA per (token t, hc copy c):
//   rstd = rsqrt(mean(h^2) + eps) * rsqrt(mean(key^2) + eps)       (over dim, fp32)
//   dot  = sum(h * q * k * key) * rstd / sqrt(dim)
//   gate = sigmoid(sign(dot) * sqrt(max(|dot|, clamp)))            (0 where the mask is off)
//   out  = h + gate * value                                        (rounded to out's type)
// x, out [T, hc, D]; kv [T, (hc + 1) * D] = hc keys then the shared value.
template <typename T> __device__ __forceinline__ float ld_f(const T *p);
template <> __device__ __forceinline__ float ld_f<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return __bfloat162float(*p);
}

template <typename TX, typename TKV>
__global__ void __launch_bounds__(256) k_engram_gate(const TX *__restrict__ x,
                                                     const TKV *__restrict__ kv,
                                                     const float *__restrict__ qw,
                                                     const float *__restrict__ kw,
                                                     const uint8_t *__restrict__ mask, int hc,
                                                     int64_t D, float eps, float clamp,
                                                     TX *__restrict__ out) {
  const int64_t t = blockIdx.x / hc;
  const int c = int(blockIdx.x % hc);
  const TX *h = x + (t * hc + c) * D;
  const TKV *key = kv + t * (hc + 1) * D + c * D;
  const TKV *val = kv + t * (hc + 1) * D + (int64_t)hc * D;
  const float *q = qw + (int64_t)c * D, *k = kw + (int64_t)c * D;
  float shh = 0.0f, skk = 0.0f, sd = 0.0f;
  for (int64_t j = threadIdx.x; j < D; j += blockDim.x) {
    const float hv = ld_f(h + j), kv_ = ld_f(key + j);
    shh = fmaf(hv, hv, shh);
    skk = fmaf(kv_, kv_, skk);
    sd = fmaf(hv * (q[j] * k[j]), kv_, sd);
  }
  __shared__ float red[3][8];
  __shared__ float s_gate;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    shh += __shfl_xor_sync(0xffffffffu, shh, o);
    skk += __shfl_xor_sync(0xffffffffu, skk, o);
    sd += __shfl_xor_sync(0xffffffffu, sd, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][w] = shh;
    red[1][w] = skk;
    red[2][w] = sd;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.0f, b = 0.0f, d = 0.0f;
    for (int i = 0; i < int(blockDim.x >> 5); ++i) {
      a += red[0][i];
      b += red[1][i];
      d += red[2][i];
    }
    const float inv_d = 1.0f / float(D);
    const float rstd = rsqrtf(a * inv_d + eps) * rsqrtf(b * inv_d + eps);
    const float dot = d * rstd * rsqrtf(float(D));
    const float mag = sqrtf(fmaxf(fabsf(dot), clamp));
    float g = 1.0f / (1.0f + expf(dot < 0.0f ? mag : -mag));
    if (mask && !mask[t]) g = 0.0f;
    s_gate = g;
  }
  __syncthreads();
  const float g = s_gate;
  TX *o = out + (t * hc + c) * D;
  for (int64_t j = threadIdx.x; j < D; j += blockDim.x) {
    const float v = fmaf(g, ld_f(val + j), ld_f(h + j));
    if constexpr (sizeof(TX) == 4)
      o[j] = v;
    else
      o[j] = __float2bfloat16_rn(v);
  }
}

}  // namespace dsv41
