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

// step 1: compressed ids into the caller's cache (engram.py:163-164)
__global__ void k_engram_compress(const int64_t *__restrict__ ids, int64_t B, int64_t L,
                                  int64_t start, const int64_t *__restrict__ token_map,
                                  int64_t vocab, int64_t *__restrict__ cache, int64_t max_seq) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= B * L) return;
  const int64_t b = i / L, l = i % L;
  int64_t id = ids[i];
  if (id < 0 || id >= vocab) {
    dev_flag(DSV41_DEVST_BAD_INDEX);
    id = 0;
  }
  cache[b * max_seq + start + l] = token_map[id];
}

// step 2: hashes; one thread per (b, l, layer)
__global__ void k_engram_hash(int64_t B, int64_t L, int64_t start,
                              const int64_t *__restrict__ cache, int64_t max_seq,
                              const int64_t *__restrict__ mult, const int64_t *__restrict__ primes,
                              const int64_t *__restrict__ offsets, int nL, int G, int H,
                              int64_t pad_id, int64_t *__restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= B * L * nL) return;
  const int layer = int(i % nL);
  const int64_t bl = i / nL, b = bl / L, l = bl % L;
  const int64_t pos = start + l;
  const int cols = (G - 1) * H;
  int64_t *o = out + (bl * nL + layer) * cols;
  const int64_t *mrow = mult + (int64_t)layer * G;
  bool blocked = false;
  int64_t rolling = 0;
  for (int shift = 0; shift < G; ++shift) {
    const int64_t src = pos - shift < 0 ? 0 : pos - shift;
    blocked = blocked || (pos < shift);
    const int64_t tok = blocked ? pad_id : cache[b * max_seq + src];
    const int64_t prod = tok * mrow[shift];
    rolling = shift == 0 ? prod : (rolling ^ prod);
    if (shift >= 1) {
      const int64_t *pr = primes + ((int64_t)layer * (G - 1) + (shift - 1)) * H;
      const int64_t *of = offsets + (int64_t)layer * cols + (shift - 1) * H;
      for (int h = 0; h < H; ++h) o[(shift - 1) * H + h] = rolling % pr[h] + of[h];
    }
  }
}

template <typename T> __device__ __forceinline__ void store_out(T *p, float v);
template <> __device__ __forceinline__ void store_out<float>(float *p, float v) { *p = v; }
template <> __device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16 *p, float v) {
  *p = __float2bfloat16_rn(v);
}

// One warp per gathered row; each lane decodes 8-byte chunks.  d % 8 == 0.
template <typename T>
__global__ void k_engram_gather_rows(const uint8_t *__restrict__ table,
                                     const uint8_t *__restrict__ scale, int64_t rows,
                                     int64_t row_lo, int64_t d, int64_t block,
                                     const int64_t *__restrict__ idx, int64_t n_idx,
                                     T *__restrict__ out) {
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_idx) return;
  const int64_t local = idx[warp] - row_lo;
  const bool in = local >= 0 && local < rows;
  const int64_t sb = d / block;
  T *o = out + warp * d;
  for (int64_t c = lane * 8; c < d; c += 256) {
    float f[8];
    if (in) {
      const uint64_t v = __ldg(reinterpret_cast<const unsigned long long *>(table + local * d + c));
      uint32_t h[4];
      e4m3x4_to_f16x4(uint32_t(v), h[0], h[1]);
      e4m3x4_to_f16x4(uint32_t(v >> 32), h[2], h[3]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sc = e8m0f(scale[local * sb + (c + j) / block]);
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

// One warp per token; D_PER_LANE = d / 32 values per lane (d = 32 * D_PER_LANE,
// D_PER_LANE % 8 == 0); rows summed in column order, fp32.
template <typename T, int D_PER_LANE>
__global__ void __launch_bounds__(256) k_engram_gather_sum(
    const uint8_t *__restrict__ table, const uint8_t *__restrict__ scale, int64_t rows,
    int64_t row_lo, int64_t block, const int64_t *__restrict__ idx, int64_t n_tok, int n_per_tok,
    T *__restrict__ out) {
  constexpr int64_t D = 32 * D_PER_LANE;
  constexpr int CH = D_PER_LANE / 8;  // 8-byte chunks per lane per row
  const int64_t tok = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= n_tok) return;
  const int64_t sb = D / block;
  float acc[D_PER_LANE];
#pragma unroll
  for (int j = 0; j < D_PER_LANE; ++j) acc[j] = 0.0f;
  const int64_t *ti = idx + tok * n_per_tok;
  // lane owns columns [c*256 + lane*8, +8) for c in [0, CH): coalesced 256-byte spans
  for (int h = 0; h < n_per_tok; h += 4) {
    uint64_t v[4][CH];
    float sc[4][CH];
    bool in[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int hh = h + u;
      const int64_t local = hh < n_per_tok ? ti[hh] - row_lo : -1;
      in[u] = hh < n_per_tok && local >= 0 && local < rows;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int64_t col = c * 256 + lane * 8;
        v[u][c] = in[u] ? __ldg(reinterpret_cast<const unsigned long long *>(table + local * D + col))
                        : 0ull;
        sc[u][c] = in[u] ? e8m0f(scale[local * sb + col / block]) : 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (!in[u]) continue;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        uint32_t hh[4];
        e4m3x4_to_f16x4(uint32_t(v[u][c]), hh[0], hh[1]);
        e4m3x4_to_f16x4(uint32_t(v[u][c] >> 32), hh[2], hh[3]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 p = h2f2(hh[j >> 1]);
          // block >= 8 and 8 | block keep the 8 columns in one scale block
          acc[c * 8 + j] = __fadd_rn(acc[c * 8 + j], __fmul_rn((j & 1) ? p.y : p.x, sc[u][c]));
        }
      }
    }
  }
  T *o = out + tok * D;
#pragma unroll
  for (int c = 0; c < CH; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) store_out<T>(o + c * 256 + lane * 8 + j, acc[c * 8 + j]);
}

}  // namespace dsv41
