// prefill.cuh -- MoE prefill bookkeeping around the block-scaled grouped GEMM.
//
// Upstream MoE.forward (docs/reference/model.py:889-904) loops over experts and runs each
// expert on the tokens routed to it.  Here the (token, slot) pairs are sorted by expert
// once (a stable counting sort: pairs keep row-major [T, k] order inside an expert), the
// fp8 activation rows are gathered into that order, the grouped GEMMs walk per-expert
// tiles, and the combine sums every token's expert outputs in ascending expert order
// (the order of upstream's loop) before adding the shared expert.
#pragma once
#include "bsgemm.cuh"
#include "common.cuh"

namespace dsv41 {

constexpr int PF_CHUNK = 512;       // pairs per counting block (16 warps)
constexpr int PF_TILE_ROWS = 224;   // activation rows per GEMM tile (the GEMM's N)

struct PfPlan {
  int *chunk_base;     // [nchunks, E]: pairs of expert e in earlier chunks
  int *grp_off;        // [E] first sorted position of expert e
  int *grp_rt0;        // [E] first row tile of expert e (tiles of <= 224 rows, numbered in order)
  int *pair_tok;       // [P] token of sorted pair
  float *pair_w;       // [P] routing weight of sorted pair
  int *slot_pos;       // [T*k] sorted position of pair (t, j)
  int *pair_exp;       // [P] expert of sorted pair (written when non-null)
  int *row_tile;       // [P] (row tile << 8) | row within the tile, of sorted pair
  int4 *tiles[4];      // {expert, m-tile, first row, rows | row tile << 8}: gate/up wide,
                       // gate/up narrow, down wide, down narrow
  int *ntiles;         // [4] tile counts of the four lists
  int *next_tile;      // [4] work counters of the four launches (zeroed here)
};

// Tiles with at most this many rows (after rounding up to 16) go to the narrow GEMM shape.
constexpr int PF_NARROW_ROWS = 64;

__global__ void __launch_bounds__(PF_CHUNK) k_pf_count(const int32_t *__restrict__ idx, int64_t P,
                                                       int E, int *__restrict__ chunk_cnt) {
  extern __shared__ int wh[];   // [16][E]
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 16 * E; i += PF_CHUNK) wh[i] = 0;
  __syncthreads();
  const int64_t p = int64_t(blockIdx.x) * PF_CHUNK + threadIdx.x;
  if (p < P) {
    const int e = idx[p];
    if (e >= 0 && e < E) atomicAdd(&wh[warp * E + e], 1);
    else dev_flag(DSV41_DEVST_BAD_INDEX);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += PF_CHUNK) {
    int s = 0;
#pragma unroll
    for (int w = 0; w < 16; ++w) s += wh[w * E + e];
    chunk_cnt[int64_t(blockIdx.x) * E + e] = s;
  }
}

// Exclusive block-wide scan of three values per thread (1024 threads).
__device__ __forceinline__ void block_scan3(int (&v)[3], int (&excl)[3], int (&total)[3]) {
  __shared__ int wt[3][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int inc[3] = {v[0], v[1], v[2]};
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int u = __shfl_up_sync(0xffffffffu, inc[k], o);
      if (lane >= o) inc[k] += u;
    }
  }
  if (lane == 31) {
#pragma unroll
    for (int k = 0; k < 3; ++k) wt[k][wid] = inc[k];
  }
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      int t = lane < nw ? wt[k][lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += u;
      }
      wt[k][lane] = t;
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    excl[k] = inc[k] - v[k] + (wid > 0 ? wt[k][wid - 1] : 0);
    total[k] = wt[k][(blockDim.x >> 5) - 1];
  }
}

// One CTA of 1024 threads, one expert per thread (E <= 1024).  An expert with n pairs has
// ceil(n / 224) row tiles; its last tile is narrow when it holds <= 64 rows.  Each list is
// ordered expert-major, then m-tile, then row tile, so tiles that share weights or
// activations are taken close together.  The tile records are written by one warp per
// expert, its lanes striding over the expert's tiles.
__global__ void __launch_bounds__(1024) k_pf_scan(int *__restrict__ chunk_cnt, int nchunks, int E,
                                                  int mt_gu, int mt_dn, PfPlan plan) {
  __shared__ int s_off[1024], s_rt0[1024], s_wide[1024], s_nar[1024], s_run[1024];
  __shared__ int s_excl_w[1024], s_excl_n[1024];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    int c = 0;
    for (; c + 8 <= nchunks; c += 8) {   // 8 independent loads in flight
      int v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = chunk_cnt[int64_t(c + u) * E + e];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        chunk_cnt[int64_t(c + u) * E + e] = run;
        run += v[u];
      }
    }
    for (; c < nchunks; ++c) {
      const int v = chunk_cnt[int64_t(c) * E + e];
      chunk_cnt[int64_t(c) * E + e] = run;
      run += v;
    }
  }
  const int nnt = (run + PF_TILE_ROWS - 1) / PF_TILE_ROWS;
  const int tail = run - (nnt - 1) * PF_TILE_ROWS;
  const int nnar = (nnt > 0 && ((tail + 15) & ~15) <= PF_NARROW_ROWS) ? 1 : 0;
  const int nwide = nnt - nnar;
  int v[3] = {run, nwide, nnar}, excl[3], tot[3];
  block_scan3(v, excl, tot);
  // row tiles are numbered expert by expert: expert e owns [rt0, rt0 + nnt)
  const int rt0 = excl[1] + excl[2];
  if (e < E) {
    plan.grp_off[e] = excl[0];
    plan.grp_rt0[e] = rt0;
    s_off[e] = excl[0];
    s_rt0[e] = rt0;
    s_wide[e] = nwide;
    s_nar[e] = nnar;
    s_run[e] = run;
    s_excl_w[e] = excl[1];
    s_excl_n[e] = excl[2];
  }
  if (threadIdx.x == 0) {
    plan.ntiles[0] = tot[1] * mt_gu;
    plan.ntiles[1] = tot[2] * mt_gu;
    plan.ntiles[2] = tot[1] * mt_dn;
    plan.ntiles[3] = tot[2] * mt_dn;
    for (int i = 0; i < 4; ++i) plan.next_tile[i] = 0;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int ee = warp; ee < E; ee += blockDim.x >> 5) {
    const int nw = s_wide[ee], rn = s_run[ee], off = s_off[ee], r0 = s_rt0[ee];
    const int mts[2] = {mt_gu, mt_dn};
    for (int pj = 0; pj < 2; ++pj) {
      const int mt_n = mts[pj];
      int4 *tw = plan.tiles[2 * pj] + int64_t(s_excl_w[ee]) * mt_n;
      // token tile by token tile, the m-tiles of one next to each other (a CTA pair takes
      // m-tiles 2i and 2i + 1 of one token tile)
      for (int i = lane; i < mt_n * nw; i += 32) {
        const int mt = i % mt_n, j = i / mt_n;
        tw[i] = make_int4(ee, mt, off + j * PF_TILE_ROWS,
                          min(PF_TILE_ROWS, rn - j * PF_TILE_ROWS) | ((r0 + j) << 8));
      }
      if (s_nar[ee]) {
        int4 *tn = plan.tiles[2 * pj + 1] + int64_t(s_excl_n[ee]) * mt_n;
        for (int mt = lane; mt < mt_n; mt += 32)
          tn[mt] = make_int4(ee, mt, off + nw * PF_TILE_ROWS,
                             (rn - nw * PF_TILE_ROWS) | ((r0 + nw) << 8));
      }
    }
  }
}

// Stable placement: rank inside the chunk from per-warp counts and warp-level matching.
__global__ void __launch_bounds__(PF_CHUNK) k_pf_place(const int32_t *__restrict__ idx,
                                                       const float *__restrict__ w, int64_t P,
                                                       int topk, int E, PfPlan plan) {
  extern __shared__ int wh[];   // [16][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 16 * E; i += PF_CHUNK) wh[i] = 0;
  __syncthreads();
  const int64_t p = int64_t(blockIdx.x) * PF_CHUNK + threadIdx.x;
  int e = -1;
  if (p < P) {
    e = idx[p];
    if (e < 0 || e >= E) e = -1;
  }
  if (p < P && e < 0) plan.slot_pos[p] = -1;   // skipped by the combine
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wh[warp * E + e] = __popc(peers);
  __syncthreads();
  if (e >= 0) {
    int before = 0;
    for (int w2 = 0; w2 < warp; ++w2) before += wh[w2 * E + e];
    const int in_e = plan.chunk_base[int64_t(blockIdx.x) * E + e] + before + rank;
    const int pos = plan.grp_off[e] + in_e;
    plan.pair_tok[pos] = int(p / topk);
    plan.pair_w[pos] = w ? w[p] : 1.0f;
    if (plan.pair_exp) plan.pair_exp[pos] = e;
    plan.slot_pos[p] = pos;
    plan.row_tile[pos] = ((plan.grp_rt0[e] + in_e / PF_TILE_ROWS) << 8) | (in_e % PF_TILE_ROWS);
  }
}

// dst row r = src row tok[r] for the fp8 codes (K bytes); the row's ue8m0 scales (K/32) go
// to its row tile's scale atoms (the tcgen05.cp layout the GEMM bulk-copies per K stage).
// xq / xs rows are qld / sld bytes apart (K and K/32 for act_quant's output; the packed
// row size for rows received by an expert-parallel owner).
__global__ void k_pf_gather(const uint8_t *__restrict__ xq, const uint8_t *__restrict__ xs,
                            int64_t qld, int64_t sld, const int *__restrict__ tok,
                            const int *__restrict__ row_tile, int64_t R, int64_t K,
                            uint8_t *__restrict__ dq, uint8_t *__restrict__ datoms) {
  const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const int64_t t = tok[r];
  const uint4 *src = reinterpret_cast<const uint4 *>(xq + t * qld);
  uint4 *dst = reinterpret_cast<uint4 *>(dq + r * K);
  for (int64_t i = lane; i < K / 16; i += 32) dst[i] = __ldg(src + i);
  const int rt = row_tile[r] >> 8, lr = row_tile[r] & 0xFF;
  const uint32_t *ss = reinterpret_cast<const uint32_t *>(xs + t * sld);
  uint8_t *base = datoms + int64_t(rt) * (K / 128) * 1024;
  for (int64_t i = lane; i < K / 128; i += 32)   // 4 scales (one K stage) per word
    *reinterpret_cast<uint32_t *>(base + sf_atom_off(lr, int(4 * i))) = __ldg(ss + i);
}

// Expert parallelism.  A pair travels as one packed row: the token's fp8 codes (K bytes),
// their ue8m0 scales (K/32), the owner-local expert id (int32) and the routing weight (f32),
// padded to 16 bytes.  Source side: rows in expert-sorted order (so grouped by owner).
__host__ __device__ constexpr int64_t ep_row_bytes(int64_t K) {
  return (K + K / 32 + 8 + 15) / 16 * 16;
}

__global__ void k_ep_pack(const uint8_t *__restrict__ xq, const uint8_t *__restrict__ xs,
                          const int *__restrict__ pair_tok, const int *__restrict__ pair_exp,
                          const float *__restrict__ pair_w, int64_t P, int64_t K, int epr,
                          uint8_t *__restrict__ rows) {
  const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= P) return;
  const int64_t t = pair_tok[r], rb = ep_row_bytes(K);
  uint8_t *row = rows + r * rb;
  const uint4 *src = reinterpret_cast<const uint4 *>(xq + t * K);
  for (int64_t i = lane; i < K / 16; i += 32) reinterpret_cast<uint4 *>(row)[i] = __ldg(src + i);
  const uint32_t *ss = reinterpret_cast<const uint32_t *>(xs + t * (K / 32));
  for (int64_t i = lane; i < K / 128; i += 32)
    reinterpret_cast<uint32_t *>(row + K)[i] = __ldg(ss + i);
  if (lane == 0) {
    reinterpret_cast<int32_t *>(row + K + K / 32)[0] = pair_exp[r] % epr;
    reinterpret_cast<float *>(row + K + K / 32)[1] = pair_w[r];
  }
}

// Pairs per owner rank from the expert offsets: owner r holds experts [r*epr, (r+1)*epr).
__global__ void k_ep_counts(const int *__restrict__ grp_off, int E, int epr, int64_t P,
                            int world, int64_t *__restrict__ counts) {
  const int r = threadIdx.x;
  if (r >= world) return;
  const int64_t lo = grp_off[r * epr];
  const int64_t hi = (r + 1) * epr < E ? grp_off[(r + 1) * epr] : P;
  counts[r] = hi - lo;
}

// Owner side: the expert id and routing weight of each received row.
__global__ void k_ep_unpack(const uint8_t *__restrict__ rows, int64_t R, int64_t K,
                            int32_t *__restrict__ ids, float *__restrict__ w) {
  const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= R) return;
  const uint8_t *tail = rows + r * ep_row_bytes(K) + K + K / 32;
  ids[r] = reinterpret_cast<const int32_t *>(tail)[0];
  w[r] = reinterpret_cast<const float *>(tail)[1];
}

// Weight scales -> tcgen05.cp atoms, once per weight set.  Scale row of weight row r is
// r >> rshift (0: per-row fp4 scales; 5: fp8 32x32 blocks).  One thread per (atom, lane):
// a 16-byte row of atom (g, mt, kq) holds the 4 per-32 scales of K stage kq for rows
// 32c + l, c = 0..3, of the tile.  paired: the tile is 64 rows of s (c = 0, 1) and the
// same 64 rows of s2 (c = 2, 3) -- the gate/up pairing of the SwiGLU GEMM.
__global__ void k_pack_sfw(const uint8_t *__restrict__ sc, const uint8_t *__restrict__ sc2,
                           int64_t groups, int64_t rows, int64_t K, int paired, int rshift,
                           uint8_t *__restrict__ out) {
  const int64_t nkq = K / 128, mt_rows = paired ? 64 : 128, mtiles = rows / mt_rows;
  const int64_t n = groups * mtiles * nkq * 32;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int l = int(i & 31);
    const int64_t atom = i >> 5;
    const int64_t kq = atom % nkq, mt = (atom / nkq) % mtiles, g = atom / (nkq * mtiles);
    uint32_t w[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint8_t *src = (paired && c >= 2) ? sc2 : sc;
      const int64_t row = g * rows + mt * mt_rows + 32 * (paired ? (c & 1) : c) + l;
      w[c] = __ldg(reinterpret_cast<const uint32_t *>(src + (row >> rshift) * (K / 32) + 4 * kq));
    }
    *reinterpret_cast<uint4 *>(out + atom * 512 + l * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// out[t, :] = sum over the token's experts in ascending id order of Yp[pos] (bf16), then
// + Ys[t, :] (bf16, may be null); fp32 arithmetic.  8 columns per thread.
template <typename TO>
__global__ void k_pf_combine(const __nv_bfloat16 *__restrict__ Yp, const __nv_bfloat16 *__restrict__ Ys,
                             const int32_t *__restrict__ idx, const int *__restrict__ slot_pos,
                             int64_t T, int topk, int64_t D, TO *__restrict__ out) {
  const int64_t groups = D / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * groups) return;
  const int64_t t = i / groups, c0 = (i % groups) * 8;
  // the token's (expert, slot) pairs, sorted by expert id with a fixed compare-exchange
  // network (registers only; unused entries sort last), then all its rows loaded at once and
  // added in that order
  int ids[8], pos[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ids[j] = j < topk ? idx[t * topk + j] : 0x7fffffff;
    pos[j] = j < topk ? slot_pos[t * topk + j] : -1;
  }
#pragma unroll
  for (int a = 0; a < 7; ++a)
#pragma unroll
    for (int b = 0; b < 7 - a; ++b)
      if (ids[b] > ids[b + 1]) {
        const int ti = ids[b], tp = pos[b];
        ids[b] = ids[b + 1];
        pos[b] = pos[b + 1];
        ids[b + 1] = ti;
        pos[b + 1] = tp;
      }
  uint4 rv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    rv[j] = pos[j] >= 0 ? *reinterpret_cast<const uint4 *>(Yp + int64_t(pos[j]) * D + c0)
                        : make_uint4(0, 0, 0, 0);
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (pos[j] < 0) continue;
    const uint32_t wv[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      acc[2 * c] = __fadd_rn(acc[2 * c], bf_bits2f(uint16_t(wv[c] & 0xFFFF)));
      acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], bf_bits2f(uint16_t(wv[c] >> 16)));
    }
  }
  if (Ys) {
    const uint4 v = *reinterpret_cast<const uint4 *>(Ys + t * D + c0);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      acc[2 * c] = __fadd_rn(acc[2 * c], bf_bits2f(uint16_t(wv[c] & 0xFFFF)));
      acc[2 * c + 1] = __fadd_rn(acc[2 * c + 1], bf_bits2f(uint16_t(wv[c] >> 16)));
    }
  }
  if constexpr (sizeof(TO) == 4) {
    float4 *o = reinterpret_cast<float4 *>(out + t * D + c0);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  } else {
    uint4 o;
    o.x = uint32_t(f2bf_bits(acc[0])) | (uint32_t(f2bf_bits(acc[1])) << 16);
    o.y = uint32_t(f2bf_bits(acc[2])) | (uint32_t(f2bf_bits(acc[3])) << 16);
    o.z = uint32_t(f2bf_bits(acc[4])) | (uint32_t(f2bf_bits(acc[5])) << 16);
    o.w = uint32_t(f2bf_bits(acc[6])) | (uint32_t(f2bf_bits(acc[7])) << 16);
    *reinterpret_cast<uint4 *>(out + t * D + c0) = o;
  }
}

}  // namespace dsv41
