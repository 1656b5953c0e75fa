// moe.cuh -- MoE decode bookkeeping: pair plan and the weighted combine.
//
// deepseek_v41_mlx/moe.py:105-112 with mlx_lm SwitchGLU (moe.py:101-102): every
// (token t, slot j) pair runs expert indices[t, j]; expert outputs are weighted
// after the down projection and summed over j in fp32 (top-k order), then the
// shared expert is added.  The plan groups pairs by expert so that each expert's
// weights stream from HBM once per chunk of <= 16 pairs.
#pragma once
#include "common.cuh"
#include "qgemv.cuh"

namespace dsv41 {

struct MoePlan {
  int32_t *pair_tok;    // [Pmax] token of padded pair q (-1 = padding)
  int32_t *pair_row;    // [Pmax] output row t*k + j of pair q (-1 = padding)
  QChunk *gu_chunks;    // routed gate/up chunks
  QChunk *dn_chunks;    // routed down chunks
  QChunk *sgu_chunks;   // shared-expert gate/up chunks
  QChunk *sdn_chunks;   // shared-expert down chunks
  int *counts;          // [0] n_gu, [1] n_dn, [2] n_pairs_padded, [3] n_sgu, [4] n_sdn
};

// Pairs per chunk: gu_chunk = 8 * nt for gate/up (nt n8 tiles of activation rows) and
// dn_chunk = 4 * nt for down (8 H rows = 4 pairs an n8 tile, hi/lo halves), nt = 1, 2 or 4
// chosen per launch.  Experts with more pairs get more chunks.

// One CTA of 1024 threads (E <= 1024).  Deterministic: a pair's rank inside its
// expert is the number of earlier pairs (row-major over [T, k]) routed to the same
// expert.  Offsets come from block-wide exclusive scans over the experts.
// tok_map (optional): the activation row of pair p's token, instead of p / topk (expert-
// parallel owners list their received rows compactly, valid rows first).
// n_valid (optional): the pairs past this count are padding (-1) and are not read -- an
// expert-parallel owner lists its received rows first in a buffer sized for the most it
// can receive, so the plan's work follows the rows that arrived.
__global__ void __launch_bounds__(1024) k_moe_plan(const int32_t *__restrict__ indices, int64_t T,
                                                   int topk, int64_t E, MoePlan plan,
                                                   const int32_t *__restrict__ tok_map,
                                                   const int *__restrict__ n_valid, int gu_chunk,
                                                   int dn_chunk) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int sh[];
  int *cnt = sh;            // [E]
  int *poff = sh + E;       // [E] padded pair offset
  int *coff = sh + 2 * E;   // [E] gate/up chunk offset
  int *doff = sh + 3 * E;   // [E] down chunk offset
  __shared__ int wtot[3][32];
  int64_t P = T * topk;
  if (n_valid) {
    const int64_t nv = *n_valid;
    P = nv < P ? (nv > 0 ? nv : 0) : P;
  }
  const int e = threadIdx.x, lane = e & 31, wid = e >> 5;
  if (e < E) cnt[e] = 0;
  __syncthreads();
  for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
    const int ex = indices[p];
    if (ex >= 0 && ex < E) atomicAdd(&cnt[ex], 1);
    else if (ex >= E) dev_flag(DSV41_DEVST_BAD_INDEX);   // negative: a padding row, skipped
  }
  __syncthreads();
  const int n = e < E ? cnt[e] : 0;
  int v[3] = {(n + 3) & ~3, (n + gu_chunk - 1) / gu_chunk, (n + dn_chunk - 1) / dn_chunk};
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
    for (int k = 0; k < 3; ++k) wtot[k][wid] = inc[k];
  }
  __syncthreads();
  if (wid == 0) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int nw = blockDim.x >> 5;
      int t = lane < nw ? wtot[k][lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += u;
      }
      wtot[k][lane] = t;                       // inclusive prefix over warps
    }
  }
  __syncthreads();
  int excl[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) excl[k] = inc[k] - v[k] + (wid > 0 ? wtot[k][wid - 1] : 0);
  if (e < E) {
    poff[e] = excl[0];
    coff[e] = excl[1];
    doff[e] = excl[2];
  }
  if (e == blockDim.x - 1) {
    plan.counts[0] = excl[1] + v[1];
    plan.counts[1] = excl[2] + v[2];
    plan.counts[2] = excl[0] + v[0];
  }
  __syncthreads();
  // chunks and padding slots, one thread per expert
  if (e < E && n > 0) {
    for (int c = 0; c * gu_chunk < n; ++c) {
      const int q0 = poff[e] + c * gu_chunk;
      const int np = min(gu_chunk, n - c * gu_chunk);
      plan.gu_chunks[coff[e] + c] = QChunk{e, q0, np, q0};
    }
    for (int c = 0; c * dn_chunk < n; ++c) {
      const int q0 = poff[e] + c * dn_chunk;       // multiple of 4: H rows 2*q0 ..
      const int np = min(dn_chunk, n - c * dn_chunk);
      plan.dn_chunks[doff[e] + c] = QChunk{e, 2 * q0, 8 * ((np + 3) / 4), q0};
    }
    for (int q = poff[e] + n; q < poff[e] + ((n + 3) & ~3); ++q) {
      plan.pair_tok[q] = -1;
      plan.pair_row[q] = -1;
    }
  }
  // pair placement, stable (an expert's pairs in ascending p): pairs in chunks of the block;
  // a pair's rank = its expert's pairs in earlier chunks and earlier warps of this chunk
  // (a running count per expert, advanced warp by warp) + lower lanes of its own warp with
  // the same expert (warp match).  Only the warps that hold pairs take a turn.
  if (e < E) cnt[e] = 0;                       // reused as the running count
  __syncthreads();
  for (int64_t base = 0; base < P; base += blockDim.x) {
    const int64_t p = base + threadIdx.x;
    const int ex = p < P ? indices[p] : -1;
    const bool valid = ex >= 0 && ex < E;
    const unsigned grp = __match_any_sync(0xffffffffu, valid ? ex : -1);
    const int lower = __popc(grp & ((1u << lane) - 1u));
    const int64_t left = P - base;
    const int nw = int((left < int64_t(blockDim.x) ? left : int64_t(blockDim.x)) + 31) >> 5;
    int rank = 0;
    for (int w = 0; w < nw; ++w) {
      if (wid == w) {
        const int b = valid ? cnt[ex] : 0;
        __syncwarp();
        if (valid && lower == 0) cnt[ex] = b + __popc(grp);
        rank = b + lower;
      }
      __syncthreads();
    }
    if (valid) {
      const int q = poff[ex] + rank;
      plan.pair_tok[q] = tok_map ? tok_map[p] : int(p / topk);
      plan.pair_row[q] = int(p);
    }
  }
}

// out[t, n] = sum_j w[t, j] * Y[t*k + j, n] (j order, fp32) + Ys[t, n]
template <typename TO>
__global__ void k_moe_combine(const float *__restrict__ Y, const float *__restrict__ Ys,
                              const float *__restrict__ w, int64_t T, int topk, int64_t D,
                              TO *__restrict__ out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * D;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / D, n = i % D;
    float acc = 0.0f;
    for (int j = 0; j < topk; ++j)
      acc = __fadd_rn(acc, __fmul_rn(Y[(t * topk + j) * D + n], w[t * topk + j]));
    if (Ys) acc = __fadd_rn(acc, Ys[i]);
    if constexpr (sizeof(TO) == 4)
      out[i] = acc;
    else
      out[i] = __float2bfloat16_rn(acc);
  }
}

}  // namespace dsv41
