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

// Pairs per chunk: one n8 tile of activation rows for gate/up (8 pairs), and for
// down 8 H rows = 4 pairs (hi/lo halves).  Experts with more pairs get more chunks.
constexpr int MOE_GU_CHUNK = 8;
constexpr int MOE_DN_CHUNK = 4;

// One CTA of 1024 threads.  Deterministic: a pair's rank inside its expert is
// the number of earlier pairs (row-major over [T, k]) routed to the same expert.
__global__ void __launch_bounds__(1024) k_moe_plan(const int32_t *__restrict__ indices, int64_t T,
                                                   int topk, int64_t E, MoePlan plan) {
  extern __shared__ int sh[];
  int *cnt = sh;            // [E]
  int *poff = sh + E;       // [E] padded pair offset
  int *coff = sh + 2 * E;   // [E] gate/up chunk offset
  int *doff = sh + 3 * E;   // [E] down chunk offset
  const int64_t P = T * topk;
  for (int64_t e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = indices[p];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else dev_flag(DSV41_DEVST_BAD_INDEX);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int po = 0, co = 0, dn = 0;
    for (int64_t e = 0; e < E; ++e) {
      poff[e] = po;
      coff[e] = co;
      doff[e] = dn;
      po += (cnt[e] + 3) & ~3;
      co += (cnt[e] + MOE_GU_CHUNK - 1) / MOE_GU_CHUNK;
      dn += (cnt[e] + MOE_DN_CHUNK - 1) / MOE_DN_CHUNK;
    }
    plan.counts[0] = co;
    plan.counts[1] = dn;
    plan.counts[2] = po;
    const int sgu = int((T + 31) / 32), sdn = int((T + 15) / 16);
    plan.counts[3] = sgu;
    plan.counts[4] = sdn;
    for (int c = 0; c < sgu; ++c)
      plan.sgu_chunks[c] = QChunk{0, 32 * c, int(T - 32 * c < 32 ? T - 32 * c : 32), 32 * c};
    for (int c = 0; c < sdn; ++c) {
      const int nt = int(T - 16 * c < 16 ? T - 16 * c : 16);
      plan.sdn_chunks[c] = QChunk{0, 32 * c, 8 * ((nt + 3) / 4), 16 * c};
    }
  }
  __syncthreads();
  // chunks and padding slots, one thread per expert
  for (int64_t e = threadIdx.x; e < E; e += blockDim.x) {
    const int n = cnt[e];
    if (n == 0) continue;
    for (int c = 0; c * MOE_GU_CHUNK < n; ++c) {
      const int q0 = poff[e] + c * MOE_GU_CHUNK;
      const int np = min(MOE_GU_CHUNK, n - c * MOE_GU_CHUNK);
      plan.gu_chunks[coff[e] + c] = QChunk{int(e), q0, np, q0};
    }
    for (int c = 0; c * MOE_DN_CHUNK < n; ++c) {
      const int q0 = poff[e] + c * MOE_DN_CHUNK;   // multiple of 4: H rows 2*q0 ..
      const int np = min(MOE_DN_CHUNK, n - c * MOE_DN_CHUNK);
      plan.dn_chunks[doff[e] + c] = QChunk{int(e), 2 * q0, 8 * ((np + 3) / 4), q0};
    }
    for (int q = poff[e] + n; q < poff[e] + ((n + 3) & ~3); ++q) {
      plan.pair_tok[q] = -1;
      plan.pair_row[q] = -1;
    }
  }
  // pair placement
  for (int64_t p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = indices[p];
    if (e < 0 || e >= E) continue;
    int rank = 0;
    for (int64_t p2 = 0; p2 < p; ++p2) rank += (indices[p2] == e);
    const int q = poff[e] + rank;
    plan.pair_tok[q] = int(p / topk);
    plan.pair_row[q] = int(p);
  }
}

// out[t, n] = sum_j w[t, j] * Y[t*k + j, n] (j order, fp32) + Ys[t, n]
template <typename TO>
__global__ void k_moe_combine(const float *__restrict__ Y, const float *__restrict__ Ys,
                              const float *__restrict__ w, int64_t T, int topk, int64_t D,
                              TO *__restrict__ out) {
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
