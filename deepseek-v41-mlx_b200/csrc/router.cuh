// router.cuh -- MoE gate (a8): scores, sqrt-softplus / sigmoid / softmax, biased top-k.
//
// deepseek_v41_mlx/moe.py:58-74 (upstream Gate.forward docs/reference/model.py:809-827):
//   scores  = (x.f32 @ W.f32^T) / gate_temp            -- bf16 products are exact in
//                                                        fp32; accumulation is fp32
//   scores  = sqrt(softplus(scores)) | sigmoid | softmax
//   indices = top-k(scores + bias)                      -- the bias only selects
//   weights = scores[indices] / (sum + 1e-20) * route_scale
// Top-k returns experts in descending biased score; equal scores pick the lower
// expert id first.
#pragma once
#include "common.cuh"

namespace dsv41 {

// partial[ks][t][e] = sum over k in split ks of x[t, k] * W[e, k]
// one warp per (16 experts, 8 tokens, k split); K % (32 * nks) == 0
__global__ void __launch_bounds__(128) k_router_scores(const __nv_bfloat16 *__restrict__ x,
                                                       int64_t T, int64_t K,
                                                       const __nv_bfloat16 *__restrict__ w,
                                                       int64_t E, int nks,
                                                       float *__restrict__ partial) {
  pdl_wait();
  pdl_trigger();
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t etiles = (E + 15) / 16, ttiles = (T + 7) / 8;
  if (gw >= etiles * ttiles * nks) return;
  const int ks = int(gw % nks);
  const int64_t rest = gw / nks;
  const int64_t e0 = (rest % etiles) * 16, t0 = (rest / etiles) * 8;
  const int64_t klen = K / nks, kbeg = ks * klen;
  const bool ok0 = e0 + g < E, ok1 = e0 + g + 8 < E, okx = t0 + g < T;
  const uint4 z = make_uint4(0, 0, 0, 0);
  const __nv_bfloat16 *w0 = w + (e0 + g) * K + kbeg + 8 * t;
  const __nv_bfloat16 *w1 = w + (e0 + g + 8) * K + kbeg + 8 * t;
  const __nv_bfloat16 *xx = x + (t0 + g) * K + kbeg + 8 * t;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int64_t k = 0; k < klen; k += 64) {
    uint4 a0[2], a1[2], b[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const bool in = k + 32 * u < klen;
      a0[u] = (ok0 && in) ? __ldg(reinterpret_cast<const uint4 *>(w0 + k + 32 * u)) : z;
      a1[u] = (ok1 && in) ? __ldg(reinterpret_cast<const uint4 *>(w1 + k + 32 * u)) : z;
      b[u] = (okx && in) ? __ldg(reinterpret_cast<const uint4 *>(xx + k + 32 * u)) : z;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      mma_bf16(d, a0[u].x, a1[u].x, a0[u].y, a1[u].y, b[u].x, b[u].y);
      mma_bf16(d, a0[u].z, a1[u].z, a0[u].w, a1[u].w, b[u].z, b[u].w);
    }
  }
  // d[0] (e0+g, t0+2t), d[1] (e0+g, t0+2t+1), d[2] (e0+g+8, t0+2t), d[3] (e0+g+8, t0+2t+1)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t e = e0 + g + ((i & 2) ? 8 : 0), tok = t0 + 2 * t + (i & 1);
    if (e < E && tok < T) partial[((int64_t)ks * T + tok) * E + e] = d[i];
  }
}

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ float block_reduce_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
  return r;
}
__device__ __forceinline__ float block_reduce_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float r = 0.0f;
  for (int i = 0; i < nw; ++i) r += red[i];
  return r;
}

// one CTA per token, blockDim = 32 * ceil(E/32) (<= 1024)
__global__ void k_router_select(const float *__restrict__ partial, int nks, int64_t T, int64_t E,
                                const float *__restrict__ bias, int topk, int score_func,
                                float gate_temp, int norm_topk_prob, float route_scale,
                                float *__restrict__ weights, int32_t *__restrict__ indices) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ float sel_score[64];
  __shared__ int sel_idx[64];
  const int64_t tok = blockIdx.x;
  const int e = threadIdx.x;
  const bool valid = e < E;
  float s = 0.0f;
  if (valid) {
#pragma unroll 16
    for (int ks = 0; ks < nks; ++ks) s += partial[((int64_t)ks * T + tok) * E + e];   // loads in flight, adds in order
    s = __fdiv_rn(s, gate_temp);
  }
  float score;
  if (score_func == DSV41_SCORE_SOFTMAX) {
    const float m = block_reduce_max(valid ? s : -INFINITY, red);
    const float ex = valid ? expf(s - m) : 0.0f;
    const float sum = block_reduce_sum(ex, red);
    score = __fdiv_rn(ex, sum);
  } else if (score_func == DSV41_SCORE_SIGMOID) {
    score = __fdiv_rn(1.0f, 1.0f + expf(-s));
  } else {
    // softplus as logaddexp(s, 0) = max(s, 0) + log1p(exp(-|s|))
    const float sp = fmaxf(s, 0.0f) + log1pf(expf(-fabsf(s)));
    score = sqrtf(sp);
  }
  float biased = valid ? score + (bias ? bias[e] : 0.0f) : -INFINITY;
  if (isnan(biased)) biased = -INFINITY;
  // 1) every warp picks its own top-min(k, 32) with shuffles only (descending biased score,
  //    ties to the lower expert id) into the candidate pool
  __shared__ float cand_v[1024];
  __shared__ float cand_s[1024];
  __shared__ int cand_i[1024];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int kw = topk < 32 ? topk : 32;
  {
    float bv = biased;
    bool taken = false;
    for (int j = 0; j < kw; ++j) {
      ArgMax a{bv, (valid && !taken) ? e : 0x7fffffff};
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
        a = better(a, b);
      }
      const int src = a.i == 0x7fffffff ? 0 : a.i & 31;
      const float sc = __shfl_sync(0xffffffffu, score, src);
      if (lane == 0) {
        cand_v[w * kw + j] = a.v;
        cand_i[w * kw + j] = a.i;
        cand_s[w * kw + j] = sc;
      }
      if (e == a.i) {                             // remove from the next rounds
        bv = -INFINITY;
        taken = true;
      }
    }
  }
  __syncthreads();
  // 2) warp 0 merges the nw * kw candidates: topk rounds of argmax over the pool
  if (w == 0) {
    const int n = nw * kw;
    for (int j = 0; j < topk; ++j) {
      ArgMax a{-INFINITY, 0x7fffffff};
      int at = -1;
      for (int c = lane; c < n; c += 32) {
        const ArgMax b{cand_v[c], cand_i[c]};
        const ArgMax m = better(a, b);
        if (m.i != a.i || m.v != a.v) at = c;
        a = m;
      }
      int pos = at;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
        const int pb = __shfl_xor_sync(0xffffffffu, pos, o);
        const ArgMax m = better(a, b);
        if (m.i != a.i || m.v != a.v) pos = pb;
        a = m;
      }
      if (lane == 0) {
        sel_idx[j] = a.i;
        sel_score[j] = cand_s[pos];
        cand_v[pos] = -INFINITY;               // taken
        cand_i[pos] = 0x7fffffff;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int j = 0; j < topk; ++j) sum += sel_score[j];
    for (int j = 0; j < topk; ++j) {
      float wv = sel_score[j];
      if (norm_topk_prob && topk > 1) wv = __fdiv_rn(wv, sum + 1e-20f);
      wv = wv * route_scale;
      weights[tok * topk + j] = wv;
      indices[tok * topk + j] = sel_idx[j];
    }
  }
}

}  // namespace dsv41
