// ep_decode.cuh -- expert-parallel MoE decode over NVLink peer memory.
//
// Replaces upstream's replicate + fp32 all_reduce expert parallelism
// (docs/reference/model.py:854-904) at decode: rank r owns experts
// [r*E/ws, (r+1)*E/ws); each rank routes its own tokens and only the (token, expert)
// pairs travel, written by the source straight into the owner's receive buffer and
// returned by the owner straight into the source's return buffer (plain stores to a
// peer's memory mapped through CUDA IPC; no multicast, no collective library, no host
// synchronisation).
//
// Every rank holds one buffer (EpLayout), mapped by every peer:
//   rows  bf16 [ws][C][D]   rows sent to this rank by source s at [s][i]
//   meta  i32  [ws][C]      owner-local expert id of row [s][i]
//   cnt   i32  [ws]         rows source s sent in this step
//   back  f32  [ws][C][D]   expert outputs of this rank's pairs, from owner o at [o][i]
//   flags u64  [2][ws]      [0][s]: source s finished writing rows; [1][o]: owner o
//                           finished returning outputs (values = step sequence number)
// C = max_tokens * topk.  Steps are numbered by a per-rank device counter (seq) that every
// rank advances once per step, so flags never need clearing.  Ordering: a writer fences at
// system scope after its stores, the last CTA of a grid publishes the flag with a release
// store; the reader polls with acquire loads (bounded by wall time, then it raises the
// device status bit and moves on rather than hang).  A step's buffers are never rewritten
// before every reader is done with them: a source starts step s+1 only after it has all
// step-s outputs, which owners send only after reading the step-s rows.
#pragma once
#include "common.cuh"

namespace dsv41 {

constexpr int EP_MAX_RANKS = 64;

struct EpLayout {
  int ws;
  int64_t C, D;
  size_t rows, meta, cnt, back, flags, total;
};

inline EpLayout ep_layout(int ws, int64_t C, int64_t D) {
  EpLayout L;
  L.ws = ws;
  L.C = C;
  L.D = D;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = (off + bytes + 255) / 256 * 256;
    return o;
  };
  L.rows = take(size_t(ws) * C * D * 2);
  L.meta = take(size_t(ws) * C * 4);
  L.cnt = take(size_t(ws) * 4);
  L.back = take(size_t(ws) * C * D * 4);
  L.flags = take(size_t(2) * ws * 8);
  L.total = off;
  return L;
}

struct EpPeers {
  uint8_t *base[EP_MAX_RANKS];   // every rank's buffer, this rank's own at [rank]
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Copy `bytes` (a multiple of 16) from src to dst with the whole CTA, 16-byte vectors.
__device__ __forceinline__ void cta_copy16(void *dst, const void *src, int64_t bytes) {
  const uint4 *s = reinterpret_cast<const uint4 *>(src);
  uint4 *d = reinterpret_cast<uint4 *>(dst);
  for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldg(s + i);
}

// Last CTA of a (owner/source) column publishes `flag` after every CTA's stores.
__device__ __forceinline__ void ep_publish(unsigned *done, int col, int ncta,
                                           unsigned long long *flag, unsigned long long seq) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();                       // this CTA's peer stores, system-visible
    const unsigned prev = atomicAdd(done + col, 1u);
    if (prev == unsigned(ncta - 1)) {
      done[col] = 0;                              // ready for the next step
      __threadfence_system();
      st_release_sys_u64(flag, seq);
    }
  }
}

// Source side.  grid (ws owners, nb CTAs per owner), 256 threads, dynamic smem P ints.
// Each CTA lists the pairs routed to its owner in (token, slot) order (a stable block
// compaction), CTA 0 of the owner writes the owner-local expert ids, the count and this
// rank's slot_pos (row o*C + i of pair p in the return buffer), and all CTAs copy the
// token rows into the owner's receive buffer.
__global__ void __launch_bounds__(256) k_ep_dispatch(
    const __nv_bfloat16 *__restrict__ x, const int32_t *__restrict__ idx, int T, int k, int epr,
    int rank, EpLayout L, EpPeers peers, const unsigned long long *__restrict__ dseq,
    int32_t *__restrict__ slot_pos, unsigned *__restrict__ done) {
  extern __shared__ int plist[];
  __shared__ int wsum[8];
  __shared__ int s_n;
  const int o = blockIdx.x, b = blockIdx.y, nb = gridDim.y;
  const int P = T * k, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (P + 255) / 256, p0 = min(P, tid * per), p1 = min(P, p0 + per);
  int c = 0;
  for (int p = p0; p < p1; ++p) {
    const int e = idx[p];
    c += (e >= 0 && e / epr == o);
  }
  int inc = c;
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, inc, s);
    if (lane >= s) inc += u;
  }
  if (lane == 31) wsum[wid] = inc;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < wid; ++w) before += wsum[w];
  int pos = before + inc - c;
  for (int p = p0; p < p1; ++p) {
    const int e = idx[p];
    if (e >= 0 && e / epr == o) plist[pos++] = p;
  }
  if (tid == 255) s_n = pos;
  __syncthreads();
  const int n = s_n;
  uint8_t *dst = peers.base[o];
  const unsigned long long seq = *dseq + 1;
  if (b == 0) {
    int32_t *meta = reinterpret_cast<int32_t *>(dst + L.meta) + (int64_t)rank * L.C;
    for (int i = tid; i < n; i += blockDim.x) {
      const int p = plist[i];
      slot_pos[p] = int32_t(o * L.C + i);
      meta[i] = idx[p] - o * epr;
    }
    if (tid == 0) reinterpret_cast<int32_t *>(dst + L.cnt)[rank] = n;
  }
  __nv_bfloat16 *rows = reinterpret_cast<__nv_bfloat16 *>(dst + L.rows) + (int64_t)rank * L.C * L.D;
  for (int i = b; i < n; i += nb)
    cta_copy16(rows + (int64_t)i * L.D, x + (int64_t)(plist[i] / k) * L.D, L.D * 2);
  ep_publish(done, o, nb,
             reinterpret_cast<unsigned long long *>(dst + L.flags) + rank, seq);
}

// Wait until flags[which][s] reached this step for every rank s (one thread per rank).
__global__ void k_ep_wait(const uint8_t *own, EpLayout L, int which,
                          const unsigned long long *__restrict__ dseq) {
  const int s = threadIdx.x;
  if (s >= L.ws) return;
  const unsigned long long seq = *dseq + 1;
  const unsigned long long *f =
      reinterpret_cast<const unsigned long long *>(own + L.flags) + which * L.ws + s;
  if (ld_acquire_sys_u64(f) >= seq) return;
  const uint64_t t0 = globaltimer_ns();
  const unsigned long long lim = g_wait_ns;
  for (uint32_t it = 0; it < (1u << 26); ++it) {
    __nanosleep(128);
    if (ld_acquire_sys_u64(f) >= seq) return;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > lim) break;
  }
  dev_flag(DSV41_DEVST_TIMEOUT);
}

// Received rows of source s, before it: the rows of sources 0 .. s-1 (compact order).
__device__ __forceinline__ int ep_rows_before(const uint8_t *own, const EpLayout &L, int s) {
  const int32_t *cnt = reinterpret_cast<const int32_t *>(own + L.cnt);
  int b = 0;
  for (int r = 0; r < s; ++r) b += cnt[r];
  return b;
}

// Owner side: the received rows listed compactly, source by source -- ids[j] the owner-local
// expert of the j-th valid row and rowmap[j] its row in the receive buffer; -1 ids after
// the last valid row (padding), and their count in *n_valid, so the plan reads only the
// rows that arrived.
__global__ void k_ep_ids(const uint8_t *own, EpLayout L, int32_t *__restrict__ ids,
                         int32_t *__restrict__ rowmap, int *__restrict__ n_valid) {
  const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int32_t *cnt = reinterpret_cast<const int32_t *>(own + L.cnt);
  if (j == 0) *n_valid = ep_rows_before(own, L, L.ws);     // every received row
  if (j >= L.ws * L.C) return;
  int64_t before = 0;
  for (int s = 0; s < L.ws; ++s) {
    const int n = cnt[s];
    if (j < before + n) {
      const int64_t row = s * L.C + (j - before);
      ids[j] = reinterpret_cast<const int32_t *>(own + L.meta)[row];
      rowmap[j] = int32_t(row);
      return;
    }
    before += n;
  }
  ids[j] = -1;
  rowmap[j] = 0;
}

// Owner side.  grid (ws sources, nb), 256 threads: the fp32 outputs of source s's rows
// (compact rows before(s) + i) go back into source s's return buffer at [this rank][i].
__global__ void __launch_bounds__(256) k_ep_return(
    const float *__restrict__ Y, const uint8_t *own, int rank, EpLayout L, EpPeers peers,
    const unsigned long long *__restrict__ dseq, unsigned *__restrict__ done) {
  const int s = blockIdx.x, b = blockIdx.y, nb = gridDim.y;
  const int n = reinterpret_cast<const int32_t *>(own + L.cnt)[s];
  const int64_t y0 = ep_rows_before(own, L, s);       // Y rows are in compact order
  uint8_t *dst = peers.base[s];
  const unsigned long long seq = *dseq + 1;
  float *back = reinterpret_cast<float *>(dst + L.back) + (int64_t)rank * L.C * L.D;
  for (int i = b; i < n; i += nb)
    cta_copy16(back + (int64_t)i * L.D, Y + (y0 + i) * L.D, L.D * 4);
  ep_publish(done, s, nb,
             reinterpret_cast<unsigned long long *>(dst + L.flags) + L.ws + rank, seq);
}

// Source side: out[t] = sum_j w[t, j] * back[slot_pos[t*k + j]] (j order, fp32) + Ys[t],
// the single-GPU combine's operations; then the step counter advances.
template <typename TO>
__global__ void k_ep_combine_decode(const uint8_t *own, EpLayout L, const int32_t *__restrict__ slot_pos,
                                    const float *__restrict__ w, const float *__restrict__ Ys,
                                    int64_t T, int topk, TO *__restrict__ out,
                                    unsigned long long *__restrict__ dseq) {
  const float *back = reinterpret_cast<const float *>(own + L.back);
  const int64_t D = L.D;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < T * D;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / D, n = i % D;
    float acc = 0.0f;
    for (int j = 0; j < topk; ++j)
      acc = __fadd_rn(acc, __fmul_rn(back[(int64_t)slot_pos[t * topk + j] * D + n], w[t * topk + j]));
    if (Ys) acc = __fadd_rn(acc, Ys[i]);
    if constexpr (sizeof(TO) == 4)
      out[i] = acc;
    else
      out[i] = __float2bfloat16_rn(acc);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *dseq += 1;   // read again only by the next step
}

}  // namespace dsv41
