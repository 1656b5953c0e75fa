// common.cuh -- shared device/host helpers for libdsv41q (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "dsv41q.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libdsv41q is written for sm_100a (B200) only"
#endif

namespace dsv41 {

// ------------------------------------------------------------------ host error state
static thread_local char g_last_error[512] = "";

static inline int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static inline int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return DSV41_OK;
  return set_error(DSV41_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define DSV41_CHECK_LAUNCH(what)                                                \
  do {                                                                          \
    cudaError_t _e = cudaGetLastError();                                        \
    if (_e != cudaSuccess) return ::dsv41::cuda_status(_e, what);               \
  } while (0)

#define DSV41_LAUNCH(call, what)                                                \
  do {                                                                          \
    cudaError_t _le = (call);                                                   \
    if (_le != cudaSuccess) return ::dsv41::cuda_status(_le, what);             \
  } while (0)

#define DSV41_REQUIRE(cond, code, ...)                                          \
  do {                                                                          \
    if (!(cond)) return ::dsv41::set_error(code, __VA_ARGS__);                  \
  } while (0)

static inline bool aligned(const void *p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

static inline int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ------------------------------------------------------------------ device status flags
// bit 0: a bounded wait ran out; bit 1: an input id was out of range.
__device__ unsigned int g_dev_status;

#define DSV41_DEVST_TIMEOUT 1u
#define DSV41_DEVST_BAD_INDEX 2u

__device__ __forceinline__ void dev_flag(unsigned int bit) { atomicOr(&g_dev_status, bit); }

// ------------------------------------------------------------------ scalar decode
// ue8m0 byte -> 2^(b-127) as fp32 (b=0 -> 2^-127 subnormal, b=255 -> +inf, as
// mx.power(2, b-127) gives for the reference's e8m0_to_float).
__device__ __forceinline__ float e8m0f(uint32_t b) {
  return __uint_as_float(b ? (b << 23) : 0x00400000u);
}

// two e4m3 codes (low byte -> .x) -> exact f16x2
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// four e4m3 codes of a word -> two f16x2 (bytes 0,1 -> h0; bytes 2,3 -> h1)
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t w, uint32_t &h0, uint32_t &h1) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\tcvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(w));
}

// eight e2m1 nibbles of a word -> four f16x2 (byte b -> h_b; low nibble -> .x)
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t &h0, uint32_t &h1,
                                                uint32_t &h2, uint32_t &h3) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
}

__device__ __forceinline__ float2 h2f2(uint32_t h) {
  __half2 v = *reinterpret_cast<__half2 *>(&h);
  return __half22float2(v);
}

// Packed fp32 pairs (sm_100 f32x2 instructions): lane 0 in the low word.  Each lane is one
// IEEE round-to-nearest multiply / add, no flush to zero -- the same bits as __fmul_rn /
// __fadd_rn on the two lanes -- at one instruction for the pair.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  return (uint64_t(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float f32x2_lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float f32x2_hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }

__device__ __forceinline__ uint16_t f2bf_bits(float f) {
  __nv_bfloat16 b = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&b);
}

__device__ __forceinline__ float bf_bits2f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ float round_bf16f(float f) { return bf_bits2f(f2bf_bits(f)); }

// ------------------------------------------------------------------ mma.sync f16 / bf16
// D = A(16x16, row) * B(16x8, col) + C; fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(  // pure register computation: free to be scheduled between the loads
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(  // pure register computation
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ mbarrier / TMA
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wall-time limit of every bounded device wait, per device (dsv41_set_wait_limit_ns;
// default 2 s).
#define DSV41_WAIT_NS 2000000000ull
__device__ unsigned long long g_wait_ns = DSV41_WAIT_NS;

// Bounded wait: gives up after g_wait_ns of wall time (checked every 256 polls) or
// 2^26 polls, whichever comes first.  On expiry the device status flag is raised and
// false is returned so the caller can bail out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const unsigned long long lim = g_wait_ns;
  for (uint32_t i = 1; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > lim) break;
  }
  dev_flag(DSV41_DEVST_TIMEOUT);
  return false;
}

// The same wait, which also gives up as soon as *abort (a shared-memory flag that a warp of
// this CTA sets when its own wait ran out) is non-zero, so that the CTA's warps give up
// together instead of leaving some of them at a barrier the others never reach.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t *bar, uint32_t parity,
                                                   const volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const unsigned long long lim = g_wait_ns;
  for (uint32_t i = 1; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && (*abort != 0 || globaltimer_ns() - t0 > lim)) break;
  }
  dev_flag(DSV41_DEVST_TIMEOUT);
  return false;
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2D tiled TMA load global -> shared (this CTA), completes on `bar`.  No
// multicast anywhere in this library.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// The same copy issued by one lane that elect.sync picks from a converged warp: every lane
// runs the calling loop, so its operands stay warp-uniform (issuing from a single-lane branch
// costs the issuing thread far more per instruction).
__device__ __forceinline__ void tma_load_2d_el(void *dst, const CUtensorMap *map, uint64_t *bar,
                                               int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// L2 prefetch of a tensor-map box (no shared memory, no barrier), one elected lane.
__device__ __forceinline__ void tma_prefetch_2d_el(const CUtensorMap *map, int32_t x, int32_t y) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];\n\t}" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_el(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------ programmatic launch
// Kernels of the decode chain are launched with programmatic stream serialization: the next
// kernel may launch while this one drains, runs its prologue (barrier init, tensor-map
// prefetch), then waits in pdl_wait() for the previous grid to finish and flush before it
// touches any data another kernel wrote.  Without the launch attribute both are no-ops.
// Opt-in (DSV41_PDL=1): on the B200 decode chain it measured no faster than plain launches
// inside a CUDA graph (T=64 layer 1.40 ms with, 1.34 ms without).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

static inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("DSV41_PDL");
    on = (e && e[0] == '1') ? 1 : 0;
  }
  return on == 1;
}

// The launch with programmatic stream serialization when `on`, else a plain launch.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl_if(bool on, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                        size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = on ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t st, Args... args) {
  return launch_pdl_if(pdl_enabled(), kernel, grid, block, smem, st, args...);
}

// ------------------------------------------------------------------ host: tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

static inline int get_encoder() {
  if (g_encode_tiled) return DSV41_OK;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
    return set_error(DSV41_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return DSV41_OK;
}

// 2D tensor map, 128-byte swizzle unless told otherwise.  inner = elements per row,
// outer = rows, row_bytes = stride, box = {box_inner, box_outer}.
static inline int make_tmap_2d(CUtensorMap *m, const void *base, CUtensorMapDataType dt,
                               uint64_t inner, uint64_t outer, uint64_t row_bytes,
                               uint32_t box_inner, uint32_t box_outer,
                               CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  int st = get_encoder();
  if (st) return st;
  if (!aligned(base, 16) || (row_bytes % 16) != 0)
    return set_error(DSV41_ERR_MISALIGNED, "TMA base must be 16-byte aligned and row stride a "
                                           "multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode_tiled(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DSV41_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSV41_OK;
}

// ------------------------------------------------------------------ host: launch timing
// Optional per-kernel timing with CUDA events recorded on the launching stream
// around each hot kernel (enabled by dsv41_prof_enable; off by default).
struct ProfRec {
  const char *name;
  cudaEvent_t a, b;
};
static constexpr int PROF_CAP = 4096;
static ProfRec g_prof[PROF_CAP];
static int g_prof_n = 0;
static bool g_prof_on = false;
static char g_prof_sel[512] = "";   // comma-separated kernel names to time; empty = all
static long long g_prof_launches = 0;

// whether `name` is one of the comma-separated names in g_prof_sel (or the list is empty)
static inline bool prof_selected(const char *name) {
  if (!g_prof_sel[0]) return true;
  const size_t n = strlen(name);
  for (const char *p = g_prof_sel; *p;) {
    const char *e = strchr(p, ',');
    const size_t len = e ? size_t(e - p) : strlen(p);
    if (len == n && strncmp(p, name, n) == 0) return true;
    if (!e) break;
    p = e + 1;
  }
  return false;
}

struct ProfScope {
  int slot = -1;
  cudaStream_t st;
  ProfScope(const char *name, cudaStream_t s) : st(s) {
    if (!g_prof_on) return;
    ++g_prof_launches;
    if (g_prof_n >= PROF_CAP || !prof_selected(name)) return;
    slot = g_prof_n++;
    ProfRec &r = g_prof[slot];
    r.name = name;
    if (!r.a) cudaEventCreate(&r.a);
    if (!r.b) cudaEventCreate(&r.b);
    // while the stream is being captured, the records become event nodes of the graph
    // (recorded at every replay of it); otherwise plain stream records
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    cudaEventRecordWithFlags(r.a, st, flags);
  }
  ~ProfScope() {
    if (slot >= 0) cudaEventRecordWithFlags(g_prof[slot].b, st, flags);
  }
  unsigned flags = cudaEventRecordDefault;
};

static inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
static inline size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

}  // namespace dsv41
