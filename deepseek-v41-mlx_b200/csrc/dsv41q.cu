// dsv41q.cu -- C ABI of libdsv41q (declared in include/dsv41q.h).  Single
// translation unit: the kernels live in the *.cuh files included below.
#include "common.cuh"
#include "dequant.cuh"
#include "act_quant.cuh"
#include "engram.cuh"
#include "qgemv.cuh"
#include "router.cuh"
#include "moe.cuh"
#include "bsgemm.cuh"
#include "prefill.cuh"
#include "ep_decode.cuh"
#include "quantize.cuh"
#include "aqgemm.cuh"
#include "a16gemm.cuh"
#include "gemv_m1.cuh"

#include <mutex>

using namespace dsv41;

#define STREAM(s) (reinterpret_cast<cudaStream_t>(s))

extern "C" const char *dsv41_get_last_error(void) { return g_last_error; }
extern "C" int dsv41_abi_version(void) { return 1; }

extern "C" int dsv41_device_status(void *stream, uint32_t *flags_out) {
  DSV41_REQUIRE(flags_out, DSV41_ERR_BAD_ARG, "flags_out is NULL");
  unsigned int v = 0, z = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_dev_status, sizeof(v), 0,
                                            cudaMemcpyDeviceToHost, STREAM(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(STREAM(stream));
  if (e == cudaSuccess)
    e = cudaMemcpyToSymbolAsync(g_dev_status, &z, sizeof(z), 0, cudaMemcpyHostToDevice,
                                STREAM(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(STREAM(stream));
  *flags_out = v;
  return cuda_status(e, "dsv41_device_status");
}

extern "C" int dsv41_set_wait_limit_ns(uint64_t ns) {
  DSV41_REQUIRE(ns == 0 || (ns >= 100000ull && ns <= 60000000000ull), DSV41_ERR_BAD_ARG,
                "wait limit must be 0 (default) or within [1e5, 6e10] ns");
  const unsigned long long v = ns ? ns : DSV41_WAIT_NS;
  return cuda_status(cudaMemcpyToSymbol(g_wait_ns, &v, sizeof(v)), "dsv41_set_wait_limit_ns");
}

// ======================================================================= profiling

extern "C" int dsv41_prof_enable(int on) {
  g_prof_on = on != 0;
  return DSV41_OK;
}

extern "C" int dsv41_prof_reset(void) {
  g_prof_n = 0;
  g_prof_launches = 0;
  return DSV41_OK;
}

extern "C" int dsv41_prof_select(const char *names) {
  const size_t n = names ? strlen(names) : 0;
  DSV41_REQUIRE(n < sizeof(g_prof_sel), DSV41_ERR_BAD_ARG, "name list longer than %zu bytes",
                sizeof(g_prof_sel) - 1);
  if (n) memcpy(g_prof_sel, names, n);
  g_prof_sel[n] = 0;
  return DSV41_OK;
}

extern "C" long long dsv41_prof_launches(void) { return g_prof_launches; }

extern "C" int dsv41_prof_report(char *buf, size_t cap) {
  DSV41_REQUIRE(buf && cap > 0, DSV41_ERR_BAD_ARG, "NULL buffer");
  // aggregate per name: launches and total milliseconds
  const char *names[64];
  int count[64];
  double total[64];
  int nn = 0;
  for (int i = 0; i < g_prof_n; ++i) {
    cudaError_t e = cudaEventSynchronize(g_prof[i].b);
    if (e != cudaSuccess) return cuda_status(e, "prof sync");
    float ms = 0.0f;
    e = cudaEventElapsedTime(&ms, g_prof[i].a, g_prof[i].b);
    if (e != cudaSuccess) return cuda_status(e, "prof elapsed");
    int j = 0;
    while (j < nn && strcmp(names[j], g_prof[i].name) != 0) ++j;
    if (j == nn) {
      if (nn == 64) continue;
      names[nn] = g_prof[i].name;
      count[nn] = 0;
      total[nn] = 0.0;
      ++nn;
    }
    count[j] += 1;
    total[j] += ms;
  }
  size_t off = 0;
  buf[0] = 0;
  for (int j = 0; j < nn && off < cap; ++j)
    off += snprintf(buf + off, cap - off, "%s %d %.6f\n", names[j], count[j], total[j]);
  return DSV41_OK;
}

// ======================================================================= decode

extern "C" int dsv41_e8m0_to_float(const uint8_t *scale, int64_t n, float *out, void *stream) {
  DSV41_REQUIRE(n >= 0, DSV41_ERR_BAD_SHAPE, "n < 0");
  if (n == 0) return DSV41_OK;
  DSV41_REQUIRE(scale && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  k_e8m0_to_float<<<grid_for(n), 256, 0, STREAM(stream)>>>(scale, n, out);
  DSV41_CHECK_LAUNCH("e8m0_to_float");
  return DSV41_OK;
}

extern "C" int dsv41_dequant_fp8_block(const uint8_t *w, const uint8_t *s, int64_t rows,
                                       int64_t cols, int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(rows >= 0 && cols >= 0, DSV41_ERR_BAD_SHAPE, "negative shape");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (rows == 0 || cols == 0) return DSV41_OK;
  DSV41_REQUIRE(w && s && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  const bool vec = (cols % 8 == 0) && aligned(w, 8);
  const int64_t n = vec ? rows * cols / 8 : rows * cols;
  cudaStream_t st = STREAM(stream);
  if (out_dtype == DSV41_F32) {
    if (vec) k_dequant_fp8_block<float, true><<<grid_for(n), 256, 0, st>>>(w, s, rows, cols, (float *)out);
    else k_dequant_fp8_block<float, false><<<grid_for(n), 256, 0, st>>>(w, s, rows, cols, (float *)out);
  } else {
    if (vec) k_dequant_fp8_block<__nv_bfloat16, true><<<grid_for(n), 256, 0, st>>>(w, s, rows, cols, (__nv_bfloat16 *)out);
    else k_dequant_fp8_block<__nv_bfloat16, false><<<grid_for(n), 256, 0, st>>>(w, s, rows, cols, (__nv_bfloat16 *)out);
  }
  DSV41_CHECK_LAUNCH("dequant_fp8_block");
  return DSV41_OK;
}

static int fp4_launch(const uint8_t *p, const uint8_t *s, int64_t rows, int64_t cols,
                      int out_dtype, void *out, void *stream, const char *what) {
  DSV41_REQUIRE(rows >= 0 && cols >= 0 && cols % 2 == 0, DSV41_ERR_BAD_SHAPE,
                "%s: cols must be even (two values per byte)", what);
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (rows == 0 || cols == 0) return DSV41_OK;
  DSV41_REQUIRE(p && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  const bool vec = (cols % 8 == 0) && aligned(p, 4);
  const int64_t n = vec ? rows * cols / 8 : rows * cols;
  cudaStream_t st = STREAM(stream);
  if (out_dtype == DSV41_F32) {
    if (vec) k_dequant_fp4<float, true><<<grid_for(n), 256, 0, st>>>(p, s, rows, cols, (float *)out);
    else k_dequant_fp4<float, false><<<grid_for(n), 256, 0, st>>>(p, s, rows, cols, (float *)out);
  } else {
    if (vec) k_dequant_fp4<__nv_bfloat16, true><<<grid_for(n), 256, 0, st>>>(p, s, rows, cols, (__nv_bfloat16 *)out);
    else k_dequant_fp4<__nv_bfloat16, false><<<grid_for(n), 256, 0, st>>>(p, s, rows, cols, (__nv_bfloat16 *)out);
  }
  DSV41_CHECK_LAUNCH(what);
  return DSV41_OK;
}

extern "C" int dsv41_unpack_fp4(const uint8_t *packed, int64_t rows, int64_t cols, float *out,
                                void *stream) {
  return fp4_launch(packed, nullptr, rows, cols, DSV41_F32, out, stream, "unpack_fp4");
}

extern "C" int dsv41_dequant_fp4(const uint8_t *packed, const uint8_t *s, int64_t rows,
                                 int64_t cols, int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(s, DSV41_ERR_BAD_ARG, "scale is NULL");
  return fp4_launch(packed, s, rows, cols, out_dtype, out, stream, "dequant_fp4");
}

extern "C" int dsv41_dequant_fp8_rows(const uint8_t *w, const uint8_t *s, int64_t rows,
                                      int64_t d, int64_t block, float *out, void *stream) {
  DSV41_REQUIRE(rows >= 0 && d >= 0 && block > 0 && d % block == 0, DSV41_ERR_BAD_SHAPE,
                "d must be a multiple of block");
  if (rows == 0 || d == 0) return DSV41_OK;
  DSV41_REQUIRE(w && s && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  k_dequant_fp8_rows<<<grid_for(rows * d), 256, 0, STREAM(stream)>>>(w, s, rows, d, block, out);
  DSV41_CHECK_LAUNCH("dequant_fp8_rows");
  return DSV41_OK;
}

extern "C" int dsv41_dequant_affine(const uint32_t *wq, const void *scales, const void *biases,
                                    int sb_dtype, int64_t rows, int64_t cols, int bits, int group,
                                    int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(bits >= 1 && bits <= 8, DSV41_ERR_BAD_ARG, "bits must be in [1, 8]");
  DSV41_REQUIRE(group > 0 && rows >= 0 && cols >= 0 && cols % group == 0 &&
                    (cols * bits) % 32 == 0,
                DSV41_ERR_BAD_SHAPE, "cols must be a multiple of group and cols*bits of 32");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  DSV41_REQUIRE(sb_dtype == DSV41_F32 || sb_dtype == DSV41_BF16 || sb_dtype == DSV41_F16,
                DSV41_ERR_BAD_DTYPE, "sb_dtype must be F32, BF16 or F16");
  if (rows == 0 || cols == 0) return DSV41_OK;
  DSV41_REQUIRE(wq && scales && biases && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  const int64_t n = rows * cols;
  cudaStream_t st = STREAM(stream);
#define AFF_LAUNCH(T, SB) \
  k_dequant_affine<T, SB><<<grid_for(n), 256, 0, st>>>(wq, scales, biases, rows, cols, bits, group, (T *)out)
  if (out_dtype == DSV41_F32) {
    if (sb_dtype == DSV41_F32) AFF_LAUNCH(float, 0);
    else if (sb_dtype == DSV41_BF16) AFF_LAUNCH(float, 1);
    else AFF_LAUNCH(float, 2);
  } else {
    if (sb_dtype == DSV41_F32) AFF_LAUNCH(__nv_bfloat16, 0);
    else if (sb_dtype == DSV41_BF16) AFF_LAUNCH(__nv_bfloat16, 1);
    else AFF_LAUNCH(__nv_bfloat16, 2);
  }
#undef AFF_LAUNCH
  DSV41_CHECK_LAUNCH("dequant_affine");
  return DSV41_OK;
}

// ======================================================================= act_quant

extern "C" int dsv41_quantize_affine(const void *w, int dtype, int64_t rows, int64_t cols,
                                     int group, int bits, uint32_t *wq, void *scales,
                                     void *biases, void *stream) {
  DSV41_REQUIRE(dtype == DSV41_BF16 || dtype == DSV41_F32, DSV41_ERR_BAD_DTYPE,
                "dtype must be BF16 or F32");
  DSV41_REQUIRE(group == 32 || group == 64 || group == 128, DSV41_ERR_UNSUPPORTED,
                "group must be 32, 64 or 128");
  DSV41_REQUIRE(bits == 2 || bits == 4 || bits == 8, DSV41_ERR_UNSUPPORTED,
                "bits must be 2, 4 or 8");
  DSV41_REQUIRE(rows >= 0 && cols >= 0 && cols % group == 0, DSV41_ERR_BAD_SHAPE,
                "cols must be a multiple of group");
  if (rows == 0 || cols == 0) return DSV41_OK;
  DSV41_REQUIRE(w && wq && scales && biases, DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("quantize_affine", st);
  if (aligned(w, 16) && aligned(wq, 16)) {
    // a thread per group, 16-byte loads (rows of 32k elements stay aligned)
    const unsigned tb = unsigned(ceil_div(rows * (cols / group), 256));
#define QT(T, G, B)                                                                             \
  k_quantize_affine_t<T, G, B><<<tb, 256, 0, st>>>(static_cast<const T *>(w), rows, cols, wq, \
                                                   static_cast<T *>(scales),                  \
                                                   static_cast<T *>(biases))
#define QTB(T, G)                                                                               \
  do {                                                                                          \
    if (bits == 2) QT(T, G, 2);                                                                 \
    else if (bits == 4) QT(T, G, 4);                                                            \
    else QT(T, G, 8);                                                                           \
  } while (0)
#define QTG(T)                                                                                  \
  do {                                                                                          \
    if (group == 32) QTB(T, 32);                                                                \
    else if (group == 64) QTB(T, 64);                                                           \
    else QTB(T, 128);                                                                           \
  } while (0)
    if (dtype == DSV41_BF16) QTG(__nv_bfloat16);
    else QTG(float);
#undef QTG
#undef QTB
#undef QT
    DSV41_CHECK_LAUNCH("quantize_affine");
    return DSV41_OK;
  }
  // unaligned input or output: a warp per group, element loads
  const unsigned blocks = unsigned(ceil_div(rows * (cols / group) * 32, 256));
#define QA(T, V)                                                                                 \
  k_quantize_affine<T, V><<<blocks, 256, 0, st>>>(static_cast<const T *>(w), rows, cols, bits, \
                                                  wq, static_cast<T *>(scales),                \
                                                  static_cast<T *>(biases))
  if (dtype == DSV41_BF16) {
    if (group == 32) QA(__nv_bfloat16, 1);
    else if (group == 64) QA(__nv_bfloat16, 2);
    else QA(__nv_bfloat16, 4);
  } else {
    if (group == 32) QA(float, 1);
    else if (group == 64) QA(float, 2);
    else QA(float, 4);
  }
#undef QA
  DSV41_CHECK_LAUNCH("quantize_affine");
  return DSV41_OK;
}

extern "C" int dsv41_act_quant_fp8(const void *x, int64_t M, int64_t K, int block,
                                   int round_scale, uint8_t *q, void *s, int s_dtype,
                                   void *deq_out, void *stream) {
  DSV41_REQUIRE(block == 32 || block == 64 || block == 128, DSV41_ERR_BAD_ARG,
                "block must be 32, 64 or 128");
  DSV41_REQUIRE(M >= 0 && K >= 0 && K % block == 0, DSV41_ERR_BAD_SHAPE,
                "K must be a multiple of block");
  DSV41_REQUIRE(s_dtype == DSV41_F32 || (s_dtype == DSV41_U8 && round_scale), DSV41_ERR_BAD_DTYPE,
                "scale dtype must be F32, or U8 (ue8m0) with round_scale");
  if (M == 0 || K == 0) return DSV41_OK;
  DSV41_REQUIRE(x && q && s, DSV41_ERR_BAD_ARG, "NULL pointer");
  const int64_t warps = M * (K / block);
  const unsigned blocks = unsigned((warps * 32 + 255) / 256);
  cudaStream_t st = STREAM(stream);
  const __nv_bfloat16 *xb = reinterpret_cast<const __nv_bfloat16 *>(x);
  __nv_bfloat16 *dq = reinterpret_cast<__nv_bfloat16 *>(deq_out);
  const int su8 = s_dtype == DSV41_U8;
  if (aligned(x, 16) && aligned(q, 8) && (!dq || aligned(dq, 16))) {
    const unsigned vb = unsigned(ceil_div(M * (K / 8), 256));
    if (block == 32)
      k_act_quant_v8<4><<<vb, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq, nullptr, 1);
    else if (block == 64)
      k_act_quant_v8<8><<<vb, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq, nullptr, 1);
    else
      k_act_quant_v8<16><<<vb, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq, nullptr, 1);
  } else if (block == 32) {
    k_act_quant<1><<<blocks, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq);
  } else if (block == 64) {
    k_act_quant<2><<<blocks, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq);
  } else {
    k_act_quant<4><<<blocks, 256, 0, st>>>(xb, M, K, round_scale, q, s, su8, dq);
  }
  DSV41_CHECK_LAUNCH("act_quant_fp8");
  return DSV41_OK;
}

// ======================================================================= qgemv host side

namespace {

struct WsCarve {
  uint8_t *base;
  size_t cap, off;
  bool ok = true;
  template <typename T> T *take(size_t count) {
    off = align_up(off, 256);
    T *p = reinterpret_cast<T *>(base + off);
    off += count * sizeof(T);
    if (off > cap) ok = false;
    return p;
  }
};

constexpr int QG_MAX_SPLIT = 16;

template <int WF, int NMAT, int NT>
int qgemv_launch(const char *name, const CUtensorMap &w0, const CUtensorMap &w1, const CUtensorMap &x8,
                 const CUtensorMap &x16, const CUtensorMap &x32, const QParams &p, int max_items,
                 cudaStream_t st) {
  using Cfg = QCfg<WF, NMAT, NT>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemv<WF, NMAT, NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "qgemv smem attribute");
    attr_set[dev] = true;
  }
  int grid = QG_MIN_CTAS * num_sms();
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  // vector scale loads when every stage is full and scale rows are NG-aligned
  QParams pv = p;
  constexpr int NG = Fmt<WF>::NG;
  bool sv = (p.K % Fmt<WF>::KS == 0) && (p.sld % NG == 0);
  if (WF == WF_FP4)
    sv = sv && aligned(p.scale[0], 8) && aligned(p.scale[NMAT - 1], 8);
  else if (WF == WF_FP8B)
    sv = sv && aligned(p.scale[0], 4) && aligned(p.scale[NMAT - 1], 4);
  else
    sv = sv && aligned(p.aff_s, 2 * NG) && aligned(p.aff_b, 2 * NG);
  pv.svec = sv ? 1 : 0;
  ProfScope prof(name, st);
  DSV41_LAUNCH(launch_pdl_if(pdl_enabled() || pv.pdl_early != 0, k_qgemv<WF, NMAT, NT>, dim3(grid),
                             dim3(QG_THREADS), Cfg::SMEM, st, w0, w1, x8, x16, x32, pv),
               "qgemv");
  DSV41_CHECK_LAUNCH("qgemv");
  return DSV41_OK;
}

// x16 tensor maps for box heights 8 / 16 / 32
int make_x_maps(CUtensorMap (&m)[3], const void *x16, int64_t rows, int64_t K) {
  const uint32_t boxes[3] = {8, 16, 32};
  for (int i = 0; i < 3; ++i) {
    int st = make_tmap_2d(&m[i], x16, CU_TENSOR_MAP_DATA_TYPE_UINT16, (uint64_t)K,
                          (uint64_t)(rows < 1 ? 1 : rows), (uint64_t)K * 2, 64, boxes[i]);
    if (st) return st;
  }
  return DSV41_OK;
}

int weight_map(CUtensorMap *m, const void *w, int64_t rows, int64_t row_bytes) {
  return make_tmap_2d(m, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)row_bytes, (uint64_t)rows,
                      (uint64_t)row_bytes, 128, QG_ROWS);
}

// K splits per tile: the smallest split count whose items fill the resident CTA
// slots in whole waves at >= 85% (items / (waves * slots)), else the best one;
// splits keep >= 4 K stages each.
int pick_nsplit(int64_t base_items, int kstages) {
  const int64_t slots = QG_MIN_CTAS * (int64_t)num_sms();
  int64_t cap = kstages / 4;
  if (cap < 1) cap = 1;
  if (cap > QG_MAX_SPLIT) cap = QG_MAX_SPLIT;
  int64_t best = 1;
  double best_eff = -1.0;
  for (int64_t ns = 1; ns <= cap; ++ns) {
    const int64_t items = base_items * ns;
    const int64_t waves = (items + slots - 1) / slots;
    const double eff = double(items) / double(waves * slots);
    if (eff >= 0.85) return int(ns);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = ns;
    }
  }
  return int(best);
}

struct GemvWs {
  __half *x16;
  float *xscale, *xsum, *partial;
  int *counters;
};

// split-K fragments of the dense GEMV: floats for tiles x chunks x the launch's split count
// (the larger of the counts for 128- and 256-column K stages, the two stage widths of the
// formats) x 128 threads x 16 (NMAT 1 x NT <= 4 x 4); none when neither splits
size_t gemv_partial_floats(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ceil_div(N, QG_ROWS), nch = ceil_div(M, 32);
  const int a = pick_nsplit(tiles * nch, int(ceil_div(K, 128)));
  const int b = pick_nsplit(tiles * nch, int(ceil_div(K, 256)));
  const int ns = a > b ? a : b;
  return ns > 1 ? size_t(tiles) * nch * ns * 32 * QG_CW * 16 : 0;
}

size_t gemv_ws_bytes(int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = ceil_div(N, QG_ROWS), nch = ceil_div(M, 32);
  size_t b = 0;
  b += align_up((size_t)M * K * 2, 256);
  b += align_up((size_t)M * 4, 256);
  b += align_up((size_t)M * ceil_div(K, 64) * 4, 256);
  b += align_up(gemv_partial_floats(M, N, K) * 4, 256);
  b += align_up((size_t)tiles * nch * 4, 256);
  return b + 256;
}

template <int WF>
int gemv_common(const void *x, int64_t M, int64_t K, const void *w, int64_t w_row_bytes,
                const uint8_t *s, int64_t sld, const void *aff_s, const void *aff_b, int64_t N,
                int out_dtype, void *y, void *workspace, size_t ws_bytes, cudaStream_t st) {
  constexpr int KS = Fmt<WF>::KS;
  DSV41_REQUIRE(M >= 0 && N >= 0 && K >= 0, DSV41_ERR_BAD_SHAPE, "negative shape");
  DSV41_REQUIRE(K % Fmt<WF>::GK == 0, DSV41_ERR_BAD_SHAPE, "K must be a multiple of %d",
                Fmt<WF>::GK);
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (M == 0 || N == 0) return DSV41_OK;
  DSV41_REQUIRE(x && w && y, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(N <= (int64_t)INT32_MAX && M <= (int64_t)INT32_MAX / 2, DSV41_ERR_BAD_SHAPE,
                "shape too large");
  DSV41_REQUIRE(workspace && ws_bytes >= gemv_ws_bytes(M, N, K), DSV41_ERR_WORKSPACE,
                "workspace too small: need %zu bytes", gemv_ws_bytes(M, N, K));
  const int64_t tiles = ceil_div(N, QG_ROWS), nch = ceil_div(M, 32);
  WsCarve wc{reinterpret_cast<uint8_t *>(workspace), ws_bytes, 0};
  GemvWs ws;
  ws.x16 = wc.take<__half>(M * K);
  ws.xscale = wc.take<float>(M);
  ws.xsum = wc.take<float>(M * ceil_div(K, 64));
  ws.partial = wc.take<float>(gemv_partial_floats(M, N, K));
  ws.counters = wc.take<int>(tiles * nch);
  DSV41_REQUIRE(wc.ok, DSV41_ERR_WORKSPACE, "workspace too small");

  constexpr bool AFF = WF == WF_AFF4 || WF == WF_AFF8;
  const int perm = WF == WF_AFF4 ? 4 : (WF == WF_AFF8 ? 8 : 0);
  QParams p{};
  p.scale[0] = s;
  p.scale[1] = s;
  p.aff_s = reinterpret_cast<const uint16_t *>(aff_s);
  p.aff_b = reinterpret_cast<const uint16_t *>(aff_b);
  p.N = N;
  p.K = K;
  p.sld = sld;
  p.tiles = int(tiles);
  p.kstages = int(ceil_div(K, KS));
  p.nsplit = pick_nsplit(tiles * nch, p.kstages);
  {  // tuning: DSV41_GEMV_MAX_SPLIT caps the K splits (never above the workspace's sizing)
    static int cap = -1;
    if (cap < 0) {
      const char *e = getenv("DSV41_GEMV_MAX_SPLIT");
      cap = e ? atoi(e) : 0;
    }
    if (cap > 0 && p.nsplit > cap) p.nsplit = cap;
  }
  // The prep kernel also zeroes the split-K tickets, and the GEMV is launched as its
  // programmatic dependent: the GEMV's first weight copies are issued while the prep runs.
  { ProfScope prof("qx_prep", st);
  DSV41_LAUNCH(launch_pdl(k_qx_prep, dim3(unsigned(M)), dim3(256), 0, st,
                          reinterpret_cast<const __nv_bfloat16 *>(x), M, K,
                          static_cast<const int32_t *>(nullptr), static_cast<const int *>(nullptr),
                          ws.x16, ws.xscale, AFF ? ws.xsum : static_cast<float *>(nullptr), perm,
                          p.nsplit > 1 ? ws.counters : static_cast<int *>(nullptr),
                          int64_t(p.nsplit > 1 ? tiles * nch : 0)),
               "qx_prep"); }
  DSV41_CHECK_LAUNCH("qx_prep");

  CUtensorMap wm, xm[3];
  int rc = weight_map(&wm, w, N, w_row_bytes);
  if (rc) return rc;
  rc = make_x_maps(xm, ws.x16, M, K);
  if (rc) return rc;

  p.xscale = ws.xscale;
  p.xsum = ws.xsum;
  p.chunks = nullptr;
  p.nchunks_host = int(nch);
  p.dense_m = int(M);
  p.dense_rows = 32;
  p.epi = out_dtype == DSV41_F32 ? EPI_STORE_F32 : EPI_STORE_BF16;
  p.out = y;
  p.ldo = N;
  p.partial = ws.partial;
  p.counters = ws.counters;
  p.pdl_early = 1;
  const int items = int(tiles * nch * p.nsplit);
  if (M <= 8) return qgemv_launch<WF, 1, 1>("qgemv_dense", wm, wm, xm[0], xm[1], xm[2], p, items, st);
  if (M <= 16) return qgemv_launch<WF, 1, 2>("qgemv_dense", wm, wm, xm[0], xm[1], xm[2], p, items, st);
  return qgemv_launch<WF, 1, 4>("qgemv_dense", wm, wm, xm[0], xm[1], xm[2], p, items, st);
}

}  // namespace

extern "C" size_t dsv41_gemv_workspace_size(int64_t M, int64_t N, int64_t K) {
  return gemv_ws_bytes(M, N, K);
}

extern "C" int dsv41_gemv_fp8_block(const void *x, int64_t M, int64_t K, const uint8_t *w,
                                    const uint8_t *s, int64_t N, int out_dtype, void *y,
                                    void *workspace, size_t workspace_bytes, void *stream) {
  DSV41_REQUIRE(s || M == 0 || N == 0, DSV41_ERR_BAD_ARG, "scale is NULL");
  // one activation row: the CUDA-core kernel (no activation prep, no workspace use)
  if (M == 1 && N > 0 && K > 0 && K % 32 == 0 && K <= 16384 && x && w && y && aligned(x, 16) &&
      aligned(w, 16) && (out_dtype == DSV41_F32 || out_dtype == DSV41_BF16)) {
    DSV41_REQUIRE(N <= (int64_t)INT32_MAX, DSV41_ERR_BAD_SHAPE, "shape too large");
    cudaStream_t st = STREAM(stream);
    const int64_t want = ceil_div(N, int64_t(GM1_THREADS / 32));
    const unsigned grid = unsigned(std::min<int64_t>(want, 2 * int64_t(num_sms())));
    ProfScope prof("gemv_fp8_m1", st);
    const uint16_t *xs = static_cast<const uint16_t *>(x);
    if (out_dtype == DSV41_F32)
      k_gemv_byte_m1<false, float><<<grid, GM1_THREADS, size_t(K) * 2, st>>>(
          xs, K, w, s, nullptr, K / 32, N, (float *)y);
    else
      k_gemv_byte_m1<false, __nv_bfloat16><<<grid, GM1_THREADS, size_t(K) * 2, st>>>(
          xs, K, w, s, nullptr, K / 32, N, (__nv_bfloat16 *)y);
    DSV41_CHECK_LAUNCH("gemv_fp8_m1");
    return DSV41_OK;
  }
  return gemv_common<WF_FP8B>(x, M, K, w, K, s, ceil_div(K, 32), nullptr, nullptr, N, out_dtype,
                              y, workspace, workspace_bytes, STREAM(stream));
}

extern "C" int dsv41_gemv_fp4(const void *x, int64_t M, int64_t K, const uint8_t *w,
                              const uint8_t *s, int64_t N, int out_dtype, void *y, void *workspace,
                              size_t workspace_bytes, void *stream) {
  DSV41_REQUIRE(s || M == 0 || N == 0, DSV41_ERR_BAD_ARG, "scale is NULL");
  return gemv_common<WF_FP4>(x, M, K, w, K / 2, s, K / 32, nullptr, nullptr, N, out_dtype, y,
                             workspace, workspace_bytes, STREAM(stream));
}

extern "C" int dsv41_gemv_affine(const void *x, int64_t M, int64_t K, const uint32_t *wq,
                                 const void *scales, const void *biases, int bits, int64_t N,
                                 int out_dtype, void *y, void *workspace, size_t workspace_bytes,
                                 void *stream) {
  DSV41_REQUIRE(bits == 4 || bits == 8, DSV41_ERR_UNSUPPORTED,
                "gemv_affine supports bits 4 and 8 (group 64)");
  DSV41_REQUIRE((scales && biases) || M == 0 || N == 0, DSV41_ERR_BAD_ARG, "NULL scales/biases");
  // one activation row, 4-bit: the CUDA-core kernel (no activation prep, no workspace use)
  if (bits == 4 && M == 1 && N > 0 && K > 0 && K % 64 == 0 && K <= 16384 && x && wq && y &&
      aligned(x, 16) && aligned(wq, 16) && (out_dtype == DSV41_F32 || out_dtype == DSV41_BF16)) {
    DSV41_REQUIRE(N <= (int64_t)INT32_MAX, DSV41_ERR_BAD_SHAPE, "shape too large");
    cudaStream_t st = STREAM(stream);
    const int64_t want = ceil_div(N, int64_t(GM1_THREADS / 32));
    const unsigned grid = unsigned(std::min<int64_t>(want, 4 * int64_t(num_sms())));
    const size_t smem = size_t(K) * 2 + size_t(K / 32) * 4;
    ProfScope prof("gemv_affine4_m1", st);
    const uint16_t *xs = static_cast<const uint16_t *>(x);
    const uint16_t *sc = static_cast<const uint16_t *>(scales);
    const uint16_t *bi = static_cast<const uint16_t *>(biases);
    if (out_dtype == DSV41_F32)
      k_gemv_affine4_m1<float><<<grid, GM1_THREADS, smem, st>>>(xs, K, wq, sc, bi, N, (float *)y);
    else
      k_gemv_affine4_m1<__nv_bfloat16><<<grid, GM1_THREADS, smem, st>>>(xs, K, wq, sc, bi, N,
                                                                       (__nv_bfloat16 *)y);
    DSV41_CHECK_LAUNCH("gemv_affine4_m1");
    return DSV41_OK;
  }
  // one activation row, 8-bit: the byte-code CUDA-core kernel in its affine form
  if (bits == 8 && M == 1 && N > 0 && K > 0 && K % 64 == 0 && K <= 16384 && x && wq && y &&
      aligned(x, 16) && aligned(wq, 16) && (out_dtype == DSV41_F32 || out_dtype == DSV41_BF16)) {
    DSV41_REQUIRE(N <= (int64_t)INT32_MAX, DSV41_ERR_BAD_SHAPE, "shape too large");
    cudaStream_t st = STREAM(stream);
    const int64_t want = ceil_div(N, int64_t(GM1_THREADS / 32));
    const unsigned grid = unsigned(std::min<int64_t>(want, 2 * int64_t(num_sms())));
    const size_t smem = size_t(K) * 2 + size_t(K / 8) * 4;
    ProfScope prof("gemv_affine8_m1", st);
    const uint16_t *xs = static_cast<const uint16_t *>(x);
    const uint8_t *wb = reinterpret_cast<const uint8_t *>(wq);
    const uint16_t *bi = static_cast<const uint16_t *>(biases);
    if (out_dtype == DSV41_F32)
      k_gemv_byte_m1<true, float><<<grid, GM1_THREADS, smem, st>>>(xs, K, wb, scales, bi, K / 64,
                                                                   N, (float *)y);
    else
      k_gemv_byte_m1<true, __nv_bfloat16><<<grid, GM1_THREADS, smem, st>>>(
          xs, K, wb, scales, bi, K / 64, N, (__nv_bfloat16 *)y);
    DSV41_CHECK_LAUNCH("gemv_affine8_m1");
    return DSV41_OK;
  }
  if (bits == 4)
    return gemv_common<WF_AFF4>(x, M, K, wq, K / 2, nullptr, K / 64, scales, biases, N, out_dtype,
                                y, workspace, workspace_bytes, STREAM(stream));
  return gemv_common<WF_AFF8>(x, M, K, wq, K, nullptr, K / 64, scales, biases, N, out_dtype, y,
                              workspace, workspace_bytes, STREAM(stream));
}

// ======================================================================= router

namespace {
int router_nks(int64_t T, int64_t K, int64_t E) {
  const int64_t base = ceil_div(E, 16) * ceil_div(T, 8);
  const int64_t target = 8 * (int64_t)num_sms();
  int64_t want = ceil_div(target, base);
  const int64_t k32 = K / 32;
  int64_t best = 1;
  for (int64_t d = 1; d <= k32 && d <= 64; ++d)
    if (k32 % d == 0 && d <= want) best = d;
  return int(best);
}
}  // namespace

extern "C" size_t dsv41_moe_route_workspace_size(int64_t T, int64_t D, int64_t E) {
  // the K-split partial scores of router_scores: router_nks(T, D, E) x T x E floats
  const int64_t nks = (T > 0 && E > 0 && D >= 32) ? router_nks(T, D, E) : 1;
  return align_up((size_t)nks * T * E * 4, 256) + 256;
}

static int route_impl(const void *x, int64_t T, int64_t D, const void *gate_w, const float *bias,
                      int64_t E, int topk, int score_func, float gate_temp, int norm_topk_prob,
                      float route_scale, float *weights, int32_t *indices, float *partial,
                      cudaStream_t st) {
  const int nks = router_nks(T, D, E);
  const int64_t warps = ceil_div(E, 16) * ceil_div(T, 8) * nks;
  { ProfScope prof("router_scores", st);
  DSV41_LAUNCH(launch_pdl(k_router_scores, dim3(unsigned(ceil_div(warps * 32, 128))), dim3(128), 0,
                          st, reinterpret_cast<const __nv_bfloat16 *>(x), T, D,
                          reinterpret_cast<const __nv_bfloat16 *>(gate_w), E, nks, partial),
               "router_scores"); }
  DSV41_CHECK_LAUNCH("router_scores");
  const int threads = int(ceil_div(E, 32) * 32);
  ProfScope prof("router_select", st);
  DSV41_LAUNCH(launch_pdl(k_router_select, dim3(unsigned(T)), dim3(threads), 0, st,
                          static_cast<const float *>(partial), nks, T, E, bias, topk, score_func,
                          gate_temp, norm_topk_prob, route_scale, weights, indices),
               "router_select");
  DSV41_CHECK_LAUNCH("router_select");
  return DSV41_OK;
}

static int route_check(int64_t T, int64_t D, int64_t E, int topk, int score_func) {
  DSV41_REQUIRE(T >= 0 && D > 0 && D % 32 == 0, DSV41_ERR_BAD_SHAPE, "D must be a multiple of 32");
  DSV41_REQUIRE(E > 0 && E <= 1024, DSV41_ERR_BAD_SHAPE, "1 <= E <= 1024");
  DSV41_REQUIRE(topk >= 1 && topk <= 64 && topk <= E, DSV41_ERR_BAD_ARG, "1 <= topk <= min(64, E)");
  DSV41_REQUIRE(score_func >= 0 && score_func <= 2, DSV41_ERR_BAD_ARG, "unknown score_func");
  return DSV41_OK;
}

extern "C" int dsv41_moe_route(const void *x, int64_t T, int64_t D, const void *gate_w,
                               const float *bias, int64_t E, int topk, int score_func,
                               float gate_temp, int norm_topk_prob, float route_scale,
                               float *weights, int32_t *indices, void *workspace,
                               size_t workspace_bytes, void *stream) {
  int rc = route_check(T, D, E, topk, score_func);
  if (rc) return rc;
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(x && gate_w && weights && indices, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(workspace && workspace_bytes >= dsv41_moe_route_workspace_size(T, D, E),
                DSV41_ERR_WORKSPACE, "workspace too small");
  DSV41_REQUIRE(aligned(x, 16) && aligned(gate_w, 16), DSV41_ERR_MISALIGNED,
                "x and gate_w must be 16-byte aligned");
  return route_impl(x, T, D, gate_w, bias, E, topk, score_func, gate_temp, norm_topk_prob,
                    route_scale, weights, indices, reinterpret_cast<float *>(workspace),
                    STREAM(stream));
}

// ======================================================================= MoE decode

namespace {

struct MoeWs {
  float *rpart, *w;
  int32_t *idx;
  MoePlan plan;
  __half *x16g, *x16, *H, *Hs;
  float *xsg, *xs, *Y, *Ys;
  float *part_gu, *part_dn, *part_sgu, *part_sdn;
  int *cnt_gu, *cnt_dn, *cnt_sgu, *cnt_sdn;
  size_t used;
  bool ok;
};

struct MoeDims {
  int64_t T, D, I, E, P, Pmax, Cmax, Tp, tiles_gu, tiles_dn;
  // what the launches use: K-split counts (routed / shared gate/up and down, router), the
  // row-pair down projection and its tiles; split-K partials are carved only where a count
  // exceeds 1; the routed kernels' n8 activation tiles per chunk (gu_nt, dn_nt: 1, 2 or 4)
  int ns_gu, ns_dn, ns_sgu, ns_sdn, nks, rowpair;
  int64_t tiles_dnx;
  int gu_nt, dn_nt;
};

// n8 tiles per routed chunk for `n` expected pairs of one expert: a chunk of 8 * nt (gate/up)
// or 4 * nt (down: hi/lo halves) pairs; every further chunk of an expert streams its weights
// again.  DSV41_MOE_CHUNK_NT="g,d" fixes both (tuning).
int chunk_nt(double n, int base) { return n <= base ? 1 : (n <= 2 * base ? 2 : 4); }

void moe_chunk_override(int &gu, int &dn) {
  static int g = -1, dd = -1;
  if (g < 0) {
    g = dd = 0;
    const char *e = getenv("DSV41_MOE_CHUNK_NT");
    int a = 0, b = 0;
    if (e && sscanf(e, "%d,%d", &a, &b) == 2 && (a == 1 || a == 2 || a == 4) &&
        (b == 1 || b == 2 || b == 4)) {
      g = a;
      dd = b;
    }
  }
  if (g) {
    gu = g;
    dn = dd;
  }
}

// expect: pairs an active expert is expected to receive (<= 0: the batch's own average,
// P over the active experts; an expert-parallel owner passes its estimate, since it is sized
// for the most rows it can receive)
MoeDims moe_dims(const dsv41_moe_config *c, int64_t T, double expect = -1.0) {
  MoeDims d;
  d.T = T;
  d.D = c->dim;
  d.I = c->inter;
  d.E = c->n_experts;
  d.P = T * c->topk;
  const int64_t act = d.P < d.E ? d.P : d.E;
  // chunks wide enough for 1.5x the expected pairs of an expert, so that most experts stream
  // their weights once
  const double avg = expect > 0 ? expect : double(d.P) / double(act > 0 ? act : 1);
  d.gu_nt = chunk_nt(1.5 * avg, 8);
  d.dn_nt = chunk_nt(1.5 * avg, 4);
  moe_chunk_override(d.gu_nt, d.dn_nt);
  d.Pmax = d.P + 3 * act;
  const int64_t c_gu = ceil_div(d.P, 8 * d.gu_nt), c_dn = ceil_div(d.P, 4 * d.dn_nt);
  d.Cmax = (c_gu > c_dn ? c_gu : c_dn) + act;
  d.Tp = ceil_div(T, 4) * 4;
  d.tiles_gu = ceil_div(d.I, QG_ROWS);
  d.tiles_dn = ceil_div(d.D, QG_ROWS);
  // routed: gate/up over all active experts' tiles; down on row pairs (two 64-row tiles of an
  // expert per item, on the two-matrix kernel) once the pair items fill a wave of CTAs,
  // which needs packed scales and dim % 128 == 0 -- below that single tiles keep more CTAs
  // streaming
  d.ns_gu = pick_nsplit(act * d.tiles_gu, int(ceil_div(d.D, Fmt<WF_FP4>::KS)));
  const int64_t pair_tiles = d.D / (2 * QG_ROWS);
  d.rowpair = ((c->flags & DSV41_MOE_PACKED_SCALES) && !(c->flags & DSV41_MOE_NO_ROWPAIR) &&
               d.D % (2 * QG_ROWS) == 0 &&
               act * pair_tiles >= QG_MIN_CTAS * (int64_t)num_sms()) ? 1 : 0;
  d.tiles_dnx = d.rowpair ? pair_tiles : d.tiles_dn;
  d.ns_dn = pick_nsplit(act * d.tiles_dnx, int(ceil_div(d.I, Fmt<WF_FP4>::KS)));
  // shared expert: dense chunks of nts n8 tiles
  const int nts = T <= 8 ? 1 : (T <= 16 ? 2 : 4);
  d.ns_sgu = pick_nsplit(ceil_div(T, 8 * nts) * d.tiles_gu, int(ceil_div(d.D, Fmt<WF_FP8B>::KS)));
  d.ns_sdn = pick_nsplit(ceil_div(T, 4 * nts) * d.tiles_dn, int(ceil_div(d.I, Fmt<WF_FP8B>::KS)));
  d.nks = T > 0 ? router_nks(T, d.D, d.E) : 1;
  return d;
}

MoeWs moe_carve(const MoeDims &d, void *base, size_t cap) {
  WsCarve wc{reinterpret_cast<uint8_t *>(base), cap, 0};
  MoeWs w;
  w.rpart = wc.take<float>(int64_t(d.nks) * d.T * d.E);
  w.w = wc.take<float>(d.P);
  w.idx = wc.take<int32_t>(d.P);
  w.plan.pair_tok = wc.take<int32_t>(d.Pmax);
  w.plan.pair_row = wc.take<int32_t>(d.Pmax);
  w.plan.gu_chunks = wc.take<QChunk>(d.Cmax);
  w.plan.dn_chunks = wc.take<QChunk>(d.Cmax);
  w.plan.sgu_chunks = wc.take<QChunk>(ceil_div(d.T, 32));
  w.plan.sdn_chunks = wc.take<QChunk>(ceil_div(d.T, 16));
  w.plan.counts = wc.take<int>(8);
  w.x16g = wc.take<__half>(d.Pmax * d.D);
  w.xsg = wc.take<float>(d.Pmax);
  w.x16 = wc.take<__half>(d.T * d.D);
  w.xs = wc.take<float>(d.T);
  w.H = wc.take<__half>(2 * d.Pmax * d.I);
  w.Hs = wc.take<__half>(2 * d.Tp * d.I);
  w.Y = wc.take<float>(d.P * d.D);
  w.Ys = wc.take<float>(d.T * d.D);
  // split-K partials, [tile][split][thread][NMAT * NT * 4 floats], only where a launch splits:
  // routed kernels NMAT * NT <= 2 x 1; shared gate/up ceil(T / 8nts) chunks of 2 x nts and
  // down ceil(T / 4nts) chunks of 1 x nts (nts <= 4) are covered by ceil(T/8) x 32 and
  // ceil(T/4) x 16 floats a thread
  const size_t ct = 32 * QG_CW;
  auto parts = [&](int64_t tiles, int ns, size_t floats) -> size_t {
    return ns > 1 ? size_t(tiles) * size_t(ns) * ct * floats : 0;
  };
  w.part_gu = wc.take<float>(parts(d.Cmax * d.tiles_gu, d.ns_gu, 8 * d.gu_nt));
  w.part_dn = wc.take<float>(parts(d.Cmax * d.tiles_dnx, d.ns_dn, 8 * d.dn_nt));
  w.part_sgu = wc.take<float>(parts(ceil_div(d.T, 8) * d.tiles_gu, d.ns_sgu, 32));
  w.part_sdn = wc.take<float>(parts(ceil_div(d.T, 4) * d.tiles_dn, d.ns_sdn, 16));
  w.cnt_gu = wc.take<int>(d.Cmax * d.tiles_gu);
  w.cnt_dn = wc.take<int>(d.Cmax * d.tiles_dn);
  w.cnt_sgu = wc.take<int>(ceil_div(d.T, 8) * d.tiles_gu);
  w.cnt_sdn = wc.take<int>(ceil_div(d.T, 4) * d.tiles_dn);
  w.used = wc.off + 256;
  w.ok = wc.ok;
  return w;
}

}  // namespace

extern "C" size_t dsv41_moe_decode_workspace_size(const dsv41_moe_config *cfg, int64_t T) {
  if (!cfg || T < 0) return 0;
  MoeDims d = moe_dims(cfg, T < 1 ? 1 : T);
  MoeWs w = moe_carve(d, nullptr, SIZE_MAX);
  return w.used;
}

namespace {

int moe_check(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, int64_t T, bool shared) {
  DSV41_REQUIRE(cfg && W, DSV41_ERR_BAD_ARG, "NULL config/weights");
  int rc = route_check(T, cfg->dim, cfg->n_experts, cfg->topk, cfg->score_func);
  if (rc) return rc;
  DSV41_REQUIRE(cfg->inter > 0 && cfg->inter % 32 == 0, DSV41_ERR_BAD_SHAPE,
                "inter must be a multiple of 32");
  DSV41_REQUIRE(cfg->swiglu_limit > 0.0f && cfg->swiglu_limit <= 255.0f, DSV41_ERR_UNSUPPORTED,
                "decode path needs 0 < swiglu_limit <= 255 (h must fit f16)");
  DSV41_REQUIRE(T <= 4096, DSV41_ERR_UNSUPPORTED, "decode path is for T <= 4096 tokens");
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(W->w1 && W->s1 && W->w3 && W->s3 && W->w2 && W->s2, DSV41_ERR_BAD_ARG,
                "NULL expert pointer");
  if (cfg->flags & DSV41_MOE_PACKED_SCALES) {
    DSV41_REQUIRE(cfg->dim % 256 == 0 && cfg->inter % 256 == 0, DSV41_ERR_BAD_SHAPE,
                  "decode-packed scales need dim and inter to be multiples of 256");
    DSV41_REQUIRE(aligned(W->s1, 16) && aligned(W->s3, 16) && aligned(W->s2, 16),
                  DSV41_ERR_MISALIGNED, "decode-packed scales must be 16-byte aligned");
  }
  DSV41_REQUIRE(!shared || (W->sw1 && W->ss1 && W->sw3 && W->ss3 && W->sw2 && W->ss2),
                DSV41_ERR_BAD_ARG, "NULL shared-expert pointer");
  return DSV41_OK;
}

// Per (host thread, device) side stream and events used to run the shared
// expert concurrently with the routed experts (fork / join on the caller's stream,
// which also works while the caller's stream is being captured into a graph).
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
static thread_local SideStream g_side[64];

int side_stream(SideStream **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  DSV41_REQUIRE(dev >= 0 && dev < 64, DSV41_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  SideStream &s = g_side[dev];
  if (!s.s) {
    e = cudaStreamCreateWithFlags(&s.s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_status(e, "side stream");
  }
  *out = &s;
  return DSV41_OK;
}

// Routed experts (SwitchGLU) for given indices -> Y[t*k + j, :] fp32 on `st`, and
// the shared expert -> Ys on `st_shared` when `shared`.
int moe_experts_impl(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, const void *x,
                     const MoeDims &d, MoeWs &ws, const int32_t *idx, float *Y, bool shared,
                     cudaStream_t st, cudaStream_t st_shared, bool routed = true,
                     const int32_t *tok_map = nullptr, const int *n_valid = nullptr) {
  const int64_t T = d.T;
  const int round = (cfg->flags & DSV41_MOE_ROUND_BF16) ? 1 : 0;
  int rc;
  if (routed) {
  // plan
  { ProfScope prof("moe_plan", st);
  DSV41_LAUNCH(launch_pdl(k_moe_plan, dim3(1), dim3(1024), 4 * d.E * sizeof(int), st,
                          static_cast<const int32_t *>(idx), T, cfg->topk, d.E, ws.plan, tok_map,
                          n_valid, 8 * d.gu_nt, 4 * d.dn_nt),
               "moe_plan"); }
  DSV41_CHECK_LAUNCH("moe_plan");
  // activations gathered per pair
  { ProfScope prof("qx_prep_gather", st);
  DSV41_LAUNCH(launch_pdl(k_qx_prep, dim3(unsigned(d.Pmax)), dim3(256), 0, st,
                          reinterpret_cast<const __nv_bfloat16 *>(x), T, d.D,
                          static_cast<const int32_t *>(ws.plan.pair_tok),
                          static_cast<const int *>(ws.plan.counts + 2), ws.x16g, ws.xsg,
                          static_cast<float *>(nullptr), 0, static_cast<int *>(nullptr), int64_t(0)),
               "qx_prep gathered"); }
  DSV41_CHECK_LAUNCH("qx_prep gathered");

  CUtensorMap m_w1, m_w3, m_w2, xg[3], hx[3];
  if ((rc = weight_map(&m_w1, W->w1, d.E * d.I, d.D / 2))) return rc;
  if ((rc = weight_map(&m_w3, W->w3, d.E * d.I, d.D / 2))) return rc;
  if ((rc = weight_map(&m_w2, W->w2, d.E * d.D, d.I / 2))) return rc;
  if ((rc = make_x_maps(xg, ws.x16g, d.Pmax, d.D))) return rc;
  if ((rc = make_x_maps(hx, ws.H, 2 * d.Pmax, d.I))) return rc;

  const int64_t active = d.P < d.E ? d.P : d.E;
  {  // routed gate/up (+SwiGLU) -> H
    QParams p{};
    p.scale[0] = W->s1;
    p.scale[1] = W->s3;
    p.N = d.I;
    p.K = d.D;
    p.sld = d.D / 32;
    p.tiles = int(d.tiles_gu);
    p.kstages = int(ceil_div(d.D, Fmt<WF_FP4>::KS));
    p.nsplit = d.ns_gu;
    p.xscale = ws.xsg;
    p.chunks = ws.plan.gu_chunks;
    p.nchunks_dev = ws.plan.counts + 0;
    p.epi = EPI_SWIGLU;
    p.out = ws.H;
    p.ldo = d.I;
    p.limit = cfg->swiglu_limit;
    p.round_gu = round;
    p.round_h = 0;
    p.partial = ws.part_gu;
    p.counters = ws.cnt_gu;
    p.spack = (cfg->flags & DSV41_MOE_PACKED_SCALES) ? 1 : 0;
    if (p.nsplit > 1) {
      cudaError_t e = cudaMemsetAsync(ws.cnt_gu, 0, sizeof(int) * d.Cmax * d.tiles_gu, st);
      if (e != cudaSuccess) return cuda_status(e, "memset");
    }
    const int items = int(d.Cmax * d.tiles_gu * p.nsplit);
    if (d.gu_nt == 1)
      rc = qgemv_launch<WF_FP4, 2, 1>("moe_expert_gate_up_fp4", m_w1, m_w3, xg[0], xg[1], xg[2], p,
                                       items, st);
    else if (d.gu_nt == 2)
      rc = qgemv_launch<WF_FP4, 2, 2>("moe_expert_gate_up_fp4", m_w1, m_w3, xg[0], xg[1], xg[2], p,
                                       items, st);
    else
      rc = qgemv_launch<WF_FP4, 2, 4>("moe_expert_gate_up_fp4", m_w1, m_w3, xg[0], xg[1], xg[2], p,
                                       items, st);
    if (rc) return rc;
  }
  {  // routed down -> Y[t*k + j]
    QParams p{};
    p.scale[0] = W->s2;
    p.scale[1] = W->s2;
    p.N = d.D;
    p.K = d.I;
    p.sld = d.I / 32;
    p.spack = (cfg->flags & DSV41_MOE_PACKED_SCALES) ? 1 : 0;
    // row pairs (two 64-row tiles of one expert per item, on the two-matrix kernel: the
    // B fragments are shared and each warp runs two independent MMA chains), as moe_dims chose
    p.rowpair = d.rowpair;
    p.tiles = int(d.tiles_dnx);
    p.kstages = int(ceil_div(d.I, Fmt<WF_FP4>::KS));
    p.nsplit = d.ns_dn;
    p.xscale = nullptr;
    p.chunks = ws.plan.dn_chunks;
    p.nchunks_dev = ws.plan.counts + 1;
    p.epi = EPI_DOWN;
    p.out = Y;
    p.ldo = d.D;
    p.pair_row = ws.plan.pair_row;
    p.partial = ws.part_dn;       // a rowpair tile's fragments fill two tiles' room
    p.counters = ws.cnt_dn;
    if (p.nsplit > 1) {
      cudaError_t e = cudaMemsetAsync(ws.cnt_dn, 0, sizeof(int) * d.Cmax * d.tiles_dn, st);
      if (e != cudaSuccess) return cuda_status(e, "memset");
    }
    const int items = int(d.Cmax * p.tiles * p.nsplit);
    if (p.rowpair) {
      if (d.dn_nt == 1)
        rc = qgemv_launch<WF_FP4, 2, 1>("moe_expert_down_fp4_pairs", m_w2, m_w2, hx[0], hx[1],
                                         hx[2], p, items, st);
      else if (d.dn_nt == 2)
        rc = qgemv_launch<WF_FP4, 2, 2>("moe_expert_down_fp4_pairs", m_w2, m_w2, hx[0], hx[1],
                                         hx[2], p, items, st);
      else
        rc = qgemv_launch<WF_FP4, 2, 4>("moe_expert_down_fp4_pairs", m_w2, m_w2, hx[0], hx[1],
                                         hx[2], p, items, st);
    } else {
      if (d.dn_nt == 1)
        rc = qgemv_launch<WF_FP4, 1, 1>("moe_expert_down_fp4", m_w2, m_w2, hx[0], hx[1], hx[2], p,
                                         items, st);
      else if (d.dn_nt == 2)
        rc = qgemv_launch<WF_FP4, 1, 2>("moe_expert_down_fp4", m_w2, m_w2, hx[0], hx[1], hx[2], p,
                                         items, st);
      else
        rc = qgemv_launch<WF_FP4, 1, 4>("moe_expert_down_fp4", m_w2, m_w2, hx[0], hx[1], hx[2], p,
                                         items, st);
    }
    if (rc) return rc;
  }
  }  // routed
  if (!shared) return DSV41_OK;
  // shared expert (fp8 32x32): gate/up -> Hs -> down -> Ys, on its own stream
  st = st_shared;
  { ProfScope prof("qx_prep", st);
  DSV41_LAUNCH(launch_pdl(k_qx_prep, dim3(unsigned(T)), dim3(256), 0, st,
                          reinterpret_cast<const __nv_bfloat16 *>(x), T, d.D,
                          static_cast<const int32_t *>(nullptr), static_cast<const int *>(nullptr),
                          ws.x16, ws.xs, static_cast<float *>(nullptr), 0,
                          static_cast<int *>(nullptr), int64_t(0)),
               "qx_prep shared"); }
  DSV41_CHECK_LAUNCH("qx_prep shared");
  CUtensorMap m_s1, m_s3, m_s2, xs[3], hs[3];
  if ((rc = weight_map(&m_s1, W->sw1, d.I, d.D))) return rc;
  if ((rc = weight_map(&m_s3, W->sw3, d.I, d.D))) return rc;
  if ((rc = weight_map(&m_s2, W->sw2, d.D, d.I))) return rc;
  if ((rc = make_x_maps(xs, ws.x16, d.T, d.D))) return rc;
  if ((rc = make_x_maps(hs, ws.Hs, 2 * d.Tp, d.I))) return rc;
  // The shared expert's chunks depend only on T (dense chunk mode), so it never
  // reads the routed plan and can run concurrently with it.
  const int nts = T <= 8 ? 1 : (T <= 16 ? 2 : 4);     // n8 tiles per chunk
  {
    QParams p{};
    p.scale[0] = W->ss1;
    p.scale[1] = W->ss3;
    p.N = d.I;
    p.K = d.D;
    p.sld = ceil_div(d.D, 32);
    p.tiles = int(d.tiles_gu);
    p.kstages = int(ceil_div(d.D, Fmt<WF_FP8B>::KS));
    const int64_t nch = ceil_div(T, 8 * nts);
    p.nsplit = d.ns_sgu;
    p.xscale = ws.xs;
    p.chunks = nullptr;
    p.nchunks_host = int(nch);
    p.dense_m = int(T);
    p.dense_rows = 8 * nts;
    p.dense_down = 0;
    p.epi = EPI_SWIGLU;
    p.out = ws.Hs;
    p.ldo = d.I;
    p.limit = cfg->swiglu_limit;
    p.round_gu = round;
    p.round_h = round;
    p.partial = ws.part_sgu;
    p.counters = ws.cnt_sgu;
    if (p.nsplit > 1) {
      cudaError_t e = cudaMemsetAsync(ws.cnt_sgu, 0, sizeof(int) * nch * d.tiles_gu, st);
      if (e != cudaSuccess) return cuda_status(e, "memset");
    }
    const int items = int(nch * d.tiles_gu * p.nsplit);
    if (nts == 1)
      rc = qgemv_launch<WF_FP8B, 2, 1>("moe_shared_gate_up_fp8", m_s1, m_s3, xs[0], xs[1], xs[2], p, items, st);
    else if (nts == 2)
      rc = qgemv_launch<WF_FP8B, 2, 2>("moe_shared_gate_up_fp8", m_s1, m_s3, xs[0], xs[1], xs[2], p, items, st);
    else
      rc = qgemv_launch<WF_FP8B, 2, 4>("moe_shared_gate_up_fp8", m_s1, m_s3, xs[0], xs[1], xs[2], p, items, st);
    if (rc) return rc;
  }
  {
    QParams p{};
    p.scale[0] = W->ss2;
    p.scale[1] = W->ss2;
    p.N = d.D;
    p.K = d.I;
    p.sld = ceil_div(d.I, 32);
    p.tiles = int(d.tiles_dn);
    p.kstages = int(ceil_div(d.I, Fmt<WF_FP8B>::KS));
    const int64_t nch = ceil_div(T, 4 * nts);          // 8*nts H rows = 4*nts tokens
    p.nsplit = d.ns_sdn;
    p.xscale = nullptr;
    p.chunks = nullptr;
    p.nchunks_host = int(nch);
    p.dense_m = int(T);
    p.dense_rows = 8 * nts;
    p.dense_down = 1;
    p.epi = EPI_DOWN;
    p.out = ws.Ys;
    p.ldo = d.D;
    p.pair_row = nullptr;
    p.npairs = int(T);
    p.round_out = round;
    p.partial = ws.part_sdn;
    p.counters = ws.cnt_sdn;
    if (p.nsplit > 1) {
      cudaError_t e = cudaMemsetAsync(ws.cnt_sdn, 0, sizeof(int) * nch * d.tiles_dn, st);
      if (e != cudaSuccess) return cuda_status(e, "memset");
    }
    const int items = int(nch * d.tiles_dn * p.nsplit);
    if (nts == 1)
      rc = qgemv_launch<WF_FP8B, 1, 1>("moe_shared_down_fp8", m_s2, m_s2, hs[0], hs[1], hs[2], p, items, st);
    else if (nts == 2)
      rc = qgemv_launch<WF_FP8B, 1, 2>("moe_shared_down_fp8", m_s2, m_s2, hs[0], hs[1], hs[2], p, items, st);
    else
      rc = qgemv_launch<WF_FP8B, 1, 4>("moe_shared_down_fp8", m_s2, m_s2, hs[0], hs[1], hs[2], p, items, st);
    if (rc) return rc;
  }
  return DSV41_OK;
}

}  // namespace

extern "C" int dsv41_moe_experts(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                 const void *x, int64_t T, const int32_t *indices, float *y,
                                 void *workspace, size_t workspace_bytes, void *stream) {
  int rc = moe_check(cfg, W, T, false);
  if (rc || T == 0) return rc;
  DSV41_REQUIRE(x && indices && y, DSV41_ERR_BAD_ARG, "NULL pointer");
  const MoeDims d = moe_dims(cfg, T);
  DSV41_REQUIRE(workspace, DSV41_ERR_WORKSPACE, "workspace is NULL");
  MoeWs ws = moe_carve(d, workspace, workspace_bytes);
  DSV41_REQUIRE(ws.ok && ws.used <= workspace_bytes, DSV41_ERR_WORKSPACE,
                "workspace too small: need %zu bytes", ws.used);
  return moe_experts_impl(cfg, W, x, d, ws, indices, y, false, STREAM(stream), STREAM(stream));
}

extern "C" int dsv41_moe_decode(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                const void *x, int64_t T, int out_dtype, void *y,
                                float *weights_out, int32_t *indices_out, void *workspace,
                                size_t workspace_bytes, void *stream) {
  const bool shared = cfg && !(cfg->flags & DSV41_MOE_NO_SHARED);
  int rc = moe_check(cfg, W, T, shared);
  if (rc || T == 0) return rc;
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  DSV41_REQUIRE(x && y && W->gate_w, DSV41_ERR_BAD_ARG, "NULL pointer");
  const MoeDims d = moe_dims(cfg, T);
  DSV41_REQUIRE(workspace, DSV41_ERR_WORKSPACE, "workspace is NULL");
  MoeWs ws = moe_carve(d, workspace, workspace_bytes);
  DSV41_REQUIRE(ws.ok && ws.used <= workspace_bytes, DSV41_ERR_WORKSPACE,
                "workspace too small: need %zu bytes", ws.used);
  DSV41_REQUIRE(aligned(x, 16) && aligned(W->gate_w, 16), DSV41_ERR_MISALIGNED,
                "x and gate_w must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  float *wts = weights_out ? weights_out : ws.w;
  int32_t *idx = indices_out ? indices_out : ws.idx;
  // the shared expert does not depend on routing: fork it onto the side stream
  SideStream *side = nullptr;
  cudaStream_t st_shared = st;
  if (shared) {
    if ((rc = side_stream(&side))) return rc;
    cudaError_t e = cudaEventRecord(side->fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->s, side->fork, 0);
    if (e != cudaSuccess) return cuda_status(e, "fork shared expert");
    st_shared = side->s;
  }
  rc = route_impl(x, T, d.D, W->gate_w, W->gate_bias, d.E, cfg->topk, cfg->score_func,
                  cfg->gate_temp, cfg->norm_topk_prob, cfg->route_scale, wts, idx, ws.rpart, st);
  if (rc) return rc;
  rc = moe_experts_impl(cfg, W, x, d, ws, idx, ws.Y, shared, st, st_shared);
  if (rc) return rc;
  if (shared) {
    cudaError_t e = cudaEventRecord(side->join, side->s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, side->join, 0);
    if (e != cudaSuccess) return cuda_status(e, "join shared expert");
  }
  const int64_t n = T * d.D;
  ProfScope prof("moe_combine", st);
  if (out_dtype == DSV41_F32)
    DSV41_LAUNCH(launch_pdl(k_moe_combine<float>, dim3(grid_for(n)), dim3(256), 0, st,
                            static_cast<const float *>(ws.Y),
                            static_cast<const float *>(shared ? ws.Ys : nullptr),
                            static_cast<const float *>(wts), T, cfg->topk, d.D, (float *)y),
                 "moe_combine");
  else
    DSV41_LAUNCH(launch_pdl(k_moe_combine<__nv_bfloat16>, dim3(grid_for(n)), dim3(256), 0, st,
                            static_cast<const float *>(ws.Y),
                            static_cast<const float *>(shared ? ws.Ys : nullptr),
                            static_cast<const float *>(wts), T, cfg->topk, d.D,
                            (__nv_bfloat16 *)y),
                 "moe_combine");
  DSV41_CHECK_LAUNCH("moe_combine");
  return DSV41_OK;
}

// ======================================================================= EP decode (peer memory)

struct dsv41_ep_ctx {
  int world = 0, rank = 0, topk = 0;
  int64_t max_tokens = 0, dim = 0;
  int device = 0;
  EpLayout L{};
  uint8_t *buf = nullptr;                 // this rank's buffer (peers map it)
  EpPeers peers{};                        // every rank's buffer as seen from this GPU
  bool opened[EP_MAX_RANKS] = {false};
  unsigned long long *dseq = nullptr;     // step counter
  unsigned *done = nullptr;               // [2][world] CTA completion counters
  bool connected = false;
};

extern "C" int dsv41_ep_create(int world, int rank, int64_t max_tokens, int topk, int64_t dim,
                               dsv41_ep_ctx **out) {
  DSV41_REQUIRE(out, DSV41_ERR_BAD_ARG, "NULL output");
  *out = nullptr;
  DSV41_REQUIRE(world >= 1 && world <= EP_MAX_RANKS && rank >= 0 && rank < world,
                DSV41_ERR_BAD_ARG, "need 1 <= world <= %d and 0 <= rank < world", EP_MAX_RANKS);
  DSV41_REQUIRE(max_tokens >= 1 && topk >= 1 && topk <= 16 && max_tokens * topk <= 8192 &&
                    dim > 0 && dim % 8 == 0,
                DSV41_ERR_UNSUPPORTED, "EP decode needs max_tokens*topk <= 8192 and 8 | dim");
  auto *c = new dsv41_ep_ctx();
  c->world = world;
  c->rank = rank;
  c->topk = topk;
  c->max_tokens = max_tokens;
  c->dim = dim;
  cudaGetDevice(&c->device);
  c->L = ep_layout(world, max_tokens * topk, dim);
  cudaError_t e = cudaMalloc(&c->buf, c->L.total);
  if (e == cudaSuccess) e = cudaMemset(c->buf, 0, c->L.total);
  if (e == cudaSuccess) e = cudaMalloc(&c->dseq, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(c->dseq, 0, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&c->done, sizeof(unsigned) * 2 * world);
  if (e == cudaSuccess) e = cudaMemset(c->done, 0, sizeof(unsigned) * 2 * world);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(c->buf);
    cudaFree(c->dseq);
    cudaFree(c->done);
    delete c;
    return cuda_status(e, "EP buffers");
  }
  c->peers.base[rank] = c->buf;
  *out = c;
  return DSV41_OK;
}

extern "C" size_t dsv41_ep_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int dsv41_ep_handle(const dsv41_ep_ctx *c, void *handle_out) {
  DSV41_REQUIRE(c && handle_out, DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, c->buf);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return DSV41_OK;
}

extern "C" int dsv41_ep_connect(dsv41_ep_ctx *c, const void *handles) {
  DSV41_REQUIRE(c && handles, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(!c->connected, DSV41_ERR_BAD_ARG, "already connected");
  const uint8_t *hb = static_cast<const uint8_t *>(handles);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    void *p = nullptr;
    const int rc = dsv41_ipc_import(hb + r * sizeof(cudaIpcMemHandle_t), &p);
    if (rc) return rc;
    c->peers.base[r] = static_cast<uint8_t *>(p);
    c->opened[r] = true;
  }
  c->connected = true;
  return DSV41_OK;
}

extern "C" int dsv41_ep_wait(const dsv41_ep_ctx *c, int which, void *stream) {
  DSV41_REQUIRE(c, DSV41_ERR_BAD_ARG, "NULL context");
  DSV41_REQUIRE(which == 0 || which == 1, DSV41_ERR_BAD_ARG,
                "which must be 0 (rows received) or 1 (outputs returned)");
  k_ep_wait<<<1, 64, 0, STREAM(stream)>>>(c->buf, c->L, which, c->dseq);
  DSV41_CHECK_LAUNCH("ep_wait");
  return DSV41_OK;
}

extern "C" int dsv41_ep_destroy(dsv41_ep_ctx *c) {
  if (!c) return DSV41_OK;
  cudaDeviceSynchronize();
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) dsv41_ipc_close(c->peers.base[r]);
  cudaFree(c->buf);
  cudaFree(c->dseq);
  cudaFree(c->done);
  delete c;
  return DSV41_OK;
}

namespace {

// The owner runs its experts on ws*C received rows (padding rows skipped), one pair each;
// every rank is taken to route about as many pairs as this one (T * topk), spread over the
// owner's experts, for the chunk width.
MoeDims ep_owner_dims_decode(const dsv41_moe_config *cfg, const dsv41_ep_ctx *c, int64_t T) {
  dsv41_moe_config lc = *cfg;
  lc.n_experts = cfg->n_experts / c->world;
  lc.topk = 1;
  const double pairs = double(T < 1 ? 1 : T) * cfg->topk;
  const double act = pairs < double(lc.n_experts) ? pairs : double(lc.n_experts);
  return moe_dims(&lc, int64_t(c->world) * c->L.C, pairs / act);
}

size_t ep_decode_ws_bytes(const dsv41_moe_config *cfg, const dsv41_ep_ctx *c, int64_t T) {
  const MoeDims dl = moe_dims(cfg, T < 1 ? 1 : T), dw = ep_owner_dims_decode(cfg, c, T);
  const size_t a = moe_carve(dl, nullptr, ~size_t(0)).used;
  const size_t b = moe_carve(dw, nullptr, ~size_t(0)).used;
  return align_up(a, 256) + align_up(b, 256) + 2 * align_up(size_t(dw.T) * 4, 256) +
         align_up(size_t(c->max_tokens) * c->topk * 4, 256) + 256;
}

}  // namespace

extern "C" size_t dsv41_moe_ep_decode_workspace_size(const dsv41_moe_config *cfg,
                                                     const dsv41_ep_ctx *ctx, int64_t T) {
  if (!cfg || !ctx || cfg->n_experts % ctx->world) return 0;
  return ep_decode_ws_bytes(cfg, ctx, T);
}

extern "C" int dsv41_moe_ep_decode(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                   dsv41_ep_ctx *c, const void *x, int64_t T, int out_dtype,
                                   void *y, float *weights_out, int32_t *indices_out,
                                   void *workspace, size_t workspace_bytes, void *stream) {
  DSV41_REQUIRE(cfg && W && c, DSV41_ERR_BAD_ARG, "NULL config/weights/context");
  DSV41_REQUIRE(c->connected, DSV41_ERR_BAD_ARG, "EP context is not connected");
  DSV41_REQUIRE(cfg->topk == c->topk && cfg->dim == c->dim && cfg->n_experts % c->world == 0,
                DSV41_ERR_BAD_SHAPE, "config does not match the EP context");
  DSV41_REQUIRE(T >= 0 && T <= c->max_tokens, DSV41_ERR_UNSUPPORTED,
                "T = %lld exceeds the context's max_tokens %lld", (long long)T,
                (long long)c->max_tokens);
  const bool shared = !(cfg->flags & DSV41_MOE_NO_SHARED);
  dsv41_moe_config lc = *cfg;                 // this rank's experts
  lc.n_experts = cfg->n_experts / c->world;
  lc.topk = 1;
  int rc = moe_check(&lc, W, 1, shared);
  if (rc) return rc;
  rc = route_check(T < 1 ? 1 : T, cfg->dim, cfg->n_experts, cfg->topk, cfg->score_func);
  if (rc) return rc;
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  DSV41_REQUIRE((x && y) || T == 0, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(W->gate_w, DSV41_ERR_BAD_ARG, "NULL router weight");
  DSV41_REQUIRE(!x || (aligned(x, 16) && aligned(W->gate_w, 16)), DSV41_ERR_MISALIGNED,
                "x and gate_w must be 16-byte aligned");
  const size_t need = ep_decode_ws_bytes(cfg, c, T);
  DSV41_REQUIRE(workspace && workspace_bytes >= need, DSV41_ERR_WORKSPACE,
                "workspace too small: need %zu bytes", need);
  cudaStream_t st = STREAM(stream);
  const MoeDims dl = moe_dims(cfg, T < 1 ? 1 : T), dw = ep_owner_dims_decode(cfg, c, T);
  WsCarve wc{static_cast<uint8_t *>(workspace), workspace_bytes, 0};
  uint8_t *ws_loc = wc.take<uint8_t>(moe_carve(dl, nullptr, ~size_t(0)).used);
  uint8_t *ws_own = wc.take<uint8_t>(moe_carve(dw, nullptr, ~size_t(0)).used);
  int32_t *ids = wc.take<int32_t>(dw.T);
  int32_t *rowmap = wc.take<int32_t>(dw.T);
  int32_t *slot_pos = wc.take<int32_t>(c->max_tokens * c->topk);
  DSV41_REQUIRE(wc.ok, DSV41_ERR_WORKSPACE, "workspace too small");
  MoeWs wl = moe_carve(dl, ws_loc, ~size_t(0));
  MoeWs wo = moe_carve(dw, ws_own, ~size_t(0));
  float *wts = weights_out ? weights_out : wl.w;
  int32_t *idx = indices_out ? indices_out : wl.idx;
  const EpLayout &L = c->L;
  const int epr = int(cfg->n_experts / c->world);

  // shared expert of this rank's tokens, on the side stream
  SideStream *side = nullptr;
  const bool do_shared = shared && T > 0;
  if (do_shared) {
    if ((rc = side_stream(&side))) return rc;
    cudaError_t e = cudaEventRecord(side->fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->s, side->fork, 0);
    if (e != cudaSuccess) return cuda_status(e, "fork shared expert");
    rc = moe_experts_impl(cfg, W, x, dl, wl, nullptr, nullptr, true, side->s, side->s, false);
    if (rc) return rc;
  }
  if (T > 0) {
    rc = route_impl(x, T, cfg->dim, W->gate_w, W->gate_bias, cfg->n_experts, cfg->topk,
                    cfg->score_func, cfg->gate_temp, cfg->norm_topk_prob, cfg->route_scale, wts,
                    idx, wl.rpart, st);
    if (rc) return rc;
  }
  // dispatch: rows into the owners' receive buffers
  const int P = int(T * cfg->topk);
  {
    ProfScope prof("ep_dispatch", st);
    // up to 64 CTAs an owner, two rows each: enough stores in flight to keep NVLink busy
    const unsigned nb =
        unsigned(std::max<int64_t>(1, std::min<int64_t>(64, ceil_div(P, 2 * c->world))));
    k_ep_dispatch<<<dim3(c->world, nb), 256, P * sizeof(int), st>>>(
        static_cast<const __nv_bfloat16 *>(x), idx, int(T), cfg->topk, epr, c->rank, L, c->peers,
        c->dseq, slot_pos, c->done);
    DSV41_CHECK_LAUNCH("ep_dispatch");
  }
  {
    ProfScope prof("ep_wait", st);
    k_ep_wait<<<1, 64, 0, st>>>(c->buf, L, 0, c->dseq);
  }
  DSV41_CHECK_LAUNCH("ep_wait dispatch");
  // owner: experts on the received rows
  {
    ProfScope prof("ep_ids", st);
    k_ep_ids<<<unsigned(ceil_div(dw.T, 256)), 256, 0, st>>>(c->buf, L, ids, rowmap,
                                                           wo.plan.counts + 5);
  }
  DSV41_CHECK_LAUNCH("ep_ids");
  float *Yr = wo.Y;
  rc = moe_experts_impl(&lc, W, c->buf + L.rows, dw, wo, ids, Yr, false, st, st, true, rowmap,
                        wo.plan.counts + 5);
  if (rc) return rc;
  {
    ProfScope prof("ep_return", st);
    // the rows each source sent are known only on the device: as many CTAs as the expected
    // rows (this rank's own pair count spread over the sources) need at two rows each
    const unsigned nb = unsigned(
        std::max<int64_t>(1, std::min<int64_t>(64, ceil_div(T * cfg->topk, 2 * c->world))));
    k_ep_return<<<dim3(c->world, nb), 256, 0, st>>>(Yr, c->buf, c->rank, L, c->peers, c->dseq,
                                                     c->done + c->world);
    DSV41_CHECK_LAUNCH("ep_return");
  }
  {
    ProfScope prof("ep_wait", st);
    k_ep_wait<<<1, 64, 0, st>>>(c->buf, L, 1, c->dseq);
  }
  DSV41_CHECK_LAUNCH("ep_wait return");
  if (do_shared) {
    cudaError_t e = cudaEventRecord(side->join, side->s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, side->join, 0);
    if (e != cudaSuccess) return cuda_status(e, "join shared expert");
  }
  {
    ProfScope prof("ep_combine", st);
    const int64_t n = T * cfg->dim;
    const unsigned g = n > 0 ? grid_for(n) : 1;
    const float *Ys = do_shared ? wl.Ys : nullptr;
    if (out_dtype == DSV41_F32)
      k_ep_combine_decode<float><<<g, 256, 0, st>>>(c->buf, L, slot_pos, wts, Ys, T, cfg->topk,
                                                    static_cast<float *>(y), c->dseq);
    else
      k_ep_combine_decode<__nv_bfloat16><<<g, 256, 0, st>>>(c->buf, L, slot_pos, wts, Ys, T,
                                                            cfg->topk,
                                                            static_cast<__nv_bfloat16 *>(y), c->dseq);
    DSV41_CHECK_LAUNCH("ep_combine");
  }
  return DSV41_OK;
}

// ======================================================================= block-scaled GEMM

namespace {

// Weight tensor map: fp4 codes as 16U4_ALIGN16B (the padded one-byte-per-code smem form
// the f8f6f4 MMA reads) or fp8 bytes; box {128 K, box_rows}.
int bs_wmap(CUtensorMap *m, const uint8_t *w, int wfmt, int64_t rows, int64_t K, uint32_t box_rows) {
  if (wfmt == BS_W_FP4) {
    DSV41_REQUIRE(aligned(w, 32), DSV41_ERR_MISALIGNED, "fp4 weights must be 32-byte aligned");
    return make_tmap_2d(m, w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, (uint64_t)K, (uint64_t)rows,
                        (uint64_t)(K / 2), 128, box_rows);
  }
  return make_tmap_2d(m, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K, (uint64_t)rows,
                      (uint64_t)K, 128, box_rows);
}

static_assert(PF_TILE_ROWS == BS_BN, "prefill tiles are GEMM tiles");

int bs_xmaps(CUtensorMap (&m)[4], const uint8_t *x, int64_t rows, int64_t K) {
  for (int i = 0; i < 4; ++i) {
    int rc = make_tmap_2d(&m[i], x, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)K,
                          (uint64_t)(rows < 1 ? 1 : rows), (uint64_t)K, 128, bs_box_rows(i));
    if (rc) return rc;
  }
  return DSV41_OK;
}

template <int WF, int EPI, bool NARROW>
int bs_launch(const char *name, const BsMaps &maps, const BsArgs &a, int grid, cudaStream_t st) {
  using Cfg = BsCfg<NARROW>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_bsgemm<WF, EPI, NARROW>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "bsgemm smem attribute");
    attr_set[dev] = true;
  }
  if (grid < 1) return DSV41_OK;
  BsArgs g = a;
  g.sf_async = (a.sw.kshift == 0 && a.sx.kshift == 0 &&
                (EPI != BS_EPI_SWIGLU || a.sw2.kshift == 0)) ? 1 : 0;
  g.nkb = a.nkb / Cfg::KSUB;
  ProfScope prof(name, st);
  k_bsgemm<WF, EPI, NARROW><<<grid, BS_THREADS, Cfg::SMEM, st>>>(maps, g);
  DSV41_CHECK_LAUNCH(name);
  return DSV41_OK;
}

int bs_grid(int tiles) { return tiles < num_sms() ? tiles : num_sms(); }

// The 2-CTA form of the wide kernel: clusters of 2 CTAs, one pair of m-tiles a cluster at a
// time (tiles from a grouped list whose m-tile count per token tile is even; every scale
// operand as atoms, loaded through maps.sfa / maps.sfb).
template <int WF, int EPI>
int bs_launch_pair(const char *name, const BsMaps &maps, const BsArgs &a, cudaStream_t st) {
  using Cfg = BsCfg<false, true>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_bsgemm<WF, EPI, false, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "bsgemm pair smem attribute");
    attr_set[dev] = true;
  }
  const int grid = num_sms() & ~1;
  if (grid < 2) return DSV41_OK;
  BsArgs g = a;
  g.sf_async = 0;
  g.nkb = a.nkb;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(BS_THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  ProfScope prof(name, st);
  DSV41_LAUNCH(cudaLaunchKernelEx(&cfg, k_bsgemm<WF, EPI, false, true>, maps, g), name);
  DSV41_CHECK_LAUNCH(name);
  return DSV41_OK;
}

// scale atoms [..][512 bytes] as a 2D byte tensor of 256-byte rows, box {256, box_rows}
int bs_atom_map(CUtensorMap *m, const uint8_t *atoms, size_t bytes, uint32_t box_rows) {
  return make_tmap_2d(m, atoms, CU_TENSOR_MAP_DATA_TYPE_UINT8, 256, uint64_t(bytes / 256), 256,
                      256, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// the 2-CTA wide kernel is on unless DSV41_NO_PAIR=1 (kept for comparisons)
bool bs_pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char *e = getenv("DSV41_NO_PAIR");
    on = (e && e[0] == '1') ? 0 : 1;
  }
  return on == 1;
}

// Dense problem: static tiles of 128 weight rows (64 + 64 in SwiGLU mode) x BN activation
// rows, the narrow shape when all activation rows fit one narrow tile.
template <int WF, int EPI>
int bs_dense_launch(const char *name, const BsMaps &maps, BsArgs a, int64_t N, int64_t M,
                    cudaStream_t st) {
  const bool narrow = M <= BS_BN_NARROW && a.nkb % BsCfg<true>::KSUB == 0;
  a.dense_bn = narrow ? BS_BN_NARROW : BS_BN;
  a.dense_nt = int(ceil_div(M, a.dense_bn));
  a.dense_tiles = int(N / (EPI == BS_EPI_SWIGLU ? 64 : BS_BM)) * a.dense_nt;
  a.dense_rows = int(M);
  a.tiles = nullptr;
  const int grid = bs_grid(a.dense_tiles);
  return narrow ? bs_launch<WF, EPI, true>(name, maps, a, grid, st)
                : bs_launch<WF, EPI, false>(name, maps, a, grid, st);
}

// Grouped problem: the wide tile list, then the narrow one, each taken from a work counter.
template <int WF, int EPI>
int bs_grouped_launch(const char *name_w, const char *name_n, const BsMaps &maps, BsArgs a,
                      const PfPlan &plan, int list, cudaStream_t st, bool pair = false) {
  a.tiles = plan.tiles[list];
  a.ntiles = plan.ntiles + list;
  a.next_tile = plan.next_tile + list;
  int rc = (pair && bs_pair_enabled() && a.sfa_atoms && a.sfb_atoms)
               ? bs_launch_pair<WF, EPI>(name_w, maps, a, st)
               : bs_launch<WF, EPI, false>(name_w, maps, a, num_sms(), st);
  if (rc) return rc;
  a.tiles = plan.tiles[list + 1];
  a.ntiles = plan.ntiles + list + 1;
  a.next_tile = plan.next_tile + list + 1;
  if (a.nkb % BsCfg<true>::KSUB != 0)   // K not a multiple of the narrow stage: wide shape
    return bs_launch<WF, EPI, false>(name_n, maps, a, num_sms(), st);
  return bs_launch<WF, EPI, true>(name_n, maps, a, num_sms(), st);
}

BsScale bs_scale(const uint8_t *p, int64_t ld, int rshift, int kblock, int64_t rows) {
  BsScale s;
  s.p = p;
  s.ld = ld;
  s.rshift = rshift;
  s.kshift = kblock == 128 ? 2 : 0;
  s.rows = rows;
  return s;
}

BsArgs bs_args(int64_t K, int64_t a_rows) {
  BsArgs a;
  memset(&a, 0, sizeof(a));
  a.nkb = int(K / BS_BK);
  a.a_rows = int(a_rows);
  return a;
}

// C[M, N] = A[M, K] . B[N, K]^T with fp8 A and fp8 / fp4 B (wfmt), ue8m0 scales.
int bs_dense(int wfmt, const uint8_t *a, const uint8_t *a_s, int a_blk, const uint8_t *b,
             const uint8_t *b_s, int b_rshift, int b_blk, int64_t M, int64_t N, int64_t K,
             void *c, int c_dtype, cudaStream_t st) {
  DSV41_REQUIRE(M >= 0 && N > 0 && K > 0 && N % 128 == 0 && K % 128 == 0, DSV41_ERR_BAD_SHAPE,
                "N and K must be positive multiples of 128");
  DSV41_REQUIRE(M <= (int64_t(1) << 30) && N < (int64_t(1) << 31),
                DSV41_ERR_BAD_SHAPE, "M or N too large");
  DSV41_REQUIRE(c_dtype == DSV41_F32 || c_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "output must be F32 or BF16");
  if (M == 0) return DSV41_OK;
  DSV41_REQUIRE(a && a_s && b && b_s && c, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(a, 16) && aligned(c, 16) && aligned(a_s, 4) && aligned(b_s, 4),
                DSV41_ERR_MISALIGNED, "a/c must be 16-byte and scales 4-byte aligned");
  BsMaps maps;
  memset(&maps, 0, sizeof(maps));
  int rc = bs_wmap(&maps.w, b, wfmt, N, K, 128);
  if (!rc) rc = bs_xmaps(maps.x, a, M, K);
  if (rc) return rc;
  BsArgs g = bs_args(K, N);
  g.sw = bs_scale(b_s, K / b_blk, b_rshift, b_blk, N);
  g.sx = bs_scale(a_s, K / a_blk, 0, a_blk, M);
  g.out = c;
  g.ldo = N;
  if (wfmt == BS_W_FP4)
    return c_dtype == DSV41_F32 ? bs_dense_launch<BS_W_FP4, BS_EPI_F32>("fp4_gemm", maps, g, N, M, st)
                                : bs_dense_launch<BS_W_FP4, BS_EPI_BF16>("fp4_gemm", maps, g, N, M, st);
  return c_dtype == DSV41_F32 ? bs_dense_launch<BS_W_FP8, BS_EPI_F32>("fp8_gemm", maps, g, N, M, st)
                              : bs_dense_launch<BS_W_FP8, BS_EPI_BF16>("fp8_gemm", maps, g, N, M, st);
}

}  // namespace

extern "C" int dsv41_fp8_gemm(const uint8_t *a, const uint8_t *a_s, const uint8_t *b,
                              const uint8_t *b_s, int64_t M, int64_t N, int64_t K, int block_size,
                              void *c, int c_dtype, void *stream) {
  DSV41_REQUIRE(block_size == 32 || block_size == 128, DSV41_ERR_BAD_ARG,
                "block_size must be 32 or 128");
  return bs_dense(BS_W_FP8, a, a_s, block_size, b, b_s, block_size == 32 ? 5 : 7, block_size, M,
                  N, K, c, c_dtype, STREAM(stream));
}

extern "C" int dsv41_fp4_gemm(const uint8_t *a, const uint8_t *a_s, const uint8_t *b,
                              const uint8_t *b_s, int64_t M, int64_t N, int64_t K,
                              int act_block_size, void *c, int c_dtype, void *stream) {
  DSV41_REQUIRE(act_block_size == 32 || act_block_size == 128, DSV41_ERR_BAD_ARG,
                "act_block_size must be 32 or 128");
  return bs_dense(BS_W_FP4, a, a_s, act_block_size, b, b_s, 0, 32, M, N, K, c, c_dtype,
                  STREAM(stream));
}

// ======================================================================= affine prefill GEMM

extern "C" int dsv41_qmm_affine(const void *x, int64_t M, int64_t K, const uint32_t *wq,
                                const void *scales, const void *biases, int bits, int64_t N,
                                int out_dtype, void *y, void *stream) {
  DSV41_REQUIRE(bits == 4 || bits == 8, DSV41_ERR_UNSUPPORTED, "bits must be 4 or 8");
  DSV41_REQUIRE(M >= 0 && K > 0 && N > 0 && K % AQ_BK == 0 && N % AQ_BM == 0,
                DSV41_ERR_BAD_SHAPE, "K must be a multiple of 64 and N of 128");
  DSV41_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31), DSV41_ERR_BAD_SHAPE,
                "shape too large");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (M == 0) return DSV41_OK;
  DSV41_REQUIRE(x && wq && scales && biases && y, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(x, 16) && aligned(wq, 16) && aligned(y, 16) && aligned(scales, 2) &&
                    aligned(biases, 2),
                DSV41_ERR_MISALIGNED, "x, wq and y must be 16-byte aligned");
  AqMaps maps;
  memset(&maps, 0, sizeof(maps));
  const uint64_t row_bytes = uint64_t(K) * bits / 8;
  int rc = make_tmap_2d(&maps.w, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, row_bytes, uint64_t(N),
                        row_bytes, AQ_BK * bits / 8, AQ_BM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!rc)
    rc = make_tmap_2d(&maps.x, x, CU_TENSOR_MAP_DATA_TYPE_UINT16, uint64_t(K), uint64_t(M),
                      uint64_t(K) * 2, AQ_BK, AQ_BN);
  if (rc) return rc;
  AqArgs a;
  memset(&a, 0, sizeof(a));
  a.nkb = int(K / AQ_BK);
  a.M = M;
  a.N = N;
  a.scale = reinterpret_cast<const uint16_t *>(scales);
  a.bias = reinterpret_cast<const uint16_t *>(biases);
  a.nt = int(ceil_div(M, AQ_BN));
  a.tiles = int(N / AQ_BM) * a.nt;
  a.out = y;
  a.ldo = N;
  cudaStream_t st = STREAM(stream);
  const int grid = a.tiles < num_sms() ? a.tiles : num_sms();
  static bool attr_set[64][4] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int v = (bits == 8 ? 2 : 0) + (out_dtype == DSV41_F32 ? 1 : 0);
  auto kern = bits == 4 ? (out_dtype == DSV41_F32 ? k_aqgemm<4, BS_EPI_F32> : k_aqgemm<4, BS_EPI_BF16>)
                        : (out_dtype == DSV41_F32 ? k_aqgemm<8, BS_EPI_F32> : k_aqgemm<8, BS_EPI_BF16>);
  if (dev >= 0 && dev < 64 && !attr_set[dev][v]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AQ_SMEM);
    if (e != cudaSuccess) return cuda_status(e, "aqgemm smem attribute");
    attr_set[dev][v] = true;
  }
  ProfScope prof("qmm_affine", st);
  kern<<<grid, AQ_THREADS, AQ_SMEM, st>>>(maps, a);
  DSV41_CHECK_LAUNCH("qmm_affine");
  return DSV41_OK;
}

// ======================================================================= MoE prefill

namespace {

struct PfDims {
  int64_t T, D, I, E, P, nchunks, cap_w, cap_n, cap_rt;
  int k;
};

// Packed weight scales (tcgen05.cp atoms, see k_pack_sfw): gate/up paired, then down.
size_t pf_packed_gu_bytes(const dsv41_moe_config *c) {
  return size_t(c->n_experts) * (c->inter / 64) * (c->dim / 128) * 512;
}
size_t pf_packed_dn_bytes(const dsv41_moe_config *c) {
  return size_t(c->n_experts) * (c->dim / 128) * (c->inter / 128) * 512;
}
// shared expert (one group), packed after the routed experts when its weights are given
size_t pf_packed_sh_off(const dsv41_moe_config *c) {
  return pf_packed_gu_bytes(c) + pf_packed_dn_bytes(c);
}
size_t pf_packed_bytes(const dsv41_moe_config *c) {
  return pf_packed_sh_off(c) + size_t(c->inter / 64) * (c->dim / 128) * 512 +
         size_t(c->dim / 128) * (c->inter / 128) * 512;
}

PfDims pf_dims(const dsv41_moe_config *cfg, int64_t T) {
  PfDims d;
  d.T = T;
  d.D = cfg->dim;
  d.I = cfg->inter;
  d.E = cfg->n_experts;
  d.k = cfg->topk;
  d.P = T * cfg->topk;
  d.nchunks = ceil_div(d.P, PF_CHUNK);
  d.cap_w = d.P / PF_TILE_ROWS + d.E + 1;       // row tiles of all experts, per m-tile
  d.cap_n = d.E;
  d.cap_rt = d.cap_w;
  return d;
}

struct PfWs {
  float *w;
  int32_t *idx;
  float *rpart;
  uint8_t *xq, *xs, *xpq, *hq, *shq;
  uint8_t *sfx_gu, *sfx_dn;   // activation scale atoms of the row tiles (gate/up, down inputs)
  uint8_t *sfx_sh, *sfh_sh;   // the same for the shared expert's dense row tiles
  uint8_t *packed;            // weight scale atoms when the caller passes none
  int32_t *ep_ids;            // expert-parallel owner: local expert of each received row
  float *ep_w;                // ... and its routing weight
  __nv_bfloat16 *yp, *ysh;
  int *chunk_cnt;
  PfPlan plan;
};

size_t pf_carve(const dsv41_moe_config *cfg, const PfDims &d, bool route, bool shared,
                bool pack, uint8_t *base, size_t cap, PfWs *ws, bool quant_x = true,
                bool ep_owner = false) {
  WsCarve c{base, cap, 0};
  PfWs w;
  memset(&w, 0, sizeof(w));
  if (route) {
    w.w = c.take<float>(d.P);
    w.idx = c.take<int32_t>(d.P);
    w.rpart = c.take<float>(dsv41_moe_route_workspace_size(d.T, d.D, d.E) / sizeof(float));
  }
  if (quant_x) {
    w.xq = c.take<uint8_t>(d.T * d.D);
    w.xs = c.take<uint8_t>(d.T * d.D / 32);
  }
  if (ep_owner) {
    w.ep_ids = c.take<int32_t>(d.P);
    w.ep_w = c.take<float>(d.P);
  }
  w.xpq = c.take<uint8_t>(d.P * d.D);
  w.hq = c.take<uint8_t>(d.P * d.I);
  w.sfx_gu = c.take<uint8_t>(d.cap_rt * (d.D / 128) * 1024);
  w.sfx_dn = c.take<uint8_t>(d.cap_rt * (d.I / 128) * 1024);
  w.yp = c.take<__nv_bfloat16>(d.P * d.D);
  if (pack) w.packed = c.take<uint8_t>(pf_packed_bytes(cfg));
  if (shared) {
    const int64_t rts = ceil_div(d.T, BS_BN);
    w.shq = c.take<uint8_t>(d.T * d.I);
    w.sfx_sh = c.take<uint8_t>(rts * (d.D / 128) * 1024);
    w.sfh_sh = c.take<uint8_t>(rts * (d.I / 128) * 1024);
    w.ysh = c.take<__nv_bfloat16>(d.T * d.D);
  }
  w.chunk_cnt = c.take<int>(d.nchunks * d.E);
  w.plan.chunk_base = w.chunk_cnt;
  w.plan.grp_off = c.take<int>(d.E);
  w.plan.grp_rt0 = c.take<int>(d.E);
  w.plan.pair_tok = c.take<int>(d.P);
  w.plan.pair_w = c.take<float>(d.P);
  w.plan.slot_pos = c.take<int>(d.P);
  w.plan.row_tile = c.take<int>(d.P);
  const int64_t mts[2] = {d.I / 64, d.D / BS_BM};
  for (int pj = 0; pj < 2; ++pj) {
    w.plan.tiles[2 * pj] = c.take<int4>(mts[pj] * d.cap_w);
    w.plan.tiles[2 * pj + 1] = c.take<int4>(mts[pj] * d.cap_n);
  }
  w.plan.ntiles = c.take<int>(4);
  w.plan.next_tile = c.take<int>(4);
  if (ws) *ws = w;
  return c.off + 256;
}

int pf_check(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, int64_t T, bool shared,
             bool routed = true) {
  DSV41_REQUIRE(cfg && W, DSV41_ERR_BAD_ARG, "NULL config/weights");
  DSV41_REQUIRE((cfg->flags & DSV41_MOE_PACKED_SCALES) == 0, DSV41_ERR_BAD_ARG,
                "prefill reads the expert scales in their release layout (no decode-packed scales)");
  int rc = route_check(T, cfg->dim, cfg->n_experts, cfg->topk, cfg->score_func);
  if (rc) return rc;
  DSV41_REQUIRE(cfg->dim % 128 == 0 && cfg->inter % 128 == 0, DSV41_ERR_BAD_SHAPE,
                "prefill needs dim and inter to be multiples of 128");
  DSV41_REQUIRE(cfg->topk <= 8, DSV41_ERR_UNSUPPORTED, "prefill supports topk <= 8");
  DSV41_REQUIRE(T * cfg->topk < (int64_t(1) << 30) && cfg->n_experts * cfg->dim < (int64_t(1) << 31),
                DSV41_ERR_BAD_SHAPE, "too many pairs or expert rows");
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(!routed || (W->w1 && W->s1 && W->w3 && W->s3 && W->w2 && W->s2),
                DSV41_ERR_BAD_ARG, "NULL expert pointer");
  DSV41_REQUIRE(!routed || (aligned(W->s1, 4) && aligned(W->s3, 4) && aligned(W->s2, 4)),
                DSV41_ERR_MISALIGNED, "expert scales must be 4-byte aligned");
  DSV41_REQUIRE(shared || routed, DSV41_ERR_BAD_ARG, "neither routed nor shared experts");
  DSV41_REQUIRE(!shared || (W->sw1 && W->ss1 && W->sw3 && W->ss3 && W->sw2 && W->ss2),
                DSV41_ERR_BAD_ARG, "NULL shared-expert pointer");
  DSV41_REQUIRE(!shared || (aligned(W->ss1, 4) && aligned(W->ss3, 4) && aligned(W->ss2, 4) &&
                            aligned(W->sw1, 16) && aligned(W->sw3, 16) && aligned(W->sw2, 16)),
                DSV41_ERR_MISALIGNED, "shared-expert weights/scales misaligned");
  return DSV41_OK;
}

}  // namespace

namespace {
int pf_pack(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, uint8_t *out,
            cudaStream_t st) {
  const int64_t E = cfg->n_experts, D = cfg->dim, I = cfg->inter;
  ProfScope prof("pf_pack_scales", st);
  if (W->s1 && W->s3 && W->s2) {
    k_pack_sfw<<<unsigned(4 * num_sms()), 256, 0, st>>>(W->s1, W->s3, E, I, D, 1, 0, out);
    DSV41_CHECK_LAUNCH("pack gate/up scales");
    k_pack_sfw<<<unsigned(4 * num_sms()), 256, 0, st>>>(W->s2, nullptr, E, D, I, 0, 0,
                                                        out + pf_packed_gu_bytes(cfg));
    DSV41_CHECK_LAUNCH("pack down scales");
  }
  if (W->ss1 && W->ss3 && W->ss2) {   // fp8 shared expert: one ue8m0 per 32x32 block
    uint8_t *sh = out + pf_packed_sh_off(cfg);
    k_pack_sfw<<<unsigned(num_sms()), 256, 0, st>>>(W->ss1, W->ss3, 1, I, D, 1, 5, sh);
    DSV41_CHECK_LAUNCH("pack shared gate/up scales");
    k_pack_sfw<<<unsigned(num_sms()), 256, 0, st>>>(W->ss2, nullptr, 1, D, I, 0, 5,
                                                    sh + size_t(I / 64) * (D / 128) * 512);
    DSV41_CHECK_LAUNCH("pack shared down scales");
  }
  return DSV41_OK;
}
}  // namespace

// ---- decode-packed expert scales (DSV41_MOE_PACKED_SCALES): s1, s3, s2 rearranged by
// k_pack_decode_sf, stored back to back [s1 | s3 | s2] with the release sizes.
extern "C" size_t dsv41_moe_decode_pack_size(const dsv41_moe_config *cfg) {
  if (!cfg || cfg->dim <= 0 || cfg->inter <= 0 || cfg->n_experts <= 0) return 0;
  const size_t gu = size_t(cfg->n_experts) * cfg->inter * (cfg->dim / 32);
  const size_t dn = size_t(cfg->n_experts) * cfg->dim * (cfg->inter / 32);
  return 2 * gu + dn;
}

extern "C" int dsv41_moe_decode_pack(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                     void *packed, size_t packed_bytes, void *stream) {
  DSV41_REQUIRE(cfg && W, DSV41_ERR_BAD_ARG, "NULL config/weights");
  DSV41_REQUIRE(cfg->dim > 0 && cfg->inter > 0 && cfg->n_experts > 0 && cfg->dim % 256 == 0 &&
                    cfg->inter % 256 == 0,
                DSV41_ERR_BAD_SHAPE, "decode-packed scales need dim and inter multiples of 256");
  DSV41_REQUIRE(W->s1 && W->s3 && W->s2 && packed, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(packed_bytes >= dsv41_moe_decode_pack_size(cfg), DSV41_ERR_BAD_ARG,
                "packed buffer too small (%zu < %zu)", packed_bytes, dsv41_moe_decode_pack_size(cfg));
  DSV41_REQUIRE(aligned(packed, 16) && aligned(W->s1, 8) && aligned(W->s3, 8) && aligned(W->s2, 8),
                DSV41_ERR_MISALIGNED, "packed must be 16-byte and scales 8-byte aligned");
  cudaStream_t st = STREAM(stream);
  const int64_t E = cfg->n_experts, D = cfg->dim, I = cfg->inter;
  uint8_t *o = static_cast<uint8_t *>(packed);
  const size_t gu = size_t(E) * I * (D / 32);
  const struct { const uint8_t *src; int64_t rows, G; uint8_t *dst; } jobs[3] = {
      {W->s1, E * I, D / 32, o}, {W->s3, E * I, D / 32, o + gu}, {W->s2, E * D, I / 32, o + 2 * gu}};
  for (const auto &j : jobs) {
    const int64_t n = j.rows * (j.G / 8);
    k_pack_decode_sf<<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(j.src, j.rows, j.G, j.dst);
    DSV41_CHECK_LAUNCH("pack_decode_sf");
  }
  return DSV41_OK;
}

extern "C" size_t dsv41_moe_prefill_pack_size(const dsv41_moe_config *cfg) {
  return cfg ? pf_packed_bytes(cfg) : 0;
}

extern "C" int dsv41_moe_prefill_pack(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                      void *packed, size_t packed_bytes, void *stream) {
  int rc = pf_check(cfg, W, 1, false);
  if (rc) return rc;
  DSV41_REQUIRE(packed && packed_bytes >= pf_packed_bytes(cfg) && aligned(packed, 16),
                DSV41_ERR_WORKSPACE, "packed buffer too small or misaligned");
  return pf_pack(cfg, W, reinterpret_cast<uint8_t *>(packed), STREAM(stream));
}

namespace {
// The routed experts of the prefill: stable sort of the pairs by expert, gather of the fp8
// rows (xq rows qld bytes apart, their scales xs rows sld bytes apart) into expert order
// with row-tile scale atoms, grouped gate/up (SwiGLU x weight -> act_quant) and down GEMMs
// -> ws.yp (bf16, sorted order).  Shared by the one-GPU layer and the expert-parallel owner.
int pf_routed(const dsv41_moe_config *cfg, const dsv41_moe_weights *W, const uint8_t *packed,
              const PfDims &d, PfWs &ws, const uint8_t *xq, int64_t qld, const uint8_t *xs,
              int64_t sld, const int32_t *ri, const float *rw, cudaStream_t st) {
  int rc = DSV41_OK;
  // stable sort of the (token, slot) pairs by expert + tile lists
  {
    ProfScope prof("pf_plan", st);
    const size_t sm = size_t(16) * d.E * sizeof(int);
    if (sm > 48 * 1024) {
      cudaFuncSetAttribute(k_pf_count, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
      cudaFuncSetAttribute(k_pf_place, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    }
    k_pf_count<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(ri, d.P, int(d.E), ws.chunk_cnt);
    DSV41_CHECK_LAUNCH("pf_count");
    k_pf_scan<<<1, 1024, 0, st>>>(ws.chunk_cnt, int(d.nchunks), int(d.E), int(d.I / 64),
                                  int(d.D / BS_BM), ws.plan);
    DSV41_CHECK_LAUNCH("pf_scan");
    k_pf_place<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(ri, rw, d.P, d.k, int(d.E), ws.plan);
    DSV41_CHECK_LAUNCH("pf_place");
  }
  {
    ProfScope prof("pf_gather", st);
    k_pf_gather<<<unsigned(ceil_div(d.P * 32, 256)), 256, 0, st>>>(
        xq, xs, qld, sld, ws.plan.pair_tok, ws.plan.row_tile, d.P, d.D, ws.xpq,
        ws.sfx_gu);
    DSV41_CHECK_LAUNCH("pf_gather");
  }
  // routed gate/up: SwiGLU * routing weight, bf16, act_quant -> hq/hs
  {
    BsMaps maps;
    memset(&maps, 0, sizeof(maps));
    rc = bs_wmap(&maps.w, W->w1, BS_W_FP4, d.E * d.I, d.D, 64);
    if (!rc) rc = bs_wmap(&maps.w2, W->w3, BS_W_FP4, d.E * d.I, d.D, 64);
    if (!rc) rc = bs_xmaps(maps.x, ws.xpq, d.P, d.D);
    if (rc) return rc;
    BsArgs a;
    memset(&a, 0, sizeof(a));
    a.nkb = int(d.D / BS_BK);
    a.a_rows = int(d.I);
    a.sw = bs_scale(W->s1, d.D / 32, 0, 32, d.E * d.I);
    a.sw2 = bs_scale(W->s3, d.D / 32, 0, 32, d.E * d.I);
    a.nkq = int(d.D / 128);
    a.mtiles = int(d.I / 64);
    a.sfa_atoms = packed;
    a.sfb_atoms = ws.sfx_gu;
    a.pw = ws.plan.pair_w;
    a.hq = ws.hq;
    a.hs_atoms = ws.sfx_dn;
    a.ldh = d.I;
    a.limit = cfg->swiglu_limit;
    // 2-CTA wide tiles: m-tiles of 64 gate + 64 up rows, taken two at a time
    const bool pair = (d.I / 64) % 2 == 0;
    if (pair) {
      rc = bs_atom_map(&maps.sfa, packed, pf_packed_gu_bytes(cfg), 2);
      if (!rc) rc = bs_atom_map(&maps.sfb, ws.sfx_gu, size_t(d.cap_rt) * (d.D / 128) * 1024, 4);
      if (rc) return rc;
    }
    rc = bs_grouped_launch<BS_W_FP4, BS_EPI_SWIGLU>("pf_gate_up_fp4", "pf_gate_up_fp4_narrow",
                                                    maps, a, ws.plan, 0, st, pair);
    if (rc) return rc;
  }
  // routed down -> yp (bf16 per pair)
  {
    BsMaps maps;
    memset(&maps, 0, sizeof(maps));
    rc = bs_wmap(&maps.w, W->w2, BS_W_FP4, d.E * d.D, d.I, 128);
    if (!rc) rc = bs_xmaps(maps.x, ws.hq, d.P, d.I);
    if (rc) return rc;
    BsArgs a;
    memset(&a, 0, sizeof(a));
    a.nkb = int(d.I / BS_BK);
    a.a_rows = int(d.D);
    a.nkq = int(d.I / 128);
    a.mtiles = int(d.D / BS_BM);
    a.sfa_atoms = packed + pf_packed_gu_bytes(cfg);
    a.sfb_atoms = ws.sfx_dn;
    a.out = ws.yp;
    a.ldo = d.D;
    const bool pair = (d.D / BS_BM) % 2 == 0;
    if (pair) {
      rc = bs_atom_map(&maps.sfa, packed + pf_packed_gu_bytes(cfg), pf_packed_dn_bytes(cfg), 2);
      if (!rc) rc = bs_atom_map(&maps.sfb, ws.sfx_dn, size_t(d.cap_rt) * (d.I / 128) * 1024, 4);
      if (rc) return rc;
    }
    rc = bs_grouped_launch<BS_W_FP4, BS_EPI_BF16>("pf_down_fp4", "pf_down_fp4_narrow", maps, a,
                                                  ws.plan, 2, st, pair);
    if (rc) return rc;
  }

  return DSV41_OK;
}
}  // namespace

namespace {
// shared-only calls carry no (token, expert) pairs
PfDims pf_dims_for(const dsv41_moe_config *cfg, int64_t T) {
  PfDims d = pf_dims(cfg, T);
  if (cfg->flags & DSV41_MOE_SHARED_ONLY) {
    d.P = 0;
    d.nchunks = 0;
  }
  return d;
}
}  // namespace

extern "C" size_t dsv41_moe_prefill_workspace_size(const dsv41_moe_config *cfg, int64_t T,
                                                   int with_routing, int with_packed) {
  if (!cfg || T <= 0) return 256;
  const bool shared = (cfg->flags & DSV41_MOE_NO_SHARED) == 0;
  const bool routed = (cfg->flags & DSV41_MOE_SHARED_ONLY) == 0;
  return pf_carve(cfg, pf_dims_for(cfg, T), routed && with_routing == 0, shared,
                  with_packed == 0, nullptr, ~size_t(0) >> 1, nullptr);
}

extern "C" int dsv41_moe_prefill(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                 const void *packed_scales, const void *x, int64_t T,
                                 const float *route_weights, const int32_t *route_indices,
                                 int out_dtype, void *y, void *workspace, size_t workspace_bytes,
                                 void *stream) {
  const bool shared = cfg && (cfg->flags & DSV41_MOE_NO_SHARED) == 0;
  const bool routed = cfg && (cfg->flags & DSV41_MOE_SHARED_ONLY) == 0;
  int rc = pf_check(cfg, W, T, shared, routed);
  if (rc) return rc;
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(!packed_scales || aligned(packed_scales, 16), DSV41_ERR_MISALIGNED,
                "packed scales must be 16-byte aligned");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "output must be F32 or BF16");
  DSV41_REQUIRE(x && y && aligned(x, 16) && aligned(y, 16), DSV41_ERR_MISALIGNED,
                "x and y must be 16-byte aligned");
  const bool route = routed && route_indices == nullptr;
  DSV41_REQUIRE(!route || W->gate_w, DSV41_ERR_BAD_ARG, "NULL gate weight");
  const PfDims d = pf_dims_for(cfg, T);
  PfWs ws;
  const size_t need = pf_carve(cfg, d, route, shared, packed_scales == nullptr,
                               reinterpret_cast<uint8_t *>(workspace), workspace_bytes, &ws);
  DSV41_REQUIRE(workspace && workspace_bytes >= need, DSV41_ERR_WORKSPACE,
                "workspace too small (%zu < %zu)", workspace_bytes, need);
  cudaStream_t st = STREAM(stream);
  const float *rw = route_weights;
  const int32_t *ri = route_indices;
  if (route) {
    DSV41_REQUIRE(aligned(W->gate_w, 16), DSV41_ERR_MISALIGNED, "gate_w must be 16-byte aligned");
    rc = route_impl(x, T, d.D, W->gate_w, W->gate_bias, d.E, d.k, cfg->score_func,
                    cfg->gate_temp, cfg->norm_topk_prob, cfg->route_scale, ws.w, ws.idx, ws.rpart,
                    st);
    if (rc) return rc;
    rw = ws.w;
    ri = ws.idx;
  }
  const uint8_t *packed = reinterpret_cast<const uint8_t *>(packed_scales);
  if (!packed) {
    rc = pf_pack(cfg, W, ws.packed, st);
    if (rc) return rc;
    packed = ws.packed;
  }
  // act_quant(x, 32, ue8m0) once per token (+ scale atoms of the shared expert's row tiles)
  {
    ProfScope prof("pf_act_quant", st);
    k_act_quant_v8<4><<<unsigned(ceil_div(d.T * (d.D / 8), 256)), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16 *>(x), d.T, d.D, 1, ws.xq, ws.xs, 1, nullptr,
        shared ? ws.sfx_sh : nullptr, BS_BN);
    DSV41_CHECK_LAUNCH("pf_act_quant");
  }
  if (routed) {
    rc = pf_routed(cfg, W, packed, d, ws, ws.xq, d.D, ws.xs, d.D / 32, ri, rw, st);
    if (rc) return rc;
  }
  if (shared) {
    BsMaps maps;
    memset(&maps, 0, sizeof(maps));
    rc = bs_wmap(&maps.w, W->sw1, BS_W_FP8, d.I, d.D, 64);
    if (!rc) rc = bs_wmap(&maps.w2, W->sw3, BS_W_FP8, d.I, d.D, 64);
    if (!rc) rc = bs_xmaps(maps.x, ws.xq, d.T, d.D);
    if (rc) return rc;
    BsArgs a = bs_args(d.D, d.I);
    a.nkq = int(d.D / 128);
    a.mtiles = int(d.I / 64);
    a.sfa_atoms = packed + pf_packed_sh_off(cfg);
    a.sfb_atoms = ws.sfx_sh;
    a.hq = ws.shq;
    a.hs_atoms = ws.sfh_sh;
    a.ldh = d.I;
    a.limit = cfg->swiglu_limit;
    rc = bs_dense_launch<BS_W_FP8, BS_EPI_SWIGLU>("pf_shared_gate_up_fp8", maps, a, d.I, d.T, st);
    if (rc) return rc;
    BsMaps m2;
    memset(&m2, 0, sizeof(m2));
    rc = bs_wmap(&m2.w, W->sw2, BS_W_FP8, d.D, d.I, 128);
    if (!rc) rc = bs_xmaps(m2.x, ws.shq, d.T, d.I);
    if (rc) return rc;
    BsArgs b = bs_args(d.I, d.D);
    b.nkq = int(d.I / 128);
    b.mtiles = int(d.D / BS_BM);
    b.sfa_atoms = packed + pf_packed_sh_off(cfg) + size_t(d.I / 64) * (d.D / 128) * 512;
    b.sfb_atoms = ws.sfh_sh;
    b.out = ws.ysh;
    b.ldo = d.D;
    rc = bs_dense_launch<BS_W_FP8, BS_EPI_BF16>("pf_shared_down_fp8", m2, b, d.D, d.T, st);
    if (rc) return rc;
  }
  {
    const int64_t n = d.T * (d.D / 8);
    ProfScope prof("pf_combine", st);
    if (out_dtype == DSV41_F32)
      k_pf_combine<float><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
          ws.yp, shared ? ws.ysh : nullptr, ri, ws.plan.slot_pos, d.T, routed ? d.k : 0, d.D,
          (float *)y);
    else
      k_pf_combine<__nv_bfloat16><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
          ws.yp, shared ? ws.ysh : nullptr, ri, ws.plan.slot_pos, d.T, routed ? d.k : 0, d.D,
          (__nv_bfloat16 *)y);
    DSV41_CHECK_LAUNCH("pf_combine");
  }
  return DSV41_OK;
}

// ======================================================================= expert-parallel prefill

namespace {
PfDims ep_owner_dims(const dsv41_moe_config *cfg, int64_t R) {
  dsv41_moe_config c = *cfg;
  c.topk = 1;
  return pf_dims(&c, R);
}
}  // namespace

// ======================================================================= prefill, port numerics
//
// The MoE layer at prefill sizes as the port computes it (deepseek_v41_mlx/moe.py:101-112):
// bf16 activations times the exactly decoded weights on kind::f16 tensor cores (a16gemm.cuh),
// expert outputs weighted and summed in top-k order after the down projection.
namespace {

struct A16Ws {
  float *w;
  int32_t *idx;
  float *rpart;
  __nv_bfloat16 *xg, *hhi, *hlo, *shi, *slo;
  float *Y, *Ys;
  int *chunk_cnt;
  PfPlan plan;
};

size_t a16_carve(const PfDims &d, bool route, bool routed, bool shared, bool round, uint8_t *base,
                 size_t cap, A16Ws *ws) {
  WsCarve c{base, cap, 0};
  A16Ws w;
  memset(&w, 0, sizeof(w));
  if (route) {
    w.w = c.take<float>(d.P);
    w.idx = c.take<int32_t>(d.P);
    w.rpart = c.take<float>(dsv41_moe_route_workspace_size(d.T, d.D, d.E) / sizeof(float));
  }
  if (routed) {
    w.xg = c.take<__nv_bfloat16>(d.P * d.D);
    w.hhi = c.take<__nv_bfloat16>(d.P * d.I);
    w.hlo = c.take<__nv_bfloat16>(d.P * d.I);     // the down projection takes the fp32 h
    w.Y = c.take<float>(d.P * d.D);
    w.chunk_cnt = c.take<int>(d.nchunks * d.E);
    w.plan.chunk_base = w.chunk_cnt;
    w.plan.grp_off = c.take<int>(d.E);
    w.plan.grp_rt0 = c.take<int>(d.E);
    w.plan.pair_tok = c.take<int>(d.P);
    w.plan.pair_w = c.take<float>(d.P);
    w.plan.slot_pos = c.take<int>(d.P);
    w.plan.row_tile = c.take<int>(d.P);
    const int64_t mts[2] = {d.I / 64, d.D / BS_BM};
    for (int pj = 0; pj < 2; ++pj) {
      w.plan.tiles[2 * pj] = c.take<int4>(mts[pj] * d.cap_w);
      w.plan.tiles[2 * pj + 1] = c.take<int4>(mts[pj] * d.cap_n);
    }
    w.plan.ntiles = c.take<int>(4);
    w.plan.next_tile = c.take<int>(4);
  }
  if (shared) {
    w.shi = c.take<__nv_bfloat16>(d.T * d.I);
    if (!round) w.slo = c.take<__nv_bfloat16>(d.T * d.I);
    w.Ys = c.take<float>(d.T * d.D);
  }
  if (ws) *ws = w;
  return c.off + 256;
}

// codes as bytes [rows, K * bits / 8], box {64 codes, box_rows}, no swizzle
int a16_wmap(CUtensorMap *m, const uint8_t *w, int wfmt, int64_t rows, int64_t K, uint32_t box_rows) {
  const uint64_t rb = wfmt == BS_W_FP4 ? uint64_t(K / 2) : uint64_t(K);
  return make_tmap_2d(m, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, rb, uint64_t(rows), rb,
                      wfmt == BS_W_FP4 ? 32u : 64u, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}
// bf16 rows [rows, K], box {64, 32 / 64 / 128 / 224 rows}, 128-byte swizzle
int a16_xmaps(CUtensorMap (&m)[4], const void *x, int64_t rows, int64_t K) {
  for (int i = 0; i < 4; ++i) {
    int rc = make_tmap_2d(&m[i], x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, uint64_t(K),
                          uint64_t(rows < 1 ? 1 : rows), uint64_t(K) * 2, 64, bs_box_rows(i));
    if (rc) return rc;
  }
  return DSV41_OK;
}

template <int WFMT, int EPI, bool HILO>
int a16_launch(const char *name, const A16Maps &maps, const A16Args &a, int grid, cudaStream_t st) {
  using Cfg = A16Cfg<WFMT, HILO>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_a16gemm<WFMT, EPI, HILO>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return cuda_status(e, "a16 smem attribute");
    attr_set[dev] = true;
  }
  ProfScope prof(name, st);
  k_a16gemm<WFMT, EPI, HILO><<<unsigned(grid < 1 ? 1 : grid), A16_THREADS, Cfg::SMEM, st>>>(maps, a);
  DSV41_CHECK_LAUNCH(name);
  return DSV41_OK;
}

A16Args a16_dense(int64_t rows, int64_t mtiles) {
  A16Args a;
  memset(&a, 0, sizeof(a));
  a.dense_nt = int(ceil_div(rows, A16_BN));
  a.dense_rows = int(rows);
  a.dense_tiles = int(mtiles) * a.dense_nt;
  return a;
}

}  // namespace

extern "C" size_t dsv41_moe_prefill_a16_workspace_size(const dsv41_moe_config *cfg, int64_t T,
                                                       int with_routing) {
  if (!cfg || T <= 0) return 256;
  const bool shared = (cfg->flags & DSV41_MOE_NO_SHARED) == 0;
  const bool routed = (cfg->flags & DSV41_MOE_SHARED_ONLY) == 0;
  const bool round = (cfg->flags & DSV41_MOE_ROUND_BF16) != 0;
  return a16_carve(pf_dims_for(cfg, T), routed && with_routing == 0, routed, shared, round,
                   nullptr, ~size_t(0) >> 1, nullptr);
}

extern "C" int dsv41_moe_prefill_a16(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                     const void *x, int64_t T, const float *route_weights,
                                     const int32_t *route_indices, int out_dtype, void *y,
                                     void *workspace, size_t workspace_bytes, void *stream) {
  const bool shared = cfg && (cfg->flags & DSV41_MOE_NO_SHARED) == 0;
  const bool routed = cfg && (cfg->flags & DSV41_MOE_SHARED_ONLY) == 0;
  int rc = pf_check(cfg, W, T, shared, routed);
  if (rc) return rc;
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "output must be F32 or BF16");
  DSV41_REQUIRE(x && y && aligned(x, 16) && aligned(y, 16), DSV41_ERR_MISALIGNED,
                "x and y must be 16-byte aligned");
  DSV41_REQUIRE(T <= (int64_t(1) << 24), DSV41_ERR_UNSUPPORTED, "T above 2^24 tokens");
  const bool round = (cfg->flags & DSV41_MOE_ROUND_BF16) != 0;
  const bool route = routed && route_indices == nullptr;
  DSV41_REQUIRE(!route || W->gate_w, DSV41_ERR_BAD_ARG, "NULL gate weight");
  DSV41_REQUIRE(!routed || route || route_weights, DSV41_ERR_BAD_ARG,
                "route_indices given without route_weights");
  const PfDims d = pf_dims_for(cfg, T);
  A16Ws ws;
  const size_t need = a16_carve(d, route, routed, shared, round,
                                reinterpret_cast<uint8_t *>(workspace), workspace_bytes, &ws);
  DSV41_REQUIRE(workspace && workspace_bytes >= need, DSV41_ERR_WORKSPACE,
                "workspace too small (%zu < %zu)", workspace_bytes, need);
  cudaStream_t st = STREAM(stream);
  const float *rw = route_weights;
  const int32_t *ri = route_indices;
  if (route) {
    DSV41_REQUIRE(aligned(W->gate_w, 16), DSV41_ERR_MISALIGNED, "gate_w must be 16-byte aligned");
    rc = route_impl(x, T, d.D, W->gate_w, W->gate_bias, d.E, d.k, cfg->score_func,
                    cfg->gate_temp, cfg->norm_topk_prob, cfg->route_scale, ws.w, ws.idx, ws.rpart,
                    st);
    if (rc) return rc;
    rw = ws.w;
    ri = ws.idx;
  }
  const int sms = num_sms();
  if (routed) {
    {  // stable sort of the (token, slot) pairs by expert + tile lists, as the a8 prefill
      ProfScope prof("a16_plan", st);
      const size_t sm = size_t(16) * d.E * sizeof(int);
      if (sm > 48 * 1024) {
        cudaFuncSetAttribute(k_pf_count, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
        cudaFuncSetAttribute(k_pf_place, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
      }
      k_pf_count<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(ri, d.P, int(d.E), ws.chunk_cnt);
      DSV41_CHECK_LAUNCH("a16 count");
      k_pf_scan<<<1, 1024, 0, st>>>(ws.chunk_cnt, int(d.nchunks), int(d.E), int(d.I / 64),
                                    int(d.D / BS_BM), ws.plan);
      DSV41_CHECK_LAUNCH("a16 scan");
      k_pf_place<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(ri, rw, d.P, d.k, int(d.E), ws.plan);
      DSV41_CHECK_LAUNCH("a16 place");
    }
    {
      ProfScope prof("a16_gather", st);
      k_a16_gather<<<unsigned(ceil_div(d.P * 32, 256)), 256, 0, st>>>(
          static_cast<const __nv_bfloat16 *>(x), ws.plan.pair_tok, d.T, d.P, d.D, ws.xg);
      DSV41_CHECK_LAUNCH("a16 gather");
    }
    // routed gate/up: SwiGLU -> h as bf16 hi + lo
    A16Maps m1;
    memset(&m1, 0, sizeof(m1));
    rc = a16_wmap(&m1.w, W->w1, BS_W_FP4, d.E * d.I, d.D, 64);
    if (!rc) rc = a16_wmap(&m1.w2, W->w3, BS_W_FP4, d.E * d.I, d.D, 64);
    if (!rc) rc = a16_xmaps(m1.x, ws.xg, d.P, d.D);
    if (rc) return rc;
    A16Args a;
    memset(&a, 0, sizeof(a));
    a.nkb = int(d.D / A16_BK);
    a.a_rows = int(d.I);
    a.s = W->s1;
    a.s2 = W->s3;
    a.sld = d.D / 32;
    a.svec = (a.sld % 16 == 0 && aligned(W->s1, 16) && aligned(W->s3, 16)) ? 1 : 0;
    a.hhi = ws.hhi;
    a.hlo = ws.hlo;
    a.ldh = d.I;
    a.round_gu = round ? 1 : 0;
    a.limit = cfg->swiglu_limit;
    for (int list = 0; list < 2; ++list) {
      a.tiles = ws.plan.tiles[list];
      a.ntiles = ws.plan.ntiles + list;
      rc = a16_launch<BS_W_FP4, A16_EPI_SWIGLU, false>("a16_gate_up_fp4", m1, a, sms, st);
      if (rc) return rc;
    }
    // routed down (input h = hi + lo) -> Y fp32 per sorted pair
    A16Maps m2;
    memset(&m2, 0, sizeof(m2));
    rc = a16_wmap(&m2.w, W->w2, BS_W_FP4, d.E * d.D, d.I, 128);
    if (!rc) rc = a16_xmaps(m2.x, ws.hhi, d.P, d.I);
    if (!rc) rc = a16_xmaps(m2.xlo, ws.hlo, d.P, d.I);
    if (rc) return rc;
    A16Args b;
    memset(&b, 0, sizeof(b));
    b.nkb = int(d.I / A16_BK);
    b.a_rows = int(d.D);
    b.s = W->s2;
    b.sld = d.I / 32;
    b.svec = (b.sld % 16 == 0 && aligned(W->s2, 16)) ? 1 : 0;
    b.out = ws.Y;
    b.ldo = d.D;
    for (int list = 2; list < 4; ++list) {
      b.tiles = ws.plan.tiles[list];
      b.ntiles = ws.plan.ntiles + list;
      rc = a16_launch<BS_W_FP4, A16_EPI_F32, true>("a16_down_fp4", m2, b, sms, st);
      if (rc) return rc;
    }
  }
  if (shared) {  // fp8 32x32 shared expert over all T rows (dense tiles)
    A16Maps m1;
    memset(&m1, 0, sizeof(m1));
    rc = a16_wmap(&m1.w, W->sw1, BS_W_FP8, d.I, d.D, 64);
    if (!rc) rc = a16_wmap(&m1.w2, W->sw3, BS_W_FP8, d.I, d.D, 64);
    if (!rc) rc = a16_xmaps(m1.x, x, d.T, d.D);
    if (rc) return rc;
    A16Args a = a16_dense(d.T, d.I / 64);
    a.nkb = int(d.D / A16_BK);
    a.a_rows = int(d.I);
    a.s = W->ss1;
    a.s2 = W->ss3;
    a.sld = ceil_div(d.D, 32);
    a.sshift = 5;
    a.svec = (a.sld % 16 == 0 && aligned(W->ss1, 16) && aligned(W->ss3, 16)) ? 1 : 0;
    a.hhi = ws.shi;
    a.hlo = ws.slo;             // null in the port's numerics: h is rounded to bf16
    a.ldh = d.I;
    a.round_gu = round ? 1 : 0;
    a.limit = cfg->swiglu_limit;
    rc = a16_launch<BS_W_FP8, A16_EPI_SWIGLU, false>("a16_shared_gate_up_fp8", m1, a,
                                                     std::min(sms, a.dense_tiles), st);
    if (rc) return rc;
    A16Maps m2;
    memset(&m2, 0, sizeof(m2));
    rc = a16_wmap(&m2.w, W->sw2, BS_W_FP8, d.D, d.I, 128);
    if (!rc) rc = a16_xmaps(m2.x, ws.shi, d.T, d.I);
    if (!rc && !round) rc = a16_xmaps(m2.xlo, ws.slo, d.T, d.I);
    if (rc) return rc;
    A16Args b = a16_dense(d.T, d.D / A16_BM);
    b.nkb = int(d.I / A16_BK);
    b.a_rows = int(d.D);
    b.s = W->ss2;
    b.sld = ceil_div(d.I, 32);
    b.sshift = 5;
    b.svec = (b.sld % 16 == 0 && aligned(W->ss2, 16)) ? 1 : 0;
    b.out = ws.Ys;
    b.ldo = d.D;
    b.round_out = round ? 1 : 0;
    if (round)
      rc = a16_launch<BS_W_FP8, A16_EPI_F32, false>("a16_shared_down_fp8", m2, b,
                                                    std::min(sms, b.dense_tiles), st);
    else
      rc = a16_launch<BS_W_FP8, A16_EPI_F32, true>("a16_shared_down_fp8", m2, b,
                                                   std::min(sms, b.dense_tiles), st);
    if (rc) return rc;
  }
  {
    const int64_t n = d.T * (d.D / 8);
    ProfScope prof("a16_combine", st);
    if (out_dtype == DSV41_F32)
      k_a16_combine<float><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
          ws.Y, shared ? ws.Ys : nullptr, rw, routed ? ws.plan.slot_pos : nullptr, d.T,
          routed ? d.k : 0, d.D, static_cast<float *>(y));
    else
      k_a16_combine<__nv_bfloat16><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
          ws.Y, shared ? ws.Ys : nullptr, rw, routed ? ws.plan.slot_pos : nullptr, d.T,
          routed ? d.k : 0, d.D, static_cast<__nv_bfloat16 *>(y));
    DSV41_CHECK_LAUNCH("a16 combine");
  }
  return DSV41_OK;
}

extern "C" size_t dsv41_moe_ep_row_bytes(int64_t dim) { return size_t(ep_row_bytes(dim)); }

extern "C" size_t dsv41_moe_ep_pack_workspace_size(const dsv41_moe_config *cfg, int64_t T) {
  if (!cfg || T <= 0) return 256;
  const PfDims d = pf_dims(cfg, T);
  WsCarve c{nullptr, ~size_t(0) >> 1, 0};
  c.take<uint8_t>(d.T * d.D);
  c.take<uint8_t>(d.T * d.D / 32);
  c.take<int>(d.nchunks * d.E);
  c.take<int>(d.E);
  c.take<int>(d.E);
  c.take<int>(d.P);
  c.take<float>(d.P);
  c.take<int>(d.P);
  c.take<int>(d.P);
  c.take<int>(8);
  return c.off + 256;
}

extern "C" int dsv41_moe_ep_pack(const dsv41_moe_config *cfg, const void *x, int64_t T,
                                 const float *route_weights, const int32_t *route_indices,
                                 int world, void *send_rows, int64_t *send_counts,
                                 int32_t *slot_pos, void *workspace, size_t workspace_bytes,
                                 void *stream) {
  DSV41_REQUIRE(cfg, DSV41_ERR_BAD_ARG, "NULL config");
  int rc = route_check(T, cfg->dim, cfg->n_experts, cfg->topk, cfg->score_func);
  if (rc) return rc;
  DSV41_REQUIRE(world >= 1 && world <= 1024 && cfg->n_experts % world == 0, DSV41_ERR_BAD_SHAPE,
                "experts must split evenly over the ranks");
  DSV41_REQUIRE(cfg->dim % 128 == 0 && cfg->topk <= 8, DSV41_ERR_BAD_SHAPE,
                "dim must be a multiple of 128, topk <= 8");
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(x && route_weights && route_indices && send_rows && send_counts && slot_pos,
                DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(x, 16) && aligned(send_rows, 16), DSV41_ERR_MISALIGNED,
                "x and send_rows must be 16-byte aligned");
  DSV41_REQUIRE(workspace && workspace_bytes >= dsv41_moe_ep_pack_workspace_size(cfg, T),
                DSV41_ERR_WORKSPACE, "workspace too small");
  const PfDims d = pf_dims(cfg, T);
  WsCarve c{reinterpret_cast<uint8_t *>(workspace), workspace_bytes, 0};
  uint8_t *xq = c.take<uint8_t>(d.T * d.D);
  uint8_t *xs = c.take<uint8_t>(d.T * d.D / 32);
  PfPlan plan;
  memset(&plan, 0, sizeof(plan));
  plan.chunk_base = c.take<int>(d.nchunks * d.E);
  plan.grp_off = c.take<int>(d.E);
  plan.grp_rt0 = c.take<int>(d.E);
  plan.pair_tok = c.take<int>(d.P);
  plan.pair_w = c.take<float>(d.P);
  plan.pair_exp = c.take<int>(d.P);
  plan.row_tile = c.take<int>(d.P);
  plan.ntiles = c.take<int>(4);
  plan.next_tile = c.take<int>(4);
  plan.slot_pos = slot_pos;
  cudaStream_t st = STREAM(stream);
  ProfScope prof("ep_pack", st);
  k_act_quant_v8<4><<<unsigned(ceil_div(d.T * (d.D / 8), 256)), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16 *>(x), d.T, d.D, 1, xq, xs, 1, nullptr, nullptr, 1);
  DSV41_CHECK_LAUNCH("ep_act_quant");
  const size_t sm = size_t(16) * d.E * sizeof(int);
  if (sm > 48 * 1024) {
    cudaFuncSetAttribute(k_pf_count, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
    cudaFuncSetAttribute(k_pf_place, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  }
  k_pf_count<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(route_indices, d.P, int(d.E), plan.chunk_base);
  DSV41_CHECK_LAUNCH("ep_count");
  k_pf_scan<<<1, 1024, 0, st>>>(plan.chunk_base, int(d.nchunks), int(d.E), 0, 0, plan);
  DSV41_CHECK_LAUNCH("ep_scan");
  k_pf_place<<<unsigned(d.nchunks), PF_CHUNK, sm, st>>>(route_indices, route_weights, d.P, d.k,
                                                       int(d.E), plan);
  DSV41_CHECK_LAUNCH("ep_place");
  k_ep_pack<<<unsigned(ceil_div(d.P * 32, 256)), 256, 0, st>>>(
      xq, xs, plan.pair_tok, plan.pair_exp, plan.pair_w, d.P, d.D, int(d.E / world),
      reinterpret_cast<uint8_t *>(send_rows));
  DSV41_CHECK_LAUNCH("ep_pack_rows");
  k_ep_counts<<<1, 1024, 0, st>>>(plan.grp_off, int(d.E), int(d.E / world), d.P, world, send_counts);
  DSV41_CHECK_LAUNCH("ep_counts");
  return DSV41_OK;
}

extern "C" size_t dsv41_moe_ep_experts_workspace_size(const dsv41_moe_config *cfg, int64_t R,
                                                      int with_packed) {
  if (!cfg || R <= 0) return 256;
  return pf_carve(cfg, ep_owner_dims(cfg, R), false, false, with_packed == 0, nullptr,
                  ~size_t(0) >> 1, nullptr, false, true);
}

extern "C" int dsv41_moe_ep_experts(const dsv41_moe_config *cfg, const dsv41_moe_weights *W,
                                    const void *packed_scales, const void *recv_rows, int64_t R,
                                    void *y, void *workspace, size_t workspace_bytes,
                                    void *stream) {
  int rc = pf_check(cfg, W, R, false, true);
  if (rc) return rc;
  if (R == 0) return DSV41_OK;
  DSV41_REQUIRE(recv_rows && y && aligned(recv_rows, 16) && aligned(y, 16), DSV41_ERR_MISALIGNED,
                "rows and y must be 16-byte aligned");
  DSV41_REQUIRE(!packed_scales || aligned(packed_scales, 16), DSV41_ERR_MISALIGNED,
                "packed scales must be 16-byte aligned");
  const PfDims d = ep_owner_dims(cfg, R);
  PfWs ws;
  const size_t need = pf_carve(cfg, d, false, false, packed_scales == nullptr,
                               reinterpret_cast<uint8_t *>(workspace), workspace_bytes, &ws,
                               false, true);
  DSV41_REQUIRE(workspace && workspace_bytes >= need, DSV41_ERR_WORKSPACE,
                "workspace too small (%zu < %zu)", workspace_bytes, need);
  cudaStream_t st = STREAM(stream);
  const uint8_t *packed = reinterpret_cast<const uint8_t *>(packed_scales);
  if (!packed) {
    rc = pf_pack(cfg, W, ws.packed, st);
    if (rc) return rc;
    packed = ws.packed;
  }
  const uint8_t *rows = reinterpret_cast<const uint8_t *>(recv_rows);
  const int64_t rb = ep_row_bytes(d.D);
  k_ep_unpack<<<unsigned(ceil_div(R, 256)), 256, 0, st>>>(rows, R, d.D, ws.ep_ids, ws.ep_w);
  DSV41_CHECK_LAUNCH("ep_unpack");
  rc = pf_routed(cfg, W, packed, d, ws, rows, rb, rows + d.D, rb, ws.ep_ids, ws.ep_w, st);
  if (rc) return rc;
  // back to arrival order: y[r] = yp[position of r] (one pair per row, bf16)
  const int64_t n = R * (d.D / 8);
  ProfScope prof("ep_unsort", st);
  k_pf_combine<__nv_bfloat16><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
      ws.yp, nullptr, ws.ep_ids, ws.plan.slot_pos, R, 1, d.D, (__nv_bfloat16 *)y);
  DSV41_CHECK_LAUNCH("ep_unsort");
  return DSV41_OK;
}

extern "C" int dsv41_moe_ep_combine(const void *back, const int32_t *slot_pos,
                                    const int32_t *route_indices, const void *shared, int64_t T,
                                    int topk, int64_t D, int out_dtype, void *y, void *stream) {
  DSV41_REQUIRE(T >= 0 && topk >= 1 && topk <= 8 && D > 0 && D % 8 == 0, DSV41_ERR_BAD_SHAPE,
                "bad shape");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "output must be F32 or BF16");
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(back && slot_pos && route_indices && y, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(back, 16) && aligned(y, 16) && (!shared || aligned(shared, 16)),
                DSV41_ERR_MISALIGNED, "buffers must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  const int64_t n = T * (D / 8);
  ProfScope prof("ep_combine", st);
  const __nv_bfloat16 *bk = reinterpret_cast<const __nv_bfloat16 *>(back);
  const __nv_bfloat16 *sh = reinterpret_cast<const __nv_bfloat16 *>(shared);
  if (out_dtype == DSV41_F32)
    k_pf_combine<float><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(bk, sh, route_indices,
                                                                    slot_pos, T, topk, D, (float *)y);
  else
    k_pf_combine<__nv_bfloat16><<<unsigned(ceil_div(n, 256)), 256, 0, st>>>(
        bk, sh, route_indices, slot_pos, T, topk, D, (__nv_bfloat16 *)y);
  DSV41_CHECK_LAUNCH("ep_combine");
  return DSV41_OK;
}

// ======================================================================= engram

extern "C" int dsv41_engram_hash(const int64_t *input_ids, int64_t B, int64_t L, int64_t start_pos,
                                 const int64_t *token_map, int64_t vocab, int64_t *ids_cache,
                                 int64_t max_seq, const int64_t *multipliers,
                                 const int64_t *primes, const int64_t *offsets, int n_layers,
                                 int max_ngram, int n_heads, int64_t pad_id, int64_t *out,
                                 void *stream) {
  DSV41_REQUIRE(B >= 0 && L >= 0 && start_pos >= 0 && start_pos + L <= max_seq,
                DSV41_ERR_BAD_SHAPE, "positions [start_pos, start_pos+L) exceed the id cache");
  DSV41_REQUIRE(n_layers >= 1 && max_ngram >= 2 && n_heads >= 1 && vocab >= 1,
                DSV41_ERR_BAD_ARG, "bad layout");
  if (B == 0 || L == 0) return DSV41_OK;
  DSV41_REQUIRE(input_ids && token_map && ids_cache && multipliers && primes && offsets && out,
                DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaStream_t st = STREAM(stream);
  const int64_t n = B * L * n_layers * (max_ngram - 1) * n_heads;
  const size_t hash_smem = sizeof(uint64_t) * size_t(n_layers) * (max_ngram - 1) * n_heads;
  DSV41_REQUIRE(hash_smem <= 48 * 1024, DSV41_ERR_UNSUPPORTED, "too many hash primes");
  k_engram_hash_cols<<<unsigned(ceil_div(n, 256)), 256, hash_smem, st>>>(
      input_ids, B, L, start_pos, token_map, vocab, ids_cache, max_seq, multipliers, primes,
      offsets, n_layers, max_ngram, n_heads, pad_id, out);
  DSV41_CHECK_LAUNCH("engram_hash");
  return DSV41_OK;
}

extern "C" int dsv41_engram_lookup_sum(const int64_t *input_ids, int64_t B, int64_t L,
                                       int64_t start_pos, const int64_t *token_map, int64_t vocab,
                                       int64_t *ids_cache, int64_t max_seq,
                                       const int64_t *multipliers, const int64_t *primes,
                                       const int64_t *offsets, const uint64_t *reciprocals,
                                       int n_layers, int layer, int max_ngram, int n_heads,
                                       int64_t pad_id, const void *packed, int64_t n_rows, int64_t row_lo,
                                       int64_t d, int64_t block, int out_dtype, void *out,
                                       void *stream) {
  DSV41_REQUIRE(B >= 0 && L >= 0 && start_pos >= 0 && start_pos + L <= max_seq,
                DSV41_ERR_BAD_SHAPE, "positions [start_pos, start_pos+L) exceed the id cache");
  DSV41_REQUIRE(n_layers >= 1 && layer >= 0 && layer < n_layers && max_ngram >= 2 &&
                    n_heads >= 1 && vocab >= 1,
                DSV41_ERR_BAD_ARG, "bad layout");
  DSV41_REQUIRE((max_ngram - 1) * n_heads <= 32 && max_ngram <= ENGRAM_MAX_G,
                DSV41_ERR_UNSUPPORTED,
                "lookup_sum needs (max_ngram - 1) * n_heads <= 32 rows a position, max_ngram <= 8");
  DSV41_REQUIRE(d == 256 || d == 512 || d == 1024, DSV41_ERR_UNSUPPORTED,
                "lookup_sum supports d in {256, 512, 1024}");
  DSV41_REQUIRE(block >= 8 && block % 8 == 0 && d % block == 0 && n_rows >= 0,
                DSV41_ERR_BAD_SHAPE, "need 8 | block and block | d");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (B == 0 || L == 0) return DSV41_OK;
  DSV41_REQUIRE(input_ids && token_map && ids_cache && multipliers && primes && offsets && out &&
                    (packed || n_rows == 0),
                DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(packed, 16) && aligned(out, 16), DSV41_ERR_MISALIGNED,
                "packed rows and out must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("engram_lookup_sum", st);
  const int G = max_ngram, H = n_heads, cols = (G - 1) * H;
  const int64_t rb = int64_t(dsv41_engram_row_bytes(d, block));
  const uint8_t *tab = static_cast<const uint8_t *>(packed);
  const unsigned blocks = unsigned(ceil_div(B * L * (d / 256) * 32, 256));
#define LS(T)                                                                                    \
  k_engram_lookup_sum<T><<<blocks, 256, 0, st>>>(                                                \
      input_ids, B, L, start_pos, token_map, vocab, ids_cache, max_seq, multipliers + layer * G, \
      primes + (int64_t)layer * cols, offsets + (int64_t)layer * cols,                          \
      reciprocals ? reciprocals + (int64_t)layer * cols : nullptr, G, H, pad_id, tab, tab + d,  \
      n_rows, row_lo, d, block, rb, rb, (T *)out)
  if (out_dtype == DSV41_F32) LS(float);
  else LS(__nv_bfloat16);
#undef LS
  DSV41_CHECK_LAUNCH("engram_lookup_sum");
  return DSV41_OK;
}

extern "C" int dsv41_engram_lookup_sum_peers(
    const int64_t *input_ids, int64_t B, int64_t L, int64_t start_pos, const int64_t *token_map,
    int64_t vocab, int64_t *ids_cache, int64_t max_seq, const int64_t *multipliers,
    const int64_t *primes, const int64_t *offsets, const uint64_t *reciprocals, int n_layers,
    int layer, int max_ngram, int n_heads, int64_t pad_id, const uint64_t *tables,
    const uint64_t *scales, int nsh, int64_t rows, int64_t total, int64_t d, int64_t block,
    int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(B >= 0 && L >= 0 && start_pos >= 0 && start_pos + L <= max_seq,
                DSV41_ERR_BAD_SHAPE, "positions [start_pos, start_pos+L) exceed the id cache");
  DSV41_REQUIRE(n_layers >= 1 && layer >= 0 && layer < n_layers && max_ngram >= 2 &&
                    n_heads >= 1 && vocab >= 1,
                DSV41_ERR_BAD_ARG, "bad layout");
  DSV41_REQUIRE((max_ngram - 1) * n_heads <= 32 && max_ngram <= ENGRAM_MAX_G,
                DSV41_ERR_UNSUPPORTED,
                "lookup_sum needs (max_ngram - 1) * n_heads <= 32 rows a position, max_ngram <= 8");
  DSV41_REQUIRE(d == 256 || d == 512 || d == 1024, DSV41_ERR_UNSUPPORTED,
                "lookup_sum supports d in {256, 512, 1024}");
  DSV41_REQUIRE(nsh >= 1 && rows >= 1 && total >= 0 && total <= rows * nsh && block >= 8 &&
                    block % 8 == 0 && d % block == 0,
                DSV41_ERR_BAD_SHAPE, "need shards, 8 | block and block | d");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (B == 0 || L == 0) return DSV41_OK;
  DSV41_REQUIRE(input_ids && token_map && ids_cache && multipliers && primes && offsets && out &&
                    tables && scales,
                DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(out, 16), DSV41_ERR_MISALIGNED, "out must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("engram_lookup_sum_peers", st);
  const int G = max_ngram, H = n_heads, cols = (G - 1) * H;
  const unsigned blocks = unsigned(ceil_div(B * L * (d / 256) * 32, 256));
  const auto *tabs = reinterpret_cast<const uint8_t *const *>(tables);
  const auto *scs = reinterpret_cast<const uint8_t *const *>(scales);
#define LSP(T)                                                                                   \
  k_engram_lookup_sum<T, true><<<blocks, 256, 0, st>>>(                                          \
      input_ids, B, L, start_pos, token_map, vocab, ids_cache, max_seq, multipliers + layer * G, \
      primes + (int64_t)layer * cols, offsets + (int64_t)layer * cols,                          \
      reciprocals ? reciprocals + (int64_t)layer * cols : nullptr, G, H, pad_id, nullptr,       \
      nullptr, rows, 0, d, block, d, d / block, (T *)out, tabs, scs, nsh, total)
  if (out_dtype == DSV41_F32) LSP(float);
  else LSP(__nv_bfloat16);
#undef LSP
  DSV41_CHECK_LAUNCH("engram_lookup_sum_peers");
  return DSV41_OK;
}

extern "C" int dsv41_engram_gather_rows(const uint8_t *table, const uint8_t *scale, int64_t rows,
                                        int64_t row_lo, int64_t d, int64_t block,
                                        const int64_t *idx, int64_t n_idx, int out_dtype,
                                        void *out, void *stream) {
  DSV41_REQUIRE(rows >= 0 && d > 0 && block > 0 && d % block == 0 && d % 8 == 0 && block % 8 == 0,
                DSV41_ERR_BAD_SHAPE, "need d %% block == 0, 8 | d, 8 | block");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (n_idx == 0) return DSV41_OK;
  DSV41_REQUIRE(table && scale && idx && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(table, 8), DSV41_ERR_MISALIGNED, "table must be 8-byte aligned");
  const unsigned blocks = unsigned(ceil_div(n_idx * 32, 256));
  if (out_dtype == DSV41_F32)
    k_engram_gather_rows<float><<<blocks, 256, 0, STREAM(stream)>>>(
        table, scale, rows, row_lo, d, block, d, d / block, idx, n_idx, (float *)out);
  else
    k_engram_gather_rows<__nv_bfloat16><<<blocks, 256, 0, STREAM(stream)>>>(
        table, scale, rows, row_lo, d, block, d, d / block, idx, n_idx, (__nv_bfloat16 *)out);
  DSV41_CHECK_LAUNCH("engram_gather_rows");
  return DSV41_OK;
}

// fp32 sum of n_per_tok rows per token (engram_gather_sum) over a table with row strides
// tld / sld bytes: a plain table (d, d / block) or packed rows received from their owners.
static int engram_sum_launch(const uint8_t *table, const uint8_t *scale, int64_t rows,
                             int64_t row_lo, int64_t d, int64_t block, int64_t tld, int64_t sld,
                             const int64_t *idx, int64_t n_tok, int n_per_tok, int out_dtype,
                             void *out, cudaStream_t st) {
  DSV41_REQUIRE(d == 256 || d == 512 || d == 1024, DSV41_ERR_UNSUPPORTED,
                "gather_sum supports d in {256, 512, 1024}");
  DSV41_REQUIRE(block >= 8 && block % 8 == 0 && d % block == 0 && rows >= 0 && n_per_tok >= 1,
                DSV41_ERR_BAD_SHAPE, "need 8 | block and block | d");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (n_tok == 0) return DSV41_OK;
  DSV41_REQUIRE(table && scale && idx && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(table, 8) && tld % 8 == 0 && aligned(out, 16), DSV41_ERR_MISALIGNED,
                "table rows must be 8-byte and out 16-byte aligned");
  ProfScope prof("engram_gather_sum", st);
  // a warp covers 256 columns
  const unsigned blocks = unsigned(ceil_div(n_tok * (d / 256) * 32, 256));
  if (out_dtype == DSV41_F32)
    k_engram_gather_sum<float><<<blocks, 256, 0, st>>>(table, scale, rows, row_lo, d, block, tld,
                                                       sld, idx, n_tok, n_per_tok, (float *)out);
  else
    k_engram_gather_sum<__nv_bfloat16><<<blocks, 256, 0, st>>>(
        table, scale, rows, row_lo, d, block, tld, sld, idx, n_tok, n_per_tok,
        (__nv_bfloat16 *)out);
  DSV41_CHECK_LAUNCH("engram_gather_sum");
  return DSV41_OK;
}

extern "C" int dsv41_engram_gather_sum(const uint8_t *table, const uint8_t *scale, int64_t rows,
                                       int64_t row_lo, int64_t d, int64_t block,
                                       const int64_t *idx, int64_t n_tok, int n_per_tok,
                                       int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(block > 0, DSV41_ERR_BAD_SHAPE, "block must be positive");
  return engram_sum_launch(table, scale, rows, row_lo, d, block, d, d / block, idx, n_tok,
                           n_per_tok, out_dtype, out, STREAM(stream));
}

// ---- CUDA IPC of a caller's allocation (any pointer inside it): the handle names the whole
// allocation, the offset locates the pointer in it.
static PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;

extern "C" int dsv41_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out) {
  DSV41_REQUIRE(ptr && handle_out && offset_out, DSV41_ERR_BAD_ARG, "NULL pointer");
  if (!g_addr_range) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
    DSV41_REQUIRE(e == cudaSuccess && fn && q == cudaDriverEntryPointSuccess, DSV41_ERR_CUDA,
                  "cuMemGetAddressRange unavailable");
    g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  DSV41_REQUIRE(r == CUDA_SUCCESS, DSV41_ERR_CUDA, "cuMemGetAddressRange failed (%d)", (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = int64_t(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return DSV41_OK;
}

// A handle is opened once per process and device; later imports of the same handle share the
// mapping (reference-counted), the last close unmaps it.
struct IpcMapping {
  int device;
  cudaIpcMemHandle_t handle;
  void *base;
  int refs;
};
static IpcMapping g_ipc[256];
static int g_ipc_n = 0;
static std::mutex g_ipc_mu;

extern "C" int dsv41_ipc_import(const void *handle, void **base_out) {
  DSV41_REQUIRE(handle && base_out, DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (int i = 0; i < g_ipc_n; ++i)
    if (g_ipc[i].refs > 0 && g_ipc[i].device == dev && !memcmp(&g_ipc[i].handle, &h, sizeof(h))) {
      ++g_ipc[i].refs;
      *base_out = g_ipc[i].base;
      return DSV41_OK;
    }
  int slot = -1;
  for (int i = 0; i < g_ipc_n && slot < 0; ++i)
    if (g_ipc[i].refs == 0) slot = i;
  if (slot < 0) {
    DSV41_REQUIRE(g_ipc_n < 256, DSV41_ERR_UNSUPPORTED, "more than 256 peer mappings");
    slot = g_ipc_n++;
  }
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
  g_ipc[slot] = IpcMapping{dev, h, *base_out, 1};
  return DSV41_OK;
}

extern "C" int dsv41_ipc_close(void *base) {
  DSV41_REQUIRE(base, DSV41_ERR_BAD_ARG, "NULL pointer");
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (int i = 0; i < g_ipc_n; ++i)
    if (g_ipc[i].refs > 0 && g_ipc[i].base == base) {
      if (--g_ipc[i].refs == 0) return cuda_status(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
      return DSV41_OK;
    }
  return set_error(DSV41_ERR_BAD_ARG, "not a mapping made by dsv41_ipc_import");
}

extern "C" int dsv41_engram_gather_sum_peers(const uint64_t *tables, const uint64_t *scales, int nsh,
                                             int64_t rows, int64_t total, int64_t d, int64_t block,
                                             const int64_t *idx, int64_t n_tok, int n_per_tok,
                                             int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(d == 256 || d == 512 || d == 1024, DSV41_ERR_UNSUPPORTED,
                "gather_sum supports d in {256, 512, 1024}");
  DSV41_REQUIRE(nsh >= 1 && rows >= 1 && total >= 0 && total <= rows * nsh && block >= 8 &&
                    block % 8 == 0 && d % block == 0 && n_per_tok >= 1,
                DSV41_ERR_BAD_SHAPE, "need shards, 8 | block and block | d");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (n_tok == 0) return DSV41_OK;
  DSV41_REQUIRE(tables && scales && idx && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(aligned(out, 16), DSV41_ERR_MISALIGNED, "out must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("engram_gather_sum_peers", st);
  const unsigned blocks = unsigned(ceil_div(n_tok * (d / 256) * 32, 256));
  const auto *tabs = reinterpret_cast<const uint8_t *const *>(tables);
  const auto *scs = reinterpret_cast<const uint8_t *const *>(scales);
  if (out_dtype == DSV41_F32)
    k_engram_gather_sum<float, true><<<blocks, 256, 0, st>>>(nullptr, nullptr, rows, 0, d, block,
                                                             d, d / block, idx, n_tok, n_per_tok,
                                                             (float *)out, tabs, scs, nsh, total);
  else
    k_engram_gather_sum<__nv_bfloat16, true><<<blocks, 256, 0, st>>>(
        nullptr, nullptr, rows, 0, d, block, d, d / block, idx, n_tok, n_per_tok,
        (__nv_bfloat16 *)out, tabs, scs, nsh, total);
  DSV41_CHECK_LAUNCH("engram_gather_sum_peers");
  return DSV41_OK;
}

extern "C" int dsv41_engram_gate(const void *x, int x_dtype, const void *kv, int kv_dtype,
                                 const float *q_weight, const float *k_weight,
                                 const uint8_t *token_mask, int64_t T, int hc, int64_t D,
                                 float eps, float clamp, void *out, void *stream) {
  DSV41_REQUIRE(T >= 0 && hc >= 1 && D >= 1, DSV41_ERR_BAD_SHAPE, "bad shape");
  DSV41_REQUIRE((x_dtype == DSV41_F32 || x_dtype == DSV41_BF16) &&
                    (kv_dtype == DSV41_F32 || kv_dtype == DSV41_BF16),
                DSV41_ERR_BAD_DTYPE, "x / kv must be F32 or BF16");
  if (T == 0) return DSV41_OK;
  DSV41_REQUIRE(x && kv && q_weight && k_weight && out, DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("engram_gate", st);
  const unsigned grid = unsigned(T * hc);
#define EG(TX, TKV)                                                                              \
  k_engram_gate<TX, TKV><<<grid, 256, 0, st>>>(static_cast<const TX *>(x), static_cast<const TKV *>(kv), \
                                               q_weight, k_weight, token_mask, hc, D, eps, clamp,  \
                                               static_cast<TX *>(out))
  if (x_dtype == DSV41_F32) {
    if (kv_dtype == DSV41_F32) EG(float, float);
    else EG(float, __nv_bfloat16);
  } else {
    if (kv_dtype == DSV41_F32) EG(__nv_bfloat16, float);
    else EG(__nv_bfloat16, __nv_bfloat16);
  }
#undef EG
  DSV41_CHECK_LAUNCH("engram_gate");
  return DSV41_OK;
}

// ---- row-sharded table: raw rows travel from their owners to the ranks that sum them
extern "C" size_t dsv41_engram_row_bytes(int64_t d, int64_t block) {
  if (d <= 0 || block <= 0) return 0;
  return size_t(align_up(size_t(d + d / block), 16));
}

extern "C" int dsv41_engram_pack_rows(const uint8_t *table, const uint8_t *scale, int64_t rows,
                                      int64_t row_lo, int64_t d, int64_t block,
                                      const int64_t *idx, int64_t n, void *out_rows,
                                      void *stream) {
  DSV41_REQUIRE(rows >= 0 && d > 0 && block > 0 && d % block == 0 && d % 16 == 0 && n >= 0,
                DSV41_ERR_BAD_SHAPE, "need block | d and 16 | d");
  if (n == 0) return DSV41_OK;
  DSV41_REQUIRE(table && scale && out_rows, DSV41_ERR_BAD_ARG, "NULL pointer");
  DSV41_REQUIRE(idx || n <= rows, DSV41_ERR_BAD_SHAPE, "without idx, n must be <= rows");
  DSV41_REQUIRE(aligned(table, 16) && aligned(out_rows, 16), DSV41_ERR_MISALIGNED,
                "table and out_rows must be 16-byte aligned");
  cudaStream_t st = STREAM(stream);
  ProfScope prof("engram_pack_rows", st);
  k_engram_pack_rows<<<unsigned(ceil_div(n * 32, 256)), 256, 0, st>>>(
      table, scale, rows, row_lo, d, block, idx, n, (uint8_t *)out_rows,
      int64_t(dsv41_engram_row_bytes(d, block)));
  DSV41_CHECK_LAUNCH("engram_pack_rows");
  return DSV41_OK;
}

extern "C" int dsv41_engram_sum_rows(const void *packed, int64_t n_rows, int64_t d, int64_t block,
                                     const int64_t *pos, int64_t n_tok, int n_per_tok,
                                     int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(d > 0 && block > 0 && d % block == 0, DSV41_ERR_BAD_SHAPE, "need block | d");
  const int64_t rb = int64_t(dsv41_engram_row_bytes(d, block));
  DSV41_REQUIRE(packed || n_rows == 0, DSV41_ERR_BAD_ARG, "NULL packed rows");
  const uint8_t *p = static_cast<const uint8_t *>(packed);
  // every position must name a received row or be negative; a NULL buffer with no rows
  // still needs a valid address for the (never read) scale pointer
  alignas(16) static const uint8_t dummy[16] = {0};
  if (!p) p = dummy;
  return engram_sum_launch(p, p + d, n_rows, 0, d, block, rb, rb, pos, n_tok, n_per_tok,
                           out_dtype, out, STREAM(stream));
}

extern "C" int dsv41_engram_dequant_rows(const void *packed, int64_t n_rows, int64_t d,
                                         int64_t block, const int64_t *pos, int64_t n,
                                         int out_dtype, void *out, void *stream) {
  DSV41_REQUIRE(d > 0 && block > 0 && d % block == 0 && d % 8 == 0 && block % 8 == 0 && n >= 0,
                DSV41_ERR_BAD_SHAPE, "need block | d, 8 | d, 8 | block");
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  if (n == 0) return DSV41_OK;
  DSV41_REQUIRE(pos && out && (packed || n_rows == 0), DSV41_ERR_BAD_ARG, "NULL pointer");
  const int64_t rb = int64_t(dsv41_engram_row_bytes(d, block));
  alignas(16) static const uint8_t dummy[16] = {0};
  const uint8_t *p = packed ? static_cast<const uint8_t *>(packed) : dummy;
  const unsigned blocks = unsigned(ceil_div(n * 32, 256));
  cudaStream_t st = STREAM(stream);
  if (out_dtype == DSV41_F32)
    k_engram_gather_rows<float><<<blocks, 256, 0, st>>>(p, p + d, n_rows, 0, d, block, rb, rb,
                                                        pos, n, (float *)out);
  else
    k_engram_gather_rows<__nv_bfloat16><<<blocks, 256, 0, st>>>(p, p + d, n_rows, 0, d, block, rb,
                                                                rb, pos, n, (__nv_bfloat16 *)out);
  DSV41_CHECK_LAUNCH("engram_dequant_rows");
  return DSV41_OK;
}

// ======================================================================= allocation-free GEMV
//
// A second entry point for the fp8 32x32 GEMV for callers that cannot hand the
// library any device memory and must not have it call cudaMalloc: hosts whose
// device memory is owned up front by their own pool or arena (cudaMalloc behind
// their back breaks their accounting and can fail once the pool has reserved the
// GPU), and FFI callers that can pass data pointers but have no allocator for a
// workspace.  Its scratch (activations as f16, split-K partial sums, split-K
// tickets) lives in the file-scope array below, which every GPU that loads this
// library holds until the process exits.
//
// Limits: 1 <= M <= 32, K % 32 == 0, M * K <= 262,144, N <= 16,384; larger
// shapes are rejected with DSV41_ERR_UNSUPPORTED (use dsv41_gemv_fp8_block with a
// workspace instead).
//
// The first call on a device looks up the array's device address for that device
// (cudaGetSymbolAddress, with that device current); make that first call before
// any stream capture.  The address is kept for the life of the process: after a
// cudaDeviceReset of that device it is stale, so do not call this entry point again
// in a process that reset the device.  All calls on a device share the one array and it keeps the
// previous call's contents: the tickets are cleared on every call, and calls whose
// kernels overlap on the GPU (different streams, no ordering between them) race on
// the array and give wrong results -- order them on one stream.
#define DSV41_NOALLOC_SCRATCH_BYTES (4u << 20)
static __device__ __align__(256) unsigned char g_noalloc_scratch[DSV41_NOALLOC_SCRATCH_BYTES];

namespace {

void *g_noalloc_ptr[64] = {nullptr};
std::mutex g_noalloc_mu;

int noalloc_scratch_ptr(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  DSV41_REQUIRE(dev >= 0 && dev < 64, DSV41_ERR_UNSUPPORTED, "device index %d >= 64", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // device `dev` is current
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return DSV41_OK;
}

template <int NT>
int noalloc_gemv_launch(const CUtensorMap &wm, const CUtensorMap (&xm)[3], QParams &p,
                        int tiles, cudaStream_t st) {
  return qgemv_launch<WF_FP8B, 1, NT>("qgemv_dense_noalloc", wm, wm, xm[0], xm[1], xm[2], p,
                                       tiles * p.nsplit, st);
}

}  // namespace

extern "C" int dsv41_gemv_fp8_block_noalloc(const void *x, int64_t M, int64_t K, const uint8_t *w,
                                            const uint8_t *s, int64_t N, int out_dtype, void *y,
                                            void *stream) {
  DSV41_REQUIRE(out_dtype == DSV41_F32 || out_dtype == DSV41_BF16, DSV41_ERR_BAD_DTYPE,
                "out_dtype must be F32 or BF16");
  DSV41_REQUIRE(M >= 0 && N >= 0 && K >= 0 && K % 32 == 0, DSV41_ERR_BAD_SHAPE,
                "negative shape, or K not a multiple of 32");
  if (M == 0 || N == 0) return DSV41_OK;          // as dsv41_gemv_fp8_block: nothing to do
  DSV41_REQUIRE(K > 0, DSV41_ERR_BAD_SHAPE, "K must be positive");
  DSV41_REQUIRE(M <= 32 && M * K <= 262144 && N <= 16384,
                DSV41_ERR_UNSUPPORTED,
                "gemv_fp8_block_noalloc: needs 1 <= M <= 32, M*K <= 262144, 1 <= N <= 16384 "
                "(got M=%lld K=%lld N=%lld); use dsv41_gemv_fp8_block with a workspace",
                (long long)M, (long long)K, (long long)N);
  DSV41_REQUIRE(x && w && s && y, DSV41_ERR_BAD_ARG, "NULL pointer");
  cudaStream_t st = STREAM(stream);
  void *base = nullptr;
  int rc = noalloc_scratch_ptr(&base);
  if (rc) return rc;

  const int NT = M <= 8 ? 1 : (M <= 16 ? 2 : 4);
  const int64_t tiles = ceil_div(N, QG_ROWS);
  WsCarve wc{reinterpret_cast<uint8_t *>(base), DSV41_NOALLOC_SCRATCH_BYTES, 0};
  __half *x16 = wc.take<__half>(M * K);
  float *xscale = wc.take<float>(32);
  int *counters = wc.take<int>(256);
  wc.off = align_up(wc.off, 256);
  float *partial = reinterpret_cast<float *>(wc.base + wc.off);
  const size_t frag_bytes = (size_t)32 * QG_CW * NT * 4 * sizeof(float);   // per tile and split
  const int64_t cap_splits = (int64_t)((DSV41_NOALLOC_SCRATCH_BYTES - wc.off) / (frag_bytes * tiles));
  DSV41_REQUIRE(wc.ok && cap_splits >= 1, DSV41_ERR_UNSUPPORTED, "shape exceeds the scratch array");

  QParams p{};
  p.scale[0] = s;
  p.scale[1] = s;
  p.N = N;
  p.K = K;
  p.sld = ceil_div(K, 32);
  p.tiles = int(tiles);
  p.kstages = int(ceil_div(K, Fmt<WF_FP8B>::KS));
  p.nsplit = pick_nsplit(tiles, p.kstages);
  if (p.nsplit > cap_splits) p.nsplit = int(cap_splits);
  p.xscale = xscale;
  p.chunks = nullptr;
  p.nchunks_host = 1;
  p.dense_m = int(M);
  p.dense_rows = 32;
  p.epi = out_dtype == DSV41_F32 ? EPI_STORE_F32 : EPI_STORE_BF16;
  p.out = y;
  p.ldo = N;
  p.partial = partial;
  p.counters = counters;
  // the array keeps the last call's contents: tickets must start at zero
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int) * 256, st);
  if (e != cudaSuccess) return cuda_status(e, "clear noalloc tickets");

  {
    ProfScope prof("qx_prep", st);
    k_qx_prep<<<unsigned(M), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16 *>(x), M, K,
                                            nullptr, nullptr, x16, xscale, nullptr, 0, nullptr, 0);
  }
  DSV41_CHECK_LAUNCH("qx_prep (noalloc)");
  CUtensorMap wm, xm[3];
  if ((rc = weight_map(&wm, w, N, K))) return rc;
  if ((rc = make_x_maps(xm, x16, M, K))) return rc;
  if (NT == 1) return noalloc_gemv_launch<1>(wm, xm, p, int(tiles), st);
  if (NT == 2) return noalloc_gemv_launch<2>(wm, xm, p, int(tiles), st);
  return noalloc_gemv_launch<4>(wm, xm, p, int(tiles), st);
}
