// qtb_engine.cu -- host runtime of the B200 decode engine: weight upload and
// repacking into tensor-core fragment order, KV page pools, stage-program
// construction, cooperative launches and the qtb_* C ABI.
//
// Build: nvcc -gencode arch=compute_100a,code=sm_100a (see the package
// Makefile).  No PyTorch, no CPU fallback: every compute path runs the
// decode_kernel in qtb_kernels.cuh.
#include "qtb_kernels.cuh"
#include "../../include/qwen3tts_b200.h"
#include "../../include/qwen_tts_cuda_b200.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstddef>
#include <cstring>
#include <string>
#include <mutex>
#include <thread>
#include <vector>
#include <algorithm>
#include <functional>
#if defined(__x86_64__) || defined(__i386__)
#include <xmmintrin.h>
#endif

using namespace qtb;

// ------------------------------------------------------------ errors -------
static thread_local std::string g_err;
// Cooperative launch of the decode kernel in 2-CTA clusters (one CTA per SM).
static void cluster_launch_config(cudaLaunchConfig_t &cfg, cudaLaunchAttribute (&at)[2], int n_sm, cudaStream_t st) {
  cfg.gridDim = dim3(n_sm);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
}

// One cluster of CL_G CTAs (the single-cluster schedule of small batches):
// the cluster is co-scheduled as a whole, so no cooperative attribute.
static void cl_launch_config(cudaLaunchConfig_t &cfg, cudaLaunchAttribute (&at)[2], cudaStream_t st) {
  cfg.gridDim = dim3(CL_G);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = SMEM_BYTES;
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL_G;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
}

// Tiled tensor maps through the driver's cuTensorMapEncodeTiled (fetched at
// run time: the library links the runtime only).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}
// A KV pool [layers][rows][128] bf16 (rows = pages x kv heads x 16) as a 3-D
// tensor of 16 x 64 boxes with the 128-byte swizzle.
static bool kv_tensor_map(CUtensorMap *out, const uint16_t *pool, int n_layers, size_t layer_elems) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || layer_elems % 128 || (uintptr_t)pool % 16) return false;
  const cuuint64_t dims[3] = {128, (cuuint64_t)(layer_elems / 128), (cuuint64_t)n_layers};
  const cuuint64_t strides[2] = {256, (cuuint64_t)layer_elems * 2};
  const cuuint32_t box[3] = {64, 16, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<uint16_t *>(pool), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int set_err(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
#define CUDA_TRY(call)                                                                          \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess)                                                                      \
      return set_err(QTB_E_CUDA, "%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_)); \
  } while (0)

extern "C" const char *qtb_last_error(void) { return g_err.c_str(); }

extern "C" int qtb_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

// ------------------------------------------ QK-norm rsqrt seeds -----------
// The reference's x86 build computes the per-head QK RMSNorm's 1 / sqrt with
// an rsqrtss seed and one Newton step (qwen_rms_norm_per_head,
// qwen_tts_kernels.c:486-577, built with -O3 -ffast-math as its Makefile
// does).  rsqrtss is implementation-defined to ~12 bits, so the device
// reproduces it from a table of this host CPU's results (qk_inv_rms in
// qtb_kernels.cuh): [exponent parity][12 leading mantissa bits] for inputs in
// [1, 4).  The table is built once per process and kept only if it
// reproduces rsqrtss on every normal input of [1, 4) (all 2^24 of them);
// otherwise, off x86, or with QTB_QK_NORM=ieee in the environment, the norm
// uses IEEE 1 / sqrtf.
constexpr int RSQ_TAB_N = 2 << 12;
static __device__ unsigned g_rsq_tab[RSQ_TAB_N];

namespace {
std::once_flag g_rsq_once;
std::vector<unsigned> g_rsq_host;   // empty: IEEE mode
std::mutex g_rsq_mu;
const unsigned *g_rsq_dev[64];      // per device, set up once
bool g_rsq_dev_done[64];
}  // namespace

static unsigned rsqrt_seed_bits(unsigned x_bits) {
#if defined(__x86_64__) || defined(__i386__)
  float x, r;
  memcpy(&x, &x_bits, 4);
  r = _mm_cvtss_f32(_mm_rsqrt_ss(_mm_set_ss(x)));
  unsigned u;
  memcpy(&u, &r, 4);
  return u;
#else
  (void)x_bits;
  return 0u;
#endif
}

static void build_rsq_table() {
  const char *env = getenv("QTB_QK_NORM");
  if (env && strcmp(env, "ieee") == 0) return;
#if defined(__x86_64__) || defined(__i386__)
  std::vector<unsigned> t(RSQ_TAB_N);
  for (unsigned par = 0; par < 2; par++)
    for (unsigned hi = 0; hi < 4096; hi++) t[(par << 12) | hi] = rsqrt_seed_bits(((127u + par) << 23) | (hi << 11));
  for (unsigned par = 0; par < 2; par++)
    for (unsigned m = 0; m < (1u << 23); m++)
      if (rsqrt_seed_bits(((127u + par) << 23) | m) != t[(par << 12) | (m >> 11)]) return;
  g_rsq_host.swap(t);
#endif
}

// Device address of the seed table on the current device (filled at the
// first call per device), or null in IEEE mode.
static int qk_rsq_table(const unsigned **out) {
  std::call_once(g_rsq_once, build_rsq_table);
  *out = nullptr;
  if (g_rsq_host.empty()) return 0;
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_err(QTB_E_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lk(g_rsq_mu);
  if (!g_rsq_dev_done[dev]) {
    void *p = nullptr;
    CUDA_TRY(cudaGetSymbolAddress(&p, g_rsq_tab));
    CUDA_TRY(cudaMemcpyToSymbol(g_rsq_tab, g_rsq_host.data(), RSQ_TAB_N * sizeof(unsigned)));
    g_rsq_dev[dev] = static_cast<const unsigned *>(p);
    g_rsq_dev_done[dev] = true;
  }
  *out = g_rsq_dev[dev];
  return 0;
}

extern "C" int qtb_qk_norm_mode(void) {
  std::call_once(g_rsq_once, build_rsq_table);
  return g_rsq_host.empty() ? 0 : 1;
}

// ------------------------------------------------------ device arena -------
struct Arena {
  std::vector<void *> ptrs;
  int alloc(void **p, size_t bytes) {
    *p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return set_err(QTB_E_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    ptrs.push_back(*p);
    return 0;
  }
  template <typename T>
  int upload(T **dst, const void *src, size_t bytes) {
    int rc = alloc((void **)dst, bytes);
    if (rc) return rc;
    cudaError_t e = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return set_err(QTB_E_CUDA, "cudaMemcpy: %s", cudaGetErrorString(e));
    return 0;
  }
  void release() {
    for (void *p : ptrs) cudaFree(p);
    ptrs.clear();
  }
};

static void parallel_for(int n, const std::function<void(int, int)> &fn) {
  unsigned hw = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  int nt = std::min<int>((int)hw, std::max(1, n / 16));
  if (nt <= 1) { fn(0, n); return; }
  std::vector<std::thread> th;
  for (int i = 0; i < nt; i++) {
    int a = (int)((long long)n * i / nt), b = (int)((long long)n * (i + 1) / nt);
    th.emplace_back(fn, a, b);
  }
  for (auto &t : th) t.join();
}

// ------------------------------------------- fragment-order repacking ------
// Tile t = 16 rows; lane l (gid = l/4, tig = l%4) of the warp holds, for each
// 16-column k-step, rows r0 = 16t+gid and r1 = r0+8 at columns c = 16s+2tig,
// c+1, c+8, c+9 (the m16n8k16 A-fragment).  The layouts below put those
// values in the lane's 16 contiguous bytes of each 512-byte warp chunk.
static inline uint16_t host_nib_q4_0(const uint8_t *blocks, int K, int r, int k) {
  const uint8_t *blk = blocks + ((size_t)r * (K / 32) + k / 32) * 18;
  const uint8_t byte = blk[2 + (k % 32) / 2];
  return (k & 1) ? (byte >> 4) : (byte & 0xf);
}
static inline uint16_t host_scale_q4_0(const uint8_t *blocks, int K, int r, int g) {
  const uint8_t *blk = blocks + ((size_t)r * (K / 32) + g) * 18;
  return (uint16_t)(blk[0] | (blk[1] << 8));
}
static inline uint16_t host_nib_i4g(const uint8_t *codes, int K, int r, int k) {
  const uint8_t byte = codes[(size_t)r * (K / 2) + k / 2];
  return (k & 1) ? (byte >> 4) : (byte & 0xf);
}

static void repack_bf16(const uint16_t *W, int rows, int K, std::vector<uint8_t> &out) {
  out.resize((size_t)rows * K * 2);
  uint16_t *o = (uint16_t *)out.data();
  const int T = rows / 16, ST = K / 16;
  parallel_for(T, [&](int t0, int t1) {
    for (int t = t0; t < t1; t++)
      for (int s = 0; s < ST; s++)
        for (int l = 0; l < 32; l++) {
          const int gid = l >> 2, tig = l & 3;
          const size_t r0 = 16 * t + gid, r1 = r0 + 8, c = 16 * s + 2 * tig;
          uint16_t *d = o + (((size_t)t * ST + s) * 32 + l) * 8;
          d[0] = W[r0 * K + c]; d[1] = W[r0 * K + c + 1];
          d[2] = W[r1 * K + c]; d[3] = W[r1 * K + c + 1];
          d[4] = W[r0 * K + c + 8]; d[5] = W[r0 * K + c + 9];
          d[6] = W[r1 * K + c + 8]; d[7] = W[r1 * K + c + 9];
        }
  });
}

static void repack_int8(const int8_t *W, int rows, int K, std::vector<uint8_t> &out) {
  out.resize((size_t)rows * K);
  uint8_t *o = out.data();
  const int T = rows / 16, CT = K / 32;
  parallel_for(T, [&](int t0, int t1) {
    for (int t = t0; t < t1; t++)
      for (int c = 0; c < CT; c++)
        for (int l = 0; l < 32; l++) {
          // the A fragment of mma m16n8k32 s8: (row gid, k 4tig..4tig+3),
          // (row gid+8, same k), then the same two at k + 16
          const int gid = l >> 2, tig = l & 3;
          const size_t r0 = 16 * t + gid, r1 = r0 + 8;
          uint8_t *d = o + (((size_t)t * CT + c) * 32 + l) * 16;
          for (int h = 0; h < 2; h++) {
            const size_t k = 32 * c + 16 * h + 4 * tig;
            for (int i = 0; i < 4; i++) {
              d[8 * h + i] = (uint8_t)W[r0 * K + k + i];
              d[8 * h + 4 + i] = (uint8_t)W[r1 * K + k + i];
            }
          }
        }
  });
}

// tcgen05 operand layout (bf16 / int8): per 128-row tile t and 128-byte K
// chunk c one 16 KB block at (t * chunks + c) * 16 KB, row r of the tile at
// (r / 8) * 1024 + (r % 8) * 128, its 16-byte units XOR-permuted by r % 8 --
// the 128-byte swizzled K-major tile the MMA reads, so one 1D bulk copy lands
// it ready in shared memory.
static void repack_tc(const uint8_t *W, int rows, int rowbytes, std::vector<uint8_t> &out) {
  const int T = rows / 128, NKC = rowbytes / 128;
  out.resize((size_t)rows * rowbytes);
  parallel_for(T, [&](int t0, int t1) {
    for (int t = t0; t < t1; t++)
      for (int c = 0; c < NKC; c++) {
        uint8_t *blk = out.data() + ((size_t)t * NKC + c) * TC_SLOT_BYTES;
        for (int r = 0; r < 128; r++) {
          const uint8_t *src = W + (size_t)(128 * t + r) * rowbytes + 128 * c;
          for (int u = 0; u < 8; u++) memcpy(blk + (r >> 3) * 1024 + (r & 7) * 128 + ((u ^ (r & 7)) << 4), src + 16 * u, 16);
        }
      }
  });
}

// Large-batch (B > 4) bf16 / int8 GEMVs run on tcgen05: every bf16 / int8
// matrix also keeps the tcgen05 operand layout.
static bool tc_enabled() { return true; }

// int4 (q4_0 or asymmetric g32): nibble getter + per-group scale/zero getters.
template <typename NibF, typename SclF, typename ZeroF>
static void repack_int4(int rows, int K, bool with_zero, NibF nib, SclF scl, ZeroF zero,
                        std::vector<uint8_t> &wout, std::vector<uint8_t> &gout) {
  wout.resize((size_t)rows * K / 2);
  const int GSZ = with_zero ? 16 : 8;
  const int T = rows / 16, CT = K / 64;
  gout.resize((size_t)T * CT * 8 * GSZ);
  uint8_t *o = wout.data();
  uint8_t *go = gout.data();
  parallel_for(T, [&](int t0, int t1) {
    for (int t = t0; t < t1; t++)
      for (int c = 0; c < CT; c++) {
        for (int l = 0; l < 32; l++) {
          const int gid = l >> 2, tig = l & 3;
          const int r0 = 16 * t + gid, r1 = r0 + 8;
          uint32_t *d = (uint32_t *)(o + (((size_t)t * CT + c) * 32 + l) * 16);
          for (int q = 0; q < 4; q++) {
            const int k = 64 * c + 16 * q + 2 * tig;
            uint32_t w = 0;
            w |= (uint32_t)nib(r0, k) << 0;      w |= (uint32_t)nib(r0, k + 1) << 16;
            w |= (uint32_t)nib(r1, k) << 4;      w |= (uint32_t)nib(r1, k + 1) << 20;
            w |= (uint32_t)nib(r0, k + 8) << 8;  w |= (uint32_t)nib(r0, k + 9) << 24;
            w |= (uint32_t)nib(r1, k + 8) << 12; w |= (uint32_t)nib(r1, k + 9) << 28;
            d[q] = w;
          }
        }
        for (int gid = 0; gid < 8; gid++) {
          const int r0 = 16 * t + gid, r1 = r0 + 8, g0 = 2 * c, g1 = 2 * c + 1;
          uint16_t *gd = (uint16_t *)(go + (((size_t)t * CT + c) * 8 + gid) * GSZ);
          gd[0] = scl(r0, g0); gd[1] = scl(r0, g1); gd[2] = scl(r1, g0); gd[3] = scl(r1, g1);
          if (with_zero) { gd[4] = zero(r0, g0); gd[5] = zero(r0, g1); gd[6] = zero(r1, g0); gd[7] = zero(r1, g1); }
        }
      }
  });
}

// ------------------------------------------------------- device matrix -----
struct DMat {
  const uint8_t *w = nullptr;
  const uint8_t *wtc = nullptr;   // tcgen05 operand layout (bf16 / int8), or null
  const float *row_scale = nullptr;
  const uint8_t *gsz = nullptr;
  int fmt = 0, rows = 0, K = 0;
  int64_t alg_bytes = 0;   // stored bytes of the reference format (weights + scales/zeros)
};

static int64_t fmt_alg_bytes(int fmt, int rows, int K) {
  switch (fmt) {
    case FMT_BF16: return (int64_t)rows * K * 2;
    case FMT_INT8: return (int64_t)rows * K + (int64_t)rows * 4;
    case FMT_Q4_0: return (int64_t)rows * (K / 32) * 18;
    case FMT_INT4G: return (int64_t)rows * (K / 32) * 20;
  }
  return 0;
}

static int check_dims(int fmt, int rows, int K) {
  if (rows <= 0 || K <= 0 || rows % 128 != 0 || K % 64 != 0)
    return set_err(QTB_E_INVALID, "matrix %dx%d: rows must be a multiple of 128 and cols of 64", rows, K);
  if (fmt < 0 || fmt > 3) return set_err(QTB_E_INVALID, "bad weight format %d", fmt);
  if (fmt == FMT_INT8 && K % 128 != 0) return set_err(QTB_E_INVALID, "int8 matrix cols %d: a multiple of 128", K);
  return 0;
}

// Upload `n` host matrices stacked along rows (same K and format) as one.
static int upload_matrix(Arena &ar, int fmt, const qtb_matrix_t *const *ms, const int *rows_each, int n, int K,
                         DMat &out) {
  int rows = 0;
  for (int i = 0; i < n; i++) {
    if (!ms[i] || !ms[i]->data) return set_err(QTB_E_INVALID, "missing weight data");
    if (rows_each[i] % 16) return set_err(QTB_E_INVALID, "row block %d not a multiple of 16", rows_each[i]);
    rows += rows_each[i];
  }
  int rc = check_dims(fmt, rows, K);
  if (rc) return rc;
  out.fmt = fmt; out.rows = rows; out.K = K;
  out.alg_bytes = fmt_alg_bytes(fmt, rows, K);
  std::vector<uint8_t> wf, gf, tcf;
  if (fmt == FMT_BF16) {
    std::vector<uint16_t> W((size_t)rows * K);
    size_t off = 0;
    for (int i = 0; i < n; i++) {
      memcpy(W.data() + off, ms[i]->data, (size_t)rows_each[i] * K * 2);
      off += (size_t)rows_each[i] * K;
    }
    repack_bf16(W.data(), rows, K, wf);
    if (tc_enabled()) repack_tc(reinterpret_cast<const uint8_t *>(W.data()), rows, K * 2, tcf);
  } else if (fmt == FMT_INT8) {
    std::vector<int8_t> W((size_t)rows * K);
    std::vector<float> sc(rows);
    size_t off = 0, ro = 0;
    for (int i = 0; i < n; i++) {
      if (!ms[i]->row_scale) return set_err(QTB_E_INVALID, "int8 matrix without row_scale");
      memcpy(W.data() + off, ms[i]->data, (size_t)rows_each[i] * K);
      memcpy(sc.data() + ro, ms[i]->row_scale, (size_t)rows_each[i] * 4);
      off += (size_t)rows_each[i] * K;
      ro += rows_each[i];
    }
    repack_int8(W.data(), rows, K, wf);
    if (tc_enabled()) repack_tc(reinterpret_cast<const uint8_t *>(W.data()), rows, K, tcf);
    float *dsc;
    if ((rc = ar.upload(&dsc, sc.data(), sc.size() * 4))) return rc;
    out.row_scale = dsc;
  } else if (fmt == FMT_Q4_0) {
    std::vector<uint8_t> Bk((size_t)rows * (K / 32) * 18);
    size_t off = 0;
    for (int i = 0; i < n; i++) {
      const size_t nb = (size_t)rows_each[i] * (K / 32) * 18;
      memcpy(Bk.data() + off, ms[i]->data, nb);
      off += nb;
    }
    const uint8_t *bp = Bk.data();
    repack_int4(rows, K, false, [&](int r, int k) { return host_nib_q4_0(bp, K, r, k); },
                [&](int r, int g) { return host_scale_q4_0(bp, K, r, g); }, [&](int, int) { return (uint16_t)0; }, wf, gf);
  } else {
    std::vector<uint8_t> C((size_t)rows * K / 2);
    std::vector<uint16_t> S((size_t)rows * (K / 32)), Z((size_t)rows * (K / 32));
    size_t off = 0, go = 0;
    for (int i = 0; i < n; i++) {
      if (!ms[i]->group_scale || !ms[i]->group_zero) return set_err(QTB_E_INVALID, "int4g32 matrix without scale/zero");
      memcpy(C.data() + off, ms[i]->data, (size_t)rows_each[i] * K / 2);
      memcpy(S.data() + go, ms[i]->group_scale, (size_t)rows_each[i] * (K / 32) * 2);
      memcpy(Z.data() + go, ms[i]->group_zero, (size_t)rows_each[i] * (K / 32) * 2);
      off += (size_t)rows_each[i] * K / 2;
      go += (size_t)rows_each[i] * (K / 32);
    }
    const uint8_t *cp = C.data();
    const uint16_t *sp = S.data(), *zp = Z.data();
    repack_int4(rows, K, true, [&](int r, int k) { return host_nib_i4g(cp, K, r, k); },
                [&](int r, int g) { return sp[(size_t)r * (K / 32) + g]; },
                [&](int r, int g) { return zp[(size_t)r * (K / 32) + g]; }, wf, gf);
  }
  uint8_t *dw;
  if ((rc = ar.upload(&dw, wf.data(), wf.size()))) return rc;
  out.w = dw;
  if (!tcf.empty()) {
    uint8_t *dt;
    if ((rc = ar.upload(&dt, tcf.data(), tcf.size()))) return rc;
    out.wtc = dt;
  }
  if (!gf.empty()) {
    uint8_t *dg;
    if ((rc = ar.upload(&dg, gf.data(), gf.size()))) return rc;
    out.gsz = dg;
  }
  return 0;
}

// ---------------------------------------------------------- the engine -----
struct DLayer {
  DMat qkv, o, gu, down;
  const float *in_norm, *post_norm, *q_norm, *k_norm;
};
struct DStack {
  int hidden = 0, n_layers = 0, n_heads = 0, n_kv = 0, head_dim = 0, inter = 0, fmt = 0;
  float eps = 1e-6f;
  std::vector<DLayer> layers;
  const float *rope_cos = nullptr, *rope_sin = nullptr;
  int rope_len = 0;
  const float *final_norm = nullptr;
  int64_t weight_bytes = 0;
  int q_dim() const { return n_heads * head_dim; }
  int kv_dim() const { return n_kv * head_dim; }
  int qkv_dim() const { return q_dim() + 2 * kv_dim(); }
};

struct qtb_engine {
  int device = 0;
  int n_sm = 0;
  int pairs = 0;   // launches run in 2-CTA clusters (K-split of small-tile int8 stages)
  int cl = 0;      // small-batch programs may run as one cluster of CL_G CTAs
  Arena ar;
  DStack talker, cp;
  int has_talker = 0, has_cp = 0;
  DMat codec_head;                 // [codebook rows used][hidden] bf16
  const uint16_t *codec_emb = nullptr;
  int codec_vocab = 0, codebook = 0;
  const float *cp_norm = nullptr;
  DMat lm_head[15];
  const uint16_t *cp_emb[15] = {};
  int cp_emb_dim = 0;
  DMat mtp;
  const float *mtp_bias = nullptr;
  int has_mtp = 0;
  const unsigned *rsq_tab = nullptr;   // QK-norm rsqrt seeds (qk_rsq_table) or null
  int codec_eos_row = 0;               // device codec-head row of the EOS token
  int has_eos = 0;
  DStack talker_pf;                    // bf16 talker weights of the prefill (when given)
  int has_talker_pf = 0;
};

static int upload_stack(qtb_engine *e, const qtb_stack_desc_t &d, DStack &s) {
  s.hidden = d.hidden; s.n_layers = d.n_layers; s.n_heads = d.n_heads; s.n_kv = d.n_kv_heads;
  s.head_dim = d.head_dim; s.inter = d.inter; s.fmt = d.fmt; s.eps = d.eps;
  if (d.head_dim != HD) return set_err(QTB_E_UNSUPPORTED, "head_dim %d (engine supports 128)", d.head_dim);
  if (d.n_kv_heads <= 0 || d.n_heads != 2 * d.n_kv_heads)
    return set_err(QTB_E_UNSUPPORTED, "GQA group %d/%d (engine supports 2 query heads per KV head)", d.n_heads, d.n_kv_heads);
  if (!d.layers) return set_err(QTB_E_INVALID, "no layers");
  int rc;
  Arena &ar = e->ar;
  s.layers.resize(d.n_layers);
  const int H = d.hidden, qd = s.q_dim(), kvd = s.kv_dim(), I = d.inter;
  for (int l = 0; l < d.n_layers; l++) {
    const qtb_layer_t &L = d.layers[l];
    DLayer &D = s.layers[l];
    const qtb_matrix_t *qkv[3] = {&L.wq, &L.wk, &L.wv};
    const int rq[3] = {qd, kvd, kvd};
    if ((rc = upload_matrix(ar, d.fmt, qkv, rq, 3, H, D.qkv))) return rc;
    const qtb_matrix_t *o[1] = {&L.wo};
    const int ro[1] = {H};
    if ((rc = upload_matrix(ar, d.fmt, o, ro, 1, qd, D.o))) return rc;
    const qtb_matrix_t *gu[1] = {&L.gate_up};
    const int rg[1] = {2 * I};
    if ((rc = upload_matrix(ar, d.fmt, gu, rg, 1, H, D.gu))) return rc;
    const qtb_matrix_t *dn[1] = {&L.down};
    const int rd[1] = {H};
    if ((rc = upload_matrix(ar, d.fmt, dn, rd, 1, I, D.down))) return rc;
    if (!L.input_norm || !L.post_attn_norm || !L.q_norm || !L.k_norm) return set_err(QTB_E_INVALID, "layer %d: missing norm", l);
    float *p;
    if ((rc = ar.upload(&p, L.input_norm, H * 4))) return rc; D.in_norm = p;
    if ((rc = ar.upload(&p, L.post_attn_norm, H * 4))) return rc; D.post_norm = p;
    if ((rc = ar.upload(&p, L.q_norm, HD * 4))) return rc; D.q_norm = p;
    if ((rc = ar.upload(&p, L.k_norm, HD * 4))) return rc; D.k_norm = p;
    s.weight_bytes += D.qkv.alg_bytes + D.o.alg_bytes + D.gu.alg_bytes + D.down.alg_bytes;
  }
  // RoPE tables: as given (bit-exact with the caller) or computed here.
  const int half = HD / 2;
  int len = d.rope_len > 0 ? d.rope_len : 8192;
  std::vector<float> cs((size_t)len * half), sn((size_t)len * half);
  if (d.rope_cos && d.rope_sin) {
    memcpy(cs.data(), d.rope_cos, cs.size() * 4);
    memcpy(sn.data(), d.rope_sin, sn.size() * 4);
  } else {
    for (int i = 0; i < half; i++) {
      const float inv = 1.0f / powf(d.rope_theta, (float)(2 * i) / (float)HD);
      for (int p = 0; p < len; p++) {
        const float ang = (float)p * inv;
        cs[(size_t)p * half + i] = cosf(ang);
        sn[(size_t)p * half + i] = sinf(ang);
      }
    }
  }
  float *pc, *ps;
  if ((rc = ar.upload(&pc, cs.data(), cs.size() * 4))) return rc;
  if ((rc = ar.upload(&ps, sn.data(), sn.size() * 4))) return rc;
  s.rope_cos = pc; s.rope_sin = ps; s.rope_len = len;
  if (d.final_norm) {
    float *p;
    if ((rc = ar.upload(&p, d.final_norm, H * 4))) return rc;
    s.final_norm = p;
  }
  return 0;
}

extern "C" void qtb_engine_destroy(qtb_engine_t *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  e->ar.release();
  delete e;
}

extern "C" int qtb_engine_create(const qtb_engine_desc_t *d, int device, qtb_engine_t **out) {
  if (!d || !out) return set_err(QTB_E_INVALID, "null argument");
  *out = nullptr;
  int ndev = 0;
  CUDA_TRY(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_err(QTB_E_INVALID, "device %d of %d", device, ndev);
  CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return set_err(QTB_E_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major, prop.minor);
  int coop = 0;
  CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
  if (!coop) return set_err(QTB_E_UNSUPPORTED, "device lacks cooperative launch");
  CUDA_TRY(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  {
    // the smallest shared-memory carveout that holds the kernel leaves the
    // rest of the SM's unified array to L1 (stack frames of the stage calls)
    cudaFuncAttributes fa;
    CUDA_TRY(cudaFuncGetAttributes(&fa, decode_kernel));
    const size_t need = (size_t)SMEM_BYTES + fa.sharedSizeBytes + 1024;
    const int pct = (int)((need * 100 + prop.sharedMemPerMultiprocessor - 1) / prop.sharedMemPerMultiprocessor);
    CUDA_TRY(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, std::min(100, pct)));
  }
  int per_sm = 0;
  CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, NTHREADS, SMEM_BYTES));
  if (per_sm < 1) return set_err(QTB_E_UNSUPPORTED, "decode kernel does not fit on an SM");

  qtb_engine *e = new qtb_engine();
  e->device = device;
  e->n_sm = prop.multiProcessorCount;
  {
    // QTB_GRID=n: run the persistent kernel on n CTAs instead of one per SM
    // (a latency-bound small batch trades bandwidth for cheaper grid barriers)
    const char *gs = getenv("QTB_GRID");
    if (gs && atoi(gs) >= 2) e->n_sm = std::min(e->n_sm, atoi(gs) & ~1);
  }
  {
    // 2-CTA clusters for the whole grid: only if all n_sm / 2 clusters can be
    // resident at once (a cooperative launch needs every CTA resident).
    // QTB_NO_CLUSTERS=1 selects the unclustered schedule (every int8 tile whole
    // in one CTA): under a kernel profiler the clustered cooperative launch did
    // not keep every CTA running at once, so its grid barrier timed out.
    const char *nc = getenv("QTB_NO_CLUSTERS");
    const bool allow = !(nc && nc[0] == '1');
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    cluster_launch_config(cfg, at, e->n_sm, nullptr);
    int ncl = 0;
    if (allow && e->n_sm % 2 == 0 &&
        cudaOccupancyMaxActiveClusters(&ncl, (const void *)decode_kernel, &cfg) == cudaSuccess && ncl >= e->n_sm / 2)
      e->pairs = 1;
    cudaGetLastError();
  }
  {
    // the single-cluster schedule, opt-in (QTB_CL=1): one cluster of CL_G
    // CTAs must fit.  Measured on B200 it is slower than the whole-GPU
    // schedule at batch 1 (c2 6.7 vs 4.7 ms per frame): 16 SMs stream the
    // weights at ~50 GB/s each, and the staging and epilogue latency per
    // stage stays, so the cheaper cluster barrier does not pay for it.
    const char *cv = getenv("QTB_CL");
    if (cv && cv[0] == '1' && e->n_sm >= CL_G &&
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute at[2];
      cl_launch_config(cfg, at, nullptr);
      int ncl = 0;
      if (cudaOccupancyMaxActiveClusters(&ncl, (const void *)decode_kernel, &cfg) == cudaSuccess && ncl >= 1) e->cl = 1;
    }
    cudaGetLastError();
  }
  int rc = 0;
  if ((rc = qk_rsq_table(&e->rsq_tab))) goto fail;
  e->has_talker = d->talker.n_layers > 0;
  if (e->has_talker) {
    if ((rc = upload_stack(e, d->talker, e->talker))) goto fail;
    if (d->talker_prefill_layers && d->talker.fmt != FMT_BF16) {
      qtb_stack_desc_t pd = d->talker;
      pd.fmt = FMT_BF16;
      pd.layers = d->talker_prefill_layers;
      if ((rc = upload_stack(e, pd, e->talker_pf))) goto fail;
      e->has_talker_pf = 1;
    }
    if (d->codec_head && d->codebook > 0) {
      // the codebook rows, then the EOS token's row (when the vocabulary has
      // one), then zero rows up to a whole 128-row tile: the special tokens the
      // reference masks never need their logits
      const int H = d->talker.hidden;
      const int rows = (d->codebook + 1 + 127) / 128 * 128;
      std::vector<uint16_t> head((size_t)rows * H, 0);
      memcpy(head.data(), d->codec_head, (size_t)d->codebook * H * 2);
      if (d->codec_vocab > QTB_CODEC_EOS)
        memcpy(head.data() + (size_t)d->codebook * H, d->codec_head + (size_t)QTB_CODEC_EOS * H, (size_t)H * 2);
      e->codec_eos_row = d->codebook;
      e->has_eos = d->codec_vocab > QTB_CODEC_EOS;
      qtb_matrix_t ch = {head.data(), nullptr, nullptr, nullptr};
      const qtb_matrix_t *m[1] = {&ch};
      const int r[1] = {rows};
      if ((rc = upload_matrix(e->ar, FMT_BF16, m, r, 1, H, e->codec_head))) goto fail;
    }
  }
  if (d->codec_embedding && d->codec_vocab > 0) {
    const int th = e->has_talker ? d->talker.hidden : d->cp_emb_dim;
    uint16_t *p;
    if ((rc = e->ar.upload(&p, d->codec_embedding, (size_t)d->codec_vocab * th * 2))) goto fail;
    e->codec_emb = p;
  }
  e->codec_vocab = d->codec_vocab;
  e->codebook = d->codebook;
  e->has_cp = d->has_cp;
  if (e->has_cp) {
    if ((rc = upload_stack(e, d->cp, e->cp))) goto fail;
    if (!d->cp_norm) { rc = set_err(QTB_E_INVALID, "cp_norm missing"); goto fail; }
    {
      float *p;
      if ((rc = e->ar.upload(&p, d->cp_norm, d->cp.hidden * 4))) goto fail;
      e->cp_norm = p;
    }
    e->cp_emb_dim = d->cp_emb_dim;
    for (int g = 0; g < 15; g++) {
      if (d->cp_lm_head[g].data) {
        const qtb_matrix_t *m[1] = {&d->cp_lm_head[g]};
        const int r[1] = {d->codebook};
        if ((rc = upload_matrix(e->ar, d->cp.fmt, m, r, 1, d->cp.hidden, e->lm_head[g]))) goto fail;
      }
      if (d->cp_codec_emb[g]) {
        uint16_t *p;
        if ((rc = e->ar.upload(&p, d->cp_codec_emb[g], (size_t)d->codebook * d->cp_emb_dim * 2))) goto fail;
        e->cp_emb[g] = p;
      }
    }
    if (d->cp_mtp_proj.data) {
      const qtb_matrix_t *m[1] = {&d->cp_mtp_proj};
      const int r[1] = {d->cp.hidden};
      if ((rc = upload_matrix(e->ar, d->cp_mtp_fmt, m, r, 1, d->cp_emb_dim, e->mtp))) goto fail;
      e->has_mtp = 1;
      if (d->cp_mtp_bias) {
        float *p;
        if ((rc = e->ar.upload(&p, d->cp_mtp_bias, d->cp.hidden * 4))) goto fail;
        e->mtp_bias = p;
      }
    }
  }
  *out = e;
  return 0;
fail:
  qtb_engine_destroy(e);
  return rc;
}

extern "C" int64_t qtb_engine_talker_weight_bytes(const qtb_engine_t *e) { return e ? e->talker.weight_bytes : 0; }
extern "C" int64_t qtb_engine_cp_pass_weight_bytes(const qtb_engine_t *e) {
  return e ? e->cp.weight_bytes + (e->has_mtp ? e->mtp.alg_bytes : 0) : 0;
}
extern "C" int64_t qtb_engine_cp_head_weight_bytes(const qtb_engine_t *e) { return e ? e->lm_head[0].alg_bytes : 0; }

// --------------------------------------------------------- the session -----
enum { PROG_TALKER = 0, PROG_CP_PASS = 1, PROG_CP_FRAME = 2, PROG_FRAME = 3, PROG_PREFILL = 4, PROG_N = 5 };
constexpr int PREFILL_CHUNK = 64;   // prompt tokens per prefill launch (the large-batch GEMV's widest batch)

struct StackBufs {
  float *x = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *hidden = nullptr, *tmp = nullptr;
  uint16_t *kpool = nullptr, *vpool = nullptr;  // [layer][n_pages][n_kv][16][128]
  int n_pages = 0;
  int *page_table = nullptr;                    // [B][pt_stride]
  int pt_stride = 0;
  int max_splits = 1, min_pps = 4;
  const void *kmap = nullptr, *vmap = nullptr;  // TMA tensor maps of the pools (device), or null
  size_t layer_pool_elems() const { return 0; }
};

// Work distribution of an attention stage: with more (slot, kv head, split)
// items than CTAs, CTAs take items from a grid-wide counter (dynamic order);
// 16 page buffers unless the program also streams small-batch GEMV weights
// (upload_prog then cuts it to 4).
static void attn_schedule(AttnArgs &a, int B, int n_sm) {
  a.dyn = (long long)B * a.n_kv * a.max_splits > n_sm ? 1 : 0;
  a.nbuf = ATT_NBUF_MAX;
}

struct qtb_session {
  qtb_engine *e = nullptr;
  int B = 0, max_ctx = 0;
  Arena ar;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  StackBufs tk, cp;
  size_t tk_layer_elems = 0, cp_layer_elems = 0;
  int *pos = nullptr;        // talker positions [B]
  int *cp_pos = nullptr;     // CP positions [B] (single-pass API)
  int *codes = nullptr;      // [B][16]
  float *cp_in = nullptr;    // [B][talker hidden] input of qtb_cp_frame
  float *pad = nullptr;      // [hidden]
  float *ws = nullptr; size_t ws_floats = 0;
  float *xsc = nullptr;      // tcgen05 stages: per-batch-row part scale and 1/rms [2][64]
  uint8_t *xop = nullptr;    // tcgen05 stages: the activation in the MMA's B-operand layout
  size_t xop_bytes = 0;
  StackBufs pf;              // prefill chunk buffers (PREFILL_CHUNK rows) over the talker's KV pools
  int *pf_pos = nullptr;     // [PREFILL_CHUNK] positions of the chunk's tokens
  PromptKV *pkv = nullptr;   // device descriptor of the prompt's f32 K/V (pkv_h: its host copy)
  PromptKV pkv_h = {};       // k, v: cudaMalloc'd on the first prefill, grown to the longest prompt
  GenState *gen = nullptr;   // codec-head generation state (device); gen_h mirrors its pointers
  GenState gen_h = {};
  int gen_on = 0;
  unsigned *sem = nullptr; int sem_n = 0;
  unsigned long long *amax_ws = nullptr;
  unsigned *amax_sem = nullptr;
  float *att_ws = nullptr;
  unsigned *att_sem = nullptr;
  Ctl *ctl = nullptr;
  Stage *prog[PROG_N] = {};
  V2Plan *plan[PROG_N] = {};   // [stage][CTA] shares of the small-batch GEMV stages
  unsigned *tc_sem[PROG_N] = {};   // per-tile counters of the split tcgen05 stages
  int tc_sem_n[PROG_N] = {};
  int prog_n[PROG_N] = {};
  int prog_G[PROG_N] = {};    // CTAs of each program's launch
  int prog_cl[PROG_N] = {};   // ... launched as one cluster (single-cluster schedule)
  int has_pad = 0;
  long long *trace = nullptr;   // per-stage clock64 trace (CTA 0), profiling only
  int trace_n = 0, trace_on = 0;
  std::vector<long long> last_ckpt;   // intra-stage checkpoints of the last profile
  std::vector<long long> last_gtrace; // per-CTA arrival times (globaltimer ns) of the last profile
  double last_ms = 0;
  int last_launches = 0;
  // pinned staging
  float *h_in = nullptr, *h_out = nullptr;
  int *h_pos = nullptr, *h_codes = nullptr;
  size_t h_in_floats = 0, h_out_floats = 0;
};

// MMA columns per batch row: bf16 weights carry the activation as bf16
// hi + mid + lo (+ a zero column) up to 16 rows, else hi + lo; the integer
// formats use fp16 hi + lo.
// MMA columns per batch row: bf16 hi/mid/lo (+0) for B <= 16; four s8 parts
// on the small-batch int8 path; f16 hi/lo otherwise.
static int parts_for(int fmt, int B, bool v2 = false) {
  if (v2 && fmt == FMT_INT8) return 4;
  return (fmt == FMT_BF16 && B <= 16) ? 4 : 2;
}
static int nch_for(int fmt, int B, bool v2 = false) {
  const int c = (parts_for(fmt, B, v2) * B + 7) / 8;
  int n = 1;
  while (n < c) n <<= 1;
  return n;
}

// Choose the k-slice count: minimise the per-warp load (rounds x slice) with
// the staged activation slice within shared memory.
static int choose_S(int T, int K, int B, int W, int fmt) {
  const int nch = nch_for(fmt, B), ent = 4 * std::min(8, parts_for(fmt, B) * B);
  int best = -1;
  double best_cost = 1e30;
  for (int S = 1; S <= 64; S <<= 1) {
    if (K % S) break;
    const int ks = K / S;
    if (ks % 64 || ks < 64) break;
    const size_t xbytes = (size_t)(ks / 16) * nch * ent * 8 + (size_t)B * (ks / 32) * 4 + 256 + 16;
    if (xbytes > (size_t)SMEM_X_BYTES) continue;
    const long long U = (long long)T * S;
    const double cost = (double)((U + W - 1) / W) * ks * (S > 1 ? 1.05 : 1.0);
    if (cost < best_cost - 1e-9) { best_cost = cost; best = S; }
  }
  return best;
}

// Small-batch GEMV path: the whole activation is staged once and the weights
// stream through the TMA ring (see gemv2_stage_t).
static bool v2_ok(int fmt, int rows, int K, int B, int G) {
  if (B > 4 || B * K > 8192) return false;   // activation staging: <= 8 quads per thread
  const int P = parts_for(fmt, B, true), nch = nch_for(fmt, B, true), ent = 4 * std::min(8, P * B);
  if (fmt == FMT_BF16 || fmt == FMT_INT8 ? nch > 2 : nch > 1) return false;
  const bool xsum = (fmt == FMT_Q4_0 || fmt == FMT_INT4G);
  // int8: one (b0, b1) pair per lane per k32 chunk and column chunk
  const size_t xb = fmt == FMT_INT8 ? (size_t)(K / 32) * nch * 32 * 8
                                    : (size_t)(K / 16) * nch * ent * 8 +
                                          (xsum ? (size_t)((B * (K / 32) + 3) & ~3) * 4 : 0);
  if (xb > (size_t)SM_X2_BYTES) return false;
  const int T = rows / 16, nt_max = (T + G - 1) / G;
  return 256 + (size_t)nt_max * (NWARPS + 1) * 16 * B * 4 <= (size_t)(SM_PAIR_OFF - SM_R_OFF);
}

// A small-batch GEMV stage on the single-cluster schedule: the activation
// staging of the small-batch path fits, and every CTA's unit results (and the
// slice sums of split tiles) fit the reduction region.
static bool cl_ok(int fmt, int rows, int K, int B) {
  if (!v2_ok(fmt, rows, K, B, 1 << 20)) return false;   // staging only (tile count checked below)
  if (rows % 16) return false;
  for (int c = 0; c < CL_G; c++) {
    const V2Plan p = cl_plan(fmt, rows, K, c, CL_G);
    const size_t units = (size_t)p.nt * p.kb, vals = (p.kb > 1) ? (size_t)p.nt : 0;
    if (256 + (units + vals) * 16 * B * 4 > (size_t)(SM_PAIR_OFF - SM_R_OFF)) return false;
  }
  return true;
}

// tcgen05 stage shape: S k-slices of kcn chunks x R row groups of 128-row tiles
// over the G CTAs, minimising the busiest CTA's copy time (a chunk is a 16 KB
// weight tile plus its N x 128-byte operand block; three chunks in flight
// stream at ~60 GB/s into one SM, measured) plus the split-K fix-up: a wait
// on the tile's other slices (~2 us) and ~1.5 us per 16-row sub-tile the CTA
// then adds up over the slices (8 sub-tiles per tile, shared by the first
// min(S, 8) slices).
struct TcShape { int S = 0, kcn = 0, R = 0; };
// The tensor-core page loop is opt-in (QTB_ATTN_TC=1, read at each program
// build / standalone call): measured on B200 it is slower than the CUDA-core
// loop (a 0.6B talker layer at 64 requests of 128-2048 positions: 202 vs 144 us).
static bool attn_tc_enabled() {
  const char *v = getenv("QTB_ATTN_TC");
  return v && v[0] == '1';
}
static bool tc_ok(const DMat &m, int B, int fmt) {
  return tc_enabled() && m.wtc && B >= 1 && B <= 64 && (fmt == FMT_BF16 || fmt == FMT_INT8) && m.rows % 128 == 0 &&
         (size_t)m.K * 4 <= (size_t)TC_NSLOT * TC_XSLOT_BYTES;   // the prep phase's row buffer
}
static TcShape tc_choose(int fmt, int rows, int K, int B, int G) {
  const int T = rows / 128, NKC = K * (fmt == FMT_INT8 ? 1 : 2) / 128;
  const int N = tc_parts(fmt) * tc_bpad(fmt, B);
  static const double sm_gbs = [] {   // QTB_TC_SM_GBS overrides the per-SM stream rate (tuning)
    const char *v = getenv("QTB_TC_SM_GBS");
    const double x = v ? atof(v) : 0.0;
    return x > 0.0 ? x : 60.0;
  }();
  const double chunk_us = (TC_SLOT_BYTES + (double)N * 128) / (sm_gbs * 1e3);
  TcShape best;
  double best_cost = 1e30;
  for (int S = 1; S <= std::min(NKC, G); S++) {
    const int kcn = (NKC + S - 1) / S;
    if ((S - 1) * kcn >= NKC) continue;   // the last slice would be empty
    const int R = std::min(T, std::max(1, G / S));
    const int tpg = (T + R - 1) / R;
    const double cost = tpg * kcn * chunk_us + (S > 1 ? 2.0 + 1.5 * tpg * ((8 + S - 1) / S) : 0.0);
    if (cost < best_cost - 1e-9) { best_cost = cost; best.S = S; best.kcn = kcn; best.R = R; }
  }
  return best;
}
static V2Plan tc_plan(const GemvArgs &g, int B, int cta, int G) {
  V2Plan p{0, 0, 0, 0, 0, 0, 0, 0};
  const TcShape sh = tc_choose(g.fmt, g.rows, g.K, B, G);
  const int T = g.rows / 128, NKC = g.K * (g.fmt == FMT_INT8 ? 1 : 2) / 128;
  const int sl = cta / sh.R, r = cta % sh.R;
  if (sh.S == 0 || sl >= sh.S) return p;
  p.t0 = (int)((long long)r * T / sh.R);
  p.nt = (int)((long long)(r + 1) * T / sh.R) - p.t0;
  p.kb = sl * sh.kcn;
  p.kc = std::min(sh.kcn, NKC - p.kb);
  p.L = p.nt * p.kc;
  p.nfill = r;      // row group
  p.pair = sl;      // k-slice
  p.pad = sh.R;
  return p;
}
// Floats of split-K partials a tcgen05 stage writes ([tile][slice][128][batch]).
static size_t tc_ws_floats(int fmt, int rows, int K, int B, int G) {
  const TcShape sh = tc_choose(fmt, rows, K, B, G);
  return sh.S > 1 ? (size_t)(rows / 128) * sh.S * 128 * tc_bpad(fmt, B) : 0;
}

struct ProgBuilder {
  qtb_session *s;
  std::vector<Stage> st;
  int err = 0;
  int cl = 0;         // single-cluster schedule (CL_G CTAs in one cluster)
  int cl_fail = 0;    // a stage this schedule cannot run was asked for
  int grid() const { return cl ? CL_G : s->e->n_sm; }
  int W() const { return grid() * NWARPS; }

  void gemv(const DMat &m, int B, const float *x, int ldx, const float *norm_w, float eps, float *y, int ldy,
            int epi, int evict_last, const float *bias = nullptr) {
    Stage S;
    memset(&S, 0, sizeof S);
    S.kind = ST_GEMV;
    S.B = B;
    GemvArgs &g = S.g;
    g.w = m.w; g.row_scale = m.row_scale; g.gsz = m.gsz; g.bias = bias;
    g.fmt = m.fmt; g.rows = m.rows; g.K = m.K;
    g.v2 = v2_ok(m.fmt, m.rows, m.K, B, grid()) ? 1 : 0;
    if (cl) {
      if (cl_ok(m.fmt, m.rows, m.K, B)) g.v2 = g.cl = 1;
      else cl_fail = 1;
    }
    if (!g.v2 && tc_ok(m, B, m.fmt)) {
      const TcShape sh = tc_choose(m.fmt, m.rows, m.K, B, grid());
      g.tc = 1;
      g.wtc = m.wtc;
      g.S = sh.S;
      g.xsc = s->xsc; g.xop = s->xop;
      g.evict_last = evict_last;
      g.x = x; g.ldx = ldx; g.norm_w = norm_w; g.eps = eps;
      g.y = y; g.ldy = ldy; g.epi = epi;
      g.ws = s->ws; g.sem = s->sem;
      g.amax_ws = s->amax_ws; g.amax_sem = s->amax_sem;
      if (sh.S < 1) { err = set_err(QTB_E_UNSUPPORTED, "no tcgen05 shape for %dx%d at B=%d", m.rows, m.K, B); return; }
      if (tc_ws_floats(m.fmt, m.rows, m.K, B, grid()) > s->ws_floats) { err = set_err(QTB_E_INVALID, "split-K workspace too small"); return; }
      if (tc_xop_bytes(m.fmt, m.K) > s->xop_bytes || B > grid() || (size_t)m.K * 4 > (size_t)TC_NSLOT * TC_XSLOT_BYTES) {
        err = set_err(QTB_E_INVALID, "tcgen05 operand staging too small (K=%d, B=%d)", m.K, B);
        return;
      }
      st.push_back(S);
      return;
    }
    g.S = g.v2 ? 1 : choose_S(m.rows / 16, m.K, B, W(), m.fmt);
    if (g.S < 1) { err = set_err(QTB_E_UNSUPPORTED, "no k-slicing fits shared memory (K=%d, B=%d)", m.K, B); return; }
    g.nch = nch_for(m.fmt, B, g.v2);
    g.parts = parts_for(m.fmt, B, g.v2);
    g.evict_last = evict_last;
    g.x = x; g.ldx = ldx; g.norm_w = norm_w; g.eps = eps;
    g.y = y; g.ldy = ldy; g.epi = epi;
    g.ws = s->ws; g.sem = s->sem;
    g.amax_ws = s->amax_ws; g.amax_sem = s->amax_sem;
    const size_t need = (size_t)(m.rows / 16) * (g.v2 ? std::max(1, grid() / std::max(1, m.rows / 16)) : g.S) * 16 * B;
    if (need > s->ws_floats) { err = set_err(QTB_E_INVALID, "split-K workspace too small"); return; }
    if (m.rows / 16 > s->sem_n) { err = set_err(QTB_E_INVALID, "semaphore array too small"); return; }
    st.push_back(S);
  }
  void argmax(const DMat &m, int B, const float *x, int ldx, const float *norm_w, float eps, int *codes,
              int code_stride, const uint16_t *emb, int emb_ld, int emb_rows, float *emb_out, int emb_out_ld,
              int evict_last) {
    gemv(m, B, x, ldx, norm_w, eps, nullptr, 0, EPI_ARGMAX, evict_last);
    if (err) return;
    GemvArgs &g = st.back().g;
    g.codes = codes; g.code_stride = code_stride;
    g.emb_table = emb; g.emb_ld = emb_ld; g.emb_rows = emb_rows; g.emb_out = emb_out; g.emb_out_ld = emb_out_ld;
  }
  void attn(const DStack &k, const StackBufs &b, int layer, int B, const int *pos_ptr, int pos_const, size_t layer_elems,
            int mode = ATT_DECODE) {
    Stage S;
    memset(&S, 0, sizeof S);
    S.kind = ST_ATTN;
    S.B = B;
    AttnArgs &a = S.a;
    a.mode = mode;
    a.qkv = b.qkv; a.ld_qkv = k.qkv_dim();
    a.out = b.attn; a.ld_out = k.q_dim();
    a.q_norm = k.layers[layer].q_norm; a.k_norm = k.layers[layer].k_norm;
    a.rope_cos = k.rope_cos; a.rope_sin = k.rope_sin; a.rope_len = k.rope_len;
    a.pos_ptr = pos_ptr; a.pos_const = pos_const;
    a.page_table = b.page_table; a.pt_stride = b.pt_stride;
    a.kpool = b.kpool + (size_t)layer * layer_elems;
    a.vpool = b.vpool + (size_t)layer * layer_elems;
    a.n_pages = b.n_pages;
    a.n_heads = k.n_heads; a.n_kv = k.n_kv;
    a.eps = k.eps; a.scale = 1.0f / sqrtf((float)HD);
    a.max_splits = b.max_splits; a.min_pps = b.min_pps;
    a.ws = s->att_ws; a.sem = s->att_sem;
    a.rsq_tab = s->e->rsq_tab;
    if (mode != ATT_DECODE) {   // prefill: one item per slot and KV head, the prompt's f32 K/V
      a.max_splits = 1; a.min_pps = 1 << 20;
      a.pkv = s->pkv; a.layer = layer;
    }
    if (cl) a.max_splits = std::max(1, std::min(a.max_splits, grid() / std::max(1, B * k.n_kv)));
    a.layer = layer;
    a.kmap = b.kmap; a.vmap = b.vmap;
    // large-batch decode attention on the tensor cores, opt-in (needs the 16
    // page buffers of a program without small-batch GEMV stages: upload_prog
    // turns it off otherwise)
    // (not the code predictor's: its items are one page of at most 16
    // positions, where the per-item set-up outweighs the page loop)
    a.tc = (mode == ATT_DECODE && B >= 8 && b.kmap && &k != &s->e->cp && attn_tc_enabled()) ? 1 : 0;
    attn_schedule(a, B, grid());
    if (mode == ATT_ATTEND) a.dyn = 0;   // static item order (attn_prefill_stage)
    st.push_back(S);
  }
  // A prompt chunk of one sequence as B slots (positions pos[i], the same page
  // table row): per layer the QKV GEMV, every token's K/V appended, then every
  // token's attention over positions <= its own, O, gate/up, down.
  void prefill_layers(const DStack &k, const StackBufs &b, int B, const int *pos_ptr, size_t layer_elems) {
    const int H = k.hidden;
    for (int l = 0; l < k.n_layers && !err; l++) {
      const DLayer &L = k.layers[l];
      gemv(L.qkv, B, b.x, H, L.in_norm, k.eps, b.qkv, k.qkv_dim(), EPI_STORE, 0);
      attn(k, b, l, B, pos_ptr, 0, layer_elems, ATT_APPEND);
      attn(k, b, l, B, pos_ptr, 0, layer_elems, ATT_ATTEND);
      gemv(L.o, B, b.attn, k.q_dim(), nullptr, k.eps, b.x, H, EPI_RESID, 0);
      gemv(L.gu, B, b.x, H, L.post_norm, k.eps, b.h, k.inter, EPI_SWIGLU, 0);
      gemv(L.down, B, b.h, k.inter, nullptr, k.eps, b.x, H, EPI_RESID, 0);
    }
  }
  void layers(const DStack &k, const StackBufs &b, int B, const int *pos_ptr, int pos_const, size_t layer_elems, int evict_last) {
    const int H = k.hidden;
    for (int l = 0; l < k.n_layers && !err; l++) {
      const DLayer &L = k.layers[l];
      gemv(L.qkv, B, b.x, H, L.in_norm, k.eps, b.qkv, k.qkv_dim(), EPI_STORE, evict_last);
      attn(k, b, l, B, pos_ptr, pos_const, layer_elems);
      gemv(L.o, B, b.attn, k.q_dim(), nullptr, k.eps, b.x, H, EPI_RESID, evict_last);
      gemv(L.gu, B, b.x, H, L.post_norm, k.eps, b.h, k.inter, EPI_SWIGLU, evict_last);
      gemv(L.down, B, b.h, k.inter, nullptr, k.eps, b.x, H, EPI_RESID, evict_last);
    }
  }
  void norm(const float *x, int ldx, const float *w, float *y, int ldy, int dim, float eps, int B) {
    Stage S;
    memset(&S, 0, sizeof S);
    S.kind = ST_NORM; S.B = B;
    S.n.x = x; S.n.ldx = ldx; S.n.w = w; S.n.y = y; S.n.ldy = ldy; S.n.dim = dim; S.n.eps = eps;
    st.push_back(S);
  }
  Stage &embed(float *dst, int ld, int dim, int B, const float *fsrc, int fsrc_ld) {
    Stage S;
    memset(&S, 0, sizeof S);
    S.kind = ST_EMBED; S.B = B;
    S.e.dst = dst; S.e.ld_dst = ld; S.e.dim = dim; S.e.fsrc = fsrc; S.e.fsrc_ld = fsrc_ld;
    st.push_back(S);
    return st.back();
  }
  static void add_tab(Stage &S, const uint16_t *tab, int ld, int rows, const int *code, int stride) {
    const int i = S.e.ntab++;
    S.e.tab[i] = tab; S.e.tab_ld[i] = ld; S.e.tab_rows[i] = rows; S.e.code[i] = code; S.e.code_stride[i] = stride;
  }
  void pos_inc(int *pos, int B) {
    Stage S;
    memset(&S, 0, sizeof S);
    S.kind = ST_POS_INC; S.B = B; S.p.pos = pos;
    st.push_back(S);
  }
};

// The code-predictor frame (qwen_cp_predict, qwen_tts_code_predictor.c:926-1045):
// pos 0 = projected talker hidden, pos 1 = projected codec embedding of code0,
// then codebooks 1..15 with the embedding of the previous code as input.
static void build_cp_frame(ProgBuilder &pb, qtb_session *s, const float *talker_hidden) {
  qtb_engine *e = s->e;
  const DStack &k = e->cp;
  StackBufs &b = s->cp;
  const int B = s->B, CH = k.hidden;
  const int TH = e->has_talker ? e->talker.hidden : e->cp_emb_dim;
  auto project = [&](const float *src, int src_ld) {
    if (e->has_mtp) pb.gemv(e->mtp, B, src, src_ld, nullptr, k.eps, b.x, CH, EPI_STORE, 1, e->mtp_bias);
    else pb.embed(b.x, CH, CH, B, src, src_ld);
  };
  // pos 0
  project(talker_hidden, TH);
  pb.layers(k, b, B, nullptr, 0, s->cp_layer_elems, 1);
  // pos 1: the talker's codec embedding of code0
  {
    float *dst = e->has_mtp ? b.tmp : b.x;
    const int dim = e->has_mtp ? TH : CH;
    Stage &S = pb.embed(dst, dim, dim, B, nullptr, 0);
    ProgBuilder::add_tab(S, e->codec_emb, TH, e->codec_vocab, s->codes, 16);
    if (e->has_mtp) pb.gemv(e->mtp, B, b.tmp, TH, nullptr, k.eps, b.x, CH, EPI_STORE, 1, e->mtp_bias);
  }
  pb.layers(k, b, B, nullptr, 1, s->cp_layer_elems, 1);
  for (int g = 0; g < 15 && !pb.err; g++) {
    const bool last = (g == 14);
    float *emb_out = e->has_mtp ? b.tmp : b.x;
    const int emb_ld = e->cp_emb_dim;
    pb.argmax(e->lm_head[g], B, b.x, CH, e->cp_norm, k.eps, s->codes + 1 + g, 16,
              last ? nullptr : e->cp_emb[g], emb_ld, e->codebook, emb_out, emb_ld, 1);
    if (last) break;
    if (e->has_mtp) pb.gemv(e->mtp, B, b.tmp, TH, nullptr, k.eps, b.x, CH, EPI_STORE, 1, e->mtp_bias);
    pb.layers(k, b, B, nullptr, g + 2, s->cp_layer_elems, 1);
  }
}

// Each CTA's share of every small-batch GEMV stage of a program ([stage][G]);
// `pairs` when the program is launched in 2-CTA clusters.
static void make_plans(const std::vector<Stage> &st, int G, bool pairs, std::vector<V2Plan> &out) {
  out.assign(st.size() * (size_t)G, V2Plan{0, 0, 0, 0, 0, 0, 0, 0});
  for (size_t i = 0; i < st.size(); i++)
    if (st[i].kind == ST_GEMV && st[i].g.tc)
      for (int c = 0; c < G; c++) out[i * G + c] = tc_plan(st[i].g, st[i].B, c, G);
  for (size_t i = 0; i < st.size(); i++)
    if (st[i].kind == ST_GEMV && st[i].g.cl)
      for (int c = 0; c < G; c++) out[i * G + c] = cl_plan(st[i].g.fmt, st[i].g.rows, st[i].g.K, c, G);
  for (size_t i = 0; i < st.size(); i++)
    if (st[i].kind == ST_GEMV && st[i].g.v2 && !st[i].g.cl)
      for (int c = 0; c < G; c++)
        out[i * G + c] = v2_plan(st[i].g.fmt, st[i].g.rows, st[i].g.K, st[i].g.norm_w != nullptr, st[i].g.epi, c, G,
                                 pairs);
}

static int upload_prog(qtb_session *s, int which, ProgBuilder &pb) {
  if (pb.err) return pb.err;
  if (pb.st.empty()) return 0;
  // the weight streamer of small-batch GEMV stages may fill the weight ring
  // during an attention stage: its page ring then stays in the activation region
  bool streams = false;
  for (const Stage &st : pb.st) streams |= (st.kind == ST_GEMV && st.g.v2);
  for (Stage &st : pb.st)
    if (st.kind == ST_ATTN && streams) { st.a.nbuf = ATT_NBUF; st.a.tc = 0; }
  // per-tile counters of the split tcgen05 stages: a disjoint range per stage,
  // zeroed at every launch of the program
  int tc_sem_n = 0;
  for (Stage &st : pb.st)
    if (st.kind == ST_GEMV && st.g.tc && st.g.S > 1) { st.g.sem_off = tc_sem_n; tc_sem_n += st.g.rows / 128; }
  if (tc_sem_n > 0) {
    unsigned *ts;
    int rc0 = s->ar.alloc((void **)&ts, (size_t)tc_sem_n * 4);
    if (rc0) return rc0;
    for (Stage &st : pb.st)
      if (st.kind == ST_GEMV && st.g.tc && st.g.S > 1) st.g.sem = ts;
    s->tc_sem[which] = ts;
  }
  s->tc_sem_n[which] = tc_sem_n;
  Stage *d;
  int rc = s->ar.upload(&d, pb.st.data(), pb.st.size() * sizeof(Stage));
  if (rc) return rc;
  std::vector<V2Plan> pl;
  make_plans(pb.st, pb.grid(), s->e->pairs != 0 && !pb.cl, pl);
  V2Plan *dp;
  if ((rc = s->ar.upload(&dp, pl.data(), pl.size() * sizeof(V2Plan)))) return rc;
  s->prog[which] = d;
  s->plan[which] = dp;
  s->prog_n[which] = (int)pb.st.size();
  s->prog_G[which] = pb.grid();
  s->prog_cl[which] = pb.cl;
  return 0;
}

static int build_programs(qtb_session *s) {
  qtb_engine *e = s->e;
  const int B = s->B;
  int rc;
  // a small-batch program runs on the single-cluster schedule when every one
  // of its stages can; otherwise (and for large batches) on the whole GPU
  auto make = [&](int which, const std::function<void(ProgBuilder &)> &fill) -> int {
    if (e->cl && B <= 4) {
      ProgBuilder pb{s};
      pb.cl = 1;
      fill(pb);
      if (!pb.err && !pb.cl_fail) return upload_prog(s, which, pb);
    }
    ProgBuilder pb{s};
    fill(pb);
    return upload_prog(s, which, pb);
  };
  if (e->has_talker) {
    const DStack &k = e->talker;
    rc = make(PROG_TALKER, [&](ProgBuilder &pb) {
      pb.layers(k, s->tk, B, s->pos, 0, s->tk_layer_elems, 0);
      pb.norm(s->tk.x, k.hidden, k.final_norm, s->tk.hidden, k.hidden, k.hidden, k.eps, B);
    });
    if (rc) return rc;
    if (s->pf.x) {
      ProgBuilder pp{s};
      const DStack &kp = e->has_talker_pf ? e->talker_pf : k;
      pp.prefill_layers(kp, s->pf, PREFILL_CHUNK, s->pf_pos, s->tk_layer_elems);
      pp.norm(s->pf.x, kp.hidden, kp.final_norm, s->pf.hidden, kp.hidden, kp.hidden, kp.eps, PREFILL_CHUNK);
      if ((rc = upload_prog(s, PROG_PREFILL, pp))) return rc;
    }
  }
  if (e->has_cp) {
    const DStack &k = e->cp;
    rc = make(PROG_CP_PASS, [&](ProgBuilder &pb) { pb.layers(k, s->cp, B, s->cp_pos, 0, s->cp_layer_elems, 1); });
    if (rc) return rc;
    rc = make(PROG_CP_FRAME, [&](ProgBuilder &pb) { build_cp_frame(pb, s, s->cp_in); });
    if (rc) return rc;
  }
  if (e->has_talker && e->codec_head.w && e->codec_emb) {
    const DStack &k = e->talker;
    rc = make(PROG_FRAME, [&](ProgBuilder &pb) {
      pb.layers(k, s->tk, B, s->pos, 0, s->tk_layer_elems, 0);
      pb.norm(s->tk.x, k.hidden, k.final_norm, s->tk.hidden, k.hidden, k.hidden, k.eps, B);
      // greedy code0 over the first `codebook` rows of the codec head
      pb.argmax(e->codec_head, B, s->tk.x, k.hidden, k.final_norm, k.eps, s->codes, 16, nullptr, 0, 0, nullptr, 0, 0);
      if (pb.err) return;
      pb.st.back().g.gen = s->gen;
      if (e->has_cp) build_cp_frame(pb, s, s->tk.hidden);
      if (pb.err) return;
      Stage &S = pb.embed(s->tk.x, k.hidden, k.hidden, B, nullptr, 0);
      ProgBuilder::add_tab(S, e->codec_emb, k.hidden, e->codec_vocab, s->codes, 16);
      if (e->has_cp)
        for (int g = 0; g < 15; g++) ProgBuilder::add_tab(S, e->cp_emb[g], e->cp_emb_dim, e->codebook, s->codes + 1 + g, 16);
      S.e.add = s->pad;
      pb.pos_inc(s->pos, B);
      pb.st.back().p.gen = s->gen;
    });
    if (rc) return rc;
  }
  return 0;
}

static int alloc_stack_bufs(qtb_session *s, const DStack &k, StackBufs &b, int B, int max_ctx, int n_pages,
                            size_t &layer_elems, int extra_tmp) {
  Arena &ar = s->ar;
  int rc;
  const size_t H = k.hidden;
  if ((rc = ar.alloc((void **)&b.x, B * H * 4))) return rc;
  if ((rc = ar.alloc((void **)&b.hidden, B * H * 4))) return rc;
  if ((rc = ar.alloc((void **)&b.qkv, (size_t)B * k.qkv_dim() * 4))) return rc;
  if ((rc = ar.alloc((void **)&b.attn, (size_t)B * k.q_dim() * 4))) return rc;
  if ((rc = ar.alloc((void **)&b.h, (size_t)B * k.inter * 4))) return rc;
  if ((rc = ar.alloc((void **)&b.tmp, (size_t)B * std::max<int>(extra_tmp, 16) * 4))) return rc;
  cudaMemset(b.x, 0, B * H * 4);
  b.pt_stride = (max_ctx + PAGE - 1) / PAGE;
  b.n_pages = n_pages > 0 ? n_pages : B * b.pt_stride;
  layer_elems = (size_t)b.n_pages * k.n_kv * PAGE * HD;
  const size_t pool = layer_elems * k.n_layers * 2;
  if ((rc = ar.alloc((void **)&b.kpool, pool))) return rc;
  if ((rc = ar.alloc((void **)&b.vpool, pool))) return rc;
  cudaMemset(b.kpool, 0, pool);
  cudaMemset(b.vpool, 0, pool);
  std::vector<int> pt((size_t)B * b.pt_stride);
  for (int i = 0; i < B; i++)
    for (int j = 0; j < b.pt_stride; j++) pt[(size_t)i * b.pt_stride + j] = (n_pages > 0) ? -1 : i * b.pt_stride + j;
  if ((rc = ar.upload(&b.page_table, pt.data(), pt.size() * 4))) return rc;
  {
    // tensor maps of the pools for the tensor-core decode attention (cudaMalloc
    // memory is 256-byte aligned, as a tensor map in global memory must be 64)
    CUtensorMap maps[2];
    if (kv_tensor_map(&maps[0], b.kpool, k.n_layers, layer_elems) &&
        kv_tensor_map(&maps[1], b.vpool, k.n_layers, layer_elems)) {
      char *d;
      if ((rc = ar.upload(&d, maps, sizeof maps))) return rc;
      b.kmap = d;
      b.vmap = d + sizeof(CUtensorMap);
    }
  }
  if (B * k.n_kv > s->e->n_sm / 2) {
    // many sequences: items of 32-64 pages taken in dynamic order keep the
    // CTAs evenly loaded whatever the length mix (pages stream across items,
    // so longer items only cut the per-item prologue and combine)
    b.max_splits = 16;
    b.min_pps = 64;
  } else {
    // at most one attention work item per CTA: a second item would double the stage
    b.max_splits = std::max(1, std::min(32, s->e->n_sm / (B * k.n_kv)));
    b.min_pps = 4;
  }
  return 0;
}

extern "C" void qtb_session_destroy(qtb_session_t *s) {
  if (!s) return;
  cudaSetDevice(s->e->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  s->ar.release();
  if (s->trace) cudaFree(s->trace);
  if (s->pkv_h.k) cudaFree(s->pkv_h.k);
  if (s->pkv_h.v) cudaFree(s->pkv_h.v);
  if (s->ev0) cudaEventDestroy(s->ev0);
  if (s->ev1) cudaEventDestroy(s->ev1);
  if (s->stream) cudaStreamDestroy(s->stream);
  cudaFreeHost(s->h_in);
  cudaFreeHost(s->h_out);
  cudaFreeHost(s->h_pos);
  cudaFreeHost(s->h_codes);
  delete s;
}

// Slots b0 .. b1 - 1 back to greedy decoding with the reference's defaults
// (top-k 50, top-p 1, LCG seed 12345: qwen_tts.c:559, qwen_tts_sampling.c:38).
static int reset_sampling(const GenState &g, int b0, int b1) {
  const int n = b1 - b0;
  std::vector<float> t(n, 0.0f), tp(n, 1.0f);
  std::vector<int32_t> tk(n, 50);
  std::vector<uint32_t> r(n, 12345u);
  CUDA_TRY(cudaMemcpy(g.temp + b0, t.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.top_k + b0, tk.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.top_p + b0, tp.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.rng + b0, r.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
  return 0;
}

extern "C" int qtb_session_create(qtb_engine_t *e, int batch, int max_ctx, int n_pages, qtb_session_t **out) {
  if (!e || !out) return set_err(QTB_E_INVALID, "null argument");
  *out = nullptr;
  if (batch < 1 || batch > 64) return set_err(QTB_E_INVALID, "batch %d outside 1..64", batch);
  CUDA_TRY(cudaSetDevice(e->device));
  qtb_session *s = new qtb_session();
  s->e = e;
  s->B = batch;
  int rc = 0;
  const int B = batch;
  if (e->has_talker) {
    if (max_ctx <= 0) max_ctx = e->talker.rope_len;
    if (max_ctx > e->talker.rope_len) max_ctx = e->talker.rope_len;
  }
  s->max_ctx = max_ctx;
  // A blocking stream: set-up work (memsets, cudaMemcpy from pageable host
  // memory, which may return before its DMA has landed) goes through the
  // legacy default stream, and the session's kernels must run behind it.
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamDefault) != cudaSuccess ||
      cudaEventCreate(&s->ev0) != cudaSuccess || cudaEventCreate(&s->ev1) != cudaSuccess) {
    rc = set_err(QTB_E_CUDA, "stream/event creation failed");
    goto fail;
  }
  {
    // workspaces sized for the largest GEMV stage of either stack
    const int W = e->n_sm * NWARPS;
    size_t ws = 16, xop = 16;
    int sem_n = 16;
    auto acc_b = [&](const DMat &m, int Bx) {
      if (!m.w) return;
      const int T = m.rows / 16;
      const int S = choose_S(T, m.K, Bx, W, m.fmt);
      if (S > 0) ws = std::max(ws, (size_t)T * S * 16 * Bx);
      ws = std::max(ws, (size_t)T * std::max(1, e->n_sm / std::max(1, T)) * 16 * Bx);
      if (tc_ok(m, Bx, m.fmt)) {
        ws = std::max(ws, tc_ws_floats(m.fmt, m.rows, m.K, Bx, e->n_sm));
        xop = std::max(xop, tc_xop_bytes(m.fmt, m.K));
      }
      sem_n = std::max(sem_n, T);
    };
    auto acc = [&](const DMat &m) { acc_b(m, B); };
    auto acc_stack = [&](const DStack &k) {
      for (const DLayer &L : k.layers) { acc(L.qkv); acc(L.o); acc(L.gu); acc(L.down); }
    };
    acc_stack(e->talker);
    for (const DLayer &L : (e->has_talker_pf ? e->talker_pf : e->talker).layers) {   // the prefill program's chunks
      acc_b(L.qkv, PREFILL_CHUNK); acc_b(L.o, PREFILL_CHUNK); acc_b(L.gu, PREFILL_CHUNK); acc_b(L.down, PREFILL_CHUNK);
    }
    acc_stack(e->cp);
    acc(e->codec_head);
    for (int g = 0; g < 15; g++) acc(e->lm_head[g]);
    acc(e->mtp);
    s->ws_floats = ws;
    s->sem_n = sem_n;
    if ((rc = s->ar.alloc((void **)&s->ws, ws * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->sem, (size_t)sem_n * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->amax_ws, (size_t)sem_n * B * 8))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->amax_sem, 64))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->ctl, sizeof(Ctl)))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->xsc, 128 * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->xop, xop))) goto fail;
    s->xop_bytes = xop;
    if ((rc = s->ar.alloc((void **)&s->pos, B * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->cp_pos, B * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->codes, (size_t)B * 16 * 4))) goto fail;
    {
      GenState &g = s->gen_h;
      g.enabled = 0;
      g.eos_row = e->codec_eos_row;
      g.eos_token = QTB_CODEC_EOS;
      g.vocab = std::max(1, e->codebook);
      g.rep_pen = 1.0f;
      g.rep_inv = 1.0f;
      if ((rc = s->ar.alloc((void **)&g.frame, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.boost_start, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.done, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.rep_count, (size_t)B * g.vocab * 2))) goto fail;
      cudaMemset(g.frame, 0, (size_t)B * 4);
      cudaMemset(g.boost_start, 0xff, (size_t)B * 4);
      cudaMemset(g.done, 0, (size_t)B * 4);
      cudaMemset(g.rep_count, 0, (size_t)B * g.vocab * 2);
      // sampling state: greedy (temperature 0) until qtb_session_set_sampling
      g.sampling = 0;
      g.ld = (g.eos_row + 1 + 3) & ~3;
      if (g.eos_row + 1 > SAMPLE_MAX_ROWS) { rc = set_err(QTB_E_UNSUPPORTED, "codec head of %d rows", g.eos_row + 1); goto fail; }
      if ((rc = s->ar.alloc((void **)&g.logits, (size_t)B * g.ld * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.temp, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.top_k, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.top_p, (size_t)B * 4))) goto fail;
      if ((rc = s->ar.alloc((void **)&g.rng, (size_t)B * 4))) goto fail;
      if ((rc = reset_sampling(g, 0, B))) goto fail;
      if ((rc = s->ar.upload(&s->gen, &g, sizeof g))) goto fail;
    }
    cudaMemset(s->sem, 0, (size_t)sem_n * 4);
    cudaMemset(s->amax_sem, 0, 64);
    cudaMemset(s->ctl, 0, sizeof(Ctl));
    cudaMemset(s->pos, 0, B * 4);
    cudaMemset(s->cp_pos, 0, B * 4);
    cudaMemset(s->codes, 0, (size_t)B * 16 * 4);
  }
  {
    int att_splits = 1, nkv = 8;
    if (e->has_talker) {
      const int mtmp = e->has_cp ? std::max(e->cp_emb_dim, e->talker.hidden) : 16;
      if ((rc = alloc_stack_bufs(s, e->talker, s->tk, B, max_ctx, n_pages, s->tk_layer_elems, mtmp))) goto fail;
      att_splits = std::max(att_splits, s->tk.max_splits);
      nkv = e->talker.n_kv;
      if ((rc = s->ar.alloc((void **)&s->pad, (size_t)e->talker.hidden * 4))) goto fail;
      cudaMemset(s->pad, 0, (size_t)e->talker.hidden * 4);
      // prefill chunks: PREFILL_CHUNK rows of activations over the same KV pools
      {
        StackBufs &p = s->pf;
        const DStack &k = e->talker;
        const size_t R = PREFILL_CHUNK;
        if ((rc = s->ar.alloc((void **)&p.x, R * k.hidden * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&p.hidden, R * k.hidden * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&p.qkv, R * k.qkv_dim() * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&p.attn, R * k.q_dim() * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&p.h, R * k.inter * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&p.page_table, R * s->tk.pt_stride * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&s->pf_pos, R * 4))) goto fail;
        if ((rc = s->ar.alloc((void **)&s->pkv, sizeof(PromptKV)))) goto fail;
        cudaMemset(s->pf_pos, 0, R * 4);
        cudaMemset(s->pkv, 0, sizeof(PromptKV));
        cudaMemset(p.page_table, 0, R * s->tk.pt_stride * 4);
        p.kpool = s->tk.kpool; p.vpool = s->tk.vpool;
        p.kmap = s->tk.kmap; p.vmap = s->tk.vmap;
        p.n_pages = s->tk.n_pages; p.pt_stride = s->tk.pt_stride;
        p.max_splits = 16; p.min_pps = 64;
        att_splits = std::max(att_splits, p.max_splits);
      }
    }
    if (e->has_cp) {
      const int th = e->has_talker ? e->talker.hidden : e->cp_emb_dim;
      if ((rc = s->ar.alloc((void **)&s->cp_in, (size_t)B * th * 4))) goto fail;
      const int cp_ctx = std::min(64, e->cp.rope_len);
      if ((rc = alloc_stack_bufs(s, e->cp, s->cp, B, cp_ctx, 0, s->cp_layer_elems, e->cp_emb_dim + e->talker.hidden))) goto fail;
      s->cp.max_splits = 1;
      nkv = std::max(nkv, e->cp.n_kv);
    }
    const int Ba = e->has_talker ? std::max(B, PREFILL_CHUNK) : B;
    if ((rc = s->ar.alloc((void **)&s->att_ws, (size_t)Ba * nkv * att_splits * 2 * (HD + 2) * 4))) goto fail;
    if ((rc = s->ar.alloc((void **)&s->att_sem, (size_t)Ba * nkv * 4))) goto fail;
    cudaMemset(s->att_sem, 0, (size_t)Ba * nkv * 4);
  }
  {
    const int H = e->has_talker ? e->talker.hidden : e->cp.hidden;
    s->h_in_floats = (size_t)B * std::max(std::max(H, e->has_cp ? e->cp.hidden : 0), e->cp_emb_dim) + 16;
    s->h_out_floats = s->h_in_floats;
    if (cudaMallocHost(&s->h_in, s->h_in_floats * 4) != cudaSuccess ||
        cudaMallocHost(&s->h_out, s->h_out_floats * 4) != cudaSuccess ||
        cudaMallocHost(&s->h_pos, (size_t)B * 4) != cudaSuccess ||
        cudaMallocHost(&s->h_codes, (size_t)B * 16 * 4) != cudaSuccess) {
      rc = set_err(QTB_E_OOM, "pinned host allocation failed");
      goto fail;
    }
  }
  if ((rc = build_programs(s))) goto fail;
  if (cudaDeviceSynchronize() != cudaSuccess) { rc = set_err(QTB_E_CUDA, "session init sync failed"); goto fail; }
  *out = s;
  return 0;
fail:
  qtb_session_destroy(s);
  return rc;
}

extern "C" int qtb_session_batch(const qtb_session_t *s) { return s ? s->B : 0; }
extern "C" int qtb_tc_plan(int fmt, int rows, int cols, int batch, int grid, int cta, int out[6]) {
  if (!out || grid < 1 || cta < 0 || cta >= grid || cols < 1) return set_err(QTB_E_INVALID, "bad argument");
  if ((fmt != FMT_BF16 && fmt != FMT_INT8) || rows % 128 != 0 || batch < 1 || batch > 64 ||
      cols % tc_kchunk(fmt) != 0)
    return set_err(QTB_E_UNSUPPORTED, "not a tcgen05 GEMV shape");
  GemvArgs g;
  memset(&g, 0, sizeof g);
  g.fmt = fmt; g.rows = rows; g.K = cols;
  const V2Plan p = tc_plan(g, batch, cta, grid);
  out[0] = p.t0; out[1] = p.nt; out[2] = p.kb; out[3] = p.kc; out[4] = p.pair;
  out[5] = tc_choose(fmt, rows, cols, batch, grid).S;
  return 0;
}

extern "C" int qtb_session_program_grid(const qtb_session_t *s, int which) {
  if (!s || which < 0 || which >= PROG_N || !s->prog[which]) return 0;
  return s->prog_cl[which] ? -s->prog_G[which] : s->prog_G[which];
}
extern "C" int qtb_session_n_pages(const qtb_session_t *s) { return s ? s->tk.n_pages : 0; }
extern "C" double qtb_session_last_ms(const qtb_session_t *s) { return s ? s->last_ms : 0.0; }
extern "C" int qtb_session_last_launches(const qtb_session_t *s) { return s ? s->last_launches : 0; }

extern "C" int qtb_session_max_ctx(const qtb_session_t *s) { return s ? s->max_ctx : 0; }
extern "C" qtb_engine_t *qtb_session_engine(qtb_session_t *s) { return s ? s->e : nullptr; }
extern "C" int qtb_session_get_dec_x(qtb_session_t *s, float *out) {
  if (!s || !out || !s->e->has_talker) return set_err(QTB_E_INVALID, "bad argument");
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(out, s->tk.x, (size_t)s->B * s->e->talker.hidden * 4, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int qtb_session_set_pages(qtb_session_t *s, int b, const int32_t *pages, int n) {
  if (!s || !pages || b < 0 || b >= s->B) return set_err(QTB_E_INVALID, "bad slot");
  if (n < 0 || n > s->tk.pt_stride) return set_err(QTB_E_INVALID, "page count %d > %d", n, s->tk.pt_stride);
  for (int i = 0; i < n; i++)
    if (pages[i] < 0 || pages[i] >= s->tk.n_pages) return set_err(QTB_E_INVALID, "page id %d out of pool [0,%d)", pages[i], s->tk.n_pages);
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(s->tk.page_table + (size_t)b * s->tk.pt_stride, pages, (size_t)n * 4, cudaMemcpyHostToDevice));
  return 0;
}

extern "C" int qtb_session_set_pos(qtb_session_t *s, const int32_t *pos) {
  if (!s || !pos) return set_err(QTB_E_INVALID, "null argument");
  for (int b = 0; b < s->B; b++)
    if (pos[b] < 0 || pos[b] >= s->max_ctx) return set_err(QTB_E_INVALID, "position %d outside [0,%d)", pos[b], s->max_ctx);
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(s->pos, pos, (size_t)s->B * 4, cudaMemcpyHostToDevice));
  return 0;
}
extern "C" int qtb_session_get_pos(qtb_session_t *s, int32_t *pos) {
  if (!s || !pos) return set_err(QTB_E_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(pos, s->pos, (size_t)s->B * 4, cudaMemcpyDeviceToHost));
  return 0;
}

// Clear the device error flag at the start of every API call.
static int begin_call(qtb_session *s) {
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemsetAsync(s->ctl, 0, sizeof(Ctl), s->stream));
  return 0;
}

// Launch program `which` n_iters times as ONE cooperative persistent kernel.
static int launch_prog(qtb_session *s, int which, int n_iters, bool timed) {
  if (!s->prog[which]) return set_err(QTB_E_UNSUPPORTED, "program %d not available for this engine", which);
  const int G = s->prog_G[which] ? s->prog_G[which] : s->e->n_sm;
  int cl = s->prog_cl[which];
  if ((long long)n_iters * s->prog_n[which] * G > 0x3fffffffLL)
    return set_err(QTB_E_INVALID, "too many iterations for one launch");
  CUDA_TRY(cudaMemsetAsync(&s->ctl->bar_count, 0, sizeof(unsigned), s->stream));
  CUDA_TRY(cudaMemsetAsync(&s->ctl->att_work, 0, 2 * sizeof(unsigned), s->stream));   // att_work, ibar
  if (s->tc_sem_n[which] > 0)
    CUDA_TRY(cudaMemsetAsync(s->tc_sem[which], 0, (size_t)s->tc_sem_n[which] * sizeof(unsigned), s->stream));
  const Stage *prog = s->prog[which];
  const V2Plan *plan = s->plan[which];
  int n_st = s->prog_n[which];
  Ctl *ctl = s->ctl;
  long long *trace = s->trace_on ? s->trace : nullptr;
  void *args[] = {(void *)&prog, (void *)&plan, (void *)&n_st, (void *)&n_iters, (void *)&ctl, (void *)&trace,
                  (void *)&cl};
  if (timed) CUDA_TRY(cudaEventRecord(s->ev0, s->stream));
  if (cl) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    cl_launch_config(cfg, at, s->stream);
    CUDA_TRY(cudaLaunchKernelExC(&cfg, (const void *)decode_kernel, args));
  } else if (s->e->pairs) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    cluster_launch_config(cfg, at, s->e->n_sm, s->stream);
    CUDA_TRY(cudaLaunchKernelExC(&cfg, (const void *)decode_kernel, args));
  } else {
    CUDA_TRY(cudaLaunchCooperativeKernel((const void *)decode_kernel, dim3(s->e->n_sm), dim3(NTHREADS), args,
                                         SMEM_BYTES, s->stream));
  }
  if (timed) CUDA_TRY(cudaEventRecord(s->ev1, s->stream));
  s->last_launches = 1;
  return 0;
}

static int finish(qtb_session *s, bool timed) {
  CUDA_TRY(cudaStreamSynchronize(s->stream));
  if (timed) {
    float ms = 0;
    cudaEventElapsedTime(&ms, s->ev0, s->ev1);
    s->last_ms = ms;
  }
  Ctl h;
  CUDA_TRY(cudaMemcpy(&h, s->ctl, sizeof(Ctl), cudaMemcpyDeviceToHost));
  if (h.err)
    return set_err(QTB_E_DEVICE, "decode kernel error %d at stage %d (info %d)", h.err, h.err_stage, h.err_info);
  return 0;
}

extern "C" int qtb_talker_step(qtb_session_t *s, const float *embeds, const int32_t *pos, float *hidden_out,
                               float *dec_x_out) {
  if (!s || !embeds) return set_err(QTB_E_INVALID, "null argument");
  if (!s->e->has_talker) return set_err(QTB_E_UNSUPPORTED, "engine has no talker");
  const int B = s->B, H = s->e->talker.hidden;
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  if (pos) {
    for (int b = 0; b < B; b++)
      if (pos[b] < 0 || pos[b] >= s->max_ctx) return set_err(QTB_E_INVALID, "position %d outside [0,%d)", pos[b], s->max_ctx);
    memcpy(s->h_pos, pos, (size_t)B * 4);
    CUDA_TRY(cudaMemcpyAsync(s->pos, s->h_pos, (size_t)B * 4, cudaMemcpyHostToDevice, s->stream));
  }
  memcpy(s->h_in, embeds, (size_t)B * H * 4);
  CUDA_TRY(cudaMemcpyAsync(s->tk.x, s->h_in, (size_t)B * H * 4, cudaMemcpyHostToDevice, s->stream));
  int rc = launch_prog(s, PROG_TALKER, 1, true);
  if (rc) return rc;
  if (hidden_out) CUDA_TRY(cudaMemcpyAsync(hidden_out, s->tk.hidden, (size_t)B * H * 4, cudaMemcpyDeviceToHost, s->stream));
  if (dec_x_out) CUDA_TRY(cudaMemcpyAsync(dec_x_out, s->tk.x, (size_t)B * H * 4, cudaMemcpyDeviceToHost, s->stream));
  return finish(s, true);
}

extern "C" int qtb_cp_pass(qtb_session_t *s, float *x, const int32_t *pos) {
  if (!s || !x || !pos) return set_err(QTB_E_INVALID, "null argument");
  if (!s->e->has_cp) return set_err(QTB_E_UNSUPPORTED, "engine has no code predictor");
  const int B = s->B, CH = s->e->cp.hidden;
  for (int b = 0; b < B; b++)
    if (pos[b] < 0 || pos[b] >= 64 || pos[b] >= s->e->cp.rope_len) return set_err(QTB_E_INVALID, "CP position %d outside [0,64)", pos[b]);
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  memcpy(s->h_pos, pos, (size_t)B * 4);
  CUDA_TRY(cudaMemcpyAsync(s->cp_pos, s->h_pos, (size_t)B * 4, cudaMemcpyHostToDevice, s->stream));
  memcpy(s->h_in, x, (size_t)B * CH * 4);
  CUDA_TRY(cudaMemcpyAsync(s->cp.x, s->h_in, (size_t)B * CH * 4, cudaMemcpyHostToDevice, s->stream));
  int rc = launch_prog(s, PROG_CP_PASS, 1, true);
  if (rc) return rc;
  CUDA_TRY(cudaMemcpyAsync(s->h_out, s->cp.x, (size_t)B * CH * 4, cudaMemcpyDeviceToHost, s->stream));
  rc = finish(s, true);
  if (rc) return rc;
  memcpy(x, s->h_out, (size_t)B * CH * 4);
  return 0;
}

extern "C" int qtb_cp_frame(qtb_session_t *s, const float *talker_hidden, const int32_t *code0, int32_t *codes_out) {
  if (!s || !talker_hidden || !code0 || !codes_out) return set_err(QTB_E_INVALID, "null argument");
  qtb_engine *e = s->e;
  if (!e->has_cp || !s->prog[PROG_CP_FRAME]) return set_err(QTB_E_UNSUPPORTED, "engine has no code predictor");
  if (!e->codec_emb) return set_err(QTB_E_UNSUPPORTED, "engine has no talker codec embedding (needed for code0)");
  const int B = s->B;
  const int TH = e->has_talker ? e->talker.hidden : e->cp_emb_dim;
  for (int b = 0; b < B; b++)
    if (code0[b] < 0 || code0[b] >= e->codec_vocab) return set_err(QTB_E_INVALID, "code0 %d outside the codec vocabulary", code0[b]);
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  memcpy(s->h_in, talker_hidden, (size_t)B * TH * 4);
  CUDA_TRY(cudaMemcpyAsync(s->cp_in, s->h_in, (size_t)B * TH * 4, cudaMemcpyHostToDevice, s->stream));
  for (int b = 0; b < B; b++) s->h_codes[b * 16] = code0[b];
  CUDA_TRY(cudaMemcpy2DAsync(s->codes, 16 * 4, s->h_codes, 16 * 4, 4, B, cudaMemcpyHostToDevice, s->stream));
  int rc = launch_prog(s, PROG_CP_FRAME, 1, true);
  if (rc) return rc;
  CUDA_TRY(cudaMemcpyAsync(s->h_codes, s->codes, (size_t)B * 16 * 4, cudaMemcpyDeviceToHost, s->stream));
  rc = finish(s, true);
  if (rc) return rc;
  for (int b = 0; b < B; b++) memcpy(codes_out + (size_t)b * 15, s->h_codes + (size_t)b * 16 + 1, 15 * 4);
  return 0;
}

extern "C" int qtb_prefill(qtb_session_t *s, int b, const float *embeds, int n, int pos0, float *hidden_out,
                           float *dec_x_out) {
  if (!s || !embeds || n < 1) return set_err(QTB_E_INVALID, "bad argument");
  if (!s->prog[PROG_PREFILL]) return set_err(QTB_E_UNSUPPORTED, "engine has no talker");
  if (b < 0 || b >= s->B) return set_err(QTB_E_INVALID, "bad slot %d", b);
  if (pos0 < 0 || pos0 + n > s->max_ctx) return set_err(QTB_E_INVALID, "positions [%d,%d) outside [0,%d)", pos0, pos0 + n, s->max_ctx);
  const int H = s->e->talker.hidden, R = PREFILL_CHUNK, pts = s->tk.pt_stride;
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  // every chunk row reads and appends through slot b's page table
  std::vector<int32_t> row(pts);
  CUDA_TRY(cudaMemcpy(row.data(), s->tk.page_table + (size_t)b * pts, (size_t)pts * 4, cudaMemcpyDeviceToHost));
  for (int i = 0; i <= (pos0 + n - 1) / PAGE; i++)
    if (row[i] < 0 || row[i] >= s->tk.n_pages) return set_err(QTB_E_INVALID, "slot %d has no page for position %d", b, 16 * i);
  std::vector<int32_t> pt((size_t)R * pts);
  for (int r = 0; r < R; r++) memcpy(pt.data() + (size_t)r * pts, row.data(), (size_t)pts * 4);
  CUDA_TRY(cudaMemcpyAsync(s->pf.page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice, s->stream));
  // the prompt's f32 K/V, positions pos0 .. pos0 + n - 1 of every layer
  const DStack &tk = s->e->talker;
  if (s->pkv_h.cap < n) {
    CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (s->pkv_h.k) cudaFree(s->pkv_h.k);
    if (s->pkv_h.v) cudaFree(s->pkv_h.v);
    s->pkv_h = PromptKV{nullptr, nullptr, 0, 0};
    const int cap = (n + R - 1) / R * R;
    const size_t bytes = (size_t)tk.n_layers * tk.n_kv * cap * HD * sizeof(float);
    CUDA_TRY(cudaMalloc((void **)&s->pkv_h.k, bytes));
    CUDA_TRY(cudaMalloc((void **)&s->pkv_h.v, bytes));
    s->pkv_h.cap = cap;
  }
  s->pkv_h.p0 = pos0;
  CUDA_TRY(cudaMemcpyAsync(s->pkv, &s->pkv_h, sizeof(PromptKV), cudaMemcpyHostToDevice, s->stream));
  std::vector<float> x((size_t)R * H);
  std::vector<int32_t> pos(R);
  int rc = 0;
  CUDA_TRY(cudaEventRecord(s->ev0, s->stream));
  for (int c0 = 0; c0 < n; c0 += R) {
    const int m = std::min(R, n - c0);
    // rows past the chunk's last token repeat it (same position, same K/V bytes)
    for (int r = 0; r < R; r++) {
      const int t = c0 + std::min(r, m - 1);
      memcpy(x.data() + (size_t)r * H, embeds + (size_t)t * H, (size_t)H * 4);
      pos[r] = pos0 + t;
    }
    CUDA_TRY(cudaMemcpyAsync(s->pf.x, x.data(), x.size() * 4, cudaMemcpyHostToDevice, s->stream));
    CUDA_TRY(cudaMemcpyAsync(s->pf_pos, pos.data(), (size_t)R * 4, cudaMemcpyHostToDevice, s->stream));
    if ((rc = launch_prog(s, PROG_PREFILL, 1, false))) return rc;
    // the copies above reuse host buffers: wait before the next chunk refills them
    CUDA_TRY(cudaStreamSynchronize(s->stream));
    if (c0 + m == n) {
      if (hidden_out)
        CUDA_TRY(cudaMemcpy(hidden_out, s->pf.hidden + (size_t)(m - 1) * H, (size_t)H * 4, cudaMemcpyDeviceToHost));
      if (dec_x_out)
        CUDA_TRY(cudaMemcpy(dec_x_out, s->pf.x + (size_t)(m - 1) * H, (size_t)H * 4, cudaMemcpyDeviceToHost));
    }
  }
  CUDA_TRY(cudaEventRecord(s->ev1, s->stream));
  s->last_launches = (n + R - 1) / R;
  const int32_t np = pos0 + n;
  CUDA_TRY(cudaMemcpy(s->pos + b, &np, 4, cudaMemcpyHostToDevice));
  return finish(s, true);
}

extern "C" int qtb_session_begin_generation(qtb_session_t *s, const int32_t *expected_frames, float rep_penalty) {
  if (!s) return set_err(QTB_E_INVALID, "null session");
  if (!s->e->has_eos) return set_err(QTB_E_UNSUPPORTED, "the codec vocabulary has no EOS token (%d)", QTB_CODEC_EOS);
  if (!(rep_penalty > 0.0f)) return set_err(QTB_E_INVALID, "repetition penalty %g", (double)rep_penalty);
  const int B = s->B;
  std::vector<int32_t> bs(B, -1);
  for (int b = 0; b < B && expected_frames; b++) bs[b] = expected_frames[b] > 0 ? 2 * expected_frames[b] : -1;
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(s->gen_h.boost_start, bs.data(), (size_t)B * 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(s->gen_h.frame, 0, (size_t)B * 4));
  CUDA_TRY(cudaMemset(s->gen_h.done, 0, (size_t)B * 4));
  CUDA_TRY(cudaMemset(s->gen_h.rep_count, 0, (size_t)B * s->gen_h.vocab * 2));
  { int rc = reset_sampling(s->gen_h, 0, B); if (rc) return rc; }
  s->gen_h.sampling = 0;
  GenState g = s->gen_h;
  g.enabled = 1;
  g.rep_pen = rep_penalty;
  g.rep_inv = 1.0f / rep_penalty;   // the reference's build multiplies by this reciprocal
  CUDA_TRY(cudaMemcpy(s->gen, &g, sizeof g, cudaMemcpyHostToDevice));
  s->gen_on = 1;
  return 0;
}

extern "C" int qtb_session_reset_slot(qtb_session_t *s, int b, int32_t expected_frames, int active) {
  if (!s || b < 0 || b >= s->B) return set_err(QTB_E_INVALID, "bad slot");
  if (!s->gen_on) return set_err(QTB_E_INVALID, "qtb_session_begin_generation first");
  CUDA_TRY(cudaSetDevice(s->e->device));
  const int32_t z = 0, d = active ? 0 : 2, bs = expected_frames > 0 ? 2 * expected_frames : -1;
  CUDA_TRY(cudaMemcpy(s->gen_h.frame + b, &z, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(s->gen_h.done + b, &d, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(s->gen_h.boost_start + b, &bs, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(s->gen_h.rep_count + (size_t)b * s->gen_h.vocab, 0, (size_t)s->gen_h.vocab * 2));
  return reset_sampling(s->gen_h, b, b + 1);
}

extern "C" int qtb_session_set_sampling(qtb_session_t *s, int b, float temperature, int32_t top_k, float top_p,
                                        uint32_t seed) {
  if (!s || b < 0 || b >= s->B) return set_err(QTB_E_INVALID, "bad slot");
  if (!s->gen_on) return set_err(QTB_E_INVALID, "qtb_session_begin_generation first");
  if (!(temperature >= 0.0f) || !(top_p > 0.0f))
    return set_err(QTB_E_INVALID, "temperature %g, top-p %g", (double)temperature, (double)top_p);
  CUDA_TRY(cudaSetDevice(s->e->device));
  const GenState &g = s->gen_h;
  CUDA_TRY(cudaMemcpy(g.temp + b, &temperature, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.top_k + b, &top_k, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.top_p + b, &top_p, 4, cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(g.rng + b, &seed, 4, cudaMemcpyHostToDevice));
  if (temperature >= 1e-6f && !s->gen_h.sampling) {   // the codec head keeps its logits from now on
    s->gen_h.sampling = 1;
    const int one = 1;
    CUDA_TRY(cudaMemcpy(reinterpret_cast<char *>(s->gen) + offsetof(GenState, sampling), &one, sizeof one,
                        cudaMemcpyHostToDevice));
  }
  return 0;
}

extern "C" int qtb_session_get_rng(qtb_session_t *s, uint32_t *state) {
  if (!s || !state) return set_err(QTB_E_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(state, s->gen_h.rng, (size_t)s->B * 4, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int qtb_session_set_slot_pos(qtb_session_t *s, int b, int32_t pos) {
  if (!s || b < 0 || b >= s->B) return set_err(QTB_E_INVALID, "bad slot");
  if (pos < 0 || pos >= s->max_ctx) return set_err(QTB_E_INVALID, "position %d outside [0,%d)", pos, s->max_ctx);
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(s->pos + b, &pos, 4, cudaMemcpyHostToDevice));
  return 0;
}

extern "C" int qtb_session_set_embed(qtb_session_t *s, int b, const float *embed) {
  if (!s || !embed || b < 0 || b >= s->B || !s->e->has_talker) return set_err(QTB_E_INVALID, "bad argument");
  CUDA_TRY(cudaSetDevice(s->e->device));
  const int H = s->e->talker.hidden;
  CUDA_TRY(cudaMemcpy(s->tk.x + (size_t)b * H, embed, (size_t)H * 4, cudaMemcpyHostToDevice));
  return 0;
}

extern "C" int qtb_session_get_done(qtb_session_t *s, int32_t *done) {
  if (!s || !done) return set_err(QTB_E_INVALID, "null argument");
  CUDA_TRY(cudaSetDevice(s->e->device));
  CUDA_TRY(cudaMemcpy(done, s->gen_h.done, (size_t)s->B * 4, cudaMemcpyDeviceToHost));
  for (int b = 0; b < s->B; b++) done[b] = done[b] != 0;   // 1: EOS in the last frame, 2: stopped before
  return 0;
}

extern "C" int qtb_decode_frames(qtb_session_t *s, const float *embeds, const float *pad, int n_frames,
                                 int32_t *codes_out, float *last_hidden_out) {
  if (!s || n_frames < 1) return set_err(QTB_E_INVALID, "bad argument");
  qtb_engine *e = s->e;
  if (!s->prog[PROG_FRAME]) return set_err(QTB_E_UNSUPPORTED, "engine lacks codec head / embeddings for whole frames");
  const int B = s->B, H = e->talker.hidden;
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  int32_t hp[64];
  CUDA_TRY(cudaMemcpy(hp, s->pos, (size_t)B * 4, cudaMemcpyDeviceToHost));
  for (int b = 0; b < B; b++)
    if (hp[b] + n_frames > s->max_ctx) return set_err(QTB_E_INVALID, "slot %d would pass max_ctx %d", b, s->max_ctx);
  if (embeds) {
    memcpy(s->h_in, embeds, (size_t)B * H * 4);
    CUDA_TRY(cudaMemcpyAsync(s->tk.x, s->h_in, (size_t)B * H * 4, cudaMemcpyHostToDevice, s->stream));
  }
  if (pad) CUDA_TRY(cudaMemcpyAsync(s->pad, pad, (size_t)H * 4, cudaMemcpyHostToDevice, s->stream));
  int rc = 0;
  if (codes_out) {
    // one launch per frame so every frame's codes can be read back
    std::vector<int32_t> done((size_t)(n_frames + 1) * B, 0);
    if (s->gen_on) CUDA_TRY(cudaMemcpyAsync(done.data(), s->gen_h.done, (size_t)B * 4, cudaMemcpyDeviceToHost, s->stream));
    CUDA_TRY(cudaEventRecord(s->ev0, s->stream));
    for (int f = 0; f < n_frames; f++) {
      if ((rc = launch_prog(s, PROG_FRAME, 1, false))) return rc;
      CUDA_TRY(cudaMemcpyAsync(codes_out + (size_t)f * B * 16, s->codes, (size_t)B * 16 * 4, cudaMemcpyDeviceToHost, s->stream));
      if (s->gen_on)
        CUDA_TRY(cudaMemcpyAsync(done.data() + (size_t)(f + 1) * B, s->gen_h.done, (size_t)B * 4, cudaMemcpyDeviceToHost,
                                 s->stream));
    }
    CUDA_TRY(cudaEventRecord(s->ev1, s->stream));
    s->last_launches = n_frames;
    if (s->gen_on) {
      // a slot that sampled EOS reports it as its code0 of that frame, with no
      // code-predictor codes (the reference stops before them), and -1 after
      CUDA_TRY(cudaStreamSynchronize(s->stream));
      for (int f = 0; f < n_frames; f++)
        for (int b = 0; b < B; b++) {
          int32_t *c = codes_out + ((size_t)f * B + b) * 16;
          if (done[(size_t)f * B + b]) {
            for (int g = 0; g < 16; g++) c[g] = -1;
          } else if (done[(size_t)(f + 1) * B + b]) {
            c[0] = QTB_CODEC_EOS;
            for (int g = 1; g < 16; g++) c[g] = -1;
          }
        }
    }
  } else {
    if ((rc = launch_prog(s, PROG_FRAME, n_frames, true))) return rc;
  }
  if (last_hidden_out)
    CUDA_TRY(cudaMemcpyAsync(last_hidden_out, s->tk.hidden, (size_t)B * H * 4, cudaMemcpyDeviceToHost, s->stream));
  return finish(s, true);
}

// ------------------------------------------------ KV scatter / gather ------
__global__ void kv_copy_kernel(uint16_t *pool, const int *pt, int pt_stride, int n_kv, size_t layer_elems,
                               uint16_t *host_layout, int layer_stride, int len, int n_layers, int to_pool) {
  const int kvd = n_kv * HD;
  const size_t total = (size_t)n_layers * len * kvd;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % kvd);
    const size_t lp = i / kvd;
    const int p = (int)(lp % len), l = (int)(lp / len);
    const int page = pt[p / PAGE];
    const int g = c / HD, d = c % HD;
    uint16_t *pp = pool + (size_t)l * layer_elems + (((size_t)page * n_kv + g) * PAGE + p % PAGE) * HD + d;
    uint16_t *hp = host_layout + ((size_t)l * layer_stride + p) * kvd + c;
    if (to_pool) *pp = *hp; else *hp = *pp;
  }
}

static int kv_transfer(qtb_session *s, StackBufs &b, const DStack &k, size_t layer_elems, int slot, uint16_t *kh,
                       uint16_t *vh, int layer_stride, int len, int to_pool) {
  if (slot < 0 || slot >= s->B || !kh || !vh) return set_err(QTB_E_INVALID, "bad slot/pointer");
  if (len < 0 || len > b.pt_stride * PAGE || len > layer_stride) return set_err(QTB_E_INVALID, "length %d out of range", len);
  if (len == 0) return 0;
  CUDA_TRY(cudaSetDevice(s->e->device));
  std::vector<int> pt(b.pt_stride);
  CUDA_TRY(cudaMemcpy(pt.data(), b.page_table + (size_t)slot * b.pt_stride, pt.size() * 4, cudaMemcpyDeviceToHost));
  for (int i = 0; i < (len + PAGE - 1) / PAGE; i++)
    if (pt[i] < 0 || pt[i] >= b.n_pages) return set_err(QTB_E_INVALID, "slot %d has no page for positions %d..", slot, i * PAGE);
  const size_t n = (size_t)k.n_layers * layer_stride * k.kv_dim();
  uint16_t *dh = nullptr;
  CUDA_TRY(cudaMalloc(&dh, n * 2));
  int rc = 0;
  const int *dpt = b.page_table + (size_t)slot * b.pt_stride;
  for (int kvsel = 0; kvsel < 2 && !rc; kvsel++) {
    uint16_t *host = kvsel ? vh : kh;
    uint16_t *pool = kvsel ? b.vpool : b.kpool;
    if (to_pool && cudaMemcpy(dh, host, n * 2, cudaMemcpyHostToDevice) != cudaSuccess) { rc = set_err(QTB_E_CUDA, "kv upload"); break; }
    kv_copy_kernel<<<512, 256, 0, s->stream>>>(pool, dpt, b.pt_stride, k.n_kv, layer_elems, dh, layer_stride, len,
                                                k.n_layers, to_pool);
    if (cudaStreamSynchronize(s->stream) != cudaSuccess) { rc = set_err(QTB_E_CUDA, "kv copy kernel: %s", cudaGetErrorString(cudaGetLastError())); break; }
    if (!to_pool && cudaMemcpy(host, dh, n * 2, cudaMemcpyDeviceToHost) != cudaSuccess) { rc = set_err(QTB_E_CUDA, "kv download"); break; }
  }
  cudaFree(dh);
  return rc;
}

extern "C" int qtb_session_upload_kv(qtb_session_t *s, int b, const uint16_t *k, const uint16_t *v, int layer_stride, int len) {
  if (!s || !s->e->has_talker) return set_err(QTB_E_INVALID, "no talker");
  return kv_transfer(s, s->tk, s->e->talker, s->tk_layer_elems, b, (uint16_t *)k, (uint16_t *)v, layer_stride, len, 1);
}
extern "C" int qtb_session_download_kv(qtb_session_t *s, int b, uint16_t *k, uint16_t *v, int layer_stride, int len) {
  if (!s || !s->e->has_talker) return set_err(QTB_E_INVALID, "no talker");
  return kv_transfer(s, s->tk, s->e->talker, s->tk_layer_elems, b, k, v, layer_stride, len, 0);
}
extern "C" int qtb_session_download_cp_kv(qtb_session_t *s, int b, uint16_t *k, uint16_t *v, int layer_stride, int len) {
  if (!s || !s->e->has_cp) return set_err(QTB_E_INVALID, "no code predictor");
  return kv_transfer(s, s->cp, s->e->cp, s->cp_layer_elems, b, k, v, layer_stride, len, 0);
}

// ---------------------------------------------- standalone kernel entries --
struct MiniRun {
  Arena ar;
  cudaStream_t st = nullptr;
  ~MiniRun() {
    if (st) cudaStreamDestroy(st);
    ar.release();
  }
};

extern "C" int qtb_codec_sample_host(const float *logits, int batch, int n, const float *temperature,
                                     const int32_t *top_k, const float *top_p, uint32_t *rng, int32_t *out) {
  if (!logits || !temperature || !top_k || !top_p || !rng || !out) return set_err(QTB_E_INVALID, "null argument");
  if (batch < 1 || batch > 64 || n < 1 || n > SAMPLE_MAX_ROWS) return set_err(QTB_E_INVALID, "batch %d, %d rows", batch, n);
  MiniRun mr;
  CUDA_TRY(cudaStreamCreateWithFlags(&mr.st, cudaStreamDefault));
  GenState g = {};
  g.eos_row = n - 1;
  g.ld = n;
  int rc;
  int32_t *dout;
  GenState *dg;
  if ((rc = mr.ar.upload(&g.logits, logits, (size_t)batch * n * 4))) return rc;
  if ((rc = mr.ar.upload(&g.temp, temperature, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.upload(&g.top_k, top_k, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.upload(&g.top_p, top_p, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.upload(&g.rng, rng, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&dout, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.upload(&dg, &g, sizeof g))) return rc;
  sample_kernel<<<batch, 32, 0, mr.st>>>(dg, dout);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaStreamSynchronize(mr.st));
  CUDA_TRY(cudaMemcpy(out, dout, (size_t)batch * 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(rng, g.rng, (size_t)batch * 4, cudaMemcpyDeviceToHost));
  return 0;
}

static int run_single_stage(MiniRun &mr, const Stage &S) {
  int rc;
  Stage *dp;
  Ctl *ctl;
  if ((rc = mr.ar.upload(&dp, &S, sizeof S))) return rc;
  if ((rc = mr.ar.alloc((void **)&ctl, sizeof(Ctl)))) return rc;
  CUDA_TRY(cudaMemset(ctl, 0, sizeof(Ctl)));
  int dev = 0, nsm = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  CUDA_TRY(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  std::vector<V2Plan> pl;
  make_plans(std::vector<Stage>{S}, nsm, false, pl);
  V2Plan *dplan;
  if ((rc = mr.ar.upload(&dplan, pl.data(), pl.size() * sizeof(V2Plan)))) return rc;
  const Stage *prog = dp;
  const V2Plan *plan = dplan;
  int n_st = 1, n_it = 1;
  long long *trace = nullptr;
  int cl0 = 0;
  void *args[] = {(void *)&prog, (void *)&plan, (void *)&n_st, (void *)&n_it, (void *)&ctl, (void *)&trace, (void *)&cl0};
  CUDA_TRY(cudaLaunchCooperativeKernel((const void *)decode_kernel, dim3(nsm), dim3(NTHREADS), args, SMEM_BYTES, mr.st));
  CUDA_TRY(cudaStreamSynchronize(mr.st));
  Ctl h;
  CUDA_TRY(cudaMemcpy(&h, ctl, sizeof h, cudaMemcpyDeviceToHost));
  if (h.err) return set_err(QTB_E_DEVICE, "kernel error %d (info %d)", h.err, h.err_info);
  return 0;
}

extern "C" int qtb_gemv_host(int fmt, const qtb_matrix_t *w, int rows, int cols, const float *x, int batch, float *y) {
  if (!w || !x || !y || batch < 1 || batch > 64) return set_err(QTB_E_INVALID, "bad argument");
  MiniRun mr;
  CUDA_TRY(cudaStreamCreateWithFlags(&mr.st, cudaStreamDefault));   // behind the legacy-stream uploads
  int dev = 0, nsm = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  DMat m;
  const qtb_matrix_t *ms[1] = {w};
  const int re[1] = {rows};
  int rc = upload_matrix(mr.ar, fmt, ms, re, 1, cols, m);
  if (rc) return rc;
  float *dx, *dy, *ws, *xsc;
  uint8_t *xop;
  unsigned *sem;
  const int T = rows / 16;
  const bool v2 = v2_ok(fmt, rows, cols, batch, nsm);
  const bool tc = !v2 && tc_ok(m, batch, fmt);
  const int S = v2 ? std::max(1, nsm / T)
                   : tc ? tc_choose(fmt, rows, cols, batch, nsm).S : choose_S(T, cols, batch, nsm * NWARPS, fmt);
  if (S < 1) return set_err(QTB_E_UNSUPPORTED, "no k-slicing fits");
  const size_t ws_floats = tc ? std::max<size_t>(16, tc_ws_floats(fmt, rows, cols, batch, nsm)) : (size_t)T * S * 16 * batch;
  if ((rc = mr.ar.upload(&dx, x, (size_t)batch * cols * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&dy, (size_t)batch * rows * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&ws, ws_floats * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&xsc, 128 * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&xop, tc ? tc_xop_bytes(fmt, cols) : 16))) return rc;
  if ((rc = mr.ar.alloc((void **)&sem, (size_t)T * 4))) return rc;
  CUDA_TRY(cudaMemset(sem, 0, (size_t)T * 4));
  Stage st;
  memset(&st, 0, sizeof st);
  st.kind = ST_GEMV;
  st.B = batch;
  GemvArgs &g = st.g;
  g.w = m.w; g.row_scale = m.row_scale; g.gsz = m.gsz;
  g.fmt = fmt; g.rows = rows; g.K = cols; g.S = v2 ? 1 : S; g.nch = nch_for(fmt, batch, v2); g.parts = parts_for(fmt, batch, v2);
  g.v2 = v2 ? 1 : 0;
  g.tc = tc ? 1 : 0;
  g.wtc = m.wtc;
  g.xsc = xsc; g.xop = xop;
  g.x = dx; g.ldx = cols; g.y = dy; g.ldy = rows; g.epi = EPI_STORE; g.ws = ws; g.sem = sem;
  if ((rc = run_single_stage(mr, st))) return rc;
  CUDA_TRY(cudaMemcpy(y, dy, (size_t)batch * rows * 4, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int qtb_attention_host(const float *qkv, int batch, int n_heads, int n_kv, int head_dim, const float *q_norm,
                                  const float *k_norm, float eps, const float *rope_cos, const float *rope_sin, int rope_len,
                                  uint16_t *kpages, uint16_t *vpages, int n_pages, const int32_t *page_table, int pt_stride,
                                  const int32_t *pos, int max_splits, float *out) {
  if (!qkv || !q_norm || !k_norm || !rope_cos || !rope_sin || !kpages || !vpages || !page_table || !pos || !out)
    return set_err(QTB_E_INVALID, "null argument");
  if (head_dim != HD || n_heads != 2 * n_kv || batch < 1 || batch > 64 || max_splits < 1 || max_splits > 64)
    return set_err(QTB_E_UNSUPPORTED, "shape not supported");
  for (int b = 0; b < batch; b++) {
    if (pos[b] < 0 || pos[b] >= rope_len || pos[b] >= pt_stride * PAGE) return set_err(QTB_E_INVALID, "position out of range");
    for (int i = 0; i <= pos[b] / PAGE; i++) {
      const int p = page_table[(size_t)b * pt_stride + i];
      if (p < 0 || p >= n_pages) return set_err(QTB_E_INVALID, "page table entry %d out of pool", p);
    }
  }
  MiniRun mr;
  CUDA_TRY(cudaStreamCreateWithFlags(&mr.st, cudaStreamDefault));   // behind the legacy-stream uploads
  const int qd = n_heads * HD, kvd = n_kv * HD, qkvd = qd + 2 * kvd;
  const size_t pool = (size_t)n_pages * n_kv * PAGE * HD;
  int rc;
  float *dqkv, *dqn, *dkn, *dcos, *dsin, *dout, *ws;
  uint16_t *dk, *dv;
  int *dpt, *dpos;
  unsigned *sem;
  if ((rc = mr.ar.upload(&dqkv, qkv, (size_t)batch * qkvd * 4))) return rc;
  if ((rc = mr.ar.upload(&dqn, q_norm, HD * 4))) return rc;
  if ((rc = mr.ar.upload(&dkn, k_norm, HD * 4))) return rc;
  if ((rc = mr.ar.upload(&dcos, rope_cos, (size_t)rope_len * (HD / 2) * 4))) return rc;
  if ((rc = mr.ar.upload(&dsin, rope_sin, (size_t)rope_len * (HD / 2) * 4))) return rc;
  if ((rc = mr.ar.upload(&dk, kpages, pool * 2))) return rc;
  if ((rc = mr.ar.upload(&dv, vpages, pool * 2))) return rc;
  if ((rc = mr.ar.upload(&dpt, page_table, (size_t)batch * pt_stride * 4))) return rc;
  if ((rc = mr.ar.upload(&dpos, pos, (size_t)batch * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&dout, (size_t)batch * qd * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&ws, (size_t)batch * n_kv * max_splits * 2 * (HD + 2) * 4))) return rc;
  if ((rc = mr.ar.alloc((void **)&sem, (size_t)batch * n_kv * 4))) return rc;
  CUDA_TRY(cudaMemset(sem, 0, (size_t)batch * n_kv * 4));
  Stage st;
  memset(&st, 0, sizeof st);
  st.kind = ST_ATTN;
  st.B = batch;
  AttnArgs &a = st.a;
  a.qkv = dqkv; a.ld_qkv = qkvd; a.out = dout; a.ld_out = qd;
  a.q_norm = dqn; a.k_norm = dkn; a.rope_cos = dcos; a.rope_sin = dsin; a.rope_len = rope_len;
  a.pos_ptr = dpos; a.page_table = dpt; a.pt_stride = pt_stride;
  a.kpool = dk; a.vpool = dv; a.n_pages = n_pages; a.n_heads = n_heads; a.n_kv = n_kv;
  a.eps = eps; a.scale = 1.0f / sqrtf((float)HD); a.max_splits = max_splits; a.min_pps = 1;
  a.ws = ws; a.sem = sem;
  if ((rc = qk_rsq_table(&a.rsq_tab))) return rc;
  {
    int dev = 0, nsm = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    attn_schedule(a, batch, nsm);
  }
  if (batch >= 8 && attn_tc_enabled()) {   // the tensor-core page loop, as large-batch sessions run it
    CUtensorMap maps[2];
    if (kv_tensor_map(&maps[0], dk, 1, pool) && kv_tensor_map(&maps[1], dv, 1, pool)) {
      char *d;
      if ((rc = mr.ar.upload(&d, maps, sizeof maps))) return rc;
      a.kmap = d; a.vmap = d + sizeof(CUtensorMap); a.layer = 0; a.tc = 1;
    }
  }
  if ((rc = run_single_stage(mr, st))) return rc;
  CUDA_TRY(cudaMemcpy(out, dout, (size_t)batch * qd * 4, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(kpages, dk, pool * 2, cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemcpy(vpages, dv, pool * 2, cudaMemcpyDeviceToHost));
  return 0;
}

extern "C" int qtb_engine_talker_layers(const qtb_engine_t *e) { return e ? e->talker.n_layers : 0; }
extern "C" int qtb_engine_talker_kv_dim(const qtb_engine_t *e) { return e ? e->talker.kv_dim() : 0; }

// Stage-level profile of one iteration of a program (0 talker step, 1 CP pass,
// 2 CP frame, 3 whole frame): per-stage SM clock cycles between grid barriers
// (CTA 0's clock) and each stage's kind (1 GEMV, 2 ATTN, 3 EMBED, 4 NORM,
// 5 POS_INC) and, for GEMV stages, rows * 65536 + K in `shape`.
extern "C" int qtb_session_profile(qtb_session_t *s, int which, long long *cycles, int *kind, int64_t *shape, int max_stages) {
  if (!s || which < 0 || which >= PROG_N || !s->prog[which]) return set_err(QTB_E_INVALID, "bad program");
  const int n = s->prog_n[which];
  if (n > max_stages) return set_err(QTB_E_INVALID, "need %d stage slots", n);
  CUDA_TRY(cudaSetDevice(s->e->device));
  const int need = (n + 1) + n * NCKPT + 2 * n * s->e->n_sm;
  if (!s->trace || s->trace_n < need) {
    if (s->trace) cudaFree(s->trace);
    s->trace = nullptr;
    CUDA_TRY(cudaMalloc(&s->trace, (size_t)need * 8));
    s->trace_n = need;
  }
  CUDA_TRY(cudaMemset(s->trace, 0, (size_t)need * 8));
  { int rc0 = begin_call(s); if (rc0) return rc0; }
  if (const char *tc = getenv("QTB_TRACE_CTA")) {   // checkpoints of another CTA than 0
    const int cta = atoi(tc);
    CUDA_TRY(cudaMemcpyAsync(&s->ctl->trace_cta, &cta, sizeof cta, cudaMemcpyHostToDevice, s->stream));
  }
  s->trace_on = 1;
  int rc = launch_prog(s, which, 1, true);
  s->trace_on = 0;
  if (rc) return rc;
  if ((rc = finish(s, true))) return rc;
  std::vector<long long> t(need);
  CUDA_TRY(cudaMemcpy(t.data(), s->trace, (size_t)need * 8, cudaMemcpyDeviceToHost));
  s->last_ckpt.assign(t.begin() + n + 1, t.begin() + n + 1 + n * NCKPT);
  s->last_gtrace.assign(t.begin() + n + 1 + n * NCKPT, t.end());
  std::vector<Stage> st(n);
  CUDA_TRY(cudaMemcpy(st.data(), s->prog[which], (size_t)n * sizeof(Stage), cudaMemcpyDeviceToHost));
  long long prev = t[n];
  for (int i = 0; i < n; i++) {
    cycles[i] = t[i] - prev;
    prev = t[i];
    kind[i] = st[i].kind;
    shape[i] = st[i].kind == ST_GEMV ? (int64_t)st[i].g.rows * 65536 + st[i].g.K : 0;
  }
  return n;
}

// Intra-stage checkpoints (NCKPT per stage, clock64 of CTA 0 or of CTA $QTB_TRACE_CTA,
// 0 = not reached) of the
// last qtb_session_profile call.
extern "C" int qtb_session_profile_checkpoints(qtb_session_t *s, long long *out, int max_vals) {
  if (!s) return set_err(QTB_E_INVALID, "null session");
  const int n = std::min<int>((int)s->last_ckpt.size(), max_vals);
  for (int i = 0; i < n; i++) out[i] = s->last_ckpt[i];
  return n;
}

// Per-CTA barrier-arrival times (global timer, ns) of the last profile:
// [stage][cta].
extern "C" int qtb_session_profile_arrivals(qtb_session_t *s, long long *out, int max_vals) {
  if (!s) return set_err(QTB_E_INVALID, "null session");
  const int n = std::min<int>((int)s->last_gtrace.size(), max_vals);
  for (int i = 0; i < n; i++) out[i] = s->last_gtrace[i];
  return n;
}

// ------------------------------------------------------------------------
// qtb_attention_noalloc: the standalone attention stage of qtb_attention_host
// on caller-owned device buffers, with the launch's own scratch (stage
// descriptor, control block, split-combine workspace and semaphores) in one
// fixed file-scope device array instead of fresh allocations.  Limits:
// batch <= 4, n_kv <= 16, max_splits <= 16 (the workspace bound below).
// The array is shared by every call on a device: calls that overlap in time
// (two streams, two host threads) race on it.  The first call on a device
// looks the array up and sets the kernel attributes; make it before any
// stream capture.
namespace {
constexpr int NOALLOC_MAX_B = 4, NOALLOC_MAX_KV = 16, NOALLOC_MAX_SPLITS = 16;
constexpr size_t NOALLOC_DESC_OFF = 0;                                     // Stage
constexpr size_t NOALLOC_CTL_OFF = 1024;                                   // Ctl
constexpr size_t NOALLOC_SEM_OFF = NOALLOC_CTL_OFF + 1024;                 // unsigned [B][n_kv]
constexpr size_t NOALLOC_WS_OFF = NOALLOC_SEM_OFF + 1024;                  // float workspace
constexpr size_t NOALLOC_WS_BYTES =
    (size_t)NOALLOC_MAX_B * NOALLOC_MAX_KV * NOALLOC_MAX_SPLITS * 2 * (HD + 2) * sizeof(float);
constexpr size_t NOALLOC_BYTES = NOALLOC_WS_OFF + NOALLOC_WS_BYTES;        // 1,068,032 bytes (~1.04 MB)
static_assert(NOALLOC_BYTES == 1068032, "the documented size of the fixed scratch array");
static_assert(sizeof(Stage) <= 1024 && sizeof(Ctl) <= 1024, "scratch layout");
static_assert((size_t)NOALLOC_MAX_B * NOALLOC_MAX_KV * sizeof(unsigned) <= 1024, "scratch layout");
constexpr int NOALLOC_MAX_DEV = 64;
std::mutex g_noalloc_mu;
unsigned char *g_noalloc_addr[NOALLOC_MAX_DEV];   // per device, looked up once
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

extern "C" int qtb_attention_noalloc(const float *qkv, int batch, int n_heads, int n_kv, int head_dim,
                                     const float *q_norm, const float *k_norm, float eps, const float *rope_cos,
                                     const float *rope_sin, int rope_len, uint16_t *kpages, uint16_t *vpages,
                                     int n_pages, const int32_t *page_table, int pt_stride, const int32_t *pos,
                                     int max_splits, float *out, void *stream) {
  if (!qkv || !q_norm || !k_norm || !rope_cos || !rope_sin || !kpages || !vpages || !page_table || !pos || !out)
    return set_err(QTB_E_INVALID, "null argument");
  if (head_dim != HD || n_heads != 2 * n_kv || rope_len < 1 || n_pages < 1 || pt_stride < 1)
    return set_err(QTB_E_UNSUPPORTED, "shape not supported");
  if (batch < 1 || batch > NOALLOC_MAX_B || n_kv < 1 || n_kv > NOALLOC_MAX_KV || max_splits < 1 ||
      max_splits > NOALLOC_MAX_SPLITS)
    return set_err(QTB_E_INVALID, "beyond the fixed scratch: batch <= %d, n_kv <= %d, max_splits <= %d",
                   NOALLOC_MAX_B, NOALLOC_MAX_KV, NOALLOC_MAX_SPLITS);
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= NOALLOC_MAX_DEV) return set_err(QTB_E_UNSUPPORTED, "device index %d", dev);
  unsigned char *base;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {   // first call on this device (current): set-up
      void *p = nullptr;
      CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
      CUDA_TRY(cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
      g_noalloc_addr[dev] = static_cast<unsigned char *>(p);
    }
    base = g_noalloc_addr[dev];
  }
  int nsm = 0;
  CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Stage *dstage = reinterpret_cast<Stage *>(base + NOALLOC_DESC_OFF);
  Ctl *ctl = reinterpret_cast<Ctl *>(base + NOALLOC_CTL_OFF);
  unsigned *sem = reinterpret_cast<unsigned *>(base + NOALLOC_SEM_OFF);
  float *ws = reinterpret_cast<float *>(base + NOALLOC_WS_OFF);
  const int qd = n_heads * HD, kvd = n_kv * HD;
  Stage s;
  memset(&s, 0, sizeof s);
  s.kind = ST_ATTN;
  s.B = batch;
  AttnArgs &a = s.a;
  a.qkv = qkv; a.ld_qkv = qd + 2 * kvd; a.out = out; a.ld_out = qd;
  a.q_norm = q_norm; a.k_norm = k_norm; a.rope_cos = rope_cos; a.rope_sin = rope_sin; a.rope_len = rope_len;
  a.pos_ptr = pos; a.page_table = page_table; a.pt_stride = pt_stride;
  a.kpool = kpages; a.vpool = vpages; a.n_pages = n_pages; a.n_heads = n_heads; a.n_kv = n_kv;
  a.eps = eps; a.scale = 1.0f / sqrtf((float)HD); a.max_splits = max_splits; a.min_pps = 1;
  a.ws = ws; a.sem = sem;
  {
    const int rc = qk_rsq_table(&a.rsq_tab);   // set up on this device's first call
    if (rc) return rc;
  }
  attn_schedule(a, batch, nsm);
  // the control block and the split semaphores must start at zero; the
  // descriptor is copied from this stack frame (synchronously, so the frame
  // may go away when the call returns)
  CUDA_TRY(cudaMemsetAsync(ctl, 0, sizeof(Ctl), st));
  CUDA_TRY(cudaMemsetAsync(sem, 0, (size_t)batch * n_kv * sizeof(unsigned), st));
  CUDA_TRY(cudaMemcpyAsync(dstage, &s, sizeof s, cudaMemcpyHostToDevice, st));
  const Stage *prog = dstage;
  int n_st = 1, n_it = 1;
  long long *trace = nullptr;
  const V2Plan *plan = nullptr;   // an attention stage reads no GEMV plan
  int cl0 = 0;
  void *args[] = {(void *)&prog, (void *)&plan, (void *)&n_st, (void *)&n_it, (void *)&ctl, (void *)&trace, (void *)&cl0};
  CUDA_TRY(cudaLaunchCooperativeKernel((const void *)decode_kernel, dim3(nsm), dim3(NTHREADS), args, SMEM_BYTES, st));
  Ctl h;
  CUDA_TRY(cudaMemcpyAsync(&h, ctl, sizeof h, cudaMemcpyDeviceToHost, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  if (h.err) return set_err(QTB_E_DEVICE, "kernel error %d (info %d)", h.err, h.err_info);
  return 0;
}

// ------------------------------------------------------------------------
// The reference's per-op CUDA backend (qwen_tts_cuda.h:23-35, defined in
// qwen_tts_cuda.c:67-141): y = W x and Y = W X for host bf16 weights and host
// f32 activations, behind the backend vtable (qwen_tts_backend.h:34-49).
// Like the reference, each weight is uploaded once and kept resident, cached
// by its host pointer; here it is stored in the engine's bf16 fragment order
// (rows padded to 128, columns to 64 with zeros) and the product runs as one
// GEMV stage of the decode kernel.  X and Y are row-major [cols][B] and
// [rows][B] as in the reference; B <= 64.
namespace {
struct OpWeight {
  const void *key;
  int rows, cols;
  DMat m;
};
struct OpCtx {
  int device = 0, nsm = 0;
  Arena weights;
  std::vector<OpWeight> cache;
  cudaStream_t st = nullptr;
  float *dx = nullptr, *dy = nullptr, *ws = nullptr, *xsc = nullptr;
  uint8_t *xop = nullptr;
  unsigned *sem = nullptr;
  Ctl *ctl = nullptr;
  Stage *dstage = nullptr;
  V2Plan *dplan = nullptr;
  size_t x_cap = 0, y_cap = 0, ws_cap = 0, sem_cap = 0, xsc_cap = 0, xop_cap = 0;
};

int op_grow(void **p, size_t *cap, size_t need) {
  if (*cap >= need) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(p, need);
  if (e != cudaSuccess) return set_err(QTB_E_OOM, "cudaMalloc(%zu): %s", need, cudaGetErrorString(e));
  *cap = need;
  return 0;
}

int op_matmat(OpCtx *c, float *Y, const uint16_t *W, const float *X, int rows, int cols, int B) {
  if (!c || !Y || !W || !X || rows < 1 || cols < 1 || B < 1 || B > 64) return set_err(QTB_E_INVALID, "bad argument");
  CUDA_TRY(cudaSetDevice(c->device));
  const int rp = (rows + 127) / 128 * 128, cp = (cols + 63) / 64 * 64;   // upload_matrix granularity
  const OpWeight *ow = nullptr;
  for (const OpWeight &o : c->cache)
    if (o.key == W && o.rows == rows && o.cols == cols) { ow = &o; break; }
  if (!ow) {
    std::vector<uint16_t> pad((size_t)rp * cp, 0);
    for (int r = 0; r < rows; r++) memcpy(pad.data() + (size_t)r * cp, W + (size_t)r * cols, (size_t)cols * 2);
    qtb_matrix_t hm;
    memset(&hm, 0, sizeof hm);
    hm.data = pad.data();
    const qtb_matrix_t *ms[1] = {&hm};
    const int re[1] = {rp};
    OpWeight o;
    o.key = W; o.rows = rows; o.cols = cols;
    int rc = upload_matrix(c->weights, FMT_BF16, ms, re, 1, cp, o.m);
    if (rc) return rc;
    c->cache.push_back(o);
    ow = &c->cache.back();
  }
  const int T = rp / 16;
  const bool v2 = v2_ok(FMT_BF16, rp, cp, B, c->nsm);
  const bool tc = !v2 && tc_ok(ow->m, B, FMT_BF16);
  const int S = v2 ? std::max(1, c->nsm / T)
                   : tc ? tc_choose(FMT_BF16, rp, cp, B, c->nsm).S : choose_S(T, cp, B, c->nsm * NWARPS, FMT_BF16);
  if (S < 1) return set_err(QTB_E_UNSUPPORTED, "no k-slicing fits (cols %d, B %d)", cols, B);
  const size_t ws_floats = tc ? std::max<size_t>(16, tc_ws_floats(FMT_BF16, rp, cp, B, c->nsm)) : (size_t)T * S * 16 * B;
  int rc;
  if ((rc = op_grow((void **)&c->dx, &c->x_cap, (size_t)B * cp * 4))) return rc;
  if ((rc = op_grow((void **)&c->dy, &c->y_cap, (size_t)B * rp * 4))) return rc;
  if ((rc = op_grow((void **)&c->ws, &c->ws_cap, ws_floats * 4))) return rc;
  if ((rc = op_grow((void **)&c->xsc, &c->xsc_cap, 128 * 4))) return rc;
  if ((rc = op_grow((void **)&c->xop, &c->xop_cap, tc ? tc_xop_bytes(FMT_BF16, cp) : 16))) return rc;
  if ((rc = op_grow((void **)&c->sem, &c->sem_cap, (size_t)T * 4))) return rc;
  // X [cols][B] -> [B][cp] (zero-padded columns)
  std::vector<float> xt((size_t)B * cp, 0.f), yt((size_t)B * rp);
  for (int k = 0; k < cols; k++)
    for (int b = 0; b < B; b++) xt[(size_t)b * cp + k] = X[(size_t)k * B + b];
  CUDA_TRY(cudaMemcpyAsync(c->dx, xt.data(), xt.size() * 4, cudaMemcpyHostToDevice, c->st));
  CUDA_TRY(cudaMemsetAsync(c->sem, 0, (size_t)T * 4, c->st));
  CUDA_TRY(cudaMemsetAsync(c->ctl, 0, sizeof(Ctl), c->st));
  Stage s;
  memset(&s, 0, sizeof s);
  s.kind = ST_GEMV;
  s.B = B;
  GemvArgs &g = s.g;
  g.w = ow->m.w; g.fmt = FMT_BF16; g.rows = rp; g.K = cp; g.S = v2 ? 1 : S;
  g.nch = nch_for(FMT_BF16, B, v2); g.parts = parts_for(FMT_BF16, B, v2); g.v2 = v2 ? 1 : 0;
  g.tc = tc ? 1 : 0; g.wtc = ow->m.wtc; g.xsc = c->xsc; g.xop = c->xop;
  g.x = c->dx; g.ldx = cp; g.y = c->dy; g.ldy = rp; g.epi = EPI_STORE; g.ws = c->ws; g.sem = c->sem;
  CUDA_TRY(cudaMemcpyAsync(c->dstage, &s, sizeof s, cudaMemcpyHostToDevice, c->st));
  std::vector<V2Plan> pl;
  make_plans(std::vector<Stage>{s}, c->nsm, false, pl);
  CUDA_TRY(cudaMemcpyAsync(c->dplan, pl.data(), pl.size() * sizeof(V2Plan), cudaMemcpyHostToDevice, c->st));
  const Stage *prog = c->dstage;
  const V2Plan *plan = c->dplan;
  int n_st = 1, n_it = 1;
  long long *trace = nullptr;
  Ctl *ctl = c->ctl;
  int cl0 = 0;
  void *args[] = {(void *)&prog, (void *)&plan, (void *)&n_st, (void *)&n_it, (void *)&ctl, (void *)&trace, (void *)&cl0};
  CUDA_TRY(cudaLaunchCooperativeKernel((const void *)decode_kernel, dim3(c->nsm), dim3(NTHREADS), args, SMEM_BYTES, c->st));
  Ctl h;
  CUDA_TRY(cudaMemcpyAsync(&h, c->ctl, sizeof h, cudaMemcpyDeviceToHost, c->st));
  CUDA_TRY(cudaMemcpyAsync(yt.data(), c->dy, yt.size() * 4, cudaMemcpyDeviceToHost, c->st));
  CUDA_TRY(cudaStreamSynchronize(c->st));
  if (h.err) return set_err(QTB_E_DEVICE, "kernel error %d (info %d)", h.err, h.err_info);
  for (int r = 0; r < rows; r++)
    for (int b = 0; b < B; b++) Y[(size_t)r * B + b] = yt[(size_t)b * rp + r];
  return 0;
}
}  // namespace

extern "C" int qwen_cuda_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) return 0;
  int dev = 0;
  if (const char *d = getenv("QWEN_CUDA_DEVICE")) dev = atoi(d);
  cudaDeviceProp p;
  if (dev < 0 || dev >= n || cudaGetDeviceProperties(&p, dev) != cudaSuccess) return 0;
  return p.major == 10 ? 1 : 0;
}

extern "C" void *qwen_cuda_init(void) {
  OpCtx *c = new OpCtx();
  if (const char *d = getenv("QWEN_CUDA_DEVICE")) c->device = atoi(d);
  int rc = 0;
  cudaDeviceProp p;
  if (cudaSetDevice(c->device) != cudaSuccess || cudaGetDeviceProperties(&p, c->device) != cudaSuccess || p.major != 10) {
    set_err(QTB_E_UNSUPPORTED, "no sm_100 device %d", c->device);
    rc = 1;
  } else {
    c->nsm = p.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->st, cudaStreamDefault) != cudaSuccess ||   // behind legacy-stream uploads
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess ||
        c->weights.alloc((void **)&c->ctl, sizeof(Ctl)) || c->weights.alloc((void **)&c->dstage, sizeof(Stage)) ||
        c->weights.alloc((void **)&c->dplan, (size_t)c->nsm * sizeof(V2Plan)))
      rc = 1;
  }
  if (rc) {
    fprintf(stderr, "qwen3tts_b200: qwen_cuda_init failed: %s\n", qtb_last_error());
    if (c->st) cudaStreamDestroy(c->st);
    c->weights.release();
    delete c;
    return nullptr;
  }
  return c;
}

extern "C" void qwen_cuda_free(void *ctx) {
  OpCtx *c = static_cast<OpCtx *>(ctx);
  if (!c) return;
  cudaSetDevice(c->device);
  if (c->st) cudaStreamSynchronize(c->st);
  for (void *p : {(void *)c->dx, (void *)c->dy, (void *)c->ws, (void *)c->sem, (void *)c->xsc, (void *)c->xop})
    if (p) cudaFree(p);
  if (c->st) cudaStreamDestroy(c->st);
  c->weights.release();
  delete c;
}

extern "C" void qwen_cuda_matmat_bf16(void *ctx, float *Y, const uint16_t *W, const float *X, int rows, int cols, int B) {
  const int rc = op_matmat(static_cast<OpCtx *>(ctx), Y, W, X, rows, cols, B);
  qtb_ref_set_error(rc);
  if (rc) fprintf(stderr, "qwen3tts_b200: qwen_cuda_matmat_bf16 failed (%d): %s\n", rc, qtb_last_error());
}

extern "C" void qwen_cuda_matvec_bf16(void *ctx, float *y, const uint16_t *W, const float *x, int rows, int cols) {
  qwen_cuda_matmat_bf16(ctx, y, W, x, rows, cols, 1);
}
