// laya_b200: host runtime + C ABI (see include/laya_b200.h).
//
// The engine owns the resident weights, one device workspace shared by every shape class,
// pinned staging buffers, and an LRU of shape-class slots, each holding the class's tensor
// maps and (once captured) its CUDA graph.  Only one forward pass runs at a time on the
// engine's stream, so all classes can share the workspace: a class whose layout does not fit
// grows it, which drops the graphs that pointed into the old one.
//
// Reference counterparts: laya_cuda/runtime.py (Runtime, Slot), laya_cuda/laya.py:195-245
// (head buffers and forward), laya_cuda/ops.py (launch glue).
#include <cuda.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/laya_b200.h"
#include "gemm.cuh"
#include "rowops.cuh"
#include "tc_attention.cuh"
#include "gemm_ln.cuh"
#include "checkpoint.cuh"

using namespace laya;

namespace {

// ---------------------------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------------------------
thread_local std::string g_create_error;

struct Failure {
  int code;
  std::string msg;
};

[[noreturn]] void fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Failure{code, buf};
}

#define CK(call)                                                                                    \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) fail(LAYA_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));     \
  } while (0)

// Residual GEMMs of classes up to this many rows may split K across CTAs (their partial sums are
// added, in split order, by the LayerNorm that follows), so small batches fill the SMs.
constexpr int kSplitRowsMax = 2048;
constexpr int kMaxSplits = 8;

// ---------------------------------------------------------------------------------------------
// Driver entry point for tensor-map encoding (no link-time dependency on libcuda).
// ---------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess) fail(LAYA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D K-major operand [rows][cols] of 16-bit elements, box {64, box_rows}, 128-byte swizzle.
CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int box_rows, bool bf16) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || (cols * 2) % 16 != 0)
    fail(LAYA_ERR_INVALID, "TMA operand must be 16-byte aligned with rows a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                           const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(LAYA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

// 2-D fp32 tensor [rows][cols] with row stride ld elements, box {32 columns, 32 rows}, 128-byte
// swizzle: the residual chunks of the fused residual + LayerNorm epilogue.
CUtensorMap make_map_f32(const float* ptr, int64_t rows, int64_t cols, int64_t ld) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || (ld * 4) % 16 != 0 || cols % 32 != 0)
    fail(LAYA_ERR_INVALID, "residual must be 16-byte aligned, its row stride and width multiples of 4 and 32 floats");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(LAYA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return m;
}

int sm_count(int device) {
  static std::map<int, int> cache;
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  cache[device] = n;
  return n;
}

// Process-wide launch options (laya_set_launch_options): programmatic dependent launch on every
// kernel (on by default), and the wait limit every pipelined kernel's bounded waits use
// (0: the kernels' default of 2 s).  Passes captured into CUDA graphs keep the options in effect
// at capture.
std::atomic<bool> g_pdl{true};
std::atomic<unsigned long long> g_wait_ns{0};
bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed); }
unsigned long long wait_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

// Warps (= rows) per block of the row kernels: 8, or fewer when that leaves SMs idle, so that a
// small class's rows spread over the whole GPU (one row per warp either way).
int row_warps(int rows) {
  int device = 0;
  CK(cudaGetDevice(&device));
  const int sms = sm_count(device);
  int w = kRowWarps;
  while (w > 1 && rows < w * sms) w /= 2;
  return w;
}

template <typename... KArgs, typename... Args>
void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// ---------------------------------------------------------------------------------------------
// Kernel dispatch
// ---------------------------------------------------------------------------------------------
template <typename T, int BN, int EPI, int NI>
void launch_gemm_ni(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t st) {
  static uint64_t configured = 0;  // one bit per device
  auto kern = gemm_kernel<BN, EPI, T, NI>;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (!(configured & (1ull << dev))) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::kSmemBytes));
    configured |= 1ull << dev;
  }
  launch_k(kern, dim3(grid), dim3(kGemmThreads), GemmCfg<BN>::kSmemBytes, st, ta, tb, a);
}

// MMA issuers of a 1-CTA GEMM: one thread's tcgen05.mma stream runs about one instruction per
// ~100 ns whatever the column tile, so grids in which every CTA has a single tile of 64 or 128
// columns spread its k-blocks over 4 or 2 issuing threads (independent accumulators added
// before the epilogue).  Larger grids keep one issuer and double-buffered accumulators.
int gemm_issuers(int bn, int tiles, int grid, int k_blocks) {
  if (tiles > grid) return 1;
  if (bn == 64) return k_blocks >= 4 ? 4 : 1;
  if (bn == 128) return k_blocks >= 2 ? 2 : 1;
  return 1;
}

template <typename T, int BN, int EPI>
void launch_gemm_inst(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t st) {
  const int tiles = ((a.M + kBM - 1) / kBM) * (a.N / BN) * a.splits;
  const int ni = gemm_issuers(BN, tiles, grid, a.K / kBK / a.splits);
  constexpr int kMulti = BN == 64 ? 4 : BN == 128 ? 2 : 1;
  if constexpr (kMulti > 1) {
    if (ni == kMulti) return launch_gemm_ni<T, BN, EPI, kMulti>(ta, tb, a, grid, st);
  }
  launch_gemm_ni<T, BN, EPI, 1>(ta, tb, a, grid, st);
}

// CTA-pair GEMM: clusters of 2 (cta_group::2), plus programmatic serialisation.
template <typename T, int BN, int EPI>
void launch_gemm_pair_inst(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t st) {
  static uint64_t configured = 0;  // one bit per device
  auto kern = gemm_pair_kernel<BN, EPI, T>;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (!(configured & (1ull << dev))) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmPairCfg<BN>::kSmemBytes));
    configured |= 1ull << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = GemmPairCfg<BN>::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, kern, ta, tb, a));
}

template <typename T, int BN>
void launch_gemm_pair_bn(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                         cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: launch_gemm_pair_inst<T, BN, EPI_STORE>(ta, tb, a, grid, st); break;
    case EPI_RELU: launch_gemm_pair_inst<T, BN, EPI_RELU>(ta, tb, a, grid, st); break;
    case EPI_GELU: launch_gemm_pair_inst<T, BN, EPI_GELU>(ta, tb, a, grid, st); break;
    case EPI_GEGLU: launch_gemm_pair_inst<T, BN, EPI_GEGLU>(ta, tb, a, grid, st); break;
    case EPI_QKV: launch_gemm_pair_inst<T, BN, EPI_QKV>(ta, tb, a, grid, st); break;
    case EPI_RESIDUAL: launch_gemm_pair_inst<T, BN, EPI_RESIDUAL>(ta, tb, a, grid, st); break;
    default: fail(LAYA_ERR_INVALID, "epilogue %d has no CTA-pair variant", epi);
  }
}

// Residual GEMM + LayerNorm: clusters of C = N/BN CTAs own 128-row blocks (persistent, as many
// clusters as can be resident at once, at most one per row block).
template <int C, int BN, typename T>
void launch_gemm_ln_inst(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tr, const GemmLnArgs& a,
                         cudaStream_t st) {
  static uint64_t configured = 0;  // one bit per device
  static int max_clusters[64] = {};
  auto kern = gemm_ln_kernel<C, BN, T>;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = GemmLnCfg<C, BN>::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  if (!(configured & (1ull << dev))) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmLnCfg<C, BN>::kSmemBytes));
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    cfg.gridDim = dim3(C * (sms / C));
    cfg.numAttrs = 1;
    int n = 0;
    CK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_clusters[dev & 63] = n > 0 ? n : 1;
    configured |= 1ull << dev;
  }
  const int m_blocks = (a.M + kBM - 1) / kBM;
  const int clusters = std::min(m_blocks, max_clusters[dev & 63]);
  cfg.gridDim = dim3(C * clusters);
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tr, a));
}

// Column block of the fused residual + LayerNorm GEMM for row width N and depth K (0: not
// supported).  256-column blocks (3-stage ring) for short K; 192 (4-stage ring) for long K.
int ln_block_n(int N, int K) {
  const bool b256 = N % 256 == 0 && N / 256 <= 4, b192 = N % 192 == 0 && N / 192 <= 4;
  if (b256 && (K <= 1024 || !b192)) return 256;
  if (b192) return 192;
  return 0;
}

template <typename T>
void launch_gemm_ln(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tr, const GemmLnArgs& args, int bn,
                    cudaStream_t st) {
  GemmLnArgs a = args;
  a.wait_ns = wait_ns();
  const int c = a.N / bn;
  if (bn == 256 && c == 1) launch_gemm_ln_inst<1, 256, T>(ta, tb, tr, a, st);
  else if (bn == 256 && c == 2) launch_gemm_ln_inst<2, 256, T>(ta, tb, tr, a, st);
  else if (bn == 256 && c == 3) launch_gemm_ln_inst<3, 256, T>(ta, tb, tr, a, st);
  else if (bn == 256 && c == 4) launch_gemm_ln_inst<4, 256, T>(ta, tb, tr, a, st);
  else if (bn == 192 && c == 1) launch_gemm_ln_inst<1, 192, T>(ta, tb, tr, a, st);
  else if (bn == 192 && c == 2) launch_gemm_ln_inst<2, 192, T>(ta, tb, tr, a, st);
  else if (bn == 192 && c == 3) launch_gemm_ln_inst<3, 192, T>(ta, tb, tr, a, st);
  else if (bn == 192 && c == 4) launch_gemm_ln_inst<4, 192, T>(ta, tb, tr, a, st);
  else fail(LAYA_ERR_INVALID, "fused residual + LayerNorm: N=%d is not 1-4 blocks of 192 or 256 columns", a.N);
}

// The fused residual + LayerNorm GEMM (gemm_ln.cuh) serves classes that do not split K, for the
// residual GEMMs with K <= kLnMaxK (the attention output projection).  For the FFN-down GEMM
// (K = 3072) the residual GEMM followed by the row LayerNorm measured about 3% faster than the
// fused kernel on the throughput workload; for the attention output the fused kernel is about
// 4% faster.
constexpr int kLnMaxK = 1024;

// Rows from which GEMMs always run as CTA pairs with 256 x 256 tiles; below, plan_small picks the
// tile (1-CTA or pair) and split-K.
constexpr int kPairMinRows = 2048;

template <typename T, int BN>
void launch_gemm_bn(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid, cudaStream_t st) {
  switch (epi) {
    case EPI_STORE: launch_gemm_inst<T, BN, EPI_STORE>(ta, tb, a, grid, st); break;
    case EPI_RELU: launch_gemm_inst<T, BN, EPI_RELU>(ta, tb, a, grid, st); break;
    case EPI_GELU: launch_gemm_inst<T, BN, EPI_GELU>(ta, tb, a, grid, st); break;
    case EPI_GEGLU:
      if (BN < 128) fail(LAYA_ERR_INVALID, "GeGLU epilogue needs a column tile of at least 128");
      launch_gemm_inst<T, BN, EPI_GEGLU>(ta, tb, a, grid, st);
      break;
    case EPI_QKV: launch_gemm_inst<T, BN, EPI_QKV>(ta, tb, a, grid, st); break;
    case EPI_RESIDUAL: launch_gemm_inst<T, BN, EPI_RESIDUAL>(ta, tb, a, grid, st); break;
    case EPI_PARTIAL: launch_gemm_inst<T, BN, EPI_PARTIAL>(ta, tb, a, grid, st); break;
    default: fail(LAYA_ERR_INVALID, "unknown epilogue %d", epi);
  }
}

// tb: W tensor map with BN-row boxes (1-CTA kernel) or BN/2-row boxes (pair kernel).
template <typename T>
void launch_gemm(int epi, int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int sms,
                 cudaStream_t st, bool pair = false) {
  GemmArgs a = args;
  a.wait_ns = wait_ns();
  if (a.K % kBK != 0 || a.N % bn != 0 || a.M <= 0) fail(LAYA_ERR_INVALID, "GEMM shape %dx%dx%d not tileable", a.M, a.N, a.K);
  if ((a.K / kBK) % a.splits != 0) fail(LAYA_ERR_INVALID, "split-K %d does not divide %d k-blocks", a.splits, a.K / kBK);
  if (pair) {
    if (a.splits != 1 || (bn != 128 && bn != 256)) fail(LAYA_ERR_INVALID, "no CTA-pair variant for this GEMM");
    const int tiles = ((a.M + 2 * kBM - 1) / (2 * kBM)) * (a.N / bn);
    const int grid = 2 * std::min(tiles, sms / 2);
    if (bn == 256) launch_gemm_pair_bn<T, 256>(epi, ta, tb, a, grid, st);
    else launch_gemm_pair_bn<T, 128>(epi, ta, tb, a, grid, st);
    return;
  }
  const int tiles = ((a.M + kBM - 1) / kBM) * (a.N / bn) * a.splits;
  const int grid = std::min(tiles, sms);
  switch (bn) {
    case 64: launch_gemm_bn<T, 64>(epi, ta, tb, a, grid, st); break;
    case 128: launch_gemm_bn<T, 128>(epi, ta, tb, a, grid, st); break;
    case 256: launch_gemm_bn<T, 256>(epi, ta, tb, a, grid, st); break;
    default: fail(LAYA_ERR_INVALID, "unsupported column tile %d", bn);
  }
}

// Column tile: the largest tile that still keeps the SMs busy.
int pick_bn(int M, int N, int epi, int sms) {
  const int mb = (M + kBM - 1) / kBM;
  int best = 0;
  double best_score = -1;
  for (int bn : {256, 128, 64}) {
    if (N % bn) continue;
    if (epi == EPI_GEGLU && bn < 128) continue;
    const int tiles = mb * (N / bn);
    const int waves = (tiles + sms - 1) / sms;
    const double util = (double)tiles / ((double)waves * sms);
    const double eff = bn == 256 ? 1.0 : bn == 128 ? 0.92 : 0.8;
    const double score = util * eff;
    if (score > best_score + 1e-9) { best_score = score; best = bn; }
  }
  if (!best) fail(LAYA_ERR_INVALID, "no column tile divides N=%d", N);
  return best;
}

// Tile plan of a GEMM of a small class (fewer than kPairMinRows rows), where every CTA runs about
// one tile, so latency and per-CTA work decide.  Per-CTA globaltimer traces of 512-row passes
// fitted this model of one wave (all constants measured on B200 there):
//   ~1.2 us from the dependency wait to the first full stage, then the operand tiles at
//   max(per-CTA bytes / ~107 GB/s into one SM (~65 GB/s for a CTA of a pair),
//       bytes of all running CTAs / ~10.5 TB/s from L2),
//   then the epilogue, ~0.8 us + ~0.1 us per 1024 accumulators of the CTA;
// plus, for split-K, the fp32 partials written here and read back by the LayerNorm.  Candidates:
// 1-CTA tiles 128 x {64,128,256}, CTA pairs 256 x {128,256} (each CTA loads half of the weight
// rows) and, where allowed, split-K factors with at most one wave.
struct TilePlan {
  bool pair = false;
  int bn = 0;
  int splits = 1;
};
TilePlan plan_small(int M, int N, int K, int epi, bool split_ok, bool pair_ok, int sms) {
  constexpr double kSmRate = 107e9, kPairSmRate = 65e9, kL2Rate = 10.5e12, kSmFlops = 14e12;
  constexpr double kLatency = 1.2e-6, kEpiFixed = 0.8e-6, kEpiPerAcc = 0.1e-6 / 1024;
  const int kb = K / kBK;
  TilePlan best;
  double best_t = 1e30;
  for (int pair = 0; pair <= (pair_ok ? 1 : 0); ++pair) {
    for (int bn : {64, 128, 256}) {
      if (N % bn || (epi == EPI_GEGLU && bn < 128) || (pair && bn < 128)) continue;
      for (int s = 1; s <= (split_ok && !pair ? kMaxSplits : 1); ++s) {
        if (kb % s || (s > 1 && kb / s < 3)) continue;
        const int rows_tile = pair ? 2 * kBM : kBM;
        const int tiles = ((M + rows_tile - 1) / rows_tile) * (N / bn) * s;
        const int slots = pair ? sms / 2 : sms;
        if (s > 1 && tiles > slots) continue;
        const int waves = (tiles + slots - 1) / slots;
        const double kk = (double)(K / s);
        const double cta_bytes = (std::min(M, kBM) + (pair ? bn / 2 : bn)) * kk * 2.0;
        const double concurrent = (double)std::min(tiles, slots) * (pair ? 2 : 1) * cta_bytes;
        const double load = std::max(std::max(cta_bytes / (pair ? kPairSmRate : kSmRate), concurrent / kL2Rate),
                                     2.0 * kBM * bn * kk / kSmFlops);
        double t = waves * (kLatency + load + kEpiFixed + kEpiPerAcc * kBM * bn);
        if (s > 1) t += 2.0 * s * (double)M * N * 4.0 / kL2Rate;
        if (t < best_t * (1 - 1e-9)) { best_t = t; best.pair = pair; best.bn = bn; best.splits = s; }
      }
    }
  }
  if (!best.bn) fail(LAYA_ERR_INVALID, "no column tile divides N=%d", N);
  return best;
}

// Tensor maps of the tcgen05 attention over a qkv buffer of M tokens: 128-row boxes of the q/k
// planes (query tiles, and key blocks of 128), 64-row boxes (key blocks of 64), and 64 dims x
// 64 keys boxes of V^T.
struct AttnMaps {
  CUtensorMap q, k64, vt;
};
AttnMaps attn_maps(const void* qkv, int M, int heads, bool bf) {
  const int64_t hm = (int64_t)heads * M;
  AttnMaps m;
  m.q = make_map(qkv, 3 * hm, 64, kTcQ, bf);
  m.k64 = make_map(qkv, 3 * hm, 64, 64, bf);
  m.vt = make_map(static_cast<const uint8_t*>(qkv) + (size_t)2 * hm * 64 * 2, (int64_t)heads * 64, M, 64, bf);
  return m;
}

template <typename T, int KB>
void launch_tc_attention_kb(const AttnMaps& maps, const TcAttnArgs& a, int n_tiles, cudaStream_t st) {
  using Cfg = TcAttnCfg<KB>;
  static uint64_t configured = 0;  // one bit per device
  auto kern = tc_attention_kernel<T, KB>;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (!(configured & (1ull << dev))) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kBytes));
    configured |= 1ull << dev;
  }
  const CUtensorMap& tk = KB == 64 ? maps.k64 : maps.q;
  if (a.splits == 1) {
    launch_k(kern, dim3(a.heads, n_tiles), dim3(kTcThreads), Cfg::kBytes, st, maps.q, tk, maps.vt, a);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.heads, n_tiles, a.splits);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = Cfg::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = a.splits;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, kern, maps.q, tk, maps.vt, a));
}

// Key-block size of the tcgen05 attention: 128 keys (two CTAs per SM, half the serial chain of
// blocks per tile) for grids that fit the SMs' resident slots at that occupancy, the batch-1
// classes; 64 keys (four CTAs per SM to hide latency) for the rest.  Measured on 512-token
// passes: 64-key blocks cost ~20 us per pass; on the throughput workload 128-key blocks cost 30%.
int attention_block_keys(int heads, int n_tiles, int splits, int sms) {
  return heads * n_tiles * splits <= TcAttnCfg<128>::kCtasPerSm * sms ? 128 : 64;
}

// The persistent 64-key kernel: a grid of the SMs' resident CTA slots (4 per SM), or, with
// `fewest`, of as few CTAs as hold kTcItems work items each (a test form: long item lists).
template <typename T>
void launch_tc_attention_persistent(const AttnMaps& maps, const TcAttnArgs& args, int n_tiles, cudaStream_t st,
                                    int sms, bool fewest) {
  static uint64_t configured = 0;  // one bit per device
  auto kern = tc_attention_persistent_kernel<T>;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (!(configured & (1ull << dev))) {
    CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TcPersistCfg::kBytes));
    configured |= 1ull << dev;
  }
  const int64_t work = (int64_t)args.heads * n_tiles;
  if (work <= 0) return;
  const int64_t least = (work + kTcItems - 1) / kTcItems;
  const int64_t grid = fewest ? least : std::max(least, std::min(work, (int64_t)TcPersistCfg::kCtasPerSm * sms));
  TcAttnArgs a = args;
  a.n_tiles = n_tiles;
  launch_k(kern, dim3((unsigned)grid), dim3(kTcThreads), TcPersistCfg::kBytes, st, maps.q, maps.k64, maps.vt, a);
}

// Large grids of whole tiles (no key split, no gathered queries) run the persistent 64-key
// kernel; `mode` 0 keeps one tile per CTA, 2 forces the persistent kernel with its fewest CTAs.
template <typename T>
void launch_tc_attention(const AttnMaps& maps, const TcAttnArgs& args, int n_tiles, cudaStream_t st, int sms,
                         int mode = 1) {
  TcAttnArgs a = args;
  a.wait_ns = wait_ns();
  a.n_tiles = n_tiles;
  if (n_tiles > 65535) fail(LAYA_ERR_INVALID, "%d attention tiles exceed the grid limit", n_tiles);
  if (a.splits != 1 && a.splits != 2 && a.splits != 4) fail(LAYA_ERR_INVALID, "attention key split %d (1, 2 or 4)", a.splits);
  const bool whole = a.splits == 1 && !a.q_index;
  if (mode == 2) {
    if (!whole) fail(LAYA_ERR_INVALID, "the persistent attention kernel runs whole tiles only");
    launch_tc_attention_persistent<T>(maps, a, n_tiles, st, sms, true);
  } else if (attention_block_keys(a.heads, n_tiles, a.splits, sms) == 128) {
    launch_tc_attention_kb<T, 128>(maps, a, n_tiles, st);
  } else if (whole && mode == 1) {
    launch_tc_attention_persistent<T>(maps, a, n_tiles, st, sms, false);
  } else {
    launch_tc_attention_kb<T, 64>(maps, a, n_tiles, st);
  }
}

// Key split of the tcgen05 attention for grids that leave SMs idle (batch-1 classes): global
// attention over rows of 384+ keys runs each tile's key blocks on 2 CTAs while the split grid
// still fits the SMs' resident CTA slots.
// Window-64 tiles (at most four blocks) stay whole: a split costs a merge through distributed
// shared memory that measured more than the blocks it saves there.
int attention_splits(int heads, int n_tiles, int sms, int window, int row_keys) {
  if (window >= 0 || row_keys < 384) return 1;
  // Four CTAs per tile measured slower than two at batch 1 (512 tokens: 0.696 vs 0.681 ms per
  // pass): the second merge round costs more than the blocks it saves.
  return heads * n_tiles * 2 <= TcAttnCfg<128>::kCtasPerSm * sms ? 2 : 1;
}

// Row kernels are instantiated per width (d = 32 * NPL, d a multiple of 64 up to 1024).
#define LAYA_FOR_EACH_WIDTH(X) X(2) X(4) X(6) X(8) X(10) X(12) X(14) X(16) X(18) X(20) X(22) X(24) X(26) X(28) X(30) X(32)

template <typename T>
void launch_embed(const int* ids, const float* table, const float* gamma, float eps, int rows, int d, int vocab,
                  float* residual, T* x, int* err, cudaStream_t st) {
  const int warps = row_warps(rows);
  const int grid = (rows + warps - 1) / warps;
  switch (d / 32) {
#define LAYA_EMBED_CASE(N)                                                                                  \
  case N:                                                                                                   \
    launch_k(embed_norm_kernel<N, T>, dim3(grid), dim3(warps * 32), 0, st, ids, table, gamma, eps, rows, d,     \
             vocab, residual, x, err);                                                                      \
    break;
    LAYA_FOR_EACH_WIDTH(LAYA_EMBED_CASE)
#undef LAYA_EMBED_CASE
    default: fail(LAYA_ERR_INVALID, "unsupported width %d", d);
  }
}

template <typename T>
void launch_norm(const NormArgs& a, cudaStream_t st) {
  if (a.d % 64 || a.d > 1024) fail(LAYA_ERR_INVALID, "unsupported width %d", a.d);
  const int warps = row_warps(a.rows);
  const int grid = (a.rows + warps - 1) / warps;
  const bool partials = a.splits > 0, fused = a.fused_final != 0;
  switch (a.d / 32) {
#define LAYA_NORM_CASE(N)                                                                                  \
  case N:                                                                                                  \
    if (fused && partials) launch_k(norm_kernel<N, T, true, true>, dim3(grid), dim3(warps * 32), 0, st, a); \
    else if (fused) launch_k(norm_kernel<N, T, false, true>, dim3(grid), dim3(warps * 32), 0, st, a);       \
    else if (partials) launch_k(norm_kernel<N, T, true, false>, dim3(grid), dim3(warps * 32), 0, st, a);    \
    else launch_k(norm_kernel<N, T, false, false>, dim3(grid), dim3(warps * 32), 0, st, a);                 \
    break;
    LAYA_FOR_EACH_WIDTH(LAYA_NORM_CASE)
#undef LAYA_NORM_CASE
    default: fail(LAYA_ERR_INVALID, "unsupported width %d", a.d);
  }
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
int span16(int n) { return (n + 15) / 16 * 16; }

// ---------------------------------------------------------------------------------------------
// Packing (runtime.py:15-25, 52-68)
// ---------------------------------------------------------------------------------------------
void shape_class(const int32_t* lengths, const int32_t* marker_counts, int n, int& rows, int& batch, int& options) {
  if (n <= 0) fail(LAYA_ERR_INVALID, "no items");
  int64_t total = 0;
  int kmax = 0;
  for (int i = 0; i < n; ++i) {
    if (lengths[i] <= 0) fail(LAYA_ERR_INVALID, "item %d is empty", i);
    total += span16(lengths[i]);
    kmax = std::max(kmax, (int)marker_counts[i]);
  }
  const int step = total <= 256 ? 32 : total <= 512 ? 64 : 128;
  if (total > (1 << 30)) fail(LAYA_ERR_INVALID, "request too large");
  rows = (int)((total + step - 1) / step * step);
  auto pow2 = [](int v, int low) { int p = 1; while (p < v) p <<= 1; return std::max(low, p); };
  batch = pow2(n, 1);
  options = pow2(std::max(kmax, 1), 8);
}

// Attention tiles of `tile_q` queries: a row of span S gives ceil(S / tile_q) tiles, the tokens
// past the last row ceil(rest / tile_q) zero-fill tiles.
int tiles_capacity(int rows, int batch, int tile_q) { return (rows + (tile_q - 16) * batch + tile_q - 1) / tile_q + 1; }

struct PackLayout {
  int64_t ids, positions, rows_, kinds, starts, lengths, counts, indices, tiles128, total;
};
PackLayout pack_layout(int m, int b, int k) {
  PackLayout p;
  int64_t o = 0;
  p.ids = o; o += m;
  p.positions = o; o += m;
  p.rows_ = o; o += m;
  p.kinds = o; o += m;
  p.starts = o; o += b;
  p.lengths = o; o += b;
  p.counts = o; o += b;
  p.indices = o; o += (int64_t)b * (k + 1);
  o = (o + 3) / 4 * 4;  // int4 alignment of the tile tables
  p.tiles128 = o; o += 4LL * tiles_capacity(m, b, kTcQ);     // tcgen05 attention
  p.total = o;
  return p;
}

int build_tiles(const int32_t* starts, const int32_t* lengths, int n_rows, int M, int tile_q, int32_t* tiles,
                int capacity) {
  int t = 0, end = 0;
  auto put = [&](int a, int b, int r) {
    if (t >= capacity) return false;
    tiles[4 * t] = a; tiles[4 * t + 1] = b; tiles[4 * t + 2] = r; tiles[4 * t + 3] = 0;
    ++t;
    return true;
  };
  // Rows longest first: the attention grid runs tiles in table order (all heads of a tile
  // together), so the longest global-attention tiles start first and the short ones fill the
  // last wave.
  std::vector<int> order(n_rows);
  for (int r = 0; r < n_rows; ++r) order[r] = r;
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return lengths[x] > lengths[y]; });
  for (int r : order) {
    const int s = starts[r], sp = span16(lengths[r]);
    for (int q = 0; q < sp; q += tile_q)
      if (!put(s + q, std::min(s + q + tile_q, s + sp), r)) return -1;
    end = std::max(end, s + sp);
  }
  for (int q = end; q < M; q += tile_q)
    if (!put(q, std::min(q + tile_q, M), -1)) return -1;
  const int used = t;
  while (t < capacity) put(0, 0, -2);
  return used;
}

void pack(const int32_t* tokens, const int32_t* lengths, const int32_t* markers, const int32_t* marker_counts,
          const int32_t* kinds, int n, int pad, int m, int b, int k, int max_len, int32_t* out) {
  const PackLayout L = pack_layout(m, b, k);
  int32_t* ids = out + L.ids;
  std::fill(out, out + L.total, 0);
  std::fill(ids, ids + m, pad);
  std::fill(out + L.rows_, out + L.rows_ + m, -1);
  int offset = 0;
  int64_t tok = 0, mk = 0;
  for (int r = 0; r < n; ++r) {
    const int len = lengths[r], cnt = marker_counts[r];
    if (len <= 0 || len > max_len) fail(LAYA_ERR_INVALID, "item %d has %d tokens (max_len %d)", r, len, max_len);
    if (cnt < 0 || cnt > k) fail(LAYA_ERR_INVALID, "item %d has %d options (class %d)", r, cnt, k);
    if (kinds[r] < 0 || kinds[r] > 2) fail(LAYA_ERR_INVALID, "item %d has question type %d", r, kinds[r]);
    const int end = offset + span16(len);
    if (end > m) fail(LAYA_ERR_INVALID, "items exceed %d packed rows", m);
    std::copy(tokens + tok, tokens + tok + len, ids + offset);
    for (int t = offset; t < end; ++t) {
      out[L.positions + t] = t - offset;
      out[L.rows_ + t] = r;
      out[L.kinds + t] = kinds[r];
    }
    out[L.starts + r] = offset;
    out[L.lengths + r] = len;
    out[L.counts + r] = cnt;
    int32_t* ind = out + L.indices + (int64_t)r * (k + 1);
    for (int j = 0; j <= k; ++j) ind[j] = offset;
    for (int j = 0; j < cnt; ++j) {
      const int pos = markers[mk + j];
      if (pos < 0 || pos >= len) fail(LAYA_ERR_INVALID, "item %d marker %d out of range", r, pos);
      ind[j + 1] = offset + pos;
    }
    tok += len;
    mk += cnt;
    offset = end;
  }
  if (build_tiles(out + L.starts, out + L.lengths, n, m, kTcQ, out + L.tiles128, tiles_capacity(m, b, kTcQ)) < 0)
    fail(LAYA_ERR_INVALID, "attention tile table overflow");
}

// ---------------------------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------------------------
struct Tensor {
  void* ptr = nullptr;
  int dtype = LAYA_DTYPE_F32;  // storage dtype
  std::vector<int64_t> shape;
  size_t bytes = 0;
  bool arena = false;          // inside the engine's weight arena (laya_load_checkpoint), not freed alone
};

struct ClassLayout {
  int m = 0, b = 0, k = 0, count = 0, tiles128 = 0;
  PackLayout pack{};
  size_t packed, residual, x, qkv, attn, ff, sel, selx, scored, ffsel, partials, hidden, out, total;
  bool has_partials = false;
  size_t n_out_floats;  // logits b*(k+1) + acts b*n_act + 1 error word
};

struct Slot {
  int m, b, k;
  ClassLayout L;
  cudaGraphExec_t graph = nullptr;
  bool maps_ready = false;
  size_t maps_ws = 0;  // workspace generation the maps point into
  CUtensorMap map_x, map_attn, map_ff, map_selx, map_scored, map_ffsel, map_residual;
  AttnMaps attn_maps;
  int launches = 0;
};

// Kernel families for laya_profile_read.
enum Family : int {
  FAM_GEMM_QKV = 0, FAM_GEMM_ATTN_OUT = 1, FAM_GEMM_FFN_UP = 2, FAM_GEMM_FFN_DOWN = 3, FAM_GEMM_HEAD = 4,
  FAM_ATTENTION = 5, FAM_ROWS = 6, FAM_HEAD_TAIL = 7, kFamilies = 8
};
// Classes with more packed rows than this run eagerly under capture mode "auto": their kernels
// are long enough that launch overhead is negligible, and a graph per distinct large class
// would cost a capture per batch.
constexpr int kAutoGraphRows = 8192;

struct ProfEvent {
  int family;
  cudaEvent_t a, b;
  double flops;
};

// One forward pass submitted by laya_submit and not yet collected: its pinned staging buffers,
// events and result metadata.  Two exist, so the host can pack and launch a pass while the
// previous one runs.
struct Inflight {
  bool busy = false;
  int64_t ticket = 0;
  int n_items = 0, m = 0, b = 0, k = 0;
  int32_t* h_packed = nullptr;
  size_t h_packed_cap = 0;
  float* h_out = nullptr;
  size_t h_out_cap = 0;
  size_t n_out_floats = 0;
  cudaEvent_t ev_start = nullptr, ev_end = nullptr, done = nullptr;
  bool miss = false, captured = false, replay = false;
  int launches = 0;
};

struct Engine {
  laya_config cfg{};
  int device = 0;
  int limit = 16;
  int sms = 148;
  bool finalized = false;
  cudaStream_t stream = nullptr;
  std::unordered_map<std::string, Tensor> weights;
  std::map<std::string, std::vector<int64_t>> expected;
  float4* rope_tab[2] = {nullptr, nullptr};  // global / local theta, [16][rope_rows] (see GemmArgs)
  int rope_rows = 0;
  uint8_t* ws = nullptr;
  void* arena = nullptr;       // every weight of the last laya_load_checkpoint, one allocation
  size_t ws_bytes = 0;
  size_t ws_generation = 0;
  Inflight inflight[2];
  int64_t next_ticket = 1;
  std::list<std::tuple<int, int, int>> lru;  // front = least recently used
  std::map<std::tuple<int, int, int>, std::unique_ptr<Slot>> slots;
  std::map<std::tuple<const void*, int>, CUtensorMap> wmaps;
  std::string error;
  bool profiling = false;
  std::vector<ProfEvent> prof_pending;
  std::vector<cudaEvent_t> prof_pool;
  double prof_ms[kFamilies] = {};
  double prof_flops[kFamilies] = {};
  int64_t prof_launches[kFamilies] = {};
  int launches = 0;

  bool bf16() const { return cfg.precision == LAYA_PRECISION_BF16; }
  int d() const { return cfg.width; }
  int F() const { return cfg.intermediate; }
  int ffw() const { return std::max(cfg.intermediate, 4 * cfg.width); }
  size_t owned() const {
    size_t s = ws_bytes;
    for (auto& kv : weights) s += kv.second.bytes;
    for (int i = 0; i < 2; ++i) if (rope_tab[i]) s += (size_t)rope_rows * 16 * sizeof(float4);
    return s;
  }
};

void build_expected(Engine& e) {
  const laya_config& c = e.cfg;
  const int64_t w = c.width, f = c.intermediate;
  auto& s = e.expected;
  s["encoder.embeddings.tok_embeddings.weight"] = {c.vocab, w};
  s["encoder.embeddings.norm.weight"] = {w};
  s["encoder.final_norm.weight"] = {w};
  s["type_emb.weight"] = {3, w};
  s["temperature"] = {3};
  s["scorer.0.weight"] = {w};
  s["scorer.0.bias"] = {w};
  s["scorer.1.weight"] = {w, w};
  s["scorer.1.bias"] = {w};
  s["scorer.3.weight"] = {1, w};
  s["scorer.3.bias"] = {1};
  s["act_head.0.weight"] = {256, w + 4};
  s["act_head.0.bias"] = {256};
  s["act_head.2.weight"] = {c.n_act, 256};
  s["act_head.2.bias"] = {c.n_act};
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    s[p + "attn.Wqkv.weight"] = {3 * w, w};
    s[p + "attn.Wo.weight"] = {w, w};
    s[p + "mlp.Wi.weight"] = {2 * f, w};
    s[p + "mlp.Wo.weight"] = {w, f};
    s[p + "mlp_norm.weight"] = {w};
    if (i) s[p + "attn_norm.weight"] = {w};
  }
  for (int i = 0; i < c.head_layers; ++i) {
    const std::string p = "head.layers." + std::to_string(i) + ".";
    s[p + "self_attn.in_proj_weight"] = {3 * w, w};
    s[p + "self_attn.in_proj_bias"] = {3 * w};
    s[p + "self_attn.out_proj.weight"] = {w, w};
    s[p + "self_attn.out_proj.bias"] = {w};
    s[p + "linear1.weight"] = {4 * w, w};
    s[p + "linear1.bias"] = {4 * w};
    s[p + "linear2.weight"] = {w, 4 * w};
    s[p + "linear2.bias"] = {w};
    s[p + "norm1.weight"] = {w};
    s[p + "norm1.bias"] = {w};
    s[p + "norm2.weight"] = {w};
    s[p + "norm2.bias"] = {w};
  }
}

// 16-bit GEMM operands; everything else (norms, embeddings, biases, the head tail) stays fp32.
bool stored_16bit(const std::string& name) {
  if (name.find("norm") != std::string::npos) return false;
  if (name.size() >= 5 && name.compare(name.size() - 5, 5, ".bias") == 0) return false;
  if (name.size() >= 5 && name.compare(name.size() - 5, 5, "_bias") == 0) return false;
  if (name == "type_emb.weight" || name == "encoder.embeddings.tok_embeddings.weight") return false;
  if (name.rfind("scorer.0.", 0) == 0 || name.rfind("scorer.3.", 0) == 0 || name.rfind("act_head.", 0) == 0) return false;
  return true;
}

float half_bits_to_float(uint16_t h, bool bf16) {
  if (bf16) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  // IEEE binary16 -> binary32
  const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, u;
  if (exp == 0) {
    if (man == 0) u = sign;
    else {
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) u = sign | 0x7F800000 | (man << 13);
  else u = sign | ((exp + 112) << 23) | (man << 13);
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t float_to_half_bits(float f, bool bf16) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (bf16) {
    if ((u & 0x7FFFFFFF) > 0x7F800000) return 0x7FC0;  // NaN
    const uint32_t lsb = (u >> 16) & 1;
    return (uint16_t)((u + 0x7FFF + lsb) >> 16);       // round to nearest even
  }
  const uint32_t sign = (u >> 16) & 0x8000;
  const uint32_t a = u & 0x7FFFFFFF;
  if (a > 0x7F800000) return (uint16_t)(sign | 0x7E00);
  if (a >= 0x477FF000) return (uint16_t)(sign | 0x7C00);  // overflow -> inf (ties above max)
  if (a < 0x38800000) {                                    // subnormal or zero
    if (a < 0x33000000) return (uint16_t)sign;
    const uint32_t e = a >> 23;
    const uint32_t m = (a & 0x7FFFFF) | 0x800000;
    const int shift = 126 - (int)e;  // 14 + (113 - e)
    uint32_t v = m >> (shift);
    const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (v & 1))) ++v;
    return (uint16_t)(sign | v);
  }
  uint32_t v = ((a - 0x38000000) >> 13);
  const uint32_t rem = a & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (v & 1))) ++v;
  return (uint16_t)(sign | v);
}

void* dev_alloc(size_t bytes) {
  void* p = nullptr;
  CK(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
  return p;
}

void drop_graphs(Engine& e);

// ---------------------------------------------------------------------------------------------
// Checkpoint load (replaces runtime.py:147-158: safetensors read, per-tensor checks, upload)
// ---------------------------------------------------------------------------------------------
struct MappedFile {
  int fd = -1;
  void* base = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (base) munmap(base, size);
    if (fd >= 0) close(fd);
  }
};

// Pinned host chunk, the device chunk it is uploaded into when the values need converting, and
// the event that says both are free again.
struct LoadStage {
  void* host = nullptr;
  void* dev = nullptr;
  cudaEvent_t done = nullptr;
  ~LoadStage() {
    if (done) cudaEventDestroy(done);
    if (host) cudaFreeHost(host);
    if (dev) cudaFree(dev);
  }
};

// memcpy split over host threads (a single thread copies from the page cache at a fraction of
// what the host can do).
void parallel_copy(void* dst, const void* src, size_t n) {
  static const int threads = std::max(1, std::min(16, (int)std::thread::hardware_concurrency()));
  if (n < (size_t(4) << 20) || threads == 1) {
    memcpy(dst, src, n);
    return;
  }
  const size_t per = (n / threads + 4095) & ~size_t(4095);
  std::vector<std::thread> pool;
  for (size_t off = 0; off < n; off += per) {
    const size_t len = std::min(per, n - off);
    pool.emplace_back([=] { memcpy(static_cast<char*>(dst) + off, static_cast<const char*>(src) + off, len); });
  }
  for (auto& t : pool) t.join();
}

void release_weights(Engine& e) {
  CK(cudaStreamSynchronize(e.stream));
  drop_graphs(e);
  for (auto& kv : e.weights)
    if (kv.second.ptr && !kv.second.arena) cudaFree(kv.second.ptr);
  e.weights.clear();
  e.wmaps.clear();
  if (e.arena) CK(cudaFree(e.arena));
  e.arena = nullptr;
  e.finalized = false;
}

// The parsed header of a mapped safetensors file (offsets checked against the file size).
struct Checkpoint {
  MappedFile file;
  std::map<std::string, StEntry> entries;
  uint64_t data0 = 0;
  const uint8_t* bytes() const { return static_cast<const uint8_t*>(file.base); }
};

void open_checkpoint(const char* path, Checkpoint& c) {
  MappedFile& f = c.file;
  f.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (f.fd < 0) fail(LAYA_ERR_INVALID, "cannot open %s: %s", path, strerror(errno));
  struct stat sb;
  if (fstat(f.fd, &sb) != 0) fail(LAYA_ERR_INVALID, "cannot stat %s", path);
  f.size = (size_t)sb.st_size;
  if (f.size < 8) fail(LAYA_ERR_INVALID, "%s is not a safetensors file", path);
  f.base = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, f.fd, 0);
  if (f.base == MAP_FAILED) {
    f.base = nullptr;
    fail(LAYA_ERR_INVALID, "cannot map %s", path);
  }
  madvise(f.base, f.size, MADV_SEQUENTIAL);
  const uint8_t* file = c.bytes();
  uint64_t header = 0;
  for (int i = 7; i >= 0; --i) header = (header << 8) | file[i];  // little-endian length
  if (header > f.size - 8) fail(LAYA_ERR_INVALID, "%s: header length %llu exceeds the file", path, (unsigned long long)header);
  try {
    c.entries = StHeaderParser(reinterpret_cast<const char*>(file + 8), (size_t)header).parse();
  } catch (const std::exception& x) {
    fail(LAYA_ERR_INVALID, "%s: %s", path, x.what());
  }
  c.data0 = 8 + header;
  for (auto& kv : c.entries) {
    const StEntry& en = kv.second;
    uint64_t elems = 1;
    for (int64_t v : en.shape) elems *= (uint64_t)v;
    if (en.end - en.begin != elems * st_dtype_bytes(en.dtype) || c.data0 + en.end > f.size)
      fail(LAYA_ERR_INVALID, "%s: data of tensor %s is out of range", path, kv.first.c_str());
  }
}

// Reads a safetensors checkpoint into the engine: checks names and shapes against the
// adapter's tensor list (the reference's messages), places every tensor in one device arena,
// and streams the file through two pinned chunks: while chunk i uploads (and converts on the
// device), chunk i+1 is copied out of the mapped file by several host threads.
void load_checkpoint(Engine& e, const char* path) {
  Checkpoint ck;
  open_checkpoint(path, ck);
  const std::map<std::string, StEntry>& entries = ck.entries;
  const uint8_t* file = ck.bytes();
  const uint64_t data0 = ck.data0;
  std::set<std::string> want, got;
  for (auto& kv : e.expected) want.insert(kv.first);
  for (auto& kv : entries) got.insert(kv.first);
  if (want != got) fail(LAYA_ERR_INVALID, "Checkpoint tensor names do not match the Laya adapter");
  struct Planned {
    std::string name;
    const StEntry* src;
    int64_t elems, rows, cols;
    int store;         // kStoreF32 / F16 / BF16
    int64_t interleave;
    size_t offset, bytes;
  };
  std::vector<Planned> plan;
  size_t arena_bytes = 0;
  for (auto& kv : entries) {
    const StEntry& en = kv.second;
    if (en.shape != e.expected[kv.first]) fail(LAYA_ERR_INVALID, "Incompatible tensor shape: %s", kv.first.c_str());
    int64_t elems = 1;
    for (int64_t v : en.shape) elems *= v;
    if (kv.first == "temperature") continue;  // calibration is read by the adapter (laya.py:145-150)
    Planned p;
    p.name = kv.first;
    p.src = &en;
    p.elems = elems;
    p.rows = en.shape.size() >= 2 ? en.shape[0] : 1;
    p.cols = elems / std::max<int64_t>(p.rows, 1);
    const bool is16 = stored_16bit(kv.first);
    p.store = !is16 ? kStoreF32 : e.bf16() ? kStoreBF16 : kStoreF16;
    p.interleave = kv.first.find("mlp.Wi.weight") != std::string::npos ? p.rows / 2 : 0;
    if (p.interleave % 64) fail(LAYA_ERR_INVALID, "intermediate size must be a multiple of 64");
    p.bytes = (size_t)elems * (is16 ? 2 : 4);
    p.offset = arena_bytes;
    arena_bytes = align_up(arena_bytes + p.bytes, 256);
    plan.push_back(p);
  }
  // Stream the file in order, so the page cache and the disk read sequentially.
  std::sort(plan.begin(), plan.end(), [](const Planned& a, const Planned& b) { return a.src->begin < b.src->begin; });

  release_weights(e);
  e.arena = dev_alloc(arena_bytes);
  constexpr size_t kChunk = size_t(32) << 20;
  LoadStage stage[2];
  for (auto& s : stage) {
    CK(cudaHostAlloc(&s.host, kChunk, cudaHostAllocDefault));
    s.dev = dev_alloc(kChunk);
    CK(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
  }
  bool used[2] = {false, false};
  int next = 0;
  for (const Planned& p : plan) {
    const int esz = st_dtype_bytes(p.src->dtype);
    const bool direct = p.interleave == 0 && ((p.store == kStoreF32 && p.src->dtype == StDtype::F32) ||
                                              (p.store == kStoreF16 && p.src->dtype == StDtype::F16) ||
                                              (p.store == kStoreBF16 && p.src->dtype == StDtype::BF16));
    uint8_t* dst = static_cast<uint8_t*>(e.arena) + p.offset;
    const int64_t row_bytes = p.cols * esz;
    const int64_t rows_per_chunk = std::max<int64_t>(1, (int64_t)kChunk / row_bytes);
    if (row_bytes > (int64_t)kChunk) fail(LAYA_ERR_INVALID, "tensor %s has rows longer than the staging chunk", p.name.c_str());
    for (int64_t r0 = 0; r0 < p.rows; r0 += rows_per_chunk) {
      const int64_t nr = std::min(rows_per_chunk, p.rows - r0);
      const size_t nbytes = (size_t)(nr * row_bytes);
      LoadStage& s = stage[next];
      if (used[next]) CK(cudaEventSynchronize(s.done));
      used[next] = true;
      next ^= 1;
      parallel_copy(s.host, file + data0 + p.src->begin + (size_t)(r0 * row_bytes), nbytes);
      if (direct) {
        CK(cudaMemcpyAsync(dst + (size_t)(r0 * row_bytes), s.host, nbytes, cudaMemcpyHostToDevice, e.stream));
      } else {
        CK(cudaMemcpyAsync(s.dev, s.host, nbytes, cudaMemcpyHostToDevice, e.stream));
        const int64_t n = nr * p.cols;
        const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)e.sms * 8);
        convert_rows_kernel<<<grid, 256, 0, e.stream>>>(s.dev, (int)p.src->dtype, dst, p.store, r0, nr, p.cols,
                                                         p.interleave);
        CK(cudaGetLastError());
      }
      CK(cudaEventRecord(s.done, e.stream));
    }
  }
  CK(cudaStreamSynchronize(e.stream));
  for (const Planned& p : plan) {
    Tensor t;
    t.ptr = static_cast<uint8_t*>(e.arena) + p.offset;
    t.shape = p.src->shape;
    t.bytes = p.bytes;
    t.arena = true;
    t.dtype = p.store == kStoreF32 ? LAYA_DTYPE_F32 : p.store == kStoreBF16 ? LAYA_DTYPE_BF16 : LAYA_DTYPE_F16;
    e.weights[p.name] = t;
  }
}

void drop_graphs(Engine& e) {
  for (auto& kv : e.slots) {
    if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    kv.second->graph = nullptr;
    kv.second->maps_ready = false;
  }
}

ClassLayout make_layout(const Engine& e, int m, int b, int k) {
  ClassLayout L;
  L.m = m; L.b = b; L.k = k;
  L.count = b * (k + 1);
  L.tiles128 = tiles_capacity(m, b, kTcQ);
  L.pack = pack_layout(m, b, k);
  const size_t d = e.d(), es = 2, A = 256;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes, A); return at; };
  L.packed = take(L.pack.total * 4);
  L.residual = take((size_t)m * d * 4);
  L.x = take((size_t)m * d * es);
  L.qkv = take((size_t)3 * m * d * es);
  L.attn = take((size_t)m * d * es);
  L.ff = take((size_t)m * e.ffw() * es);
  L.sel = take((size_t)L.count * d * 4);
  L.selx = take((size_t)L.count * d * es);
  L.scored = take((size_t)L.count * d * es);
  L.ffsel = take((size_t)L.count * 4 * d * es);
  L.has_partials = m <= kSplitRowsMax;
  L.partials = take(L.has_partials ? (size_t)kMaxSplits * std::max(m, L.count) * d * 4 : 0);
  L.hidden = take((size_t)b * kActHidden * 4);
  // logits [b][k+1], acts [b][n_act], the error word, then the head tail's per-question
  // arrival counters (zeroed with the error word at the start of every pass).
  L.n_out_floats = (size_t)b * (k + 1) + (size_t)b * e.cfg.n_act + 1;
  L.out = take((L.n_out_floats + b) * 4);
  L.total = o;
  return L;
}

void ensure_workspace(Engine& e, size_t bytes) {
  if (bytes <= e.ws_bytes) return;
  CK(cudaStreamSynchronize(e.stream));
  drop_graphs(e);
  if (e.ws) CK(cudaFree(e.ws));
  e.ws = nullptr;
  e.ws_bytes = 0;
  const size_t want = align_up(bytes + bytes / 8, 1 << 20);
  e.ws = static_cast<uint8_t*>(dev_alloc(want));
  e.ws_bytes = want;
  ++e.ws_generation;
}

// Pinned staging of a free in-flight record (none of its copies is pending).  Capacities grow to
// powers of two: pinning and unpinning are slow and cudaFreeHost synchronises the device, so a
// stream of slightly growing classes must not reallocate every time.
size_t pow2_at_least(size_t n) {
  size_t c = 4096;
  while (c < n) c <<= 1;
  return c;
}
void ensure_host(Inflight& r, size_t ints, size_t floats) {
  ints = pow2_at_least(ints);
  floats = pow2_at_least(floats);
  if (ints > r.h_packed_cap) {
    if (r.h_packed) CK(cudaFreeHost(r.h_packed));
    r.h_packed = nullptr;
    CK(cudaHostAlloc(reinterpret_cast<void**>(&r.h_packed), ints * 4, cudaHostAllocDefault));
    r.h_packed_cap = ints;
  }
  if (floats > r.h_out_cap) {
    if (r.h_out) CK(cudaFreeHost(r.h_out));
    r.h_out = nullptr;
    CK(cudaHostAlloc(reinterpret_cast<void**>(&r.h_out), floats * 4, cudaHostAllocDefault));
    r.h_out_cap = floats;
  }
}

const Tensor& W(const Engine& e, const std::string& name) {
  auto it = e.weights.find(name);
  if (it == e.weights.end() || !it->second.ptr) fail(LAYA_ERR_STATE, "tensor %s not loaded", name.c_str());
  return it->second;
}
const float* Wf(const Engine& e, const std::string& name) {
  const Tensor& t = W(e, name);
  return static_cast<const float*>(t.ptr);
}

const CUtensorMap& weight_map(Engine& e, const std::string& name, int bn) {
  const Tensor& t = W(e, name);
  auto key = std::make_tuple((const void*)t.ptr, bn);
  auto it = e.wmaps.find(key);
  if (it != e.wmaps.end()) return it->second;
  CUtensorMap m = make_map(t.ptr, t.shape[0], t.shape[1], bn, e.bf16());
  return e.wmaps.emplace(key, m).first->second;
}

void prepare_maps(Engine& e, Slot& s) {
  if (s.maps_ready && s.maps_ws == e.ws_generation) return;
  const ClassLayout& L = s.L;
  const bool bf = e.bf16();
  const int d = e.d();
  s.map_x = make_map(e.ws + L.x, L.m, d, kBM, bf);
  s.map_attn = make_map(e.ws + L.attn, L.m, d, kBM, bf);
  s.map_ff = make_map(e.ws + L.ff, L.m, e.F(), kBM, bf);
  s.map_selx = make_map(e.ws + L.selx, L.count, d, kBM, bf);
  s.map_scored = make_map(e.ws + L.scored, L.count, d, kBM, bf);
  s.map_ffsel = make_map(e.ws + L.ffsel, L.count, 4 * d, kBM, bf);
  s.map_residual = make_map_f32(reinterpret_cast<const float*>(e.ws + L.residual), L.m, d, d);
  // Attention: Q/K rows of the qkv buffer ([3*heads*m][64], 128-row boxes) and V^T
  // ([heads*64][m], 64x64 boxes), both 128-byte swizzled.
  s.attn_maps = attn_maps(e.ws + L.qkv, L.m, e.cfg.heads, bf);
  s.maps_ready = true;
  s.maps_ws = e.ws_generation;
}

cudaEvent_t prof_event(Engine& e) {
  if (!e.prof_pool.empty()) {
    cudaEvent_t ev = e.prof_pool.back();
    e.prof_pool.pop_back();
    return ev;
  }
  cudaEvent_t ev;
  CK(cudaEventCreate(&ev));
  return ev;
}

// Wraps one launch: counts it and, when profiling an eager pass, brackets it with events.
template <typename F>
void launch(Engine& e, bool prof, int family, double flops, F&& f) {
  ProfEvent pe{family, nullptr, nullptr, flops};
  if (prof) {
    pe.a = prof_event(e);
    pe.b = prof_event(e);
    CK(cudaEventRecord(pe.a, e.stream));
  }
  f();
  ++e.launches;
  if (prof) {
    CK(cudaEventRecord(pe.b, e.stream));
    e.prof_pending.push_back(pe);
  }
}

void prof_resolve(Engine& e) {
  if (e.prof_pending.empty()) return;
  CK(cudaStreamSynchronize(e.stream));
  for (auto& p : e.prof_pending) {
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, p.a, p.b));
    e.prof_ms[p.family] += ms;
    e.prof_flops[p.family] += p.flops;
    e.prof_launches[p.family] += 1;
    e.prof_pool.push_back(p.a);
    e.prof_pool.push_back(p.b);
  }
  e.prof_pending.clear();
}

template <typename T>
void gemm(Engine& e, bool prof, int family, int epi, const CUtensorMap& ta, const std::string& wname, int M, void* out,
          int ldo, float* residual, int ldr, const float* bias, int* err, int rope = -1, const int* positions = nullptr) {
  const Tensor& w = W(e, wname);
  const int N = (int)w.shape[0], K = (int)w.shape[1];
  // Large classes run every epilogue on the CTA pair (the FFN-down residual GEMM measured 440 ->
  // 402 ms per throughput step against the 1-CTA kernel: half the weight rows per CTA); small
  // classes keep residual GEMMs on the 1-CTA kernel, where plan_small may split K.
  const bool pair_ok = epi != EPI_RESIDUAL || M >= kPairMinRows;
  int bn;
  bool pair;
  if (M < kPairMinRows) {
    const TilePlan plan = plan_small(M, N, K, epi, false, pair_ok, e.sms);
    bn = plan.bn;
    pair = plan.pair;
  } else {
    pair = pair_ok && N % 256 == 0;
    bn = pair ? 256 : pick_bn(M, N, epi, e.sms);
  }
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.splits = 1;
  a.out = out; a.ldo = ldo; a.residual = residual; a.ldr = ldr; a.bias = bias;
  a.heads = e.cfg.heads;
  if (rope >= 0) { a.rope_tab = e.rope_tab[rope]; a.rope_rows = e.rope_rows; }
  a.positions = positions;
  a.err = err;
  const CUtensorMap& tb = weight_map(e, wname, pair ? bn / 2 : bn);
  launch(e, prof, family, 2.0 * M * N * K, [&] { launch_gemm<T>(epi, bn, ta, tb, a, e.sms, e.stream, pair); });
}

template <typename T>
void gemm_partial(Engine& e, bool prof, int family, const CUtensorMap& ta, const std::string& wname, int M, int splits,
                  int bn, float* partials, int* err) {
  const Tensor& w = W(e, wname);
  const int N = (int)w.shape[0], K = (int)w.shape[1];
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.splits = splits;
  a.residual = partials; a.ldr = N; a.err = err;
  const CUtensorMap& tb = weight_map(e, wname, bn);
  launch(e, prof, family, 2.0 * M * N * K, [&] { launch_gemm<T>(EPI_PARTIAL, bn, ta, tb, a, e.sms, e.stream); });
}

// The whole forward pass of one shape class (runtime.py:90-113 + laya.py:214-245), enqueued
// on the engine stream.  Used eagerly and inside graph capture.
template <typename T>
void enqueue_forward(Engine& e, Slot& s, bool prof) {
  const ClassLayout& L = s.L;
  const laya_config& c = e.cfg;
  const int m = L.m, d = c.width, count = L.count;
  uint8_t* ws = e.ws;
  const int32_t* in = reinterpret_cast<const int32_t*>(ws + L.packed);
  const int* ids = in + L.pack.ids;
  const int* positions = in + L.pack.positions;
  const int* kinds = in + L.pack.kinds;
  const int* starts = in + L.pack.starts;
  const int* lengths = in + L.pack.lengths;
  const int* counts = in + L.pack.counts;
  const int* indices = in + L.pack.indices;
  const int4* tiles128 = reinterpret_cast<const int4*>(in + L.pack.tiles128);
  float* residual = reinterpret_cast<float*>(ws + L.residual);
  T* x = reinterpret_cast<T*>(ws + L.x);
  T* qkv = reinterpret_cast<T*>(ws + L.qkv);
  T* attn = reinterpret_cast<T*>(ws + L.attn);
  T* ff = reinterpret_cast<T*>(ws + L.ff);
  float* sel = reinterpret_cast<float*>(ws + L.sel);
  T* selx = reinterpret_cast<T*>(ws + L.selx);
  T* scored = reinterpret_cast<T*>(ws + L.scored);
  T* ffsel = reinterpret_cast<T*>(ws + L.ffsel);
  float* partials = L.has_partials ? reinterpret_cast<float*>(ws + L.partials) : nullptr;
  float* outf = reinterpret_cast<float*>(ws + L.out);
  float* logits = outf;
  float* acts = outf + (size_t)L.b * (L.k + 1);
  int* err = reinterpret_cast<int*>(acts + (size_t)L.b * c.n_act);

  int* arrivals = err + 1;
  CK(cudaMemsetAsync(err, 0, sizeof(int) * (1 + (size_t)L.b), e.stream));
  launch(e, prof, FAM_ROWS, 0, [&] {
    launch_embed<T>(ids, Wf(e, "encoder.embeddings.tok_embeddings.weight"), Wf(e, "encoder.embeddings.norm.weight"),
                    c.eps, m, d, c.vocab, residual, x, err, e.stream);
  });

  // gathered: only the rows gather_rows_kernel reads (each question's CLS and marker tokens)
  // attend; the other rows of `attn` are left as they are (global attention only).
  auto attention = [&](int window, bool gathered) {
    TcAttnArgs a{};
    a.qk = qkv; a.out = attn; a.tiles = tiles128; a.starts = starts; a.lengths = lengths;
    a.M = m; a.heads = c.heads; a.window = window; a.err = err;
    int n_tiles = L.tiles128;
    if (gathered) {
      a.q_index = indices; a.q_per_row = L.k + 1; a.q_tiles = (L.k + 1 + kTcQ - 1) / kTcQ;
      n_tiles = L.b * a.q_tiles;
    }
    a.splits = attention_splits(c.heads, n_tiles, e.sms, window, m / L.b);
    launch(e, prof, FAM_ATTENTION, 0, [&] { launch_tc_attention<T>(s.attn_maps, a, n_tiles, e.stream, e.sms); });
  };
  // A residual GEMM whose sum the next norm must still add: split count and the GEMM bias.
  struct Pending { int splits = 0; const float* bias = nullptr; };
  auto norm = [&](float* res, int rows, const float* g, const float* b, float eps, T* out, Pending pend) {
    NormArgs a{};
    a.residual = res; a.partials = pend.splits ? partials : nullptr; a.splits = pend.splits;
    a.partial_bias = pend.bias;
    a.gamma1 = g; a.beta1 = b; a.eps1 = eps; a.fused_final = 0;
    a.x = out; a.rows = rows; a.d = d;
    launch(e, prof, FAM_ROWS, 0, [&] { launch_norm<T>(a, e.stream); });
  };
  // residual += A W^T + bias: the fused residual epilogue, or, for small classes, split-K
  // partials that the following norm adds.
  auto residual_gemm = [&](int family, const CUtensorMap& ta, const std::string& wname, int rows, float* res,
                           const float* bias) -> Pending {
    const Tensor& w = W(e, wname);
    const int N = (int)w.shape[0], K = (int)w.shape[1];
    if (partials && rows <= kSplitRowsMax && N == d) {
      const TilePlan plan = plan_small(rows, N, K, EPI_PARTIAL, true, false, e.sms);
      if (plan.splits > 1) {
        gemm_partial<T>(e, prof, family, ta, wname, rows, plan.splits, plan.bn, partials, err);
        return Pending{plan.splits, bias};
      }
    }
    gemm<T>(e, prof, family, EPI_RESIDUAL, ta, wname, rows, nullptr, 0, res, d, bias, err);
    return Pending{};
  };

  // residual += A W^T + bias, then x = LN(residual): one fused kernel when the class does not
  // split K, else the residual GEMM (or its split-K partials) followed by the norm kernel.
  auto residual_ln = [&](int family, const CUtensorMap& ta, const std::string& wname, const float* bias,
                         const float* gamma, const float* beta, float eps) {
    const Tensor& w = W(e, wname);
    const int bn = ln_block_n((int)w.shape[0], (int)w.shape[1]);
    if (!bn || m <= kSplitRowsMax || w.shape[1] > kLnMaxK) {
      const Pending pend = residual_gemm(family, ta, wname, m, residual, bias);
      norm(residual, m, gamma, beta, eps, x, pend);
      return;
    }
    GemmLnArgs a{};
    a.M = m; a.N = (int)w.shape[0]; a.K = (int)w.shape[1];
    a.residual = residual; a.ldr = d; a.bias = bias; a.gamma = gamma; a.beta = beta; a.eps = eps;
    a.x = x; a.ldx = d; a.err = err;
    const CUtensorMap tb = weight_map(e, wname, bn);
    launch(e, prof, family, 2.0 * m * a.N * a.K, [&] { launch_gemm_ln<T>(ta, tb, s.map_residual, a, bn, e.stream); });
  };

  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    const bool local = i % c.global_every != 0;
    gemm<T>(e, prof, FAM_GEMM_QKV, EPI_QKV, s.map_x, p + "attn.Wqkv.weight", m, qkv, 0, nullptr, 0, nullptr, err, local ? 1 : 0, positions);
    attention(local ? c.window : -1, false);
    residual_ln(FAM_GEMM_ATTN_OUT, s.map_attn, p + "attn.Wo.weight", nullptr, Wf(e, p + "mlp_norm.weight"), nullptr,
                c.eps);
    gemm<T>(e, prof, FAM_GEMM_FFN_UP, EPI_GEGLU, s.map_x, p + "mlp.Wi.weight", m, ff, e.F(), nullptr, 0, nullptr, err);
    if (i + 1 < c.layers) {
      residual_ln(FAM_GEMM_FFN_DOWN, s.map_ff, p + "mlp.Wo.weight", nullptr,
                  Wf(e, "encoder.layers." + std::to_string(i + 1) + ".attn_norm.weight"), nullptr, c.eps);
    } else {
      const Pending pend = residual_gemm(FAM_GEMM_FFN_DOWN, s.map_ff, p + "mlp.Wo.weight", m, residual, nullptr);
      // encoder.final_norm -> residual; residual += type_emb[kind]; x = head.layers.0.norm1(residual)
      NormArgs a{};
      a.residual = residual;
      a.partials = pend.splits ? partials : nullptr; a.splits = pend.splits; a.partial_bias = pend.bias;
      a.gamma1 = Wf(e, "encoder.final_norm.weight"); a.beta1 = nullptr; a.eps1 = c.eps;
      a.fused_final = 1; a.type_emb = Wf(e, "type_emb.weight"); a.kinds = kinds;
      a.gamma2 = Wf(e, "head.layers.0.norm1.weight"); a.beta2 = Wf(e, "head.layers.0.norm1.bias"); a.eps2 = 1e-5f;
      a.x = x; a.rows = m; a.d = d;
      launch(e, prof, FAM_ROWS, 0, [&] { launch_norm<T>(a, e.stream); });
    }
  }

  Pending head_pend;
  for (int i = 0; i < c.head_layers; ++i) {
    const std::string p = "head.layers." + std::to_string(i) + ".";
    if (i > 0) norm(residual, m, Wf(e, p + "norm1.weight"), Wf(e, p + "norm1.bias"), 1e-5f, x, Pending{});
    gemm<T>(e, prof, FAM_GEMM_HEAD, EPI_QKV, s.map_x, p + "self_attn.in_proj_weight", m, qkv, 0, nullptr, 0,
            Wf(e, p + "self_attn.in_proj_bias"), err);
    // The last head layer only needs the attention rows that are gathered next.
    attention(-1, i + 1 == c.head_layers);
    if (i + 1 == c.head_layers) {
      launch(e, prof, FAM_ROWS, 0, [&] {
        launch_k(gather_rows_kernel<T>, dim3(count), dim3(256), 0, e.stream, (const float*)residual, (const T*)attn,
                 indices, count, d, m, sel, scored, err);
      });
      Pending pend = residual_gemm(FAM_GEMM_HEAD, s.map_scored, p + "self_attn.out_proj.weight", count, sel,
                                   Wf(e, p + "self_attn.out_proj.bias"));
      norm(sel, count, Wf(e, p + "norm2.weight"), Wf(e, p + "norm2.bias"), 1e-5f, selx, pend);
      gemm<T>(e, prof, FAM_GEMM_HEAD, EPI_RELU, s.map_selx, p + "linear1.weight", count, ffsel, 4 * d, nullptr, 0,
              Wf(e, p + "linear1.bias"), err);
      head_pend = residual_gemm(FAM_GEMM_HEAD, s.map_ffsel, p + "linear2.weight", count, sel, Wf(e, p + "linear2.bias"));
    } else {
      Pending pend = residual_gemm(FAM_GEMM_HEAD, s.map_attn, p + "self_attn.out_proj.weight", m, residual,
                                   Wf(e, p + "self_attn.out_proj.bias"));
      norm(residual, m, Wf(e, p + "norm2.weight"), Wf(e, p + "norm2.bias"), 1e-5f, x, pend);
      gemm<T>(e, prof, FAM_GEMM_HEAD, EPI_RELU, s.map_x, p + "linear1.weight", m, ff, 4 * d, nullptr, 0, Wf(e, p + "linear1.bias"), err);
      const CUtensorMap ffmap = make_map(ff, m, 4 * d, kBM, e.bf16());
      // The next head layer's norm1 reads the residual directly, so this GEMM never splits.
      gemm<T>(e, prof, FAM_GEMM_HEAD, EPI_RESIDUAL, ffmap, p + "linear2.weight", m, nullptr, 0, residual, d,
              Wf(e, p + "linear2.bias"), err);
    }
  }
  norm(sel, count, Wf(e, "scorer.0.weight"), Wf(e, "scorer.0.bias"), 1e-5f, selx, head_pend);
  gemm<T>(e, prof, FAM_GEMM_HEAD, EPI_GELU, s.map_selx, "scorer.1.weight", count, scored, d, nullptr, 0, Wf(e, "scorer.1.bias"), err);
  TailArgs t{};
  t.selected = sel; t.scored = scored; t.counts = counts;
  t.w3 = Wf(e, "scorer.3.weight"); t.b3 = Wf(e, "scorer.3.bias");
  t.wa0 = Wf(e, "act_head.0.weight"); t.ba0 = Wf(e, "act_head.0.bias");
  t.wa2 = Wf(e, "act_head.2.weight"); t.ba2 = Wf(e, "act_head.2.bias");
  t.logits = logits; t.acts = acts; t.k = L.k; t.d = d; t.n_act = c.n_act;
  t.hidden = reinterpret_cast<float*>(ws + L.hidden); t.arrivals = arrivals;
  const size_t tail_smem = ((size_t)(L.k + 1) + d + 4 + kActHidden) * sizeof(float);
  launch(e, prof, FAM_HEAD_TAIL, 0, [&] {
    const int parts = L.b * kTailPartsSmall <= 4 * e.sms ? kTailPartsSmall : kTailPartsLarge;
    launch_k(head_tail_kernel<T>, dim3(L.b, parts), dim3(kTailThreads), tail_smem, e.stream, t);
  });
}

void forward(Engine& e, Slot& s, bool prof) {
  if (e.bf16()) enqueue_forward<__nv_bfloat16>(e, s, prof);
  else enqueue_forward<__half>(e, s, prof);
}

// The slot of a class.  Graph runs use the LRU (inserting, and evicting the least recently
// used class when full); eager runs use a cached slot when there is one and otherwise a
// transient slot that is not cached, so large one-off classes never evict graphs.
Slot& get_slot(Engine& e, int m, int b, int k, bool cache, bool& miss, std::unique_ptr<Slot>& transient) {
  auto key = std::make_tuple(m, b, k);
  auto it = e.slots.find(key);
  miss = it == e.slots.end();
  if (miss && !cache) {
    transient = std::make_unique<Slot>();
    transient->m = m; transient->b = b; transient->k = k;
    transient->L = make_layout(e, m, b, k);
    return *transient;
  }
  if (miss) {
    if ((int)e.slots.size() >= e.limit) {
      CK(cudaStreamSynchronize(e.stream));
      auto victim = e.lru.front();
      e.lru.pop_front();
      auto& vs = e.slots[victim];
      if (vs->graph) cudaGraphExecDestroy(vs->graph);
      e.slots.erase(victim);
    }
    auto s = std::make_unique<Slot>();
    s->m = m; s->b = b; s->k = k;
    s->L = make_layout(e, m, b, k);
    it = e.slots.emplace(key, std::move(s)).first;
  } else {
    e.lru.remove(key);
  }
  e.lru.push_back(key);
  return *it->second;
}

// Capture modes of laya_predict / laya_forward_device: 0 eager, 1 graph, 2 auto.
bool wants_graph(int capture, int rows) { return capture == 1 || (capture == 2 && rows <= kAutoGraphRows); }

// Runs one pass of slot `s` whose inputs are already in the workspace.  Returns the launch count.
int run_slot(Engine& e, Slot& s, bool capture, bool& captured) {
  captured = false;
  prepare_maps(e, s);
  if (capture) {
    if (!s.graph) {
      cudaGraph_t g = nullptr;
      const int before = e.launches;
      CK(cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal));
      try {
        forward(e, s, false);
      } catch (...) {
        cudaStreamEndCapture(e.stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      CK(cudaStreamEndCapture(e.stream, &g));
      cudaError_t r = cudaGraphInstantiate(&s.graph, g, 0);
      cudaGraphDestroy(g);
      if (r != cudaSuccess) { s.graph = nullptr; fail(LAYA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(r)); }
      s.launches = e.launches - before;
      e.launches = before;
      captured = true;
    }
    CK(cudaGraphLaunch(s.graph, e.stream));
    return s.launches;
  }
  const int before = e.launches;
  forward(e, s, e.profiling);
  return e.launches - before;
}

}  // namespace

struct laya_engine {
  Engine impl;
};

namespace {
int finish_error(laya_engine* h, const Failure& f) {
  if (h) h->impl.error = f.msg;
  else g_create_error = f.msg;
  return f.code;
}
}  // namespace

#define API_BEGIN try {
#define API_END(h)                                                   \
  }                                                                  \
  catch (const Failure& f) { return finish_error(h, f); }            \
  catch (const std::exception& x) { return finish_error(h, Failure{LAYA_ERR_CUDA, x.what()}); } \
  return LAYA_OK;

extern "C" {

int laya_create(const laya_config* cfg, int device, int max_cached_shapes, laya_engine** out) {
  API_BEGIN
  if (!cfg || !out) fail(LAYA_ERR_INVALID, "null argument");
  *out = nullptr;
  const laya_config& c = *cfg;
  if (c.width <= 0 || c.width % 64 || c.width > 1024 || c.heads * 64 != c.width)
    fail(LAYA_ERR_INVALID, "width must be heads x 64 and at most 1024");
  if (c.layers <= 0 || c.intermediate <= 0 || c.intermediate % 64 || c.global_every <= 0 || c.window < 0)
    fail(LAYA_ERR_INVALID, "invalid encoder geometry");
  if (c.max_len <= 0 || c.max_len > 1024 || c.head_layers < 1 || c.n_act < 1 || c.n_act > 64 || c.vocab <= 0)
    fail(LAYA_ERR_INVALID, "invalid context budget or decision head");
  if (c.precision != LAYA_PRECISION_BF16 && c.precision != LAYA_PRECISION_F16) fail(LAYA_ERR_INVALID, "bad precision");
  if (max_cached_shapes < 1 || max_cached_shapes > 64) fail(LAYA_ERR_INVALID, "max_cached_shapes must be 1..64");
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) fail(LAYA_ERR_NO_DEVICE, "no CUDA device");
  if (device < 0 || device >= n) fail(LAYA_ERR_NO_DEVICE, "device %d not present", device);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) fail(LAYA_ERR_NO_DEVICE, "%s is sm_%d%d; this build targets sm_100a (B200)", prop.name, prop.major, prop.minor);
  CK(cudaSetDevice(device));
  auto h = std::make_unique<laya_engine>();
  Engine& e = h->impl;
  e.cfg = c;
  e.device = device;
  e.limit = max_cached_shapes;
  e.sms = sm_count(device);
  build_expected(e);
  CK(cudaStreamCreateWithFlags(&e.stream, cudaStreamNonBlocking));

  *out = h.release();
  API_END(nullptr)
}

int laya_load_tensor(laya_engine* h, const char* name, int dtype, const int64_t* shape, int ndim, const void* host) {
  API_BEGIN
  if (!h || !name || !host || (ndim > 0 && !shape)) fail(LAYA_ERR_INVALID, "null argument");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  auto it = e.expected.find(name);
  if (it == e.expected.end()) fail(LAYA_ERR_INVALID, "Checkpoint tensor names do not match the Laya adapter: %s", name);
  std::vector<int64_t> sh(shape, shape + ndim);
  if (sh != it->second) fail(LAYA_ERR_INVALID, "Incompatible tensor shape: %s", name);
  if (std::string(name) == "temperature") return LAYA_OK;
  int64_t count = 1;
  for (auto v : sh) count *= v;
  std::vector<float> vals((size_t)count);
  if (dtype == LAYA_DTYPE_F32) memcpy(vals.data(), host, (size_t)count * 4);
  else if (dtype == LAYA_DTYPE_F16 || dtype == LAYA_DTYPE_BF16) {
    const uint16_t* s = static_cast<const uint16_t*>(host);
    for (int64_t i = 0; i < count; ++i) vals[i] = half_bits_to_float(s[i], dtype == LAYA_DTYPE_BF16);
  } else fail(LAYA_ERR_INVALID, "unsupported dtype %d", dtype);
  Tensor t;
  t.shape = sh;
  const std::string n(name);
  const bool is16 = stored_16bit(n);
  std::vector<uint16_t> packed;
  const void* src = vals.data();
  if (is16) {
    packed.resize((size_t)count);
    const bool geglu = n.find("mlp.Wi.weight") != std::string::npos;
    if (geglu) {
      // Interleave gate/up rows in 64-row blocks so one column tile holds matching pairs.
      const int64_t F = sh[0] / 2, K = sh[1];
      for (int64_t blk = 0; blk < F / 64; ++blk)
        for (int half = 0; half < 2; ++half)
          for (int64_t r = 0; r < 64; ++r) {
            const int64_t src_row = half * F + blk * 64 + r, dst_row = blk * 128 + half * 64 + r;
            for (int64_t c = 0; c < K; ++c) packed[dst_row * K + c] = float_to_half_bits(vals[src_row * K + c], e.bf16());
          }
    } else {
      for (int64_t i = 0; i < count; ++i) packed[i] = float_to_half_bits(vals[i], e.bf16());
    }
    src = packed.data();
    t.dtype = e.bf16() ? LAYA_DTYPE_BF16 : LAYA_DTYPE_F16;
    t.bytes = (size_t)count * 2;
  } else {
    t.dtype = LAYA_DTYPE_F32;
    t.bytes = (size_t)count * 4;
  }
  auto old = e.weights.find(n);
  if (old != e.weights.end() && old->second.ptr) {
    if (!old->second.arena) CK(cudaFree(old->second.ptr));
    e.wmaps.clear();
  }
  t.ptr = dev_alloc(t.bytes);
  CK(cudaMemcpy(t.ptr, src, t.bytes, cudaMemcpyHostToDevice));
  e.weights[n] = t;
  e.finalized = false;
  API_END(h)
}

int laya_scan_checkpoint(const char* path, int64_t* tensors, int64_t* elements) {
  API_BEGIN
  if (!path || !tensors || !elements) fail(LAYA_ERR_INVALID, "null argument");
  Checkpoint ck;
  open_checkpoint(path, ck);
  int64_t n = 0;
  for (auto& kv : ck.entries) {
    int64_t c = 1;
    for (int64_t v : kv.second.shape) c *= v;
    n += c;
  }
  *tensors = (int64_t)ck.entries.size();
  *elements = n;
  API_END(nullptr)
}

int laya_load_checkpoint(laya_engine* h, const char* path) {
  API_BEGIN
  if (!h || !path) fail(LAYA_ERR_INVALID, "null argument");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  load_checkpoint(e, path);
  API_END(h)
}

int laya_finalize(laya_engine* h) {
  API_BEGIN
  if (!h) fail(LAYA_ERR_INVALID, "null engine");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  for (auto& kv : e.expected)
    if (kv.first != "temperature" && !e.weights.count(kv.first)) fail(LAYA_ERR_INVALID, "missing tensor %s", kv.first.c_str());
  if (e.F() % 64) fail(LAYA_ERR_INVALID, "intermediate size must be a multiple of 64");
  // RoPE tables cover every position a packed row can hold (runtime.py:159-165):
  // freq_j = 1 / theta^(2j/64) in fp32, angle = pos * freq_j in fp32.
  e.rope_rows = span16(e.cfg.max_len);
  const float thetas[2] = {e.cfg.theta_global, e.cfg.theta_local};
  for (int t = 0; t < 2; ++t) {
    // [16][rope_rows] x (cos f_2k, cos f_2k+1, sin f_2k, sin f_2k+1): see GemmArgs::rope_tab.
    std::vector<float> tab((size_t)e.rope_rows * 64);
    for (int j = 0; j < 32; ++j) {
      const float expo = (float)(2 * j) / 64.0f;
      const float freq = 1.0f / powf(thetas[t], expo);
      for (int pos = 0; pos < e.rope_rows; ++pos) {
        const float angle = (float)pos * freq;
        float* q = &tab[((size_t)(j >> 1) * e.rope_rows + pos) * 4];
        q[j & 1] = (float)cos((double)angle);
        q[2 + (j & 1)] = (float)sin((double)angle);
      }
    }
    if (e.rope_tab[t]) cudaFree(e.rope_tab[t]);
    e.rope_tab[t] = static_cast<float4*>(dev_alloc(tab.size() * 4));
    CK(cudaMemcpy(e.rope_tab[t], tab.data(), tab.size() * 4, cudaMemcpyHostToDevice));
  }
  drop_graphs(e);
  e.finalized = true;
  API_END(h)
}

int laya_shape_class(const int32_t* lengths, const int32_t* marker_counts, int n_items, int32_t* rows, int32_t* batch,
                     int32_t* options) {
  API_BEGIN
  int m, b, k;
  shape_class(lengths, marker_counts, n_items, m, b, k);
  *rows = m; *batch = b; *options = k;
  API_END(nullptr)
}

int64_t laya_packed_ints(int rows, int batch, int options) { return pack_layout(rows, batch, options).total; }

int laya_pack(const int32_t* tokens, const int32_t* lengths, const int32_t* markers, const int32_t* marker_counts,
              const int32_t* kinds, int n_items, int pad_id, int rows, int batch, int options, int32_t* packed) {
  API_BEGIN
  if (n_items > batch) fail(LAYA_ERR_INVALID, "more items than the batch class");
  pack(tokens, lengths, markers, marker_counts, kinds, n_items, pad_id, rows, batch, options, 1024, packed);
  API_END(nullptr)
}

namespace {
// Packs the items into a free in-flight record, enqueues H2D, the forward pass and D2H on the
// engine stream, and returns the record's ticket.  Nothing here waits for the GPU except a
// workspace growth or a graph eviction (both synchronise the stream first).
int64_t submit(Engine& e, const int32_t* tokens, const int32_t* lengths, const int32_t* markers,
               const int32_t* marker_counts, const int32_t* kinds, int n_items, int capture) {
  if (!e.finalized) fail(LAYA_ERR_STATE, "engine not finalised");
  if (!tokens || !lengths || !marker_counts || !kinds) fail(LAYA_ERR_INVALID, "null argument");
  Inflight* r = !e.inflight[0].busy ? &e.inflight[0] : !e.inflight[1].busy ? &e.inflight[1] : nullptr;
  if (!r) fail(LAYA_ERR_STATE, "two passes are in flight: collect one first");
  CK(cudaSetDevice(e.device));
  int m, b, k;
  shape_class(lengths, marker_counts, n_items, m, b, k);
  const bool graph = wants_graph(capture, m);
  bool miss = false;
  std::unique_ptr<Slot> transient;  // launches copy everything they need; safe to drop after enqueue
  Slot& s = get_slot(e, m, b, k, graph, miss, transient);
  ensure_workspace(e, s.L.total);
  ensure_host(*r, (size_t)s.L.pack.total, s.L.n_out_floats);
  if (!r->done) {
    CK(cudaEventCreate(&r->ev_start));
    CK(cudaEventCreate(&r->ev_end));
    CK(cudaEventCreateWithFlags(&r->done, cudaEventDisableTiming));
  }
  // The pad id is the tokenizer's [PAD]; padded positions are never attended by real tokens.
  pack(tokens, lengths, markers, marker_counts, kinds, n_items, 0, m, b, k, e.cfg.max_len, r->h_packed);
  CK(cudaMemcpyAsync(e.ws + s.L.packed, r->h_packed, (size_t)s.L.pack.total * 4, cudaMemcpyHostToDevice, e.stream));
  bool captured = false;
  CK(cudaEventRecord(r->ev_start, e.stream));
  r->launches = run_slot(e, s, graph, captured);
  CK(cudaEventRecord(r->ev_end, e.stream));
  CK(cudaMemcpyAsync(r->h_out, e.ws + s.L.out, s.L.n_out_floats * 4, cudaMemcpyDeviceToHost, e.stream));
  CK(cudaEventRecord(r->done, e.stream));
  r->busy = true;
  r->ticket = e.next_ticket++;
  r->n_items = n_items; r->m = m; r->b = b; r->k = k;
  r->n_out_floats = s.L.n_out_floats;
  r->miss = miss; r->captured = captured; r->replay = graph && s.graph != nullptr;
  return r->ticket;
}

// Waits for the pass of `ticket` and copies its outputs: logits [n_items][k] (options of the
// class; the CLS slot is dropped) and acts [n_items][n_act].
void collect(Engine& e, int64_t ticket, float* logits_out, float* acts_out, laya_metrics* metrics) {
  Inflight* r = nullptr;
  for (auto& x : e.inflight)
    if (x.busy && x.ticket == ticket) r = &x;
  if (!r) fail(LAYA_ERR_INVALID, "no pass in flight with ticket %lld", (long long)ticket);
  CK(cudaSetDevice(e.device));
  const cudaError_t sync = cudaEventSynchronize(r->done);
  r->busy = false;
  if (sync != cudaSuccess) fail(LAYA_ERR_CUDA, "forward pass: %s", cudaGetErrorString(sync));
  prof_resolve(e);
  const int b = r->b, k = r->k;
  const float* outf = r->h_out;
  const int errword = *reinterpret_cast<const int*>(outf + (size_t)b * (k + 1) + (size_t)b * e.cfg.n_act);
  if (errword) fail(LAYA_ERR_DEVICE, "device error %d during the forward pass", errword);
  if (logits_out && acts_out) {
    for (int i = 0; i < r->n_items; ++i) {
      memcpy(logits_out + (size_t)i * k, outf + (size_t)i * (k + 1) + 1, (size_t)k * 4);
      memcpy(acts_out + (size_t)i * e.cfg.n_act, outf + (size_t)b * (k + 1) + (size_t)i * e.cfg.n_act,
             (size_t)e.cfg.n_act * 4);
    }
  }
  if (metrics) {
    float ms = 0;
    CK(cudaEventElapsedTime(&ms, r->ev_start, r->ev_end));
    metrics->gpu_ms = ms;
    metrics->rows = r->m; metrics->batch = b; metrics->options = k;
    metrics->cache_miss = r->miss;
    metrics->graph_capture = r->captured;
    metrics->graph_replay = r->replay;
    metrics->kernel_launches = r->launches;
    metrics->owned_gpu_bytes = e.owned();
  }
}
}  // namespace

int laya_predict(laya_engine* h, const int32_t* tokens, const int32_t* lengths, const int32_t* markers,
                 const int32_t* marker_counts, const int32_t* kinds, int n_items, int capture, float* logits_out,
                 float* acts_out, laya_metrics* metrics) {
  API_BEGIN
  if (!h) fail(LAYA_ERR_INVALID, "null engine");
  if (!logits_out || !acts_out) fail(LAYA_ERR_INVALID, "null argument");
  Engine& e = h->impl;
  const int64_t ticket = submit(e, tokens, lengths, markers, marker_counts, kinds, n_items, capture);
  collect(e, ticket, logits_out, acts_out, metrics);
  API_END(h)
}

int laya_submit(laya_engine* h, const int32_t* tokens, const int32_t* lengths, const int32_t* markers,
                const int32_t* marker_counts, const int32_t* kinds, int n_items, int capture, int64_t* ticket) {
  API_BEGIN
  if (!h || !ticket) fail(LAYA_ERR_INVALID, "null argument");
  *ticket = submit(h->impl, tokens, lengths, markers, marker_counts, kinds, n_items, capture);
  API_END(h)
}

int laya_collect(laya_engine* h, int64_t ticket, float* logits_out, float* acts_out, laya_metrics* metrics) {
  API_BEGIN
  if (!h || !logits_out || !acts_out) fail(LAYA_ERR_INVALID, "null argument");
  collect(h->impl, ticket, logits_out, acts_out, metrics);
  API_END(h)
}

int laya_forward_device(laya_engine* h, const int32_t* packed, int rows, int batch, int options, int capture,
                        float* logits_dev, float* acts_dev) {
  API_BEGIN
  if (!h || !packed) fail(LAYA_ERR_INVALID, "null argument");
  Engine& e = h->impl;
  if (!e.finalized) fail(LAYA_ERR_STATE, "engine not finalised");
  CK(cudaSetDevice(e.device));
  const bool graph = wants_graph(capture, rows);
  bool miss = false;
  std::unique_ptr<Slot> transient;
  Slot& s = get_slot(e, rows, batch, options, graph, miss, transient);
  ensure_workspace(e, s.L.total);
  CK(cudaMemcpyAsync(e.ws + s.L.packed, packed, (size_t)s.L.pack.total * 4, cudaMemcpyDeviceToDevice, e.stream));
  bool captured = false;
  run_slot(e, s, graph, captured);
  const float* outf = reinterpret_cast<const float*>(e.ws + s.L.out);
  if (logits_dev)
    CK(cudaMemcpyAsync(logits_dev, outf, (size_t)batch * (options + 1) * 4, cudaMemcpyDeviceToDevice, e.stream));
  if (acts_dev)
    CK(cudaMemcpyAsync(acts_dev, outf + (size_t)batch * (options + 1), (size_t)batch * e.cfg.n_act * 4,
                       cudaMemcpyDeviceToDevice, e.stream));
  API_END(h)
}

int laya_reserve(laya_engine* h, int rows, int batch, int options) {
  API_BEGIN
  if (!h || rows <= 0 || batch <= 0 || options <= 0) fail(LAYA_ERR_INVALID, "bad reservation");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  ensure_workspace(e, make_layout(e, rows, batch, options).total);
  API_END(h)
}

void* laya_stream(laya_engine* h) { return h ? (void*)h->impl.stream : nullptr; }

int laya_set_profiling(laya_engine* h, int enabled) {
  API_BEGIN
  if (!h) fail(LAYA_ERR_INVALID, "null engine");
  h->impl.profiling = enabled != 0;
  API_END(h)
}

int laya_profile_read(laya_engine* h, int family, double* total_ms, int64_t* launches, double* flops) {
  API_BEGIN
  if (!h || family < 0 || family >= kFamilies) fail(LAYA_ERR_INVALID, "bad profile family");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  prof_resolve(e);
  if (total_ms) *total_ms = e.prof_ms[family];
  if (launches) *launches = e.prof_launches[family];
  if (flops) *flops = e.prof_flops[family];
  API_END(h)
}

int laya_read_tensor(laya_engine* h, const char* name, float* out, int64_t count) {
  API_BEGIN
  if (!h || !name || !out) fail(LAYA_ERR_INVALID, "null argument");
  Engine& e = h->impl;
  CK(cudaSetDevice(e.device));
  auto it = e.weights.find(name);
  if (it == e.weights.end()) fail(LAYA_ERR_INVALID, "tensor %s not loaded", name);
  const Tensor& t = it->second;
  int64_t n = 1;
  for (auto v : t.shape) n *= v;
  if (count != n) fail(LAYA_ERR_INVALID, "tensor %s has %lld values", name, (long long)n);
  if (t.dtype == LAYA_DTYPE_F32) {
    CK(cudaMemcpy(out, t.ptr, (size_t)n * 4, cudaMemcpyDeviceToHost));
  } else {
    std::vector<uint16_t> tmp((size_t)n);
    CK(cudaMemcpy(tmp.data(), t.ptr, (size_t)n * 2, cudaMemcpyDeviceToHost));
    const bool geglu = std::string(name).find("mlp.Wi.weight") != std::string::npos;
    const int64_t K = t.shape.size() > 1 ? t.shape[1] : 1, F = t.shape[0] / 2;
    for (int64_t i = 0; i < n; ++i) {
      int64_t src = i;
      if (geglu) {  // undo the gate/up interleave
        const int64_t row = i / K, c = i % K, half = row / F, r = row % F;
        src = ((r / 64) * 128 + half * 64 + r % 64) * K + c;
      }
      out[i] = half_bits_to_float(tmp[(size_t)src], t.dtype == LAYA_DTYPE_BF16);
    }
  }
  API_END(h)
}

int laya_cached_shapes(laya_engine* h, int32_t* count) {
  API_BEGIN
  if (!h || !count) fail(LAYA_ERR_INVALID, "null argument");
  *count = (int32_t)h->impl.slots.size();
  API_END(h)
}

int laya_pool_bytes(laya_engine* h, uint64_t* used, uint64_t* total) {
  API_BEGIN
  if (!h) fail(LAYA_ERR_INVALID, "null engine");
  const uint64_t v = h->impl.owned();
  if (used) *used = v;
  if (total) *total = v;
  API_END(h)
}

int laya_destroy(laya_engine* h) {
  if (!h) return LAYA_OK;
  Engine& e = h->impl;
  int rc = LAYA_OK;
  if (cudaSetDevice(e.device) != cudaSuccess) rc = LAYA_ERR_CUDA;
  if (e.stream) cudaStreamSynchronize(e.stream);
  for (auto& kv : e.slots)
    if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
  e.slots.clear();
  for (auto& kv : e.weights)
    if (kv.second.ptr && !kv.second.arena) cudaFree(kv.second.ptr);
  e.weights.clear();
  for (int i = 0; i < 2; ++i) {
    if (e.rope_tab[i]) cudaFree(e.rope_tab[i]);
  }
  if (e.ws) cudaFree(e.ws);
  if (e.arena) cudaFree(e.arena);
  for (auto& r : e.inflight) {
    if (r.h_packed) cudaFreeHost(r.h_packed);
    if (r.h_out) cudaFreeHost(r.h_out);
    if (r.ev_start) cudaEventDestroy(r.ev_start);
    if (r.ev_end) cudaEventDestroy(r.ev_end);
    if (r.done) cudaEventDestroy(r.done);
  }
  for (auto& p : e.prof_pending) { cudaEventDestroy(p.a); cudaEventDestroy(p.b); }
  for (auto ev : e.prof_pool) cudaEventDestroy(ev);

  if (e.stream) cudaStreamDestroy(e.stream);
  delete h;
  return rc;
}

const char* laya_last_error(laya_engine* h) { return h ? h->impl.error.c_str() : g_create_error.c_str(); }

int laya_set_launch_options(int programmatic_launch, uint64_t wait_limit_ns) {
  if (programmatic_launch != 0 && programmatic_launch != 1) return LAYA_ERR_INVALID;
  g_pdl.store(programmatic_launch != 0);
  g_wait_ns.store(wait_limit_ns);
  return LAYA_OK;
}

// ---------------------------------------------------------------------------------------------
// Kernel-level entry points
// ---------------------------------------------------------------------------------------------
int laya_op_gemm(int precision, int epi, const void* x, const void* w, int M, int N, int K, void* out, int ldo,
                 float* residual, int ldr, const float* bias, int heads, const float* rope_tab, int rope_rows,
                 const int32_t* positions, int splits, int block_n, int* err, void* stream) {
  API_BEGIN
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const int sms = sm_count(dev);
  const bool bf = precision == LAYA_PRECISION_BF16;
  if (splits < 1) splits = 1;
  // block_n < 0 selects the CTA-pair kernel with |block_n| columns per tile.
  const bool pair = block_n < 0;
  const int bn = block_n > 0 ? block_n : block_n < 0 ? -block_n : pick_bn(M, N, epi, sms);
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.splits = splits;
  a.out = out; a.ldo = ldo; a.residual = residual; a.ldr = ldr; a.bias = bias;
  a.heads = heads; a.rope_tab = reinterpret_cast<const float4*>(rope_tab); a.rope_rows = rope_rows;
  a.positions = positions;
  if (rope_tab && (reinterpret_cast<uintptr_t>(rope_tab) & 15)) fail(LAYA_ERR_INVALID, "rope_tab must be 16-byte aligned");
  a.err = err;
  const CUtensorMap ta = make_map(x, M, K, kBM, bf);
  const CUtensorMap tb = make_map(w, N, K, pair ? bn / 2 : bn, bf);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf) launch_gemm<__nv_bfloat16>(epi, bn, ta, tb, a, sms, st, pair);
  else launch_gemm<__half>(epi, bn, ta, tb, a, sms, st, pair);
  API_END(nullptr)
}

int laya_op_gemm_ln(int precision, const void* x, const void* w, int M, int N, int K, float* residual, int ldr,
                    const float* bias, const float* gamma, const float* beta, float eps, void* out, int ldo, int* err,
                    void* stream) {
  API_BEGIN
  if (!residual || !gamma || !out) fail(LAYA_ERR_INVALID, "null argument");
  const bool bf = precision == LAYA_PRECISION_BF16;
  GemmLnArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.residual = residual; a.ldr = ldr; a.bias = bias; a.gamma = gamma; a.beta = beta; a.eps = eps;
  a.x = out; a.ldx = ldo; a.err = err;
  const CUtensorMap ta = make_map(x, M, K, kBM, bf);
  const int bn = ln_block_n(N, K);
  if (!bn) fail(LAYA_ERR_INVALID, "fused residual + LayerNorm: N=%d is not 1-4 blocks of 192 or 256 columns", N);
  const CUtensorMap tb = make_map(w, N, K, bn, bf);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const CUtensorMap tr = make_map_f32(residual, M, N, ldr);
  if (bf) launch_gemm_ln<__nv_bfloat16>(ta, tb, tr, a, bn, st);
  else launch_gemm_ln<__half>(ta, tb, tr, a, bn, st);
  API_END(nullptr)
}

int laya_interleave_geglu(const uint16_t* src, uint16_t* dst, int F, int K) {
  API_BEGIN
  if (F % 64) fail(LAYA_ERR_INVALID, "F must be a multiple of 64");
  for (int blk = 0; blk < F / 64; ++blk)
    for (int half = 0; half < 2; ++half)
      for (int r = 0; r < 64; ++r)
        memcpy(dst + ((size_t)blk * 128 + half * 64 + r) * K, src + ((size_t)half * F + blk * 64 + r) * K, (size_t)K * 2);
  API_END(nullptr)
}

int laya_attention_tiles(const int32_t* starts, const int32_t* lengths, int n_rows, int M, int tile_q, int32_t* tiles,
                         int capacity) {
  if (tile_q != kTcQ) return -1;
  return build_tiles(starts, lengths, n_rows, M, tile_q, tiles, capacity);
}

int laya_op_attention(int precision, int impl, const void* qkv, void* out, const int32_t* tiles, int n_tiles,
                      const int32_t* starts, const int32_t* lengths, int M, int heads, int window, int* err,
                      void* stream) {
  API_BEGIN
  if (impl < 1 || impl > 6)
    fail(LAYA_ERR_INVALID,
         "attention impl %d (1: forward-pass rule, 2: no key split, 3: 2-way, 4: 4-way key split, 5: one tile per "
         "CTA, 6: persistent, fewest CTAs)", impl);
  const bool bf = precision == LAYA_PRECISION_BF16;
  const AttnMaps maps = attn_maps(qkv, M, heads, bf);
  TcAttnArgs t{};
  t.qk = qkv; t.out = out; t.tiles = reinterpret_cast<const int4*>(tiles); t.starts = starts; t.lengths = lengths;
  t.M = M; t.heads = heads; t.window = window; t.err = err;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  t.splits = impl == 2 || impl >= 5 ? 1 : impl == 3 ? 2 : impl == 4 ? 4 : attention_splits(heads, n_tiles, sm_count(dev), window, M);
  const int mode = impl == 5 ? 0 : impl == 6 ? 2 : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf) launch_tc_attention<__nv_bfloat16>(maps, t, n_tiles, st, sm_count(dev), mode);
  else launch_tc_attention<__half>(maps, t, n_tiles, st, sm_count(dev), mode);
  API_END(nullptr)
}

int laya_op_attention_gathered(int precision, const void* qkv, void* out, const int32_t* q_index, int q_per_row,
                               const int32_t* starts, const int32_t* lengths, int n_rows, int M, int heads, int* err,
                               void* stream) {
  API_BEGIN
  if (q_per_row <= 0 || n_rows <= 0) fail(LAYA_ERR_INVALID, "gathered attention needs rows and queries");
  const bool bf = precision == LAYA_PRECISION_BF16;
  const AttnMaps maps = attn_maps(qkv, M, heads, bf);
  TcAttnArgs t{};
  t.qk = qkv; t.out = out; t.starts = starts; t.lengths = lengths;
  t.M = M; t.heads = heads; t.window = -1; t.err = err;
  t.q_index = q_index; t.q_per_row = q_per_row; t.q_tiles = (q_per_row + kTcQ - 1) / kTcQ;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  t.splits = attention_splits(heads, n_rows * t.q_tiles, sm_count(dev), -1, M / n_rows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf) launch_tc_attention<__nv_bfloat16>(maps, t, n_rows * t.q_tiles, st, sm_count(dev));
  else launch_tc_attention<__half>(maps, t, n_rows * t.q_tiles, st, sm_count(dev));
  API_END(nullptr)
}

int laya_op_embed_norm(int precision, const int32_t* ids, const float* table, const float* gamma, float eps, int rows,
                       int width, int vocab, float* residual, void* x, int* err, void* stream) {
  API_BEGIN
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (precision == LAYA_PRECISION_BF16)
    launch_embed<__nv_bfloat16>(ids, table, gamma, eps, rows, width, vocab, residual, static_cast<__nv_bfloat16*>(x), err, st);
  else launch_embed<__half>(ids, table, gamma, eps, rows, width, vocab, residual, static_cast<__half*>(x), err, st);
  API_END(nullptr)
}

int laya_op_head_tail(int precision, const float* selected, const void* scored, const int32_t* counts, int batch,
                      int options, int width, const float* w3, const float* b3, const float* wa0, const float* ba0,
                      const float* wa2, const float* ba2, int n_act, float* logits, float* acts, float* features,
                      float* hidden, int32_t* arrivals, void* stream) {
  API_BEGIN
  if (!selected || !scored || !counts || !w3 || !b3 || !wa0 || !ba0 || !wa2 || !ba2 || !logits || !acts || !hidden ||
      !arrivals)
    fail(LAYA_ERR_INVALID, "null argument");
  if (batch <= 0 || options <= 0 || width <= 0 || width % 8 || n_act < 1) fail(LAYA_ERR_INVALID, "bad head shape");
  TailArgs t{};
  t.selected = selected; t.scored = scored; t.counts = counts;
  t.w3 = w3; t.b3 = b3; t.wa0 = wa0; t.ba0 = ba0; t.wa2 = wa2; t.ba2 = ba2;
  t.logits = logits; t.acts = acts; t.features = features; t.hidden = hidden; t.arrivals = arrivals;
  t.k = options; t.d = width; t.n_act = n_act;
  const size_t smem = ((size_t)(options + 1) + width + 4 + kActHidden) * sizeof(float);
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const int parts = batch * kTailPartsSmall <= 4 * sm_count(dev) ? kTailPartsSmall : kTailPartsLarge;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (precision == LAYA_PRECISION_BF16)
    launch_k(head_tail_kernel<__nv_bfloat16>, dim3(batch, parts), dim3(kTailThreads), smem, st, t);
  else launch_k(head_tail_kernel<__half>, dim3(batch, parts), dim3(kTailThreads), smem, st, t);
  API_END(nullptr)
}

int laya_op_norm(int precision, float* residual, const float* partials, int splits, const float* gamma, const float* beta,
                 float eps, void* x, int rows, int width, void* stream) {
  API_BEGIN
  NormArgs a{};
  a.residual = residual; a.partials = partials; a.splits = partials ? splits : 0;
  a.gamma1 = gamma; a.beta1 = beta; a.eps1 = eps; a.fused_final = 0; a.x = x; a.rows = rows; a.d = width;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (precision == LAYA_PRECISION_BF16) launch_norm<__nv_bfloat16>(a, st);
  else launch_norm<__half>(a, st);
  API_END(nullptr)
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Split-K residual GEMM without allocation (laya_op_gemm_residual_static).
//
// Its split-K partial sums live in this file-scope device array rather than in memory the
// caller or the library allocates.  Every GPU that loads the library holds the array until the
// process exits.  In host code the symbol is only a host-side stand-in: kernels receive the
// device address obtained with cudaGetSymbolAddress, looked up once per device below.
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) float g_static_partials[LAYA_STATIC_SCRATCH_FLOATS];

namespace {

std::mutex g_static_mutex;
float* g_static_ptr[64] = {};

// Device address of g_static_partials on the current device; the first call on a device looks
// it up (with that device current) and caches it.
float* static_partials_address() {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) fail(LAYA_ERR_INVALID, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (!g_static_ptr[dev]) {
    void* ptr = nullptr;
    CK(cudaGetSymbolAddress(&ptr, g_static_partials));
    if (!ptr) fail(LAYA_ERR_CUDA, "cudaGetSymbolAddress returned no address");
    g_static_ptr[dev] = static_cast<float*>(ptr);
  }
  return g_static_ptr[dev];
}

// residual[r][c] += bias[c] + sum_s partials[s][r][c], summed in split order.  Does nothing when
// the split-K GEMM reported an error: its partials may then be only partly written.
__global__ void __launch_bounds__(256) add_partials_kernel(float* residual, const float* partials, int splits,
                                                           int rows, int cols, const float* bias, const int* err) {
  // Launched with programmatic serialisation like every kernel here: wait for the split-K GEMM.
  pdl_wait();
  if (err && *reinterpret_cast<const volatile int*>(err) != 0) return;
  const int64_t n4 = (int64_t)rows * cols / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < splits; ++sp) {
      const float4 p = reinterpret_cast<const float4*>(partials)[(int64_t)sp * n4 + i];
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    if (bias) {
      const int c = (int)((i * 4) % cols);
      acc.x += bias[c]; acc.y += bias[c + 1]; acc.z += bias[c + 2]; acc.w += bias[c + 3];
    }
    float4 r = reinterpret_cast<float4*>(residual)[i];
    r.x += acc.x; r.y += acc.y; r.z += acc.z; r.w += acc.w;
    reinterpret_cast<float4*>(residual)[i] = r;
  }
}

}  // namespace

extern "C" int laya_op_gemm_residual_static(int precision, const void* x, const void* w, int M, int N, int K,
                                            int splits, float* residual, const float* bias, int* err, void* stream) {
  API_BEGIN
  if (!x || !w || !residual) fail(LAYA_ERR_INVALID, "null argument");
  if (M <= 0 || N <= 0 || K <= 0 || splits < 1) fail(LAYA_ERR_INVALID, "bad GEMM shape %dx%dx%d split %d", M, N, K, splits);
  // The partials are added to `residual` as float4, and to `bias` four columns at a time.
  if (reinterpret_cast<uintptr_t>(residual) & 15) fail(LAYA_ERR_INVALID, "residual must be 16-byte aligned");
  if (bias && (reinterpret_cast<uintptr_t>(bias) & 15)) fail(LAYA_ERR_INVALID, "bias must be 16-byte aligned");
  if (N % 64 || K % kBK) fail(LAYA_ERR_INVALID, "N must be a multiple of 64 and K of %d", kBK);
  if ((K / kBK) % splits) fail(LAYA_ERR_INVALID, "split-K %d does not divide %d k-blocks", splits, K / kBK);
  const int64_t need = (int64_t)M * N * splits;
  if (need > LAYA_STATIC_SCRATCH_FLOATS)
    fail(LAYA_ERR_INVALID, "M*N*splits = %lld partial sums exceed the static scratch of %d floats", (long long)need,
         LAYA_STATIC_SCRATCH_FLOATS);
  int dev = 0;
  CK(cudaGetDevice(&dev));
  // The scratch address is the current device's: a stream of another device would run the
  // kernels there against this device's array.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (st) {
    int stream_dev = -1;
    CK(cudaStreamGetDevice(st, &stream_dev));
    if (stream_dev != dev) fail(LAYA_ERR_INVALID, "stream belongs to device %d, the current device is %d", stream_dev, dev);
  }
  float* partials = static_partials_address();
  const int sms = sm_count(dev);
  const bool bf = precision == LAYA_PRECISION_BF16;
  const int bn = pick_bn(M, N, EPI_PARTIAL, sms);
  GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.splits = splits;
  a.residual = partials; a.ldr = N; a.err = err;
  const CUtensorMap ta = make_map(x, M, K, kBM, bf);
  const CUtensorMap tb = make_map(w, N, K, bn, bf);
  // Every partial element read below is written by this GEMM first, so the array needs no
  // clearing between calls.
  if (bf) launch_gemm<__nv_bfloat16>(EPI_PARTIAL, bn, ta, tb, a, sms, st);
  else launch_gemm<__half>(EPI_PARTIAL, bn, ta, tb, a, sms, st);
  const int64_t n4 = (int64_t)M * N / 4;
  const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 4LL * sms);
  launch_k(add_partials_kernel, dim3(grid), dim3(256), 0, st, residual, (const float*)partials, splits, M, N, bias,
           (const int*)err);
  API_END(nullptr)
}
