// Persistent, warp-specialised tcgen05 GEMM for the encoder and head linears:
//
//   D[M, N] = A[M, K] * W[N, K]^T       (A: activations, W: PyTorch Linear weight; both K-major)
//
// with the consumer of D fused into the epilogue (RoPE + head-major layout for QKV, GeGLU for
// the FFN up-projection, residual accumulation for the attention-out and FFN down projections,
// bias + ReLU / GELU for the decision head, split-K partials for small row counts).
//
// One CTA per SM, 10 warps:
//   warp 0      TMA producer: A/W tiles (BK = 64 16-bit elements, 128-byte swizzle) into a
//               ring of shared-memory stages (no multicast).
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues tcgen05.mma
//               (M = 128, N = BN, K = 16) into one of two TMEM accumulators.
//   warps 2..9  epilogue: tcgen05.ld of the finished accumulator (warp w reads TMEM lanes
//               32*(w%4) .. +31, i.e. tile rows; warps 2-5 and 6-9 split the tile's column
//               chunks), fused transform, global stores.  Two warps per lane quarter keep the
//               epilogue (exact-erf GELU, RoPE) shorter than the next tile's MMAs.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//
// Replaces the reference's cuBLAS GemmEx calls (laya_cuda/ops.py:58-66 called from
// laya_cuda/runtime.py:77-80) and the elementwise kernels that followed them
// (kernels.cu:50-82 bias/add/activate/layout).
#pragma once
#include "common.cuh"

namespace laya {

enum EpiKind : int {
  EPI_STORE = 0,    // out = acc + bias
  EPI_RELU = 1,     // out = relu(acc + bias)
  EPI_GELU = 2,     // out = gelu(acc + bias)
  EPI_GEGLU = 3,    // W rows interleaved in 64-row blocks [gate_i, up_i]: out = gelu(gate) * up
  EPI_QKV = 4,      // (+bias) RoPE on q/k; q, k -> [heads][M][64], v -> transposed [heads][64][M]
  EPI_RESIDUAL = 5, // residual(fp32) += acc + bias
  EPI_PARTIAL = 6,  // partial[split](fp32) = acc          (split-K)
};

struct GemmArgs {
  int M, N, K;
  int splits;             // split-K factor (EPI_PARTIAL only; 1 otherwise)
  void* out;              // 16-bit output
  int ldo;                // elements
  float* residual;        // EPI_RESIDUAL target, or EPI_PARTIAL base ([splits][M][ldr])
  int ldr;
  const float* bias;      // fp32 [N] (GeGLU: unused) or nullptr
  // EPI_QKV
  int heads;
  // RoPE table or nullptr: [16][rope_rows] of (cos f_2k, cos f_2k+1, sin f_2k, sin f_2k+1) at a
  // position, frequency-pair major so a warp's rows (mostly consecutive positions) read one
  // contiguous run per pair, one 16-byte load per two rotations.
  const float4* rope_tab;
  int rope_rows;
  const int* positions;   // [M]
  int* err;               // device error word
  unsigned long long wait_ns;  // wait limit of this launch (0: kWaitTimeoutNs)
};

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 320;  // 10 warps: the busiest scheduler holds 3, so <= 168 registers
constexpr int kEpiWarps = 8;

// Per epilogue warp: a [32 rows][128 B] staging block in shared memory.  The warp's lanes own
// one tile row each (the TMEM lane layout); global memory is accessed through the block in the
// transposed mapping (lane -> row 4k + lane/8, 16-byte piece lane%8 for k = 0..7), so every
// warp-wide global access covers four whole 128-byte lines instead of 32 partial ones.
constexpr int kEpiStageBytes = 32 * 128;
constexpr int kEpiSmemBytes = kEpiWarps * kEpiStageBytes;

template <int BN>
struct GemmCfg {
  static constexpr int kStageA = kBM * kBK * 2;
  static constexpr int kStageB = BN * kBK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (192 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kOffEpi = kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffEpi + kEpiSmemBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// Byte offset of 16-byte piece j of row r in a staging block (pieces XOR-swizzled by row, so both
// the row-per-lane writes and the transposed reads are free of bank conflicts).
__device__ __forceinline__ uint32_t stage_off(int r, int j) { return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4)); }

// Lane `lane` writes its row (8 pieces) into the block; the previous contents must be consumed.
__device__ __forceinline__ void stage_put(uint8_t* buf, int lane, const uint4 (&p)[8]) {
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(buf + stage_off(lane, j)) = p[j];
  __syncwarp();
}

// Piece (row 4k + lane/8, lane%8) of the block.
__device__ __forceinline__ uint4 stage_get(const uint8_t* buf, int k, int lane) {
  return *reinterpret_cast<const uint4*>(buf + stage_off(4 * k + (lane >> 3), lane & 7));
}

__device__ __forceinline__ uint4 u4(float a, float b, float c, float d) {
  return make_uint4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d));
}
__device__ __forceinline__ float4 f4(uint4 v) {
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

// Writes a staged block of 16-bit rows (64 elements each) to dst_row(r) for tile rows r < rows.
template <typename RowPtr>
__device__ __forceinline__ void stage_store16(const uint8_t* buf, int lane, int rows, RowPtr dst_row) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 4 * k + (lane >> 3);
    if (r < rows) *reinterpret_cast<uint4*>(dst_row(r) + (lane & 7) * 8) = stage_get(buf, k, lane);
  }
}

// Residual epilogue (residual[row, n0 + ...] += accumulator + bias), software-pipelined: a warp's
// residual chunks (32 rows x 32 columns, every other chunk of the tile) are loaded two ahead in
// the coalesced mapping, the first two before the accumulator is waited on, so the fp32 read
// latency overlaps the tile's MMAs and the previous chunk's work.
template <int BN>
struct ResidualPipe {
  static constexpr int kChunks = BN / 64;
  float4 buf[2][8];

  __device__ __forceinline__ void load(const GemmArgs& a, int row0, int n0, int half, int lane, int i) {
    const float* base = a.residual + n0 + (half + 2 * i) * 32 + (lane & 7) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = row0 + 4 * k + (lane >> 3);
      buf[i & 1][k] = r < a.M ? *reinterpret_cast<const float4*>(base + (size_t)r * a.ldr) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  __device__ __forceinline__ void start(const GemmArgs& a, int row0, int n0, int half, int lane) {
    load(a, row0, n0, half, lane, 0);
    if (kChunks > 1) load(a, row0, n0, half, lane, 1);
  }

  __device__ __forceinline__ void finish(const GemmArgs& a, uint32_t tbase, int row0, int n0, int half, int lane,
                                         uint8_t* stage) {
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      const int c = half + 2 * i;
      const int col = n0 + c * 32;
      uint32_t v[32];
      tmem_ld32_async(tbase + c * 32, v);
      tmem_wait_ld(v);
      uint4 p[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.bias) bb = *reinterpret_cast<const float4*>(a.bias + col + 4 * j);
        p[j] = u4(__uint_as_float(v[4 * j]) + bb.x, __uint_as_float(v[4 * j + 1]) + bb.y,
                  __uint_as_float(v[4 * j + 2]) + bb.z, __uint_as_float(v[4 * j + 3]) + bb.w);
      }
      stage_put(stage, lane, p);
      float* base = a.residual + col + (lane & 7) * 4;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = row0 + 4 * k + (lane >> 3);
        const float4 add = f4(stage_get(stage, k, lane));
        float4 t = buf[i & 1][k];
        t.x += add.x; t.y += add.y; t.z += add.z; t.w += add.w;
        if (r < a.M) *reinterpret_cast<float4*>(base + (size_t)r * a.ldr) = t;
      }
      if (i + 2 < kChunks) load(a, row0, n0, half, lane, i + 2);
    }
  }
};

// QKV epilogue (RoPE on q and k, head-major q/k, transposed v).  The tile's columns are 64-column
// chunks, one head of q, k or v each.  The two
// warps of a TMEM lane quarter split every chunk's 32 frequency pairs, warp `half` taking pairs
// 8*half .. 8*half+7, i.e. columns [16 half, +16) and [32 + 16 half, +16) of each chunk, so all
// eight epilogue warps work on every chunk.  A row's RoPE entries depend only on its position
// and the frequency pair, not on the head, so start() loads the warp's eight entries once per
// tile, before the accumulator is waited on.
template <int BN, typename T>
struct QkvPipe {
  float4 rope[8];
  bool roped;

  __device__ __forceinline__ void start(const GemmArgs& a, int row, int n0, int half) {
    // roped: the tile starts in q or k (its later chunks may reach v, which is not rotated).
    roped = n0 / (a.heads * 64) < 2 && a.rope_tab != nullptr && row < a.M;
    if (roped) {
      const float4* rt = a.rope_tab + a.positions[row];
#pragma unroll
      for (int k = 0; k < 8; ++k) rope[k] = __ldg(rt + (size_t)(8 * half + k) * a.rope_rows);
    }
  }

  __device__ __forceinline__ void finish(const GemmArgs& a, uint32_t tbase, int row0, int n0, int half, int lane,
                                         uint8_t* stage) {
    const int row = row0 + lane;
    const int rows = min(32, a.M - row0);
    const int width = a.heads * 64;
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      const int n = n0 + 64 * c;
      const int part = n / width;
      const int head = (n - part * width) >> 6;
      float lo[16], hi[16];
      tmem_ld16x2(tbase + 64 * c + 16 * half, tbase + 64 * c + 32 + 16 * half, lo, hi);
      if (a.bias) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          lo[i] += a.bias[n + 16 * half + i];
          hi[i] += a.bias[n + 32 + 16 * half + i];
        }
      }
      if (roped && part < 2) {
        // Rotate-half RoPE: lo' = lo cos - hi sin, hi' = hi cos + lo sin (pairs of frequencies).
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 cs = make_float2(rope[k].x, rope[k].y), sn = make_float2(rope[k].z, rope[k].w);
          const float2 l = make_float2(lo[2 * k], lo[2 * k + 1]), h = make_float2(hi[2 * k], hi[2 * k + 1]);
          const float2 nl = sub2(mul2(l, cs), mul2(h, sn));
          const float2 nh = fma2(h, cs, mul2(l, sn));
          lo[2 * k] = nl.x; lo[2 * k + 1] = nl.y;
          hi[2 * k] = nh.x; hi[2 * k + 1] = nh.y;
        }
      }
      if (part < 2) {
        // q, k -> [part][heads][M][64]: this warp's half of each of its 32 rows is two 32-byte
        // runs (pieces 0,1 at byte 32 half, pieces 2,3 at byte 64 + 32 half), staged so that
        // each store covers whole 32-byte sectors.
        uint4 p[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          p[j] = make_uint4(pack2<T>(lo[8 * j + 0], lo[8 * j + 1]), pack2<T>(lo[8 * j + 2], lo[8 * j + 3]),
                            pack2<T>(lo[8 * j + 4], lo[8 * j + 5]), pack2<T>(lo[8 * j + 6], lo[8 * j + 7]));
          p[2 + j] = make_uint4(pack2<T>(hi[8 * j + 0], hi[8 * j + 1]), pack2<T>(hi[8 * j + 2], hi[8 * j + 3]),
                                pack2<T>(hi[8 * j + 4], hi[8 * j + 5]), pack2<T>(hi[8 * j + 6], hi[8 * j + 7]));
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(stage + stage_off(lane, j)) = p[j];
        __syncwarp();
        T* out = reinterpret_cast<T*>(a.out) + ((size_t)part * a.heads + head) * a.M * 64;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int r = 8 * k + (lane >> 2), j = lane & 3;
          const int col = (j < 2 ? 16 * half + 8 * j : 32 + 16 * half + 8 * (j - 2));
          if (r < rows)
            *reinterpret_cast<uint4*>(out + (size_t)(row0 + r) * 64 + col) =
                *reinterpret_cast<const uint4*>(stage + stage_off(r, j));
        }
      } else if (a.M % 8 == 0) {
        // V transposed, [heads][64][M]: the warp's 32 dims x 32 tokens go through the staging
        // block transposed (dim d' = 0..31 its 16 low then 16 high dims, 64 bytes of tokens per
        // dim), then each lane stores four 16-byte runs of 8 tokens.  M a multiple of 8 keeps
        // every run 16-byte aligned and wholly inside or wholly past the last row.
        T* vt = reinterpret_cast<T*>(a.out) + ((size_t)2 * a.heads + head) * a.M * 64;
        __syncwarp();
        T* st16 = reinterpret_cast<T*>(stage);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          st16[i * 32 + lane] = from_f32<T>(lo[i]);
          st16[(16 + i) * 32 + lane] = from_f32<T>(hi[i]);
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int piece = lane + 32 * k, dd = piece >> 2, sub = piece & 3;
          const int dim = dd < 16 ? 16 * half + dd : 32 + 16 * half + (dd - 16);
          const int t0 = row0 + 8 * sub;
          if (t0 < a.M)
            *reinterpret_cast<uint4*>(vt + (size_t)dim * a.M + t0) =
                *reinterpret_cast<const uint4*>(st16 + dd * 32 + 8 * sub);
        }
      } else if (row < a.M) {
        // Row counts that are not a multiple of 8: one 2-byte store per dim and token (each
        // dimension's 32 stores fill one 64-byte run).
        T* vt = reinterpret_cast<T*>(a.out) + ((size_t)2 * a.heads + head) * a.M * 64 + row;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          vt[(size_t)(16 * half + i) * a.M] = from_f32<T>(lo[i]);
          vt[(size_t)(32 + 16 * half + i) * a.M] = from_f32<T>(hi[i]);
        }
      }
    }
  }
};

// Epilogue of one accumulator tile for one warp: TMEM lanes row0 .. row0+31 of the tile (this
// lane: row0 + lane), columns from `tbase`, output column base n0; `half` selects every other
// column chunk (two warps share a TMEM lane quarter).  EPI_RESIDUAL and EPI_QKV are handled by
// ResidualPipe and QkvPipe.
template <int BN, int EPI, typename T>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& args, uint32_t tbase, int row0, int n0, int split,
                                              int half, int lane, uint8_t* stage) {
  const int rows = min(32, args.M - row0);  // live rows of this warp's block
  if (EPI == EPI_GEGLU) {
    // Tile columns: [gate 64 | up 64] x (BN / 128); output columns n0/2 + 64c + [0, 64).
#pragma unroll 1
    for (int c = half; c < BN / 128; c += 2) {
      uint4 p[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // Gate and up columns loaded together, one wait.
        uint32_t g[32], u[32];
        tmem_ld32_async(tbase + c * 128 + h * 32, g);
        tmem_ld32_async(tbase + c * 128 + 64 + h * 32, u);
        tmem_wait_ld(g);
        tmem_wait_ld(u);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 y = mul2(gelu_erf2(make_float2(__uint_as_float(g[i + 2 * e]), __uint_as_float(g[i + 2 * e + 1]))),
                                  make_float2(__uint_as_float(u[i + 2 * e]), __uint_as_float(u[i + 2 * e + 1])));
            w[e] = pack2<T>(y.x, y.y);
          }
          p[h * 4 + i / 8] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      stage_put(stage, lane, p);
      T* out = reinterpret_cast<T*>(args.out) + n0 / 2 + c * 64;
      stage_store16(stage, lane, rows, [&](int r) { return out + (size_t)(row0 + r) * args.ldo; });
    }
  } else if (EPI == EPI_PARTIAL) {
    // partial[split][row][col] = acc (fp32), 32 columns (128 B per row) per chunk.
#pragma unroll 1
    for (int c = half; c < BN / 32; c += 2) {
      uint32_t v[32];
      tmem_ld32_async(tbase + c * 32, v);
      tmem_wait_ld(v);
      uint4 p[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) p[j] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      stage_put(stage, lane, p);
      float* base = args.residual + ((size_t)split * args.M) * args.ldr + n0 + c * 32 + (lane & 7) * 4;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = 4 * k + (lane >> 3);
        if (r < rows) *reinterpret_cast<uint4*>(base + (size_t)(row0 + r) * args.ldr) = stage_get(stage, k, lane);
      }
    }
  } else {
    // EPI_STORE / EPI_RELU / EPI_GELU: out = act(acc + bias), 64 columns per chunk.
#pragma unroll 1
    for (int c = half; c < BN / 64; c += 2) {
      const int col = n0 + c * 64;
      uint4 p[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld32(tbase + c * 64 + h * 32, v);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float x[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float t = v[i + j] + (args.bias ? args.bias[col + h * 32 + i + j] : 0.f);
            if (EPI == EPI_RELU) t = fmaxf(t, 0.f);
            if (EPI == EPI_GELU) t = gelu_erf(t);
            x[j] = t;
          }
          p[h * 4 + i / 8] = make_uint4(pack2<T>(x[0], x[1]), pack2<T>(x[2], x[3]), pack2<T>(x[4], x[5]),
                                        pack2<T>(x[6], x[7]));
        }
      }
      stage_put(stage, lane, p);
      T* out = reinterpret_cast<T*>(args.out) + col;
      stage_store16(stage, lane, rows, [&](int r) { return out + (size_t)(row0 + r) * args.ldo; });
    }
  }
}

template <int BN, int EPI, typename T, int NI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  // NI > 1: NI threads (lane 0 of warp 1 and of epilogue warps 2..NI) issue the MMAs of a tile,
  // issuer i taking k-blocks i, i + NI, ... into its own accumulator; the epilogue warps add the
  // accumulators before the epilogue.  One thread's tcgen05.mma stream runs about one
  // instruction per ~100 ns whatever N is up to 256, so a tile of N <= 128 leaves most of the
  // tensor core idle with one issuer; independent streams from several threads run
  // concurrently.  Only for grids in which every CTA has at most one tile (the host checks), so
  // the epilogue warps are idle while they issue.  Each stage always goes to the same issuer
  // (NI divides S), so every issuer sees its stages' phases in order.
  static_assert(NI == 1 || (S % NI == 0 && NI <= kEpiWarps + 1), "issuers must divide the stages");
  constexpr int kCols = NI == 1 ? Cfg::kTmemCols : (NI * BN < 32 ? 32 : NI * BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffEpi + kEpiSmemBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint64_t* presum = bars + 2 * S + 5;  // NI > 1: every epilogue warp added its share
  uint64_t* idrain = bars + 2 * S + 6;  // [NI - 1]: drains of the extra issuers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 6 + (NI > 1 ? NI - 1 : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const unsigned long long wait_ns = wait_limit(args.wait_ns);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int m_blocks = (args.M + kBM - 1) / kBM;
  const int n_blocks = args.N / BN;
  const int splits = args.splits;
  const int k_blocks_total = args.K / kBK;
  const int k_blocks = k_blocks_total / splits;
  const int tiles = m_blocks * n_blocks * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], NI); mbar_init(&tempty[i], kEpiWarps); }
    mbar_init(drain, 1);
    mbar_init(presum, kEpiWarps);
    for (int i = 0; i + 1 < NI; ++i) mbar_init(&idrain[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
  if (warp == 1) { tmem_alloc(tmem_slot, kCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The prologue above touches no predecessor output.

  // Tile order: split outermost, then row block, then column block, so CTAs running together
  // share an A row block (it stays in L2 while all its column blocks are computed).
  auto decode = [&](int t, int& split, int& mb, int& nb) {
    split = t / (m_blocks * n_blocks);
    int r = t - split * m_blocks * n_blocks;
    mb = r / n_blocks;
    nb = r - mb * n_blocks;
  };

  // NI > 1 (one tile per CTA): issuer i's share of the tile's k-blocks into accumulator i, then
  // a commit to tfull.  Bounded waits; the caller drains its own MMAs afterwards.
  auto issue_share = [&](int i) {
    const uint32_t idesc = mma_idesc<std::is_same<T, __nv_bfloat16>::value>(kBM, BN);
    const uint32_t d_tmem = tmem_base + (uint32_t)(i * BN);
    bool ok = (int)blockIdx.x < tiles;
    for (int kb = i; kb < k_blocks && ok; kb += NI) {
      const int stage = kb % S;
      if (!mbar_wait(&full[stage], (kb / S) & 1, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + stage * Cfg::kStageA);
      const uint32_t b0 = smem_u32(sB + stage * Cfg::kStageB);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k)
        tc_mma_f16(d_tmem, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(b0 + k * 32), idesc,
                   (kb > i || k > 0) ? 1u : 0u);
      tc_commit(&empty[stage]);
    }
    if (ok) tc_commit(&tfull[0]);
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      // Weights do not depend on the previous kernel: the first tile's weight stages are loaded
      // before waiting for it, so their HBM latency overlaps the predecessor's tail.
      int pre = 0;
      if ((int)blockIdx.x < tiles) {
        int split, mb, nb; decode(blockIdx.x, split, mb, nb);
        pre = k_blocks < S ? k_blocks : S;
        for (int kb = 0; kb < pre; ++kb) {
          mbar_arrive_expect_tx(&full[kb], Cfg::kStageBytes);
          tma_load_2d(sB + kb * Cfg::kStageB, &tmB, &full[kb], (split * k_blocks + kb) * kBK, nb * BN);
        }
        // A CTA with a single tile (small classes) requests the rest of its weights into L2 at
        // once, so the ring's refills hit L2 instead of each waiting out HBM latency.
        if (tiles <= (int)gridDim.x)
          for (int kb = pre; kb < k_blocks; ++kb) tma_prefetch_l2_2d(&tmB, (split * k_blocks + kb) * kBK, nb * BN);
      }
      pdl_wait();
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int split, mb, nb; decode(t, split, mb, nb);
        for (int kb = 0; kb < k_blocks; ++kb) {
          const int kx = (split * k_blocks + kb) * kBK;
          if (t == (int)blockIdx.x && kb < pre) {
            // Stage `kb` already expects this k-block's bytes and holds its weights.
            tma_load_2d(sA + stage * Cfg::kStageA, &tmA, &full[stage], kx, mb * kBM);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrGemmProducerWait, abort_flag, wait_ns)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
            tma_load_2d(sA + stage * Cfg::kStageA, &tmA, &full[stage], kx, mb * kBM);
            tma_load_2d(sB + stage * Cfg::kStageB, &tmB, &full[stage], kx, nb * BN);
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      // Every copy issued lands before the CTA exits, also when this role finished its loads
      // but another role gave up and will not consume them.  mbar_drain is bounded by time only:
      // on an abort an abort-aware wait would return at once and leave TMA writes landing in
      // shared memory the CTA no longer owns.  On the normal path every stage has completed.
      (void)ok;
      for (int s = 0; s < S; ++s)
        if (issued & (1u << s)) mbar_drain(&full[s], (last_par >> s) & 1);
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && NI > 1) {
      issue_share(0);
      tc_commit(drain);
      mbar_drain(drain, 0);
    } else if (lane == 0) {
      const uint32_t idesc = mma_idesc<std::is_same<T, __nv_bfloat16>::value>(kBM, BN);
      int stage = 0; uint32_t phase = 0;
      int acc = 0; uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kStageA);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kStageB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            tc_mma_f16(d_tmem, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(b0 + k * 32), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // Drain: make sure no MMA is still writing TMEM when it is released (bounded by time
      // only, so it also waits after an abort).
      tc_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    pdl_wait();
    // Epilogue warps 2..9 -> TMEM lane quarter (warp % 4); `half` picks every other chunk.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stage = smem + Cfg::kOffEpi + (warp - 2) * kEpiStageBytes;
    int acc = 0; uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int split, mb, nb; decode(t, split, mb, nb);
      const int row0 = mb * kBM + quarter * 32;
      ResidualPipe<BN> rp;
      QkvPipe<BN, T> qp;
      if (EPI == EPI_RESIDUAL) rp.start(args, row0, nb * BN, half, lane);
      if (EPI == EPI_QKV) qp.start(args, row0 + lane, nb * BN, half);
      if (NI > 1 && warp - 1 < NI) {
        // Extra issuer (one tile per CTA: the loop runs once).
        if (lane == 0) {
          issue_share(warp - 1);
          tc_commit(&idrain[warp - 2]);
          mbar_drain(&idrain[warp - 2], 0);
        }
        __syncwarp();
      }
      if (!mbar_wait(&tfull[acc], acc_phase, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (NI > 1) {
        // Accumulator 0 += accumulators 1.. (those that received k-blocks): this warp adds the
        // 32-column chunks h of its lane quarter with h % 2 == half, then every epilogue warp
        // waits until all shares are in (the epilogue reads columns across the halves).
        const int used = k_blocks < NI ? k_blocks : NI;
#pragma unroll 1
        for (int h = half; h < BN / 32; h += 2) {
          uint32_t v[32];
          tmem_ld32_async(tbase + 32 * h, v);
          tmem_wait_ld(v);
          for (int i = 1; i < used; ++i) {
            uint32_t w[32];
            tmem_ld32_async(tbase + (uint32_t)(i * BN) + 32 * h, w);
            tmem_wait_ld(w);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) + __uint_as_float(w[e]));
          }
          tmem_st32(tbase + 32 * h, v);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(presum);
        if (!mbar_wait(presum, 0, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns)) break;
        tc_fence_after();
      }
      if (EPI == EPI_RESIDUAL) rp.finish(args, tbase, row0, nb * BN, half, lane, stage);
      else if (EPI == EPI_QKV) qp.finish(args, tbase, row0, nb * BN, half, lane, stage);
      else epilogue_tile<BN, EPI, T>(args, tbase, row0, nb * BN, split, half, lane, stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kCols);
}


// ---------------------------------------------------------------------------------------------
// CTA-pair variant (cluster of 2, tcgen05 cta_group::2): 256 x BN output tiles.  Each CTA loads
// its 128 rows of A and BN/2 rows of W per k-block and holds its 128 accumulator rows in its own
// TMEM; the pair leader (rank 0) issues the M=256 MMAs that read both CTAs' shared memory.  Per
// CTA this moves (128 + BN/2) x 64 operand elements per k-block for a 128 x BN share of the
// output instead of (128 + BN) x 64: a third less L2 -> shared traffic than the 1-CTA kernel.
// Used for large row counts; small classes use the 1-CTA kernel (split-K included).
//
// Barriers: full[s] lives in the leader (both CTAs' TMA loads complete on it; the leader
// expects both CTAs' bytes); empty[s] and tfull[a] live in both CTAs (the leader's MMA thread
// commits to its own and, through the peer's cluster address, to the peer's); tempty[a] lives in
// the leader (all 16 epilogue warps of the pair arrive, the peer's remotely).
// ---------------------------------------------------------------------------------------------
template <int BN>
struct GemmPairCfg {
  static constexpr int kStageA = kBM * kBK * 2;           // this CTA's 128 rows of A
  static constexpr int kStageB = (BN / 2) * kBK * 2;      // this CTA's BN/2 rows of W
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (192 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kOffEpi = kStages * kStageBytes;
  static constexpr int kSmemBytes = kOffEpi + kEpiSmemBytes + 1024 + 256;
};

template <int BN, int EPI, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs args) {
  using Cfg = GemmPairCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kStageA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffEpi + kEpiSmemBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* drain = bars + 2 * S + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const unsigned long long wait_ns = wait_limit(args.wait_ns);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  const int m_blocks = (args.M + 2 * kBM - 1) / (2 * kBM);
  const int n_blocks = args.N / BN;
  const int k_blocks = args.K / kBK;
  const int tiles = m_blocks * n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], 2 * kEpiWarps); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
  if (warp == 1) { tmem_alloc_pair(tmem_slot, Cfg::kTmemCols); tmem_relinquish_pair(); }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        const int mb = t / n_blocks, nb = t - mb * n_blocks;
        const int arow = mb * 2 * kBM + (int)rank * kBM;
        const int brow = nb * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrGemmProducerWait, abort_flag, wait_ns)) { ok = false; break; }
          const uint32_t leader_full = cluster_addr(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          tma_load_2d_pair(sA + stage * Cfg::kStageA, &tmA, leader_full, kb * kBK, arow);
          tma_load_2d_pair(sB + stage * Cfg::kStageB, &tmB, leader_full, kb * kBK, brow);
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      if (leader) {
        // Both CTAs' copies complete on the leader's full barriers: wait for them by time only,
        // on every path (see gemm_kernel).
        (void)ok;
        for (int s = 0; s < S; ++s)
          if (issued & (1u << s)) mbar_drain(&full[s], (last_par >> s) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = mma_idesc<std::is_same<T, __nv_bfloat16>::value>(2 * kBM, BN);
      int stage = 0; uint32_t phase = 0;
      int acc = 0; uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kStageA);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kStageB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            tc_mma_f16_pair(d_tmem, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(b0 + k * 32), idesc,
                            (kb > 0 || k > 0) ? 1u : 0u);
          }
          const uint32_t e = smem_u32(&empty[stage]);
          tc_commit_pair(cluster_addr(e, 0));
          tc_commit_pair(cluster_addr(e, 1));
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&tfull[acc]);
        tc_commit_pair(cluster_addr(f, 0));
        tc_commit_pair(cluster_addr(f, 1));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      tc_commit_pair(cluster_addr(smem_u32(drain), 0));
      mbar_drain(drain, 0);
    }
  } else {
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stage = smem + Cfg::kOffEpi + (warp - 2) * kEpiStageBytes;
    const uint32_t leader_tempty0 = cluster_addr(smem_u32(&tempty[0]), 0);
    const uint32_t leader_tempty1 = cluster_addr(smem_u32(&tempty[1]), 0);
    int acc = 0; uint32_t acc_phase = 0;
    for (int t = pair; t < tiles; t += pairs) {
      const int mb = t / n_blocks, nb = t - mb * n_blocks;
      const int row0 = mb * 2 * kBM + (int)rank * kBM + quarter * 32;
      ResidualPipe<BN> rp;
      QkvPipe<BN, T> qp;
      if (EPI == EPI_RESIDUAL) rp.start(args, row0, nb * BN, half, lane);
      if (EPI == EPI_QKV) qp.start(args, row0 + lane, nb * BN, half);
      if (!mbar_wait(&tfull[acc], acc_phase, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (EPI == EPI_RESIDUAL) rp.finish(args, tbase, row0, nb * BN, half, lane, stage);
      else if (EPI == EPI_QKV) qp.finish(args, tbase, row0, nb * BN, half, lane, stage);
      else epilogue_tile<BN, EPI, T>(args, tbase, row0, nb * BN, 0, half, lane, stage);
      tc_fence_before();
      __syncwarp();
      // The accumulator's TMEM columns were read to completion (tcgen05.wait::ld) before this
      // point; the tile's global stores need no ordering with the next MMAs, so the arrival is
      // relaxed and does not wait for them.
      if (lane == 0) mbar_arrive_cluster_relaxed(acc == 0 ? leader_tempty0 : leader_tempty1);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  cluster_sync();  // both CTAs done with TMEM and with the peer's barriers
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
}

}  // namespace laya
