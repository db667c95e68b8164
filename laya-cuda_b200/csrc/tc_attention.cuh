// Varlen packed attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), used by the
// forward pass.  Same semantics as the reference kernel laya_cuda/kernels.cu:90-154: rows packed
// at 16-token alignment, key j visible to query i of the same row iff j < length and
// (window < 0 or |i - j| <= window), scores scaled by 1/8, fp32 softmax, padding queries and
// tokens past the last row produce zeros.
//
// Work unit: one CTA per (128-query tile of one row, head); the host's tile table never lets a
// tile straddle rows.  4 warps, one thread per query row (warp w owns TMEM lanes [32w, 32w+32)).
// The kernel is bound by instruction latency in the softmax, not by a pipe's throughput, so for
// large grids it is laid out for many resident warps: with 64-key blocks (KB = 64) a CTA holds
// 128 TMEM columns and ~50 KB of shared memory, so four CTAs (16 warps) share an SM and hide each
// other's waits.  Small grids (batch 1), where the serial chain of blocks per tile decides,
// take 128-key blocks (KB = 128: 256 TMEM columns, two CTAs per SM, half as many blocks).
//
// TMEM per CTA: S_j = Q K_j^T for a block of KB keys in columns [0, KB) (fp32); the softmax
// reads S_j into registers and writes P_j = 2^(s log2e / 8 - m) as 16-bit pairs over its first
// KB / 2 columns; O in columns [KB, KB + 64).  The tensor core executes a CTA's MMAs in issue order, so
// the control lane issues O += P_j V_j and S_{j+1} = Q K_{j+1}^T back to back: S_{j+1} overwrites
// P_j only after the P V product has read it, and the single commit after S_{j+1} tells the
// softmax warps both that S_{j+1} is ready and that O is settled (for the rare rescale).  Per
// block the warps wait on one barrier (s_full) and arrive on one (p_full).
//
// Warp 0 also controls the pipeline (TMEM allocation; one lane issues copies and MMAs):
//   TMA   the Q tile once, then per block the K tile and the V^T tile(s) into double-buffered
//         stages (128-byte swizzle, no multicast); a stage is refilled once the commit that
//         covers the MMA reading it has been observed;
//   MMA   S_j (M=128, N=KB, K=64), O += P_j V_j (M=128, N=64, K=KB, A = P from TMEM).
// The softmax masks only 32-key chunks that straddle the window or row end and skips chunks no
// query of its warp can see; it keeps the running maximum m and sum l in fp32 (paired fp32
// instructions for the scale-and-subtract and the sums); O stays in TMEM and is rescaled (read,
// scaled, written back) only when a row maximum grows by more than 2^8, so P <= 256 and the final
// O / l is unchanged.  Key blocks start at the window's first key (rounded down to 16 tokens).
// Small grids (batch-1 classes) split each tile's key blocks over a CTA pair (TcAttnArgs::splits).
// Inputs (from the QKV GEMM epilogue): Q, K [heads][M][64] (K-major rows of 128 bytes) and V
// transposed [heads][64][M], so every shared-memory operand is K-major, as in gemm.cuh.  Every
// wait is bounded and reports through the error word.
#pragma once
#include "common.cuh"

namespace laya {

constexpr int kTcQ = 128;              // queries per CTA
constexpr int kTcThreads = 128;
constexpr float kTcRescaleLog2 = 8.f;  // O is rescaled when the row maximum grows by more than 2^8

struct TcAttnArgs {
  const void* qk;       // q, k: [heads][M][64] each (read directly only for gathered queries)
  void* out;            // [M][heads*64]
  const int4* tiles;    // (t0, t1, row, 0): 128-query tiles; row -1: zero-fill; row -2: unused
  const int* starts;
  const int* lengths;
  int M;
  int heads;
  int window;           // -1: global
  int* err;
  // Gathered queries (global attention only): when q_index is set, tile y of the grid is part
  // y % q_tiles of row y / q_tiles, whose queries are the tokens q_index[row * q_per_row + i]
  // (the decision head's CLS and marker rows); `tiles` is unused and rows of length 0 are skipped.
  const int* q_index;
  int q_per_row;
  int q_tiles;
  // 1, 2 or 4: key split.  The grid is (heads, tiles, splits) in clusters of (1, 1, splits); CTA
  // rank r of a cluster runs key blocks [r h, r h + h) of its tile (h = the blocks / splits,
  // rounded up).  The partial results merge pairwise through distributed shared memory (rank r
  // hands its unnormalised O row, running maximum and sum to rank r - step, step = 1, 2), and
  // rank 0 stores.  Shortens the serial block chain of grids that leave SMs idle.
  int splits;
  unsigned long long wait_ns;  // wait limit of this launch (0: kWaitTimeoutNs)
  int n_tiles;                 // entries of `tiles` (the persistent kernel's work list)
};

// Layout of the kernel with KB-key blocks.
template <int KB>
struct TcAttnCfg {
  static_assert(KB == 64 || KB == 128, "64- or 128-key blocks");
  static constexpr int kChunks = KB / 32;                 // 32-key chunks per block
  static constexpr int kCtasPerSm = KB == 64 ? 4 : 2;
  static constexpr int kTmemCols = KB == 64 ? 128 : 256;  // S / P: [0, KB), O: [KB, KB + 64)
  static constexpr int kQ = kTcQ * 128;                   // 16 KB: [128 queries][64 dims]
  static constexpr int kK = KB * 128;                     // per stage: [KB keys][64 dims]
  static constexpr int kV = 64 * KB * 2;                  // per stage: KB / 64 x [64 dims][64 keys]
  static constexpr int kStages = 2;
  static constexpr int kOffQ = 0, kOffK = kQ, kOffV = kQ + kStages * kK;
  static constexpr int kOffBar = kOffV + kStages * kV;
  static constexpr int kBytes = kOffBar + 256 + 1024;     // barriers + alignment slack
  // Block-relative key from which blocks every query of the warp sees in full compute their
  // exponentials on the FMA pipe (exp2_poly2) rather than the special-function unit: the last
  // eighth of the block (larger shares measured slower: the polynomial costs issue slots).
  static constexpr int kPolyKey = KB - KB / 8;
  static_assert(kCtasPerSm * (kBytes + 1024) <= 228 * 1024, "shared memory of the resident CTAs");
  static_assert(kCtasPerSm * kTmemCols <= 512, "TMEM of the resident CTAs");
};

// Softmax helpers for one thread's row of a block held in registers as NC 32-key chunks (raw
// fp32 scores).  `vis` bit c: chunk c is loaded (some query of the warp sees one of its keys);
// `full` bit c: every query of the warp sees every key of chunk c (no mask).  Both are
// warp-uniform; kAll = every chunk visible and full (the common case of global layers), which
// compiles without a branch.
//
// Masks the scores this thread's query may not see to -inf and returns the block maximum.
// Key ck + i is visible iff (unsigned)(ck + i - lo_key) <= span_keys.
template <bool kAll, int NC>
__device__ __forceinline__ float tc_block_max(uint32_t (&sx)[NC][32], uint32_t vis, uint32_t full, int kb, int lo_key,
                                              uint32_t span_keys) {
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (!kAll && !((vis >> c) & 1)) continue;
    if (!kAll && !((full >> c) & 1)) {
      const int d = kb + 32 * c - lo_key;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if ((uint32_t)(d + i) > span_keys) sx[c][i] = __float_as_uint(-INFINITY);
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2)
      mx[(i >> 1) & 7] = max3(mx[(i >> 1) & 7], __uint_as_float(sx[c][i]), __uint_as_float(sx[c][i + 1]));
  }
#pragma unroll
  for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
  return mx[0];
}

// P = 2^(s * scale - sub) for the loaded chunks (zeros for the others), stored as 16-bit pairs
// into TMEM columns p_tmem + 16c; returns the row sum of the fp32 probabilities.
template <bool kAll, typename T, int NC, int kPolyKey>
__device__ __forceinline__ float tc_block_probs(const uint32_t (&sx)[NC][32], uint32_t vis, float scale, float sub,
                                                uint32_t p_tmem) {
  float2 sm[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
  const float2 sc = make_float2(scale, scale), ns = make_float2(-sub, -sub);
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    uint32_t pk[16];
    if (kAll || ((vis >> c) & 1)) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 x = fma2(make_float2(__uint_as_float(sx[c][i]), __uint_as_float(sx[c][i + 1])), sc, ns);
        const float2 p = kAll && 32 * c + i >= kPolyKey ? exp2_poly2(x) : make_float2(ex2_approx(x.x), ex2_approx(x.y));
        sm[(i >> 1) & 3] = add2(sm[(i >> 1) & 3], p);
        pk[i >> 1] = pack2<T>(p.x, p.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) pk[i] = 0u;
    }
    tmem_st16(p_tmem + 16 * c, pk);
  }
  const float2 t = add2(add2(sm[0], sm[1]), add2(sm[2], sm[3]));
  return t.x + t.y;
}

// tmK: K rows in boxes of KB rows; tmVt: V^T in boxes of 64 keys x 64 dims.
template <typename T, int KB>
__global__ void __launch_bounds__(kTcThreads, TcAttnCfg<KB>::kCtasPerSm)
    tc_attention_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmVt, const TcAttnArgs a) {
  using Cfg = TcAttnCfg<KB>;
  constexpr int NC = Cfg::kChunks;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // The tile table, starts and lengths are written by the host before the forward pass, so they
  // are read before waiting on the previous kernel.
  const bool gathered = a.q_index != nullptr;
  int t0, t1, row, nq = kTcQ;  // nq: queries of a gathered tile
  const int* qidx = nullptr;
  if (gathered) {
    row = blockIdx.y / a.q_tiles;
    const int part = blockIdx.y - row * a.q_tiles;
    nq = min(kTcQ, a.q_per_row - part * kTcQ);
    qidx = a.q_index + (size_t)row * a.q_per_row + part * kTcQ;
    t0 = t1 = 0;
    if (a.lengths[row] == 0) return;  // unused row of the shape class
  } else {
    const int4 tile = a.tiles[blockIdx.y];  // grid: (heads, tiles), all heads of a tile together
    t0 = tile.x; t1 = tile.y; row = tile.z;
    if (row == -2) return;
  }
  const int head = blockIdx.x;
  const int width = a.heads * 64;
  T* out = reinterpret_cast<T*>(a.out);
  if (row < 0) {
    // Tokens past the last row: zeros (8 x 16 bytes per token and head).
    pdl_wait();
    for (int i = threadIdx.x; i < (t1 - t0) * 8; i += kTcThreads) {
      const int t = t0 + (i >> 3);
      *reinterpret_cast<uint4*>(out + (size_t)t * width + head * 64 + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int first = a.starts[row];
  const int valid = a.lengths[row];
  const int q0 = gathered ? 0 : t0 - first;  // row-relative index of the tile's first query
  int k_lo = 0, k_hi = valid;
  if (a.window >= 0) {
    k_lo = max(0, q0 - a.window) & ~15;  // 16-token aligned: the V^T copy's inner coordinate
    k_hi = min(valid, q0 + kTcQ + a.window);
  }
  const int all_blocks = k_hi > k_lo ? (k_hi - k_lo + KB - 1) / KB : 0;
  // Key split: this CTA's share of the tile's blocks (k_lo stays 16-aligned: KB-key steps).
  const bool split = a.splits > 1;
  const uint32_t rank = split ? cluster_rank() : 0;
  int n_blocks = all_blocks;
  if (split) {
    const int h = (all_blocks + a.splits - 1) / a.splits;
    n_blocks = max(0, min(h, all_blocks - (int)rank * h));
    k_lo += (int)rank * h * KB;
  }

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::kOffQ;
  uint8_t* sK = smem + Cfg::kOffK;
  uint8_t* sV = smem + Cfg::kOffV;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;   // [2]
  uint64_t* v_full = bar + 3;   // [2]
  uint64_t* s_full = bar + 5;   // S_j ready, and every earlier MMA (so O) complete
  uint64_t* p_full = bar + 6;   // every warp wrote P_j
  uint64_t* o_full = bar + 7;   // the last P V product complete
  uint64_t* drain = bar + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const unsigned long long wait_ns = wait_limit(a.wait_ns);

  // Thread <-> query row r = TMEM lane r: warp w owns lanes [32w, 32w + 32).
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = threadIdx.x;
  const bool ctl = warp == 0;  // the control warp: TMEM allocation, copies and MMA issue (lane 0)
  if (threadIdx.x == 0) {
    mbar_init(q_full, gathered ? 4 : 1);  // gathered: the four warps write Q
    for (int s = 0; s < 2; ++s) { mbar_init(k_full + s, 1); mbar_init(v_full + s, 1); }
    mbar_init(s_full, 1); mbar_init(p_full, 4); mbar_init(o_full, 1); mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmVt);
  }
  if (ctl) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
  const uint32_t s_tmem = tmem_base + lane_addr, p_tmem = s_tmem, o_tmem = s_tmem + KB;
  const int plane_rows = a.heads * a.M;
  int k_issued = 0, v_issued = 0;  // copies issued (control lane)
  // Copies into stage j & 1 (control lane), issued once the commit covering the MMA that last
  // read the stage has been observed (S_{j-2} for K, P_{j-2} V_{j-2} for V).
  auto load_k = [&](int j) {
    const int st = j & 1;
    mbar_arrive_expect_tx(k_full + st, Cfg::kK);
    tma_load_2d(sK + st * Cfg::kK, &tmK, k_full + st, 0, plane_rows + head * a.M + first + k_lo + j * KB);
    k_issued = j + 1;
  };
  auto load_v = [&](int j) {
    const int st = j & 1;
    mbar_arrive_expect_tx(v_full + st, Cfg::kV);
#pragma unroll
    for (int h = 0; h < KB / 64; ++h)
      tma_load_2d(sV + st * Cfg::kV + h * 64 * 128, &tmVt, v_full + st, first + k_lo + j * KB + 64 * h, head * 64);
    v_issued = j + 1;
  };
  // S_j = Q K_j^T into TMEM columns [0, KB) once K_j has landed, then commit s_full (control warp).
  auto issue_s = [&](int j) -> bool {
    if (!mbar_wait(k_full + (j & 1), (j >> 1) & 1, a.err, kErrAttnWait, abort_flag, wait_ns)) return false;
    tc_fence_after();
    if (lane == 0) {
      const uint32_t idesc_s = mma_idesc<bf>(kTcQ, KB);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK + (j & 1) * Cfg::kK);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tc_mma_f16(tmem_base, smem_desc_sw128(q_addr + k * 32), smem_desc_sw128(k_addr + k * 32), idesc_s, k > 0);
      tc_commit(s_full);
    }
    __syncwarp();
    return true;
  };
  // O (+)= P_j V_j, A = P from TMEM columns [0, KB / 2), once V_j has landed (control warp).  Not
  // committed: the commit after the next S (or o_full after the last block) covers it.
  auto issue_pv = [&](int j) -> bool {
    if (!mbar_wait(v_full + (j & 1), (j >> 1) & 1, a.err, kErrAttnWait, abort_flag, wait_ns)) return false;
    tc_fence_after();
    if (lane == 0) {
      const uint32_t idesc_o = mma_idesc<bf>(kTcQ, 64);
      const uint32_t v_addr = smem_u32(sV + (j & 1) * Cfg::kV);
#pragma unroll
      for (int k = 0; k < KB / 16; ++k)
        tc_mma_f16_ts(tmem_base + KB, tmem_base + 8 * k, smem_desc_sw128(v_addr + (k >> 2) * 64 * 128 + (k & 3) * 32),
                      idesc_o, (j | k) != 0);
    }
    __syncwarp();
    return true;
  };

  bool ok = true;
  if (ctl && lane == 0 && n_blocks > 0) {
    if (!gathered) {
      mbar_arrive_expect_tx(q_full, Cfg::kQ);
      tma_load_2d(sQ, &tmQ, q_full, 0, head * a.M + t0);
    }
    for (int j = 0; j < n_blocks && j < 2; ++j) { load_k(j); load_v(j); }
  }

  const int q = q0 + r;              // row-relative query index of this thread
  const int qa = q0 + warp * 32;     // the warp's first query
  constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
  // Keys this query may see: row-relative [lo_key, lo_key + span_keys]; an empty range (a
  // padding query of a windowed layer) sees nothing.
  int lo_key = a.window >= 0 ? q - a.window : 0;
  const int hi_key = a.window >= 0 ? min(valid - 1, q + a.window) : valid - 1;
  uint32_t span_keys = (uint32_t)(hi_key - lo_key);
  if (hi_key < lo_key) { lo_key = 1 << 30; span_keys = 0; }
  const bool warp_live = gathered ? warp * 32 < nq : qa < valid;
  // Gathered queries: this thread's token, or -1 past nq and for an index outside the packed
  // rows (reported as kErrBadIndex; its Q row is zero and nothing is stored for it).
  int qtok = -1;
  if (gathered && r < nq) {
    qtok = qidx[r];
    if ((unsigned)qtok >= (unsigned)a.M) {
      if (a.err) atomicCAS(a.err, 0, kErrBadIndex);
      qtok = -1;
    }
  }
  if (gathered && n_blocks > 0) {
    // Q row r <- token qtok (zeros for -1), written in the 128-byte swizzled K-major layout the
    // TMA would produce, then handed to the async proxy.
    const T* qsrc = reinterpret_cast<const T*>(a.qk) + ((size_t)head * a.M + (qtok >= 0 ? qtok : 0)) * 64;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = qtok >= 0 ? *reinterpret_cast<const uint4*>(qsrc + c * 8) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(sQ + r * 128 + ((c ^ (r & 7)) << 4)) = v;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
  }
  if (ctl && n_blocks > 0) ok = mbar_wait(q_full, 0, a.err, kErrAttnWait, abort_flag, wait_ns) && issue_s(0);

  float m_used = -INFINITY, l = 0.f;
  for (int j = 0; j < n_blocks; ++j) {
    const int kb = k_lo + j * KB;
    // S_j is ready, and every MMA issued before it (P_{j-1} V_{j-1}) has completed.
    ok = ok && mbar_wait(s_full, j & 1, a.err, kErrAttnWait, abort_flag, wait_ns);
    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
    tc_fence_after();
    if (ctl && lane == 0) {
      // S_j completed: its K stage takes K_{j+2}.  P_{j-1} V_{j-1} completed: its V stage takes
      // V_{j+1} (V_0 and V_1 were loaded up front).
      if (j + 2 < n_blocks) load_k(j + 2);
      if (j >= 1 && j + 1 < n_blocks) load_v(j + 1);
    }
    // Chunk c holds keys [kb + 32c, kb + 32c + 32).  vis bit c: some query of the warp sees a
    // key of the chunk; full bit c: every query of the warp sees every key.  Warp-uniform.
    uint32_t vis = 0, full = 0;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int ck = kb + 32 * c;
      if (warp_live && ck < valid && (a.window < 0 || (ck + 31 >= qa - a.window && ck <= qa + 31 + a.window)))
        vis |= 1u << c;
      if (ck + 31 < valid && (a.window < 0 || (ck >= qa + 31 - a.window && ck + 31 <= qa + a.window)))
        full |= 1u << c;
    }
    full &= vis;
    uint32_t sx[NC][32];
#pragma unroll
    for (int c = 0; c < NC; ++c)
      if ((vis >> c) & 1) tmem_ld32_async(s_tmem + 32 * c, sx[c]);
#pragma unroll
    for (int c = 0; c < NC; ++c)
      if ((vis >> c) & 1) tmem_wait_ld(sx[c]);
    const bool all = full == (1u << NC) - 1;
    const float bmax = all ? tc_block_max<true, NC>(sx, vis, full, kb, lo_key, span_keys)
                           : tc_block_max<false, NC>(sx, vis, full, kb, lo_key, span_keys);
    const float m_new = bmax * kScaleLog2;
    float alpha = 1.f;
    bool o_dirty = false;
    if (m_new > m_used + kTcRescaleLog2) {  // false while every visible key is masked
      if (m_used != -INFINITY) { alpha = ex2_approx(m_used - m_new); o_dirty = true; }
      m_used = m_new;
    }
    const float sub = m_used == -INFINITY ? 0.f : m_used;
    // P_j goes over S_j's first columns, which this warp has read (the loads above completed).
    const float sum = all ? tc_block_probs<true, T, NC, Cfg::kPolyKey>(sx, vis, kScaleLog2, sub, p_tmem)
                          : tc_block_probs<false, T, NC, Cfg::kPolyKey>(sx, vis, kScaleLog2, sub, p_tmem);
    l = l * alpha + sum;
    // Rows whose maximum grew by more than 2^8 rescale O before P_j V_j accumulates into it (O
    // is settled: s_full covered every earlier MMA, and P_j V_j waits for p_full).
    if (__any_sync(0xffffffffu, o_dirty)) {
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t o[32];
        tmem_ld32_async(o_tmem + 32 * h, o);
        tmem_wait_ld(o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        tmem_st32(o_tmem + 32 * h, o);
      }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full);
    if (ctl) {
      // Once every warp has written P_j: O += P_j V_j, then S_{j+1}, whose commit covers both
      // (after the last block, o_full is committed instead).
      ok = ok && mbar_wait(p_full, j & 1, a.err, kErrAttnWait, abort_flag, wait_ns) && issue_pv(j);
      if (ok) {
        if (j + 1 < n_blocks) {
          ok = issue_s(j + 1);
        } else {
          if (lane == 0) tc_commit(o_full);
          __syncwarp();
        }
      }
    }
  }
  // Normalise and store this row (zeros for padding queries); rows past the tile belong to
  // other tiles and are not written.
  if (ok && n_blocks > 0) {
    ok = mbar_wait(o_full, 0, a.err, kErrAttnWait, abort_flag, wait_ns);
    ok = __all_sync(0xffffffffu, ok);
  }
  uint32_t o[2][32];
  if (ok && n_blocks > 0) {
    tc_fence_after();
    tmem_ld32_async(o_tmem, o[0]);
    tmem_ld32_async(o_tmem + 32, o[1]);
    tmem_wait_ld(o[0]);
    tmem_wait_ld(o[1]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) { o[0][i] = 0u; o[1][i] = 0u; }
  }
  if (split) {
    // Pairwise merge, step = 1 (and 2 for four ranks).  Every CTA of the cluster reaches both
    // barriers of every round on every path (the early returns above are taken by all CTAs of a
    // cluster alike).  (1): every CTA's MMAs have completed, so a receiver's Q, K and V buffers
    // are free (and, after the first round, its previous round's row has been merged); the
    // sender writes its row there: 64 O values, its running maximum (log2 units), its sum and
    // its status.  (2): the rows have landed and the receiver merges them.
    constexpr int kXRow = 68;  // floats per exchanged row (16-byte multiple)
    static_assert(kTcQ * kXRow * 4 <= Cfg::kOffBar, "exchange buffer");
    float* xrow = reinterpret_cast<float*>(sQ) + r * kXRow;
    for (uint32_t step = 1; step < (uint32_t)a.splits; step *= 2) {
      const bool sender = rank % (2 * step) == step, receiver = rank % (2 * step) == 0;
      cluster_sync();
      if (sender) {
        const uint32_t dst = cluster_addr(smem_u32(xrow), rank - step);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            st_cluster_v4(dst + (h * 32 + i) * 4, make_float4(__uint_as_float(o[h][i]), __uint_as_float(o[h][i + 1]),
                                                              __uint_as_float(o[h][i + 2]), __uint_as_float(o[h][i + 3])));
        st_cluster_v4(dst + 64 * 4, make_float4(m_used, l, ok ? 1.f : 0.f, 0.f));
      }
      cluster_sync();
      if (receiver) {
        const float4 ml = *reinterpret_cast<const float4*>(xrow + 64);
        ok = ok && ml.z != 0.f;
        // Rescale both partial results to the larger maximum (a side that saw no key has
        // maximum -inf, sum 0 and O 0, and weight 0).
        const float mx = fmaxf(m_used, ml.x);
        const float w0 = m_used == -INFINITY ? 0.f : ex2_approx(m_used - mx);
        const float w1 = ml.x == -INFINITY ? 0.f : ex2_approx(ml.x - mx);
        l = l * w0 + ml.y * w1;
        m_used = mx;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 p = *reinterpret_cast<const float4*>(xrow + h * 32 + i);
            o[h][i] = __float_as_uint(__uint_as_float(o[h][i]) * w0 + p.x * w1);
            o[h][i + 1] = __float_as_uint(__uint_as_float(o[h][i + 1]) * w0 + p.y * w1);
            o[h][i + 2] = __float_as_uint(__uint_as_float(o[h][i + 2]) * w0 + p.z * w1);
            o[h][i + 3] = __float_as_uint(__uint_as_float(o[h][i + 3]) * w0 + p.w * w1);
          }
      }
    }
  }
  if (ok && rank == 0) {
    const int token = gathered ? qtok : t0 + r;
    if (gathered ? token >= 0 : token < t1) {
      const bool live = all_blocks > 0 && (gathered || q < valid) && l > 0.f;
      const float inv = live ? 1.f / l : 0.f;
      T* dst = out + (size_t)token * width + head * 64;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = live ? __uint_as_float(o[h][i + e]) * inv : 0.f;
          uint4 w;
          w.x = pack2<T>(v[0], v[1]); w.y = pack2<T>(v[2], v[3]);
          w.z = pack2<T>(v[4], v[5]); w.w = pack2<T>(v[6], v[7]);
          *reinterpret_cast<uint4*>(dst + h * 32 + i) = w;
        }
    }
  }
  if (ctl && lane == 0) {
    // Every MMA issued completes before the TMEM is released, and every copy lands before the
    // CTA exits (bounded waits).
    tc_commit(drain);
    mbar_drain(drain, 0);
    if (*abort_flag) {
      if (!gathered && n_blocks > 0) mbar_drain(q_full, 0);
      for (int j = max(0, k_issued - 2); j < k_issued; ++j) mbar_drain(k_full + (j & 1), (j >> 1) & 1);
      for (int j = max(0, v_issued - 2); j < v_issued; ++j) mbar_drain(v_full + (j & 1), (j >> 1) & 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ctl) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

// ---------------------------------------------------------------------------------------------
// Persistent form of the 64-key kernel, for grids larger than the SMs' resident CTA slots (the
// throughput classes; no key split, no gathered queries).  Work item w = (tile w / heads, head
// w % heads); CTA c runs items c, c + G, c + 2G, ... (G = the grid) in order.  The tile table
// lists the longest rows first, so every CTA's list starts with the costliest items and the
// cheap ones even out the end.
//
// One TMEM allocation, one barrier set and one K/V stage ring serve all items of a CTA: the
// block counter g runs on across items, so the copies for the next item's first blocks are
// issued as soon as their stages free up (during the current item's last blocks), the next Q
// tile is loaded as soon as the current item's last S = Q K^T has completed, and the next
// item's first S is issued right after the current item's last P V product, so that it runs
// while the warps normalise and store the current item's output.  O is reused: the next item's
// first P V product (which overwrites O) waits for p_full, which every warp reaches only after
// it has read the current item's O.
//
// Item descriptors are read once, before the dependency wait (the tile table, starts and
// lengths are written by the host), into shared memory: (t0, t1, first, valid) and
// (k_lo, blocks, head, 0); valid < 0 marks the table's zero-fill (-1) and unused (-2) entries.
constexpr int kTcItems = 128;  // work items per persistent CTA at most (the host sizes the grid)

struct TcPersistCfg : TcAttnCfg<64> {
  static constexpr int kOffItems = TcAttnCfg<64>::kOffBar + 256;
  static constexpr int kBytes = kOffItems + kTcItems * 32 + 1024;
  static_assert(kCtasPerSm * (kBytes + 1024) <= 228 * 1024, "shared memory of the resident CTAs");
};

template <typename T>
__global__ void __launch_bounds__(kTcThreads, TcPersistCfg::kCtasPerSm)
    tc_attention_persistent_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                                   const __grid_constant__ CUtensorMap tmVt, const TcAttnArgs a) {
  using Cfg = TcPersistCfg;
  constexpr int KB = 64, NC = 2;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + Cfg::kOffQ;
  uint8_t* sK = smem + Cfg::kOffK;
  uint8_t* sV = smem + Cfg::kOffV;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;   // [2]
  uint64_t* v_full = bar + 3;   // [2]
  uint64_t* s_full = bar + 5;   // S_g ready, and every earlier MMA complete
  uint64_t* p_full = bar + 6;   // every warp wrote P_g
  uint64_t* o_full = bar + 7;   // an item's last P V product complete
  uint64_t* drain = bar + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int4* items = reinterpret_cast<int4*>(smem + Cfg::kOffItems);

  const int n_work = a.n_tiles * a.heads;
  int n_mine = (int)blockIdx.x < n_work ? (n_work - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  if (n_mine > kTcItems) {  // the host sizes the grid so that this never happens
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrLaunchShape);
    n_mine = kTcItems;
  }
  for (int k = threadIdx.x; k < n_mine; k += kTcThreads) {
    const int w = blockIdx.x + k * gridDim.x;
    const int4 tile = a.tiles[w / a.heads];
    int first = 0, valid = tile.z < 0 ? tile.z : 0, k_lo = 0, blocks = 0;
    if (tile.z >= 0) {
      first = a.starts[tile.z];
      valid = a.lengths[tile.z];
      const int q0 = tile.x - first;
      int k_hi = valid;
      if (a.window >= 0) {
        k_lo = max(0, q0 - a.window) & ~15;  // 16-token aligned: the V^T copy's inner coordinate
        k_hi = min(valid, q0 + kTcQ + a.window);
      }
      blocks = k_hi > k_lo ? (k_hi - k_lo + KB - 1) / KB : 0;
    }
    items[2 * k] = make_int4(tile.x, tile.y, first, valid);
    items[2 * k + 1] = make_int4(k_lo, blocks, w % a.heads, 0);
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = threadIdx.x;
  const bool ctl = warp == 0;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) { mbar_init(k_full + s, 1); mbar_init(v_full + s, 1); }
    mbar_init(s_full, 1); mbar_init(p_full, 4); mbar_init(o_full, 1); mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmVt);
  }
  if (ctl) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();

  constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
  const uint32_t lane_addr = (uint32_t)(warp * 32) << 16;
  const uint32_t s_tmem = tmem_base + lane_addr, p_tmem = s_tmem, o_tmem = s_tmem + KB;
  // Kernel parameters stay in the constant bank: width = heads * 64, the K plane at heads * M.
  T* const out = reinterpret_cast<T*>(a.out);
  auto blocks_of = [&](int k) { return items[2 * k + 1].y; };
  auto next_item = [&](int k) {  // the first item at or after k that has key blocks
    while (k < n_mine && blocks_of(k) == 0) ++k;
    return k;
  };
  // Copy state of the control lane, kept in shared memory between its turns (registers are the
  // softmax's) and held in registers within a turn: for K and V^T the next (item, block) to
  // load as the item, its blocks still to load and the tile's coordinate (K: the row in the
  // tensor map; V^T: the first key's column, with the head's row block); the next item whose Q
  // tile to load; and `ph`: bit b (K stages 0-1, V stages 2-3, Q 4) the parity of the next copy
  // into that buffer, bit 5 + b set once a copy was issued into it (for the drain after an abort).
  struct Copies {
    int k_item, k_left, k_at, q_item;
    int v_item, v_left, v_at, v_head;
    uint32_t ph, pad0, pad1, pad2;
  };
  int4* copies_smem = reinterpret_cast<int4*>(bar + 10);  // 48 bytes, 16-byte aligned
  auto get_copies = [&]() {
    Copies c;
    const int4 x = copies_smem[0], y = copies_smem[1], z = copies_smem[2];
    c.k_item = x.x; c.k_left = x.y; c.k_at = x.z; c.q_item = x.w;
    c.v_item = y.x; c.v_left = y.y; c.v_at = y.z; c.v_head = y.w;
    c.ph = (uint32_t)z.x; c.pad0 = c.pad1 = c.pad2 = 0;
    return c;
  };
  auto put_copies = [&](const Copies& c) {
    copies_smem[0] = make_int4(c.k_item, c.k_left, c.k_at, c.q_item);
    copies_smem[1] = make_int4(c.v_item, c.v_left, c.v_at, c.v_head);
    copies_smem[2] = make_int4((int)c.ph, 0, 0, 0);
  };
  auto seek_k = [&](Copies& c, int item) {  // the first block of `item` or a later one (or the end)
    c.k_item = next_item(item);
    if (c.k_item < n_mine) {
      const int4 d0 = items[2 * c.k_item], d1 = items[2 * c.k_item + 1];
      c.k_left = d1.y;
      c.k_at = (a.heads + d1.z) * a.M + d0.z + d1.x;
    }
  };
  auto seek_v = [&](Copies& c, int item) {
    c.v_item = next_item(item);
    if (c.v_item < n_mine) {
      const int4 d0 = items[2 * c.v_item], d1 = items[2 * c.v_item + 1];
      c.v_left = d1.y;
      c.v_at = d0.z + d1.x;
      c.v_head = d1.z;
    }
  };
  auto issued = [&](Copies& c, int b) {
    c.ph ^= 1u << b;
    c.ph |= 32u << b;
  };
  auto load_k = [&](Copies& c, int block) {  // block: the block counter g of the copy
    const int st = block & 1;
    mbar_arrive_expect_tx(k_full + st, Cfg::kK);
    tma_load_2d(sK + st * Cfg::kK, &tmK, k_full + st, 0, c.k_at);
    issued(c, st);
    if (--c.k_left > 0) c.k_at += KB;
    else seek_k(c, c.k_item + 1);
  };
  auto load_v = [&](Copies& c, int block) {
    const int st = block & 1;
    mbar_arrive_expect_tx(v_full + st, Cfg::kV);
    tma_load_2d(sV + st * Cfg::kV, &tmVt, v_full + st, c.v_at, c.v_head * 64);
    issued(c, 2 + st);
    if (--c.v_left > 0) c.v_at += KB;
    else seek_v(c, c.v_item + 1);
  };
  auto load_q = [&](Copies& c) {
    const int4 d0 = items[2 * c.q_item], d1 = items[2 * c.q_item + 1];
    mbar_arrive_expect_tx(q_full, Cfg::kQ);
    tma_load_2d(sQ, &tmQ, q_full, 0, d1.z * a.M + d0.x);
    issued(c, 4);
    c.q_item = next_item(c.q_item + 1);
  };
  // S_g = Q K_g^T into TMEM columns [0, 64), then commit s_full (control warp).
  auto issue_s = [&](int g) -> bool {
    if (!mbar_wait(k_full + (g & 1), (g >> 1) & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns))) return false;
    tc_fence_after();
    if (lane == 0) {
      const uint32_t idesc_s = mma_idesc<bf>(kTcQ, KB);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK + (g & 1) * Cfg::kK);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        tc_mma_f16(tmem_base, smem_desc_sw128(q_addr + k * 32), smem_desc_sw128(k_addr + k * 32), idesc_s, k > 0);
      tc_commit(s_full);
    }
    __syncwarp();
    return true;
  };
  // O (+)= P_g V_g (A = P from TMEM columns [0, 32)); `fresh`: the item's first block.
  auto issue_pv = [&](int g, bool fresh) -> bool {
    if (!mbar_wait(v_full + (g & 1), (g >> 1) & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns))) return false;
    tc_fence_after();
    if (lane == 0) {
      const uint32_t idesc_o = mma_idesc<bf>(kTcQ, 64);
      const uint32_t v_addr = smem_u32(sV + (g & 1) * Cfg::kV);
#pragma unroll
      for (int k = 0; k < KB / 16; ++k)
        tc_mma_f16_ts(tmem_base + KB, tmem_base + 8 * k, smem_desc_sw128(v_addr + k * 32), idesc_o, !fresh || k != 0);
    }
    __syncwarp();
    return true;
  };
  bool ok = true;
  const int first_item = next_item(0);
  if (ctl && lane == 0) {
    Copies c;
    c.ph = 0;
    seek_k(c, 0);
    seek_v(c, 0);
    c.q_item = c.k_item;
    if (first_item < n_mine) {
      load_q(c);
      for (int i = 0; i < 2 && c.k_item < n_mine; ++i) load_k(c, i);
      for (int i = 0; i < 2 && c.v_item < n_mine; ++i) load_v(c, i);
    }
    put_copies(c);
  }
  if (ctl && first_item < n_mine) ok = mbar_wait(q_full, 0, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns)) && issue_s(0);

  constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
  int g = 0, seq = 0;  // key blocks and items with key blocks done so far
  for (int k = 0; k < n_mine && ok; ++k) {
    const int n_blocks = items[2 * k + 1].y;
    if (n_blocks == 0) {
      // Tokens past the last row (or a tile no key reaches): zeros; unused entries: nothing.
      const int4 d0 = items[2 * k];
      const int head = items[2 * k + 1].z;
      if (d0.w != -2)
        for (int i = threadIdx.x; i < (d0.y - d0.x) * 8; i += kTcThreads) {
          const int t = d0.x + (i >> 3);
          *reinterpret_cast<uint4*>(out + (size_t)t * (a.heads * 64) + head * 64 + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
        }
      continue;
    }
    const int valid = items[2 * k].w, k_lo = items[2 * k + 1].x;
    const int q = items[2 * k].x - items[2 * k].z + r;  // row-relative index of this thread's query
    const int qa = q - lane;                            // the warp's first query
    int lo_key = a.window >= 0 ? q - a.window : 0;
    const int hi_key = a.window >= 0 ? min(valid - 1, q + a.window) : valid - 1;
    uint32_t span_keys = (uint32_t)(hi_key - lo_key);
    if (hi_key < lo_key) { lo_key = 1 << 30; span_keys = 0; }
    const bool warp_live = qa < valid;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; j < n_blocks; ++j, ++g) {
      const int kb = k_lo + j * KB;
      ok = ok && mbar_wait(s_full, g & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns));
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      if (ctl && lane == 0) {
        // S_g completed: its K stage takes block g + 2; P_{g-1} V_{g-1} completed: its V stage
        // takes block g + 1 (blocks 0 and 1 were loaded up front, so the cursors stand at
        // exactly these blocks); after the item's last S the Q tile takes the next item's.
        Copies c = get_copies();
        if (c.k_item < n_mine) load_k(c, g + 2);
        if (g >= 1 && c.v_item < n_mine) load_v(c, g + 1);
        if (j + 1 == n_blocks && c.q_item < n_mine) load_q(c);
        put_copies(c);
      }
      uint32_t vis = 0, full = 0;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int ck = kb + 32 * c;
        if (warp_live && ck < valid && (a.window < 0 || (ck + 31 >= qa - a.window && ck <= qa + 31 + a.window)))
          vis |= 1u << c;
        if (ck + 31 < valid && (a.window < 0 || (ck >= qa + 31 - a.window && ck + 31 <= qa + a.window)))
          full |= 1u << c;
      }
      full &= vis;
      uint32_t sx[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c)
        if ((vis >> c) & 1) tmem_ld32_async(s_tmem + 32 * c, sx[c]);
#pragma unroll
      for (int c = 0; c < NC; ++c)
        if ((vis >> c) & 1) tmem_wait_ld(sx[c]);
      const bool all = full == (1u << NC) - 1;
      const float bmax = all ? tc_block_max<true, NC>(sx, vis, full, kb, lo_key, span_keys)
                             : tc_block_max<false, NC>(sx, vis, full, kb, lo_key, span_keys);
      const float m_new = bmax * kScaleLog2;
      float alpha = 1.f;
      bool o_dirty = false;
      if (m_new > m_used + kTcRescaleLog2) {
        if (m_used != -INFINITY) { alpha = ex2_approx(m_used - m_new); o_dirty = true; }
        m_used = m_new;
      }
      const float sub = m_used == -INFINITY ? 0.f : m_used;
      const float sum = all ? tc_block_probs<true, T, NC, Cfg::kPolyKey>(sx, vis, kScaleLog2, sub, p_tmem)
                            : tc_block_probs<false, T, NC, Cfg::kPolyKey>(sx, vis, kScaleLog2, sub, p_tmem);
      l = l * alpha + sum;
      if (__any_sync(0xffffffffu, o_dirty)) {
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t o[32];
          tmem_ld32_async(o_tmem + 32 * h, o);
          tmem_wait_ld(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_tmem + 32 * h, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (ctl) {
        // Every warp wrote P_g: O += P_g V_g, then the next S (this item's next block, or the
        // next item's first block once its Q tile has landed), whose commit covers both; after
        // an item's last block o_full is committed first.
        ok = ok && mbar_wait(p_full, g & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns)) && issue_pv(g, j == 0);
        if (ok) {
          if (j + 1 < n_blocks) {
            ok = issue_s(g + 1);
          } else {
            if (lane == 0) tc_commit(o_full);
            __syncwarp();
            if (next_item(k + 1) < n_mine)
              ok = mbar_wait(q_full, (seq + 1) & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns)) && issue_s(g + 1);
          }
        }
      }
    }
    if (!ok) break;
    // Normalise and store this item's rows (zeros for padding queries).
    ok = mbar_wait(o_full, seq & 1, a.err, kErrAttnWait, abort_flag, wait_limit(a.wait_ns));
    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
    tc_fence_after();
    ++seq;
    // One 32-column half of O at a time (registers: the loop keeps its state live here).
    const int token = items[2 * k].x + r;
    const bool store = token < items[2 * k].y;
    const bool live = q < valid && l > 0.f;
    const float inv = live ? 1.f / l : 0.f;
    T* dst = out + (size_t)token * (a.heads * 64) + items[2 * k + 1].z * 64;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      uint32_t o[32];
      tmem_ld32_async(o_tmem + 32 * h, o);
      tmem_wait_ld(o);
      if (store) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = live ? __uint_as_float(o[i + e]) * inv : 0.f;
          uint4 w;
          w.x = pack2<T>(v[0], v[1]); w.y = pack2<T>(v[2], v[3]);
          w.z = pack2<T>(v[4], v[5]); w.w = pack2<T>(v[6], v[7]);
          *reinterpret_cast<uint4*>(dst + h * 32 + i) = w;
        }
      }
    }
  }
  if (ctl && lane == 0) {
    // Every MMA issued completes before the TMEM is released, and every copy lands before the
    // CTA exits (bounded waits).
    tc_commit(drain);
    mbar_drain(drain, 0);
    if (*abort_flag) {
      // The last copy into each buffer has the parity before its bit's last toggle.
      // Buffers 0-3 are k_full[0..1], v_full[0..1] (barriers 1-4); buffer 4 is q_full (barrier 0).
      const uint32_t ph = get_copies().ph;
      for (int b = 0; b < 5; ++b)
        if ((ph >> (5 + b)) & 1) mbar_drain(bar + (b < 4 ? b + 1 : 0), ((ph >> b) & 1) ^ 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ctl) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

}  // namespace laya
