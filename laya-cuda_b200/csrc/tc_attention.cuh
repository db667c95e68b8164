// Varlen packed attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), used by the
// forward pass.  Same semantics as attention.cuh, which restates the reference kernel
// laya_cuda/kernels.cu:90-154: rows packed at 16-token alignment, key j visible to query i of
// the same row iff j < length and (window < 0 or |i - j| <= window), scores scaled by 1/8,
// fp32 softmax, padding queries and tokens past the last row produce zeros.
//
// Work unit: one CTA per (128-query tile of one row, head); the host's tile table never lets a
// tile straddle rows.  6 warps:
//   warp 0     TMA: the Q tile once, then per 128-key block the K tile and the V^T tile
//              (128-byte swizzle, no multicast).
//   warp 1     TMEM allocation + MMA issue (one thread): S = Q K^T (M=128, N=128, K=64) into
//              TMEM columns [0,128); O_blk = P V (M=128, N=64, K=128) into columns [128,192).
//   warps 2-5  softmax, one thread per query row: reads its S row from TMEM, online max and
//              sum in fp32, writes P (16-bit, swizzled K-major) to shared memory for the P V
//              product, and accumulates O in registers: o = o * exp2(m_old - m_new) + O_blk.
// Inputs (from the QKV GEMM epilogue): Q, K [heads][M][64] (K-major rows of 128 bytes) and V
// transposed [heads][64][M], so every MMA operand is K-major, as in gemm.cuh.  Every wait is
// bounded and reports through the error word.
#pragma once
#include "common.cuh"

namespace laya {

constexpr int kTcQ = 128;          // queries per CTA
constexpr int kTcKB = 128;         // keys per block
constexpr int kTcThreads = 192;
constexpr int kTcTmemCols = 256;   // S: [0,128), O: [128,192)

struct TcAttnArgs {
  void* out;            // [M][heads*64]
  const int4* tiles;    // (t0, t1, row, 0): 128-query tiles; row -1: zero-fill; row -2: unused
  const int* starts;
  const int* lengths;
  int M;
  int heads;
  int window;           // -1: global
  int* err;
};

struct TcAttnSmem {
  static constexpr int kQ = kTcQ * 128;            // 16 KB: [128 queries][64 dims]
  static constexpr int kK = kTcKB * 128;           // 16 KB: [128 keys][64 dims]
  static constexpr int kV = 2 * 64 * 128;          // 16 KB: two [64 dims][64 keys] tiles
  static constexpr int kP = 2 * kTcQ * 128;        // 32 KB: two [128 queries][64 keys] tiles
  static constexpr int kOffQ = 0, kOffK = kQ, kOffV = kQ + kK, kOffP = kQ + kK + kV;
  static constexpr int kOffBar = kOffP + kP;
  static constexpr int kBytes = kOffBar + 256 + 1024;  // barriers + alignment slack
};

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 2) tc_attention_kernel(const __grid_constant__ CUtensorMap tmQK,
                                                                    const __grid_constant__ CUtensorMap tmVt,
                                                                    const TcAttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + TcAttnSmem::kOffQ;
  uint8_t* sK = smem + TcAttnSmem::kOffK;
  uint8_t* sV = smem + TcAttnSmem::kOffV;
  uint8_t* sP = smem + TcAttnSmem::kOffP;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TcAttnSmem::kOffBar);
  uint64_t* q_full = bar + 0;
  uint64_t* k_full = bar + 1;
  uint64_t* k_empty = bar + 2;
  uint64_t* v_full = bar + 3;
  uint64_t* v_empty = bar + 4;
  uint64_t* s_full = bar + 5;
  uint64_t* s_free = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* o_full = bar + 8;
  uint64_t* drain = bar + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int width = a.heads * 64;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1); mbar_init(k_full, 1); mbar_init(k_empty, 1); mbar_init(v_full, 1);
    mbar_init(v_empty, 1); mbar_init(s_full, 1); mbar_init(s_free, 4); mbar_init(p_full, 4);
    mbar_init(o_full, 1); mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmQK); tma_prefetch_desc(&tmVt); }
  if (warp == 1) { tmem_alloc(tmem_slot, kTcTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  const int4 tile = a.tiles[blockIdx.x];
  const int t0 = tile.x, t1 = tile.y, row = tile.z;
  T* out = reinterpret_cast<T*>(a.out);
  int first = 0, valid = 0, q0 = 0, k_lo = 0, n_blocks = 0;
  if (row >= 0) {
    first = a.starts[row];
    valid = a.lengths[row];
    q0 = t0 - first;
    int k_hi = valid;
    if (a.window >= 0) {
      k_lo = max(0, q0 - a.window);
      k_hi = min(valid, q0 + kTcQ + a.window);
    }
    k_lo = (k_lo / kTcKB) * kTcKB;
    n_blocks = k_hi > k_lo ? (k_hi - k_lo + kTcKB - 1) / kTcKB : 0;
  }

  if (row < 0 || n_blocks == 0) {
    // Unused slot, or tokens past the last row: zeros (8 x 16 bytes per token and head).
    if (row == -1) {
      for (int i = threadIdx.x; i < (t1 - t0) * 8; i += kTcThreads) {
        const int t = t0 + (i >> 3);
        *reinterpret_cast<uint4*>(out + (size_t)t * width + head * 64 + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
      }
    }
  } else if (warp == 0) {
    if (lane == 0) {
      const int plane_rows = a.heads * a.M;
      bool ok = true;
      uint32_t k_inflight = 0, v_inflight = 0;  // 1 while a load has been issued but not consumed
      mbar_arrive_expect_tx(q_full, TcAttnSmem::kQ);
      tma_load_2d(sQ, &tmQK, q_full, 0, head * a.M + t0);
      for (int j = 0; j < n_blocks && ok; ++j) {
        const int key0 = first + k_lo + j * kTcKB;  // absolute token of the block's first key
        if (!mbar_wait(k_empty, (j & 1) ^ 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(k_full, TcAttnSmem::kK);
        tma_load_2d(sK, &tmQK, k_full, 0, plane_rows + head * a.M + key0);
        k_inflight = 1;
        if (!mbar_wait(v_empty, (j & 1) ^ 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(v_full, TcAttnSmem::kV);
        tma_load_2d(sV, &tmVt, v_full, key0, head * 64);
        tma_load_2d(sV + 64 * 128, &tmVt, v_full, key0 + 64, head * 64);
        v_inflight = 1;
      }
      if (!ok) {
        // Let copies already in flight land before the CTA exits.
        mbar_wait(q_full, 0, nullptr, 0, abort_flag);
        (void)k_inflight; (void)v_inflight;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr bool bf = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t idesc_s = mma_idesc<bf>(kTcQ, kTcKB);
      const uint32_t idesc_o = mma_idesc<bf>(kTcQ, 64);
      const uint32_t s_tmem = tmem_base, o_tmem = tmem_base + kTcKB;
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, a.err, kErrAttnWait, abort_flag);
      for (int j = 0; j < n_blocks && ok; ++j) {
        // S_j = Q K_j^T once K_j has landed and the softmax has read S_{j-1}.
        if (!mbar_wait(k_full, j & 1, a.err, kErrAttnWait, abort_flag)) break;
        if (!mbar_wait(s_free, (j & 1) ^ 1, a.err, kErrAttnWait, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tc_mma_f16(s_tmem, smem_desc_sw128(q_addr + k * 32), smem_desc_sw128(k_addr + k * 32), idesc_s, k > 0);
        tc_commit(s_full);
        tc_commit(k_empty);
        // O_j = P_j V_j once the softmax has written P_j and V_j has landed.
        if (!mbar_wait(p_full, j & 1, a.err, kErrAttnWait, abort_flag)) break;
        if (!mbar_wait(v_full, j & 1, a.err, kErrAttnWait, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f16(o_tmem, smem_desc_sw128(p_addr + c * kTcQ * 128 + k * 32),
                       smem_desc_sw128(v_addr + c * 64 * 128 + k * 32), idesc_o, (c | k) != 0);
        tc_commit(o_full);
        tc_commit(v_empty);
      }
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, abort_flag);
    }
  } else {
    // Softmax warps: thread <-> query row r (TMEM lane r).
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int q = q0 + r;                                 // row-relative query index
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_tmem = tmem_base + lane_addr, o_tmem = tmem_base + lane_addr + kTcKB;
    constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    uint8_t* p_row0 = sP + r * 128;                       // P tile 0 (keys 0-63), row r
    uint8_t* p_row1 = sP + kTcQ * 128 + r * 128;          // P tile 1 (keys 64-127), row r
    bool ok = true;
    for (int j = 0; j < n_blocks && ok; ++j) {
      const int kb = k_lo + j * kTcKB;
      if (!mbar_wait(s_full, j & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      tc_fence_after();
      // Pass 1: the row maximum over this block's visible keys.
      float bm = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32];
        tmem_ld32(s_tmem + c * 32, x);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = kb + c * 32 + i;
          bool keep = key < valid;
          if (a.window >= 0) keep = keep && abs(key - q) <= a.window;
          if (keep) bm = fmaxf(bm, x[i] * kScaleLog2);
        }
      }
      const float m_new = fmaxf(m, bm);
      const float alpha = m_new == -INFINITY ? 1.f : exp2f(m - m_new);
      const float sub = m_new == -INFINITY ? 0.f : m_new;
      // Pass 2: probabilities, their sum, and P (16-bit, 128-byte swizzled rows) in smem.
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float x[32];
        tmem_ld32(s_tmem + c * 32, x);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = kb + c * 32 + i + e;
            bool keep = key < valid;
            if (a.window >= 0) keep = keep && abs(key - q) <= a.window;
            p2[e] = keep ? exp2f(x[i + e] * kScaleLog2 - sub) : 0.f;
            sum += p2[e];
          }
          pk[i / 2] = pack2<T>(p2[0], p2[1]);
        }
        uint8_t* prow = (c < 2) ? p_row0 : p_row1;
#pragma unroll
        for (int piece = 0; piece < 4; ++piece) {
          const int logical = (c & 1) * 4 + piece;      // 16-byte piece within the 128-byte row
          const int phys = logical ^ (r & 7);
          *reinterpret_cast<uint4*>(prow + phys * 16) =
              make_uint4(pk[piece * 4], pk[piece * 4 + 1], pk[piece * 4 + 2], pk[piece * 4 + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) { mbar_arrive(s_free); mbar_arrive(p_full); }
      l = l * alpha + sum;
      m = m_new;
      if (!mbar_wait(o_full, j & 1, a.err, kErrAttnWait, abort_flag)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float o[32];
        tmem_ld32(o_tmem + h * 32, o);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[h * 32 + i] = acc[h * 32 + i] * alpha + o[i];
      }
    }
    // Normalise and store this row (zeros for padding queries); rows past the tile belong to
    // other tiles and are not written.
    const int token = t0 + r;
    if (token < t1) {
      const float inv = (ok && q < valid && l > 0.f) ? 1.f / l : 0.f;
      T* dst = out + (size_t)token * width + head * 64;
#pragma unroll
      for (int i = 0; i < 64; i += 8) {
        uint4 w;
        w.x = pack2<T>(acc[i] * inv, acc[i + 1] * inv); w.y = pack2<T>(acc[i + 2] * inv, acc[i + 3] * inv);
        w.z = pack2<T>(acc[i + 4] * inv, acc[i + 5] * inv); w.w = pack2<T>(acc[i + 6] * inv, acc[i + 7] * inv);
        *reinterpret_cast<uint4*>(dst + i) = w;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTcTmemCols);
}

}  // namespace laya
