// Residual GEMM with the following LayerNorm fused into its epilogue:
//
//   residual[M, N] += A[M, K] * W[N, K]^T + bias;   x = LN(residual) * gamma (+ beta)
//
// for the encoder's attention-out -> mlp_norm and FFN-down -> next attn_norm pairs
// (reference: runtime.py:96-108 calling linear, add and layer_norm, kernels.cu:20-49), so the
// updated residual never makes a second trip through HBM for its normalisation.
//
// A LayerNorm needs whole rows, and a row of N = C x BN fp32 accumulators does not fit one
// SM's TMEM next to a second accumulator buffer, so C CTAs form a cluster that owns a 128-row
// block: CTA `rank` computes columns [BN rank, BN rank + BN) of it (d = 768: C = 3, BN = 256
// with a 3-stage operand ring for short K, where the longer MMA per tile hides the epilogue;
// C = 4, BN = 192 with a 4-stage ring for long K, where load latency matters more).  The row
// statistics are combined through distributed shared memory: every epilogue thread computes,
// for its row and its BN/2 columns, the partial sum and the partial centred sum of squares and
// sends both to every CTA of the cluster with st.async, which counts its bytes on the
// receiving CTA's exchange mbarrier (armed once per tile with the expected byte count).  No
// release fence is involved, so the exchange does not wait for the epilogue's outstanding
// global stores.  The partials are merged with Chan's parallel-variance formula,
// M2 = sum M2_i + n sum (mean_i - mean)^2, so the result is the centred (two-pass) variance of
// the reference's LayerNorm, with one exchange per tile.
//
// Per CTA the roles are those of gemm_kernel (warp 0 TMA, warp 1 TMEM + MMA, warps 2-9
// epilogue; two BN-column TMEM accumulators so tile i's epilogue overlaps tile i+1's MMAs).
// The epilogue keeps the updated residual in the accumulator's TMEM columns between its three
// passes: (A) v = acc + bias + residual, written to HBM and back to TMEM, with this thread's
// partial sum and centred M2 (per 32-column chunk in registers, merged with Chan's formula);
// exchange; (C) x = (v - mean) * rstd * gamma (+ beta), rounded once.  Global traffic goes
// through the per-warp swizzled staging block of gemm.cuh, so it covers whole 128-byte lines.
// Clusters walk the row blocks in lock step (same order in every CTA of a cluster).
#pragma once
#include "gemm.cuh"

namespace laya {

struct GemmLnArgs {
  int M, N, K;              // N = C * BN
  float* residual;          // [M][ldr] fp32, updated in place
  int ldr;
  const float* bias;        // [N] or nullptr
  const float* gamma;       // [N]
  const float* beta;        // [N] or nullptr
  float eps;
  void* x;                  // [M][ldx] T: the normalised rows
  int ldx;
  int* err;
  unsigned long long wait_ns;  // wait limit of this launch (0: kWaitTimeoutNs)
};

template <int C, int BN>
struct GemmLnCfg {
  static_assert(BN == 192 || BN == 256, "column block of 192 or 256");
  static constexpr int kStageA = kBM * kBK * 2;
  static constexpr int kStageB = BN * kBK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = 3;
  static constexpr int kOffEpi = kStages * kStageBytes;
  static constexpr int kChunks = BN / 64;  // 32-column chunks per epilogue warp
  // Per epilogue warp, two 4 KB blocks (1024-byte aligned: the 128-byte swizzle pattern) for its
  // 32 x 32 fp32 residual chunks; the second doubles as the staging block of the LayerNorm pass.
  static constexpr int kRingBlock = 32 * 32 * 4;
  static constexpr int kRingBytes = kEpiWarps * 2 * kRingBlock;
  // Exchange: [2 parity][2C partials][128 rows][sum, M2] fp32.
  static constexpr int kOffX = kOffEpi + kRingBytes;
  static constexpr int kXBytes = 2 * 2 * C * kBM * 2 * 4;
  static constexpr uint32_t kXTxBytes = C * kEpiWarps * 32 * 8;  // received per CTA per tile
  static constexpr int kOffBar = kOffX + kXBytes;
  // The CTA's column block of gamma (fp32), read by the LayerNorm pass.
  static constexpr int kOffGB = kOffBar + 512;
  static constexpr int kSmemBytes = kOffGB + BN * 4 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory of one CTA");
};

// Asynchronous store of two floats into a cluster CTA's shared memory (cluster address `addr`,
// 8-byte aligned) whose 8 bytes complete on the mbarrier at cluster address `bar`.
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float a, float b, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "f"(a), "f"(b), "r"(bar)
               : "memory");
}

// Staging-block accessors for the coalesced <-> row-per-lane transposes (see gemm.cuh).
__device__ __forceinline__ void stage_put_co(uint8_t* buf, int k, int lane, uint4 v) {
  *reinterpret_cast<uint4*>(buf + stage_off(4 * k + (lane >> 3), lane & 7)) = v;
}
__device__ __forceinline__ uint4 stage_get_row(const uint8_t* buf, int lane, int j) {
  return *reinterpret_cast<const uint4*>(buf + stage_off(lane, j));
}

template <int C, int BN, typename T>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmR, const GemmLnArgs args) {
  using Cfg = GemmLnCfg<C, BN>;
  constexpr int NCH = Cfg::kChunks;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * Cfg::kStageA;
  float* xbuf = reinterpret_cast<float*>(smem + Cfg::kOffX);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = bars + 2 * S + 2;
  uint64_t* xbar = bars + 2 * S + 4;   // [2 parity]
  uint64_t* drain = bars + 2 * S + 6;
  uint64_t* rbar = bars + 2 * S + 7;   // [8 epilogue warps][2 blocks]: residual chunk landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 7 + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const unsigned long long wait_ns = wait_limit(args.wait_ns);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const int cid = blockIdx.x / C, n_clusters = gridDim.x / C;
  const int m_blocks = (args.M + kBM - 1) / kBM;
  const int k_blocks = args.K / kBK;
  const int nb = rank;  // this CTA's BN-column block

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&tfull[i], 1); mbar_init(&tempty[i], kEpiWarps); }
    for (int i = 0; i < 2; ++i) mbar_init(&xbar[i], 1);  // armed with expect_tx once per tile
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&rbar[i], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); tma_prefetch_desc(&tmR); }
  if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
  tc_fence_before();
  cluster_sync();  // every CTA's exchange barriers exist before the first remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0; uint32_t phase = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      // This CTA's weight slice does not depend on the previous kernel: the first tile's weight
      // stages are loaded before waiting for it.
      int pre = 0;
      if (cid < m_blocks) {
        pre = k_blocks < S ? k_blocks : S;
        for (int kb = 0; kb < pre; ++kb) {
          mbar_arrive_expect_tx(&full[kb], Cfg::kStageBytes);
          tma_load_2d(sB + kb * Cfg::kStageB, &tmB, &full[kb], kb * kBK, nb * BN);
        }
      }
      pdl_wait();
      for (int mb = cid; mb < m_blocks && ok; mb += n_clusters) {
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (mb == cid && kb < pre) {
            tma_load_2d(sA + stage * Cfg::kStageA, &tmA, &full[stage], kb * kBK, mb * kBM);
          } else {
            if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrGemmProducerWait, abort_flag, wait_ns)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
            tma_load_2d(sA + stage * Cfg::kStageA, &tmA, &full[stage], kb * kBK, mb * kBM);
            tma_load_2d(sB + stage * Cfg::kStageB, &tmB, &full[stage], kb * kBK, nb * BN);
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
      // Every copy issued lands before the CTA exits (bounded by time, on every path: another
      // role may have given up without consuming them).
      (void)ok;
      for (int s = 0; s < S; ++s)
        if (issued & (1u << s)) mbar_drain(&full[s], (last_par >> s) & 1);
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      const uint32_t idesc = mma_idesc<std::is_same<T, __nv_bfloat16>::value>(kBM, BN);
      int stage = 0; uint32_t phase = 0;
      int acc = 0; uint32_t acc_phase = 0;
      bool ok = true;
      for (int mb = cid; mb < m_blocks && ok; mb += n_clusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrGemmMmaWait, abort_flag, wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kStageA);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kStageB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            tc_mma_f16(d_tmem, smem_desc_sw128(a0 + k * 32), smem_desc_sw128(b0 + k * 32), idesc,
                       (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      tc_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // This CTA's columns of gamma (a weight: loaded before the dependency wait) into shared
    // memory, so the LayerNorm pass reads it as broadcast 16-byte loads; the eight epilogue warps
    // meet on named barrier 1 before any of them reads the copy.  (beta, absent from the
    // encoder's norms, is read from global memory when given.)
    float* s_gamma = reinterpret_cast<float*>(smem + Cfg::kOffGB);
    for (int i = threadIdx.x - 64; i < BN; i += kEpiWarps * 32) s_gamma[i] = args.gamma[nb * BN + i];
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");
    pdl_wait();
    // Epilogue warp: TMEM lane quarter q (tile rows 32q..32q+31, one per lane) and column half h
    // (this CTA's columns [h BN/2, (h+1) BN/2), NCH 32-column chunks).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    // Residual chunk j (32 rows x 32 fp32 columns) goes through ring block j & 1: a TMA load, the
    // update in place by the lanes (row-per-lane, the swizzled layout of stage_off), a TMA store.
    uint8_t* ring = smem + Cfg::kOffEpi + (warp - 2) * 2 * Cfg::kRingBlock;
    uint64_t* rb = rbar + (warp - 2) * 2;
    uint8_t* stage = ring + Cfg::kRingBlock;           // LayerNorm pass staging (ring block 1)
    uint32_t rphase = 0, rpending = 0;                 // per ring block: phase, load in flight
    const int col0 = nb * BN + half * (BN / 2);       // first global column of this warp
    constexpr float kPart = (float)(BN / 2);          // columns per partial
    const float inv_n = 1.f / (float)args.N;
    T* xout = reinterpret_cast<T*>(args.x);
    // Exchange: send this thread's partials (sum and centred M2 of its row over this warp's
    // columns) to every CTA of the cluster, wait until all C * 8 warps' partials have landed
    // here, and merge them.  The tile's exchange barrier was armed at the start of the tile.
    auto exchange = [&](int par, int lt, float sum, float m2, float& mean, float& var, bool& fine) {
      const int slot = (par * 2 * C + rank * 2 + half) * kBM + quarter * 32 + lane;
      const uint32_t local = smem_u32(xbuf + 2 * slot);
      const uint32_t bar_local = smem_u32(&xbar[par]);
#pragma unroll
      for (int c = 0; c < C; ++c) st_async_f32x2(cluster_addr(local, c), sum, m2, cluster_addr(bar_local, c));
      fine = mbar_wait(&xbar[par], (lt >> 1) & 1, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns);
      const float2* part = reinterpret_cast<const float2*>(xbuf) + (par * 2 * C) * kBM + quarter * 32 + lane;
      float total = 0.f;
#pragma unroll
      for (int i = 0; i < 2 * C; ++i) total += part[i * kBM].x;
      mean = total * inv_n;
      float acc_m2 = 0.f, spread = 0.f;
#pragma unroll
      for (int i = 0; i < 2 * C; ++i) {
        const float2 pi = part[i * kBM];
        const float d = pi.x * (1.f / kPart) - mean;
        acc_m2 += pi.y;
        spread = fmaf(d, d, spread);
      }
      var = (acc_m2 + kPart * spread) * inv_n;
    };
    // Loads residual chunk j of the block at row0 into ring block b (lane 0; rows past M read
    // as zeros).  The block must be free: no store from it still reading.
    auto res_load = [&](int b, int row0, int j) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&rb[b], Cfg::kRingBlock);
        tma_load_2d(ring + b * Cfg::kRingBlock, &tmR, &rb[b], col0 + 32 * j, row0);
      }
      rpending |= 1u << b;
    };
    auto res_wait = [&](int b) -> bool {
      const bool fine = mbar_wait(&rb[b], (rphase >> b) & 1, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns);
      rphase ^= 1u << b;
      rpending &= ~(1u << b);
      return fine;
    };
    // Every TMA store this warp issued has finished reading its ring block.
    auto stores_read = [&]() {
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
    };
    if (cid < m_blocks) {
      const int row0 = cid * kBM + quarter * 32;
      res_load(0, row0, 0);
      res_load(1, row0, 1);
    }
    int acc = 0; uint32_t acc_phase = 0;
    int lt = 0;  // local tile count
    for (int mb = cid; mb < m_blocks; mb += n_clusters, ++lt) {
      const int row0 = mb * kBM + quarter * 32;
      const int rows = min(32, args.M - row0);  // may be <= 0: the warp still takes part in the exchange
      const int par = lt & 1;
      // Arm this tile's exchange barrier with the bytes every CTA of the cluster will send here.
      // (The previous use of this parity completed: this warp waited for it.)
      if (warp == 2 && lane == 0) mbar_arrive_expect_tx(&xbar[par], Cfg::kXTxBytes);
      if (!mbar_wait(&tfull[acc], acc_phase, args.err, kErrGemmEpilogueWait, abort_flag, wait_ns)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + half * (BN / 2);
      // Pass A: v = acc + bias + residual -> HBM (residual) and TMEM (in place).  Each chunk's
      // sum and centred M2 come from its 32 values in registers (two passes) and are merged into
      // this thread's partial with Chan's formula, so no second pass over TMEM is needed.
      float pm = 0.f, pm2 = 0.f;  // running mean and M2 of this thread's partial
      bool landed = true;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int b = j & 1;
        uint8_t* blk = ring + b * Cfg::kRingBlock;
        uint32_t v[32];
        tmem_ld32_async(tbase + 32 * j, v);
        landed = res_wait(b);
        tmem_wait_ld(v);
        if (!__all_sync(0xffffffffu, landed)) break;
        // v = residual + (acc + bias), in place in the block (this lane's row, 8 x 16 bytes).
        float cs = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
          if (args.bias) bb = *reinterpret_cast<const float4*>(args.bias + col0 + 32 * j + 4 * q);
          const float4 rr = f4(*reinterpret_cast<const uint4*>(blk + stage_off(lane, q)));
          const float4 nv = make_float4(rr.x + (__uint_as_float(v[4 * q]) + bb.x),
                                        rr.y + (__uint_as_float(v[4 * q + 1]) + bb.y),
                                        rr.z + (__uint_as_float(v[4 * q + 2]) + bb.z),
                                        rr.w + (__uint_as_float(v[4 * q + 3]) + bb.w));
          *reinterpret_cast<uint4*>(blk + stage_off(lane, q)) = u4(nv.x, nv.y, nv.z, nv.w);
          v[4 * q] = __float_as_uint(nv.x); v[4 * q + 1] = __float_as_uint(nv.y);
          v[4 * q + 2] = __float_as_uint(nv.z); v[4 * q + 3] = __float_as_uint(nv.w);
          cs += (nv.x + nv.y) + (nv.z + nv.w);
        }
        // The updated chunk goes back to HBM from the block (TMA store; the lanes' writes are
        // handed to the async proxy first) and to TMEM for the LayerNorm pass.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && rows > 0) {
          tma_store_2d(&tmR, blk, col0 + 32 * j, row0);
          bulk_commit();
        }
        tmem_st32(tbase + 32 * j, v);
        const float cm = cs * (1.f / 32.f);
        float cm2 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float d = __uint_as_float(v[i]) - cm;
          cm2 = fmaf(d, d, cm2);
        }
        // Merge (32 j values, mean pm, M2 pm2) with (32 values, mean cm, M2 cm2).
        const float delta = cm - pm;
        pm += delta * (1.f / (float)(j + 1));
        pm2 += cm2 + delta * delta * (32.f * (float)j / (float)(j + 1));
        if (j + 2 < NCH) {
          stores_read();
          res_load(b, row0, j + 2);
        }
      }
      if (!__all_sync(0xffffffffu, landed)) break;
      tmem_wait_st();
      // Ring block 0 takes the next tile's chunk 0 now; block 1 is the staging block of the
      // LayerNorm pass below and takes chunk 1 after it.
      const int next0 = (mb + n_clusters) * kBM + quarter * 32;
      stores_read();
      if (mb + n_clusters < m_blocks) res_load(0, next0, 0);
      const float sum = pm * kPart, m2 = pm2;
      bool fine;
      float mean, var;
      exchange(par, lt, sum, m2, mean, var, fine);
      if (!__all_sync(0xffffffffu, fine)) break;
      const float rstd = rsqrtf(var + args.eps);
      // Pass C: x = (v - mean) * rstd * gamma (+ beta): 64 columns (128 bytes of T) per staged
      // block, and a last 32-column block (64 bytes per row) when NCH is odd.
      auto normalise = [&](int j, uint32_t (&v)[32], uint4* p) {
        tmem_wait_ld(v);
        const int c0 = half * (BN / 2) + 32 * j;  // column within this CTA's block
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const float4 g0 = *reinterpret_cast<const float4*>(s_gamma + c0 + i);
          const float4 g1 = *reinterpret_cast<const float4*>(s_gamma + c0 + i + 4);
          const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            y[e] = (__uint_as_float(v[i + e]) - mean) * rstd * g[e];
            if (args.beta) y[e] += args.beta[nb * BN + c0 + i + e];
          }
          p[i / 8] = make_uint4(pack2<T>(y[0], y[1]), pack2<T>(y[2], y[3]), pack2<T>(y[4], y[5]), pack2<T>(y[6], y[7]));
        }
      };
#pragma unroll
      for (int j = 0; j < NCH; j += 2) {
        uint4 p[8];
        const int pieces = j + 1 < NCH ? 8 : 4;
        uint32_t vb[2][32];
        tmem_ld32_async(tbase + 32 * j, vb[0]);
        if (pieces == 8) tmem_ld32_async(tbase + 32 * (j + 1), vb[1]);
        normalise(j, vb[0], p);
        if (pieces == 8) normalise(j + 1, vb[1], p + 4);
        else p[4] = p[5] = p[6] = p[7] = make_uint4(0, 0, 0, 0);
        stage_put(stage, lane, p);
        T* xo = xout + col0 + 32 * j;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 4 * k + (lane >> 3);
          if (r < rows && (lane & 7) < pieces)
            *reinterpret_cast<uint4*>(xo + (size_t)(row0 + r) * args.ldx + (lane & 7) * 8) = stage_get(stage, k, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      // The staging block takes the next tile's chunk 1 (the lanes' staging writes are ordered
      // before the copy's writes).
      if (mb + n_clusters < m_blocks) {
        fence_proxy_async_smem();
        __syncwarp();
        res_load(1, next0, 1);
      }
    }
    // Stores complete and loads landed before the CTA exits (on every path; bounded drains).
    if (lane == 0) {
      bulk_wait_all();
      for (int b = 0; b < 2; ++b)
        if ((rpending >> b) & 1) mbar_drain(&rb[b], (rphase >> b) & 1);
    }
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while a peer may still write its exchange buffer
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 512);
}

}  // namespace laya
