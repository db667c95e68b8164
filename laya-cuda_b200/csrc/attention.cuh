// Varlen packed attention over the rows of one forward pass (encoder layers and the decision
// head's self-attention), restating the semantics of the reference kernel
// laya_cuda/kernels.cu:90-154:
//   * rows are packed back to back at 16-token alignment; row r owns tokens
//     [starts[r], starts[r] + lengths[r]) and padding up to the next 16-token boundary;
//   * key j is visible to query i of the same row iff j < length and (window < 0 or |i-j| <= window);
//   * scores are scaled by 1/8 (64-wide heads), softmax in fp32;
//   * padding queries (and every token past the last row) produce exact zeros.
//
// This file holds the mma.sync variant (64-query tiles): kernel-level tests and the forward pass
// under LAYA_ATTENTION=mma_sync.  The forward pass uses the tcgen05 variant in tc_attention.cuh.
//
// Work unit: one CTA per (64-query tile of one row, head).  The host builds the tile table
// while packing the inputs, so a tile never straddles two rows and a CTA stages one K/V block
// per step that all four of its warps share.  Q and K come from the QKV GEMM epilogue in
// head-major layout [heads][M][64], V transposed [heads][64][M]; the output is token-major
// [M][heads*64] (the next GEMM's A operand).  Tensor-core math is mma.sync m16n8k16 with fp32
// accumulation; K/V blocks are double-buffered in XOR-swizzled shared memory with cp.async,
// fragments via ldmatrix.
#pragma once
#include "common.cuh"

namespace laya {

constexpr int kAttnQ = 64;        // queries per CTA (16 per warp)
constexpr int kAttnKB = 64;       // keys per block
constexpr int kAttnThreads = 128;

struct AttnArgs {
  const void* qkv;      // q, k: [heads][M][64] each; then v transposed: [heads][64][M]
  void* out;            // [M][heads*64]
  const int4* tiles;    // (t0, t1, row, 0); row -1: zero-fill [t0,t1); row -2: unused slot
  const int* starts;
  const int* lengths;
  int M;
  int heads;
  int window;           // -1: global
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `c` of row `r` in a [64][64] 16-bit tile with XOR swizzle.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// kSplitP: probabilities enter the PV product as high + low 16-bit parts (two MMAs), keeping
// fp32-level probability precision, as the reference does (kernels.cu:133-146).
template <typename T, bool kSplitP>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
  __shared__ __align__(128) uint8_t sQ[kAttnQ * 128];
  __shared__ __align__(128) uint8_t sK[2][kAttnKB * 128];
  __shared__ __align__(128) uint8_t sV[2][kAttnKB * 128];

  pdl_wait();
  const int4 tile = a.tiles[blockIdx.y];  // grid: (heads, tiles), all heads of a tile together
  const int head = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = tile.x, t1 = tile.y, row = tile.z;
  const int width = a.heads * 64;
  T* out = reinterpret_cast<T*>(a.out);
  if (row == -2) return;
  if (row < 0) {
    // Tokens past the last row: zeros (8 x 16 bytes per token and head).
    for (int i = tid; i < (t1 - t0) * 8; i += kAttnThreads) {
      const int t = t0 + (i >> 3);
      *reinterpret_cast<uint4*>(out + (size_t)t * width + head * 64 + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  const int first = a.starts[row];
  const int valid = a.lengths[row];
  const int q0 = t0 - first;                 // row-relative index of the tile's first query
  const size_t plane = (size_t)a.heads * a.M * 64;
  const T* Q = reinterpret_cast<const T*>(a.qkv) + ((size_t)head * a.M + first) * 64;
  const T* K = Q + plane;
  const T* Vt = reinterpret_cast<const T*>(a.qkv) + 2 * plane + (size_t)head * 64 * a.M + first;

  int k_lo = 0, k_hi = valid;
  if (a.window >= 0) {
    k_lo = max(0, q0 - a.window);
    k_hi = min(valid, q0 + kAttnQ + a.window);
  }
  k_lo = (k_lo / kAttnKB) * kAttnKB;
  const int n_blocks = k_hi > k_lo ? (k_hi - k_lo + kAttnKB - 1) / kAttnKB : 0;

  // Q tile: 64 rows x 8 chunks; rows past the row length load zeros.
  const uint32_t q_base = smem_u32(sQ);
  for (int i = tid; i < kAttnQ * 8; i += kAttnThreads) {
    const int r = i >> 3, c = i & 7;
    const bool ok = (q0 + r < valid) && (t0 + r < t1);
    cp_async16(q_base + swz(r, c), Q + (size_t)(ok ? q0 + r : 0) * 64 + c * 8, ok);
  }
  auto load_kv = [&](int blk, int buf) {
    const int kb = k_lo + blk * kAttnKB;
    const uint32_t kbase = smem_u32(sK[buf]), vbase = smem_u32(sV[buf]);
    for (int i = tid; i < kAttnKB * 8; i += kAttnThreads) {
      const int r = i >> 3, c = i & 7;
      const bool ok = kb + r < valid;
      const size_t off = (size_t)(ok ? kb + r : 0) * 64 + c * 8;
      cp_async16(kbase + swz(r, c), K + off, ok);
      // V^T tile: row r = dimension, chunk c = keys kb+8c .. kb+8c+7.
      const bool vok = kb + 8 * c < valid;
      cp_async16(vbase + swz(r, c), Vt + (size_t)r * a.M + (vok ? kb + 8 * c : 0), vok);
    }
  };
  if (n_blocks > 0) load_kv(0, 0);
  cp_async_commit();

  const int wq = q0 + warp * 16;               // row-relative first query of this warp
  const bool warp_live = wq < valid && (t0 + warp * 16) < t1;
  const int r0 = wq + (lane >> 2), r1 = r0 + 8;  // this thread's two query rows
  constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;

  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int blk = 0; blk < n_blocks; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < n_blocks) load_kv(blk + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (blk == 0 && warp_live) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = warp * 16 + (lane & 15);
        const int ch = c * 2 + (lane >> 4);
        ldsm_x4(q_base + swz(r, ch), qa[c][0], qa[c][1], qa[c][2], qa[c][3]);
      }
    }
    const int kb = k_lo + blk * kAttnKB;
    // Skip blocks wholly outside this warp's window.
    bool need = warp_live;
    if (a.window >= 0) need = need && (kb <= wq + 15 + a.window) && (kb + kAttnKB - 1 >= wq - a.window);
    if (need) {
      const uint32_t kbase = smem_u32(sK[buf]), vbase = smem_u32(sV[buf]);
      // 16-key groups [g_lo, g_hi] of this block that any of the warp's 16 queries can see;
      // the others are skipped in both products.  A block with every key visible to every
      // query of the warp ("interior") needs no per-element mask.
      int g_lo = 0, hi_key = valid - 1 - kb;
      if (a.window >= 0) {
        const int lo_key = wq - a.window - kb;
        hi_key = min(hi_key, wq + 15 + a.window - kb);
        g_lo = lo_key <= 0 ? 0 : lo_key >> 4;
      }
      const int g_hi = min(3, hi_key >> 4);
      const bool interior =
          kb + kAttnKB - 1 < valid && (a.window < 0 || (kb >= wq + 15 - a.window && kb + kAttnKB - 1 <= wq + a.window));
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        if (np < g_lo || np > g_hi) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = c * 2 + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + swz(key, ch), b0, b1, b2, b3);
          mma16816<T>(s[2 * np], qa[c], b0, b1);
          mma16816<T>(s[2 * np + 1], qa[c], b2, b3);
        }
      }
      // Mask and scale.
      float nm0 = m0, nm1 = m1;
      if (interior) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) s[n][e] *= kScaleLog2;
          nm0 = fmaxf(nm0, fmaxf(s[n][0], s[n][1]));
          nm1 = fmaxf(nm1, fmaxf(s[n][2], s[n][3]));
        }
      } else {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kb + n * 8 + (lane & 3) * 2 + (e & 1);
            const int q = e < 2 ? r0 : r1;
            bool keep = key < valid;
            if (a.window >= 0) keep = keep && abs(key - q) <= a.window;
            s[n][e] = keep ? s[n][e] * kScaleLog2 : -INFINITY;
          }
          nm0 = fmaxf(nm0, fmaxf(s[n][0], s[n][1]));
          nm1 = fmaxf(nm1, fmaxf(s[n][2], s[n][3]));
        }
      }
#pragma unroll
      for (int d = 1; d < 4; d <<= 1) {
        nm0 = fmaxf(nm0, __shfl_xor_sync(0xffffffffu, nm0, d));
        nm1 = fmaxf(nm1, __shfl_xor_sync(0xffffffffu, nm1, d));
      }
      const float c0 = nm0 == -INFINITY ? 1.f : exp2f(m0 - nm0);
      const float c1 = nm1 == -INFINITY ? 1.f : exp2f(m1 - nm1);
      m0 = nm0; m1 = nm1;
      l0 *= c0; l1 *= c1;
#pragma unroll
      for (int n = 0; n < 8; ++n) { o[n][0] *= c0; o[n][1] *= c0; o[n][2] *= c1; o[n][3] *= c1; }
      const float sub0 = m0 == -INFINITY ? 0.f : m0, sub1 = m1 == -INFINITY ? 0.f : m1;
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // 16-key chunk j = S n-tiles 2j, 2j+1
        if (j < g_lo || j > g_hi) continue;  // every probability of the group is 0
        uint32_t ph[4], pl[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = s[2 * j + h][e];
            p[e] = x == -INFINITY ? 0.f : exp2f(x - (e < 2 ? sub0 : sub1));
          }
          l0 += p[0] + p[1];
          l1 += p[2] + p[3];
          ph[h * 2 + 0] = pack2<T>(p[0], p[1]);
          ph[h * 2 + 1] = pack2<T>(p[2], p[3]);
          if (kSplitP) {
            const float2 a01 = unpack2_f32(ph[h * 2 + 0], (T*)nullptr);
            const float2 a23 = unpack2_f32(ph[h * 2 + 1], (T*)nullptr);
            pl[h * 2 + 0] = pack2<T>(p[0] - a01.x, p[1] - a01.y);
            pl[h * 2 + 1] = pack2<T>(p[2] - a23.x, p[3] - a23.y);
          }
        }
        // A fragment order: (r0,k0-7), (r1,k0-7), (r0,k8-15), (r1,k8-15).
        const uint32_t pa[4] = {ph[0], ph[1], ph[2], ph[3]};
        uint32_t pb[4];
        if (kSplitP) { pb[0] = pl[0]; pb[1] = pl[1]; pb[2] = pl[2]; pb[3] = pl[3]; }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int dim = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int kch = j * 2 + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(vbase + swz(dim, kch), b0, b1, b2, b3);
          mma16816<T>(o[2 * np], pa, b0, b1);
          mma16816<T>(o[2 * np + 1], pa, b2, b3);
          if (kSplitP) {
            mma16816<T>(o[2 * np], pb, b0, b1);
            mma16816<T>(o[2 * np + 1], pb, b2, b3);
          }
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Normalise and store; rows past the length (or past the tile) write zeros.
#pragma unroll
  for (int d = 1; d < 4; d <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, d);
    l1 += __shfl_xor_sync(0xffffffffu, l1, d);
  }
  const float i0 = (r0 < valid && l0 > 0.f) ? 1.f / l0 : 0.f;
  const float i1 = (r1 < valid && l1 > 0.f) ? 1.f / l1 : 0.f;
  const int tok0 = first + r0, tok1 = first + r1;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int col = head * 64 + n * 8 + (lane & 3) * 2;
    if (tok0 < t1) *reinterpret_cast<uint32_t*>(out + (size_t)tok0 * width + col) = pack2<T>(o[n][0] * i0, o[n][1] * i0);
    if (tok1 < t1) *reinterpret_cast<uint32_t*>(out + (size_t)tok1 * width + col) = pack2<T>(o[n][2] * i1, o[n][3] * i1);
  }
}

}  // namespace laya
