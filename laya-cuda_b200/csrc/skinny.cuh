// CUDA-core GEMM for a handful of rows: the decision head's gathered CLS/marker rows at small
// batches (one question: 9 rows), where a tensor-core tile would be 128 rows of which 9 are live
// and every CTA walks a serial chain of k-blocks for almost no work.
//
//   D[m][n] = sum_k X[m][k] W[n][k]   (m < M <= kSkinnyRows; X, W 16-bit, K-major)
//
// One warp per output column n over the whole K: its lanes hold the column's weight row in
// registers (16-byte vectors, loaded before the dependency wait: weights do not depend on the
// previous kernel), the CTA stages X in shared memory once, each lane accumulates its vectors'
// products for every row in fp32, and a butterfly reduction gives every lane all M sums.
// Epilogues as the tensor-core GEMM: store (+bias), ReLU, exact-erf GELU, fp32 residual +=.
// Replaces, for these rows, the cuBLAS GemmEx calls of the head (laya_cuda/laya.py:229-241).
#pragma once
#include "common.cuh"
#include "gemm.cuh"

namespace laya {

constexpr int kSkinnyRows = 16;     // most rows
constexpr int kSkinnyWarps = 8;     // output columns per CTA
constexpr int kSkinnyMaxK = 4096;   // K <= 16 vectors of 8 elements per lane
constexpr int kSkinnyVecs = kSkinnyMaxK / 256;

template <int EPI, typename T>
__global__ void __launch_bounds__(kSkinnyWarps * 32) skinny_gemm_kernel(const T* __restrict__ x,
                                                                      const T* __restrict__ w, const GemmArgs a) {
  extern __shared__ __align__(16) uint8_t skinny_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kSkinnyWarps + warp;
  const int nv = a.K / 8;  // 16-byte vectors per row
  uint4 wv[kSkinnyVecs];
#pragma unroll
  for (int i = 0; i < kSkinnyVecs; ++i) {
    const int v = lane + 32 * i;
    wv[i] = n < a.N && v < nv ? __ldg(reinterpret_cast<const uint4*>(w + (size_t)n * a.K) + v) : make_uint4(0, 0, 0, 0);
  }
  pdl_wait();
  uint4* sx = reinterpret_cast<uint4*>(skinny_smem);  // [M][nv]
  for (int i = threadIdx.x; i < a.M * nv; i += blockDim.x) {
    const int m = i / nv, v = i - m * nv;
    sx[i] = *(reinterpret_cast<const uint4*>(x + (size_t)m * a.K) + v);
  }
  __syncthreads();
  if (n >= a.N) return;
  float acc[kSkinnyRows];
#pragma unroll
  for (int m = 0; m < kSkinnyRows; ++m) acc[m] = 0.f;
#pragma unroll
  for (int i = 0; i < kSkinnyVecs; ++i) {
    const int v = lane + 32 * i;
    if (v >= nv) break;
    float2 wf[4];
    wf[0] = unpack2_f32(wv[i].x, (T*)nullptr); wf[1] = unpack2_f32(wv[i].y, (T*)nullptr);
    wf[2] = unpack2_f32(wv[i].z, (T*)nullptr); wf[3] = unpack2_f32(wv[i].w, (T*)nullptr);
#pragma unroll
    for (int m = 0; m < kSkinnyRows; ++m) {
      if (m < a.M) {
        const uint4 xv = sx[m * nv + v];
        const float2 x0 = unpack2_f32(xv.x, (T*)nullptr), x1 = unpack2_f32(xv.y, (T*)nullptr);
        const float2 x2 = unpack2_f32(xv.z, (T*)nullptr), x3 = unpack2_f32(xv.w, (T*)nullptr);
        float s = acc[m];
        s = fmaf(x0.x, wf[0].x, s); s = fmaf(x0.y, wf[0].y, s);
        s = fmaf(x1.x, wf[1].x, s); s = fmaf(x1.y, wf[1].y, s);
        s = fmaf(x2.x, wf[2].x, s); s = fmaf(x2.y, wf[2].y, s);
        s = fmaf(x3.x, wf[3].x, s); s = fmaf(x3.y, wf[3].y, s);
        acc[m] = s;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kSkinnyRows; ++m) {
    if (m < a.M) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
    }
  }
  const float bias = a.bias ? a.bias[n] : 0.f;
#pragma unroll
  for (int m = 0; m < kSkinnyRows; ++m) {
    if (m < a.M && lane == m) {
      float v = acc[m] + bias;
      if (EPI == EPI_RESIDUAL) {
        a.residual[(size_t)m * a.ldr + n] += v;
      } else {
        if (EPI == EPI_RELU) v = fmaxf(v, 0.f);
        if (EPI == EPI_GELU) v = gelu_erf(v);
        reinterpret_cast<T*>(a.out)[(size_t)m * a.ldo + n] = from_f32<T>(v);
      }
    }
  }
}

}  // namespace laya
