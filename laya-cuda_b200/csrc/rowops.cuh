// Row-wise HBM-bound kernels: embedding gather + LayerNorm, residual LayerNorms (with optional
// split-K partial reduction, final-norm + token-type + head-norm fusion), the head's row
// gather, and the decision-head tail (scorer output, option features, action head).
//
// One warp per row; each lane keeps its slice of the row in registers, so a row is read once
// and written once.  LayerNorm follows the reference (laya_cuda/kernels.cu:20-49): population
// variance of the centred values, rsqrt(var + eps), gamma, optional beta.
#pragma once
#include "common.cuh"

namespace laya {

constexpr int kRowWarps = 8;           // most rows per block (one warp per row); small classes launch
                                       // fewer warps per block so that their rows spread over more SMs

// A warp holds one row of width d = 32 * NPL (NPL even, 2..32: widths 64..1024): lane `lane`
// keeps NPL floats, in vectors of CH consecutive columns at col = j*32*CH + lane*CH.
template <int NPL>
struct RowVec {
  static constexpr int CH = (NPL % 4 == 0) ? 4 : 2;
};

template <int NPL>
__device__ __forceinline__ void row_load(const float* src, int lane, float (&v)[NPL]) {
  constexpr int CH = RowVec<NPL>::CH;
#pragma unroll
  for (int j = 0; j < NPL / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (CH == 4) {
      const float4 t = *reinterpret_cast<const float4*>(src + col);
      v[j * 4] = t.x; v[j * 4 + 1] = t.y; v[j * 4 + 2] = t.z; v[j * 4 + 3] = t.w;
    } else {
      const float2 t = *reinterpret_cast<const float2*>(src + col);
      v[j * 2] = t.x; v[j * 2 + 1] = t.y;
    }
  }
}

template <int NPL>
__device__ __forceinline__ void row_store(float* dst, int lane, const float (&v)[NPL]) {
  constexpr int CH = RowVec<NPL>::CH;
#pragma unroll
  for (int j = 0; j < NPL / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (CH == 4) *reinterpret_cast<float4*>(dst + col) = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
    else *reinterpret_cast<float2*>(dst + col) = make_float2(v[j * 2], v[j * 2 + 1]);
  }
}

template <int NPL, typename T>
__device__ __forceinline__ void row_store_t(T* dst, int lane, const float (&v)[NPL]) {
  constexpr int CH = RowVec<NPL>::CH;
#pragma unroll
  for (int j = 0; j < NPL / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (CH == 4) {
      uint2 w; w.x = pack2<T>(v[j * 4], v[j * 4 + 1]); w.y = pack2<T>(v[j * 4 + 2], v[j * 4 + 3]);
      *reinterpret_cast<uint2*>(dst + col) = w;
    } else {
      *reinterpret_cast<uint32_t*>(dst + col) = pack2<T>(v[j * 2], v[j * 2 + 1]);
    }
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// In-place LayerNorm of the lane's slice: v = (v - mean) * rsqrt(var + eps) * gamma + beta, with
// the lane's gamma / beta slices already in registers (row_load's layout; beta zeros if absent).
template <int NPL>
__device__ __forceinline__ void row_layernorm(float (&v)[NPL], const float (&g)[NPL], const float (&b)[NPL], float eps) {
  constexpr float inv_d = 1.0f / (32 * NPL);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) s += v[i];
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) { const float t = v[i] - mean; q += t * t; }
  const float inv = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
  for (int i = 0; i < NPL; ++i) v[i] = (v[i] - mean) * inv * g[i] + b[i];
}

// LayerNorm without a held beta: v = (v - mean) * rsqrt(var + eps) * gamma, then + beta loaded
// here only when given (the encoder's norms have none), so no beta slice stays live across the
// reductions.
template <int NPL>
__device__ __forceinline__ void row_layernorm_beta_late(float (&v)[NPL], const float (&g)[NPL], const float* beta,
                                                        int lane, float eps) {
  constexpr float inv_d = 1.0f / (32 * NPL);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) s += v[i];
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) { const float t = v[i] - mean; q += t * t; }
  const float inv = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
  for (int i = 0; i < NPL; ++i) v[i] = (v[i] - mean) * inv * g[i];
  if (beta) {
    constexpr int CH = RowVec<NPL>::CH;
#pragma unroll
    for (int j = 0; j < NPL / CH; ++j) {
      const int col = j * 32 * CH + lane * CH;
#pragma unroll
      for (int c = 0; c < CH; ++c) v[j * CH + c] += beta[col + c];
    }
  }
}

// Loads the lane's slice of an optional [d] vector (zeros when absent).
template <int NPL>
__device__ __forceinline__ void row_load_opt(const float* src, int lane, float (&v)[NPL]) {
  if (src) {
    row_load<NPL>(src, lane, v);
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] = 0.f;
  }
}

// residual[t] = LN_gamma(E[ids[t]]) (fp32); x[t] = residual[t] rounded to T.
// Replaces kernels.cu:16-19 + the embeddings.norm and copy passes of runtime.py:93-95.
template <int NPL, typename T>
__global__ void __launch_bounds__(kRowWarps * 32) embed_norm_kernel(const int* ids, const float* table,
                                                                    const float* gamma, float eps, int rows, int d,
                                                                    int vocab, float* residual, T* x, int* err) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  float g[NPL], z[NPL];
  row_load<NPL>(gamma, lane, g);  // a weight: loaded before waiting on the previous kernel
  row_load_opt<NPL>(nullptr, lane, z);
  pdl_wait();
  if (row >= rows) return;
  int id = ids[row];
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicCAS(err, 0, kErrBadIndex);
    id = 0;
  }
  float v[NPL];
  row_load<NPL>(table + (size_t)id * d, lane, v);
  row_layernorm<NPL>(v, g, z, eps);
  row_store<NPL>(residual + (size_t)row * d, lane, v);
  row_store_t<NPL, T>(x + (size_t)row * d, lane, v);
}

struct NormArgs {
  float* residual;          // [rows][d] fp32, updated in place
  const float* partials;    // split-K partial sums [splits][rows][d] to add first, or nullptr
  int splits;
  const float* partial_bias;  // bias [d] of the split GEMM, added with the partials (or nullptr)
  const float* gamma1; const float* beta1; float eps1;
  // Final-norm fusion (encoder.final_norm -> + type_emb[kind] -> head norm1):
  int fused_final;
  const float* type_emb; const int* kinds;
  const float* gamma2; const float* beta2; float eps2;
  void* x;                  // [rows][d] T output (may be nullptr)
  int rows, d;
};

// Normal:  residual += sum(partials) + bias; x = LN1(residual).
// Fused:   residual = LN1(residual + sum(partials) + bias) + type_emb[kind]; x = LN2(residual).
// PARTIALS selects the split-K variant (only used for small classes) and FUSED the final-norm
// fusion (once per pass, `a.fused_final`), so the common variant holds only gamma and the row in
// registers (beta, when given, is added after normalising): four 256-thread blocks fit an SM.
// Replaces kernels.cu:20-49 and kernels.cu:155-158.
template <int NPL, typename T, bool PARTIALS, bool FUSED>
__global__ void __launch_bounds__(kRowWarps * 32) norm_kernel(const NormArgs a) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  // Every independent load is issued up front, so a row costs about one memory round trip: the
  // norm weights and the split GEMM's bias (weights) before waiting on the previous kernel, then
  // the residual row and up to four partial rows together.
  float g1[NPL], b1[NPL], pb[NPL];
  row_load<NPL>(a.gamma1, lane, g1);
  if (FUSED) row_load_opt<NPL>(a.beta1, lane, b1);
  if (PARTIALS) row_load_opt<NPL>(a.partial_bias, lane, pb);
  pdl_wait();
  if (row >= a.rows) return;
  const int d = 32 * NPL;
  float* r = a.residual + (size_t)row * d;
  float v[NPL];
  row_load<NPL>(r, lane, v);
  if (PARTIALS) {
    // Partial sums in split order, then the GEMM bias, then the residual: a fixed order, so the
    // result does not depend on the batch or on scheduling.
    float acc[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) acc[i] = 0.f;
    for (int s0 = 0; s0 < a.splits; s0 += 4) {
      float p[4][NPL];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (s0 + q < a.splits) row_load<NPL>(a.partials + ((size_t)(s0 + q) * a.rows + row) * d, lane, p[q]);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (s0 + q < a.splits) {
#pragma unroll
          for (int i = 0; i < NPL; ++i) acc[i] += p[q][i];
        }
    }
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] += acc[i] + pb[i];
  }
  if (FUSED) {
    float g2[NPL], b2[NPL], t[NPL];
    row_load<NPL>(a.gamma2, lane, g2);
    row_load_opt<NPL>(a.beta2, lane, b2);
    row_load<NPL>(a.type_emb + (size_t)a.kinds[row] * d, lane, t);
    row_layernorm<NPL>(v, g1, b1, a.eps1);
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] += t[i];
    row_store<NPL>(r, lane, v);
    row_layernorm<NPL>(v, g2, b2, a.eps2);
  } else {
    if (PARTIALS) row_store<NPL>(r, lane, v);
    row_layernorm_beta_late<NPL>(v, g1, a.beta1, lane, a.eps1);
  }
  if (a.x) row_store_t<NPL, T>(reinterpret_cast<T*>(a.x) + (size_t)row * d, lane, v);
}

// selected[i] = residual[indices[i]] (fp32); scored[i] = attention[indices[i]] (T).
// Replaces kernels.cu:159-166 (gather, gather_half) as used by laya.py:226-227.
template <typename T>
__global__ void __launch_bounds__(256) gather_rows_kernel(const float* residual, const T* attention,
                                                          const int* indices, int count, int d, int rows,
                                                          float* selected, T* scored, int* err) {
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= count) return;
  int src = indices[i];
  if (src < 0 || src >= rows) {
    if (threadIdx.x == 0) atomicCAS(err, 0, kErrBadIndex);
    src = 0;
  }
  for (int c = threadIdx.x * 4; c < d; c += blockDim.x * 4) {
    *reinterpret_cast<float4*>(selected + (size_t)i * d + c) = *reinterpret_cast<const float4*>(residual + (size_t)src * d + c);
    *reinterpret_cast<uint2*>(scored + (size_t)i * d + c) = *reinterpret_cast<const uint2*>(attention + (size_t)src * d + c);
  }
}

struct TailArgs {
  const float* selected;   // [b*(k+1)][d] fp32: head output rows (CLS + markers)
  const void* scored;      // [b*(k+1)][d] T: gelu(scorer.1(LN(selected)))
  const int* counts;       // [b]
  const float* w3; const float* b3;      // scorer.3: [d], [1]
  const float* wa0; const float* ba0;    // act_head.0: [256][d+4], [256]
  const float* wa2; const float* ba2;    // act_head.2: [n_act][256], [n_act]
  float* logits;           // [b][k+1]
  float* acts;             // [b][n_act]
  float* hidden;           // [b][256] scratch: act_head.0 outputs
  int* arrivals;           // [b] zero at launch: CTAs of the question that finished their part
  float* features;         // [b][4] (p1, p1 - p2, H / log(max(c,2)), max(c,2)/255) or nullptr
  int k, d, n_act;
};

constexpr int kTailThreads = 256;
constexpr int kTailWarps = kTailThreads / 32;
// CTAs per question (gridDim.y), each owning 256/parts hidden units: 32 (one unit per warp) for
// small batches, whose few questions would otherwise leave most SMs idle; 8 for large ones.
constexpr int kTailPartsSmall = 32, kTailPartsLarge = 8;
constexpr int kActHidden = 256;

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Decision-head tail, gridDim.y CTAs per question (blockIdx.x = question, blockIdx.y = part).
// Restates laya.py:241-245 and kernels.cu:167-183 (features) in fp32:
//   logits   = scored . w3 + b3                       (every part; part 0 stores them)
//   features = [CLS row, p1, p1 - p2, H / log(max(c,2)), max(c,2)/255] over the option logits
//   hidden   = gelu(act_head.0(features))             (each part its 32 units, to global scratch)
//   acts     = act_head.2(hidden)                     (the part that finishes last)
// Dynamic shared memory: features [d+4], hidden [256], logits [k+1].
template <typename T>
__global__ void __launch_bounds__(kTailThreads) head_tail_kernel(const TailArgs a) {
  extern __shared__ float sh[];
  __shared__ int s_last;
  const int q = blockIdx.x, part = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k1 = a.k + 1, d = a.d;
  {
    // This part's act_head.0 rows do not depend on the previous kernel: start them towards L2.
    const int units = kActHidden / (int)gridDim.y;
    const char* w = reinterpret_cast<const char*>(a.wa0 + (size_t)part * units * (d + 4));
    const int lines = (int)(((size_t)units * (d + 4) * sizeof(float) + 127) / 128);
    for (int i = threadIdx.x; i < lines; i += kTailThreads)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(w + (size_t)i * 128));
  }
  pdl_wait();
  float* feat = sh;                    // [d + 4]
  float* hidden = sh + d + 4;          // [256]
  float* logit = hidden + kActHidden;  // [k1]
  const T* scored = reinterpret_cast<const T*>(a.scored);
  // scorer.3: one warp per gathered row, 8 elements per lane step.
  for (int j = warp; j < k1; j += kTailWarps) {
    const T* x = scored + ((size_t)q * k1 + j) * d;
    float s = 0.f;
    for (int c = lane * 8; c < d; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + c);
      const float4 w0 = *reinterpret_cast<const float4*>(a.w3 + c);
      const float4 w1 = *reinterpret_cast<const float4*>(a.w3 + c + 4);
      const float2 p0 = unpack2_f32(v.x, (T*)nullptr), p1 = unpack2_f32(v.y, (T*)nullptr);
      const float2 p2 = unpack2_f32(v.z, (T*)nullptr), p3 = unpack2_f32(v.w, (T*)nullptr);
      s += p0.x * w0.x + p0.y * w0.y + p1.x * w0.z + p1.y * w0.w + p2.x * w1.x + p2.y * w1.y + p3.x * w1.z + p3.y * w1.w;
    }
    s = warp_sum(s);
    if (lane == 0) {
      logit[j] = s + a.b3[0];
      if (part == 0) a.logits[(size_t)q * k1 + j] = s + a.b3[0];
    }
  }
  const float* cls = a.selected + (size_t)q * k1 * d;
  for (int c = threadIdx.x; c < d; c += kTailThreads) feat[c] = cls[c];
  __syncthreads();
  if (warp == 0) {
    // Softmax over the question's options, its entropy and top-2 probabilities, warp-parallel.
    // (The count is at most the class's option count; clamped so a bad count cannot read past
    // the logits staged in shared memory.)
    const int count = min(max(a.counts[q], 0), a.k);
    float top = -INFINITY;
    for (int j = lane; j < count; j += 32) top = fmaxf(top, logit[j + 1]);
    top = warp_max(top);
    float total = 0.f;
    for (int j = lane; j < count; j += 32) total += expf(logit[j + 1] - top);
    total = warp_sum(total);
    float entropy = 0.f, p1 = 0.f, p2 = 0.f;
    for (int j = lane; j < count; j += 32) {
      const float p = expf(logit[j + 1] - top) / total;
      entropy -= p * logf(fmaxf(p, 1e-9f));
      if (p > p1) { p2 = p1; p1 = p; } else p2 = fmaxf(p2, p);
    }
    entropy = warp_sum(entropy);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, p1, o), o2 = __shfl_xor_sync(0xffffffffu, p2, o);
      const float n2 = fmaxf(fminf(p1, o1), fmaxf(p2, o2));
      p1 = fmaxf(p1, o1);
      p2 = n2;
    }
    if (lane == 0) {
      const int c2 = count > 2 ? count : 2;
      feat[d] = p1;
      feat[d + 1] = p1 - p2;
      feat[d + 2] = entropy / logf((float)c2);
      feat[d + 3] = (float)c2 / 255.f;
      if (a.features && part == 0)
        for (int i = 0; i < 4; ++i) a.features[(size_t)q * 4 + i] = feat[d + i];
    }
  }
  __syncthreads();
  // act_head.0 + GELU for this part's hidden units: one warp per unit, float4 over d+4.
  const int kUnits = kActHidden / (int)gridDim.y;
  const int n4 = (d + 4) / 4;
  const float4* f4 = reinterpret_cast<const float4*>(feat);
  for (int u = warp; u < kUnits; u += kTailWarps) {
    const int o = part * kUnits + u;
    const float4* w = reinterpret_cast<const float4*>(a.wa0 + (size_t)o * (d + 4));
    float s = 0.f;
    for (int c = lane; c < n4; c += 32) {
      const float4 x = f4[c], y = __ldg(w + c);
      s += x.x * y.x + x.y * y.y + x.z * y.z + x.w * y.w;
    }
    s = warp_sum(s);
    if (lane == 0) a.hidden[(size_t)q * kActHidden + o] = gelu_erf(s + a.ba0[o]);
  }
  // The part that finishes last computes the action logits from all 256 hidden units.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.arrivals[q], 1) == (int)gridDim.y - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int c = threadIdx.x; c < kActHidden; c += kTailThreads) hidden[c] = __ldcg(a.hidden + (size_t)q * kActHidden + c);
  __syncthreads();
  for (int o = warp; o < a.n_act; o += kTailWarps) {
    const float* w = a.wa2 + (size_t)o * kActHidden;
    float s = 0.f;
    for (int c = lane; c < kActHidden; c += 32) s += w[c] * hidden[c];
    s = warp_sum(s);
    if (lane == 0) a.acts[(size_t)q * a.n_act + o] = s + a.ba2[o];
  }
  if (threadIdx.x == 0) a.arrivals[q] = 0;
}

}  // namespace laya
