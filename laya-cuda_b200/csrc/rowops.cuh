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

constexpr int kRowWarps = 8;           // rows per 256-thread block
constexpr int kMaxPerLane = 32;        // supports widths up to 1024

// Loads row `src` (fp32, width d) into v[0 .. d/32): element i of the lane lives at column
// lane*CH + (i/CH)*32*CH + i%CH (vectors of CH consecutive floats).
template <int CH>
__device__ __forceinline__ void row_load(const float* src, int d, int lane, float (&v)[kMaxPerLane]) {
#pragma unroll
  for (int j = 0; j < kMaxPerLane / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (col < d) {
      if (CH == 4) {
        float4 t = *reinterpret_cast<const float4*>(src + col);
        v[j * 4] = t.x; v[j * 4 + 1] = t.y; v[j * 4 + 2] = t.z; v[j * 4 + 3] = t.w;
      } else {
        float2 t = *reinterpret_cast<const float2*>(src + col);
        v[j * 2] = t.x; v[j * 2 + 1] = t.y;
      }
    }
  }
}

template <int CH>
__device__ __forceinline__ void row_store(float* dst, int d, int lane, const float (&v)[kMaxPerLane]) {
#pragma unroll
  for (int j = 0; j < kMaxPerLane / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (col < d) {
      if (CH == 4) *reinterpret_cast<float4*>(dst + col) = make_float4(v[j * 4], v[j * 4 + 1], v[j * 4 + 2], v[j * 4 + 3]);
      else *reinterpret_cast<float2*>(dst + col) = make_float2(v[j * 2], v[j * 2 + 1]);
    }
  }
}

template <int CH, typename T>
__device__ __forceinline__ void row_store_t(T* dst, int d, int lane, const float (&v)[kMaxPerLane]) {
#pragma unroll
  for (int j = 0; j < kMaxPerLane / CH; ++j) {
    const int col = j * 32 * CH + lane * CH;
    if (col < d) {
      if (CH == 4) {
        uint2 w; w.x = pack2<T>(v[j * 4], v[j * 4 + 1]); w.y = pack2<T>(v[j * 4 + 2], v[j * 4 + 3]);
        *reinterpret_cast<uint2*>(dst + col) = w;
      } else {
        *reinterpret_cast<uint32_t*>(dst + col) = pack2<T>(v[j * 2], v[j * 2 + 1]);
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// In-place LayerNorm of the lane's slice: v = (v - mean) * rsqrt(var + eps) * gamma (+ beta).
template <int CH>
__device__ __forceinline__ void row_layernorm(float (&v)[kMaxPerLane], int d, int lane, const float* gamma,
                                              const float* beta, float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i)
    if ((i / CH) * 32 * CH + lane * CH < d) s += v[i];
  const float mean = warp_sum(s) / d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i)
    if ((i / CH) * 32 * CH + lane * CH < d) { const float t = v[i] - mean; q += t * t; }
  const float inv = rsqrtf(warp_sum(q) / d + eps);
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int col = (i / CH) * 32 * CH + lane * CH + i % CH;
    if (col < d) v[i] = (v[i] - mean) * inv * gamma[col] + (beta ? beta[col] : 0.f);
  }
}

// residual[t] = LN_gamma(E[ids[t]]) (fp32); x[t] = residual[t] rounded to T.
// Replaces kernels.cu:16-19 + the embeddings.norm and copy passes of runtime.py:93-95.
template <int CH, typename T>
__global__ void __launch_bounds__(kRowWarps * 32) embed_norm_kernel(const int* ids, const float* table,
                                                                    const float* gamma, float eps, int rows, int d,
                                                                    int vocab, float* residual, T* x, int* err) {
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  int id = ids[row];
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicCAS(err, 0, kErrBadIndex);
    id = 0;
  }
  float v[kMaxPerLane];
  row_load<CH>(table + (size_t)id * d, d, lane, v);
  row_layernorm<CH>(v, d, lane, gamma, nullptr, eps);
  row_store<CH>(residual + (size_t)row * d, d, lane, v);
  row_store_t<CH>(x + (size_t)row * d, d, lane, v);
}

struct NormArgs {
  float* residual;          // [rows][d] fp32, updated in place
  const float* partials;    // split-K partial sums [splits][rows][d] to add first, or nullptr
  int splits;
  const float* gamma1; const float* beta1; float eps1;
  // Final-norm fusion (encoder.final_norm -> + type_emb[kind] -> head norm1):
  int fused_final;
  const float* type_emb; const int* kinds;
  const float* gamma2; const float* beta2; float eps2;
  void* x;                  // [rows][d] T output (may be nullptr)
  int rows, d;
};

// Normal:  residual += sum(partials); x = LN1(residual).
// Fused:   residual = LN1(residual + sum(partials)) + type_emb[kind]; x = LN2(residual).
// Replaces kernels.cu:20-49 and kernels.cu:155-158 (type_add).
template <int CH, typename T>
__global__ void __launch_bounds__(kRowWarps * 32) norm_kernel(const NormArgs a) {
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= a.rows) return;
  float* r = a.residual + (size_t)row * a.d;
  float v[kMaxPerLane];
  row_load<CH>(r, a.d, lane, v);
  for (int s = 0; s < a.splits; ++s) {
    float p[kMaxPerLane];
    row_load<CH>(a.partials + ((size_t)s * a.rows + row) * a.d, a.d, lane, p);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) v[i] += p[i];
  }
  if (a.fused_final) {
    row_layernorm<CH>(v, a.d, lane, a.gamma1, a.beta1, a.eps1);
    float t[kMaxPerLane];
    row_load<CH>(a.type_emb + (size_t)a.kinds[row] * a.d, a.d, lane, t);
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) v[i] += t[i];
    row_store<CH>(r, a.d, lane, v);
    row_layernorm<CH>(v, a.d, lane, a.gamma2, a.beta2, a.eps2);
  } else {
    if (a.splits > 0) row_store<CH>(r, a.d, lane, v);
    row_layernorm<CH>(v, a.d, lane, a.gamma1, a.beta1, a.eps1);
  }
  if (a.x) row_store_t<CH>(reinterpret_cast<T*>(a.x) + (size_t)row * a.d, a.d, lane, v);
}

// selected[i] = residual[indices[i]] (fp32); scored[i] = attention[indices[i]] (T).
// Replaces kernels.cu:159-166 (gather, gather_half) as used by laya.py:226-227.
template <typename T>
__global__ void __launch_bounds__(256) gather_rows_kernel(const float* residual, const T* attention,
                                                          const int* indices, int count, int d, int rows,
                                                          float* selected, T* scored, int* err) {
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
  int k, d, n_act;
};

constexpr int kTailThreads = 256;
constexpr int kActHidden = 256;

// One CTA per question.  Restates laya.py:241-245 and kernels.cu:167-183 (features) in fp32:
// logits = scored . w3 + b3; features = [CLS row, p1, p1 - p2, H / log(max(c,2)), max(c,2)/255]
// over the option logits; acts = act_head.2(gelu(act_head.0(features))).
template <typename T>
__global__ void __launch_bounds__(kTailThreads) head_tail_kernel(const TailArgs a) {
  extern __shared__ float sh[];
  const int q = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k1 = a.k + 1, d = a.d;
  float* logit = sh;                 // [k1]
  float* feat = sh + k1;             // [d + 4]
  float* hidden = feat + d + 4;      // [256]
  const T* scored = reinterpret_cast<const T*>(a.scored);
  for (int j = warp; j < k1; j += kTailThreads / 32) {
    const T* x = scored + ((size_t)q * k1 + j) * d;
    float s = 0.f;
    for (int c = lane; c < d; c += 32) s += to_f32(x[c]) * a.w3[c];
    s = warp_sum(s);
    if (lane == 0) { logit[j] = s + a.b3[0]; a.logits[(size_t)q * k1 + j] = s + a.b3[0]; }
  }
  const float* cls = a.selected + (size_t)q * k1 * d;
  for (int c = threadIdx.x; c < d; c += kTailThreads) feat[c] = cls[c];
  __syncthreads();
  if (threadIdx.x == 0) {
    const int count = a.counts[q];
    float top = -INFINITY, total = 0.f, p1 = 0.f, p2 = 0.f, entropy = 0.f;
    for (int j = 0; j < count; ++j) top = fmaxf(top, logit[j + 1]);
    for (int j = 0; j < count; ++j) total += expf(logit[j + 1] - top);
    for (int j = 0; j < count; ++j) {
      const float p = expf(logit[j + 1] - top) / total;
      entropy -= p * logf(fmaxf(p, 1e-9f));
      if (p > p1) { p2 = p1; p1 = p; } else p2 = fmaxf(p2, p);
    }
    const int c2 = count > 2 ? count : 2;
    feat[d] = p1;
    feat[d + 1] = p1 - p2;
    feat[d + 2] = entropy / logf((float)c2);
    feat[d + 3] = (float)c2 / 255.f;
  }
  __syncthreads();
  for (int o = warp; o < kActHidden; o += kTailThreads / 32) {
    const float* w = a.wa0 + (size_t)o * (d + 4);
    float s = 0.f;
    for (int c = lane; c < d + 4; c += 32) s += w[c] * feat[c];
    s = warp_sum(s);
    if (lane == 0) hidden[o] = gelu_erf(s + a.ba0[o]);
  }
  __syncthreads();
  for (int o = warp; o < a.n_act; o += kTailThreads / 32) {
    const float* w = a.wa2 + (size_t)o * kActHidden;
    float s = 0.f;
    for (int c = lane; c < kActHidden; c += 32) s += w[c] * hidden[c];
    s = warp_sum(s);
    if (lane == 0) a.acts[(size_t)q * a.n_act + o] = s + a.ba2[o];
  }
}

}  // namespace laya
