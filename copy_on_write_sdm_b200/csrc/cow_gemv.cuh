// cow_gemv.cuh -- matrix-vector helpers shared by the one-block-per-token decode
// kernels (readout + MLP, attention block): a block of kGemvThreads threads holds
// the token's vectors in shared memory and multiplies them by transposed
// ([in, out], row-major) weights read straight from global memory / L2.
#pragma once

#include "cow_common.cuh"

namespace {

constexpr int kGemvThreads = 1024;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxPass = 256;  // outputs per pass at most (J <= 8)

// Sum of v over the block; red holds kGemvWarps floats.
__device__ __forceinline__ float block_sum(float v, float* red, int tid) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  __syncthreads();  // red may still be read from the previous call
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kGemvThreads / 32; ++w) s += red[w];
  return s;
}

// y[j] = epi(j, sum_k in[k] * Wt[k*ld + j]) for j < N (a window of N columns of a
// row-major [K, ld] matrix), from the block's shared vector ``in``.  A pass covers
// 32*J outputs (J per lane); the 32 warps split k (warp w takes k = w, w+32, ...),
// and each lane issues a group of U x J predicated weight loads before the FMAs
// that consume them, so a phase costs ceil(K / (32 U)) dependent L2 round trips.
// The warps' partial sums meet in shared memory, where four threads per output
// add them up.
template <int J, int U, typename Epi>
__device__ __forceinline__ void gemv_cols(const float* __restrict__ in, int K, const float* __restrict__ Wt, int ld,
                                          int N, float* part, Epi epi) {
  constexpr int kWarps = kGemvThreads / 32, kPass = 32 * J;
  static_assert(kPass <= kGemvMaxPass, "pass wider than the partial-sum scratch");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int o0 = 0; o0 < N; o0 += kPass) {
    float acc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) acc[j] = 0.f;
    bool on[J];
#pragma unroll
    for (int j = 0; j < J; ++j) on[j] = o0 + lane + 32 * j < N;
    for (int k0 = warp; k0 < K; k0 += U * kWarps) {
      float w[U][J];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = k0 + u * kWarps;
        const float* row = Wt + static_cast<int64_t>(k) * ld + o0 + lane;
#pragma unroll
        for (int j = 0; j < J; ++j) w[u][j] = (k < K && on[j]) ? __ldg(row + 32 * j) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = k0 + u * kWarps;
        const float x = k < K ? in[k] : 0.f;
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = fmaf(x, w[u][j], acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) part[warp * kPass + lane + 32 * j] = acc[j];
    __syncthreads();
    // four threads per output, each adding a quarter of the warps' partials
    for (int q = tid; q < 4 * kPass; q += kGemvThreads) {
      const int o = q >> 2, r = q & 3;
      float v = 0.f;
#pragma unroll
      for (int w = r; w < kWarps; w += 4) v += part[w * kPass + o];
      v += __shfl_xor_sync(kFull, v, 1);
      v += __shfl_xor_sync(kFull, v, 2);
      if (r == 0 && o0 + o < N) epi(o0 + o, v);
    }
    __syncthreads();
  }
}

// The whole [K, N] matrix: y[o] = epi(o, sum_k in[k] * Wt[k*N + o]).
template <int J, int U, typename Epi>
__device__ __forceinline__ void gemv(const float* __restrict__ in, int K, const float* __restrict__ Wt, int N,
                                     float* part, Epi epi) {
  gemv_cols<J, U>(in, K, Wt, N, N, part, epi);
}

// out_row[o] = t1[o] + (W_2 GELU_erf(W_1 LayerNorm(t1)))[o]: the pre-norm MLP block
// (no biases in W_1, W_2) and its residual add for the block's token.  t1 [W] is in
// shared memory; s_n [W], s_h [HD], part and red are shared scratch.
__device__ __forceinline__ void mlp_residual(const float* s_t1, float* s_n, float* s_h, float* part, float* red,
                                             int W, int HD, const float* mn_w, const float* mn_b, float eps,
                                             const float* w1_t, const float* w2_t, float* out_row) {
  const int tid = threadIdx.x;
  float acc = 0.f;
  for (int k = tid; k < W; k += kGemvThreads) acc += s_t1[k];
  const float mean = block_sum(acc, red, tid) / static_cast<float>(W);
  acc = 0.f;
  for (int k = tid; k < W; k += kGemvThreads) {
    const float d = s_t1[k] - mean;
    acc += d * d;
  }
  const float rstd = rsqrtf(block_sum(acc, red, tid) / static_cast<float>(W) + eps);
  for (int k = tid; k < W; k += kGemvThreads) s_n[k] = (s_t1[k] - mean) * rstd * mn_w[k] + mn_b[k];
  __syncthreads();
  gemv<8, 4>(s_n, W, w1_t, HD, part, [&](int o, float v) { s_h[o] = 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); });
  gemv<4, 8>(s_h, HD, w2_t, W, part, [&](int o, float v) { out_row[o] = s_t1[o] + v; });
}

}  // namespace
