// cow_readout.cu -- the SDM layer's readout and the MLP block after it, fused.
//
// After the step, the reference's decode (copy_on_write_sdm/inference.py:523-536
// `_finish_faithful_sdm_step`, inference.py:658-661 the residual adds,
// model.py:25-45 `ResidualMLP`, eval mode so dropout is the identity) runs for every token
//   r      = LayerNorm_hw(readings)              per bank, eps 1e-6, then heads -> width
//   t1     = tokens + W_o (sigmoid(W_g n + b_g) * r) + b_o   (n: the controller's normalised input)
//   out    = t1 + W_2 GELU(W_1 LayerNorm_width(t1))          (no biases in the MLP)
// as about a dozen PyTorch kernels.  Here one 1024-thread block per token row does
// it all; weights are stored transposed ([in, out]) so that consecutive lanes read
// consecutive outputs of each input element.

#include "cow_common.cuh"
#include "cow_gemv.cuh"

namespace {

constexpr int kReadoutThreads = kGemvThreads;
constexpr int kReadoutMaxWidth = 512;
constexpr int kReadoutMaxHidden = 2048;

struct ReadoutLaunch {
  const float* tokens;       // [B*T, width] residual stream into the layer
  const float* normalized;   // [B*T, width] controller's normalised input
  const float* readings;     // [B*H, T, hw]
  const float* rn_w;         // [hw] readings norm
  const float* rn_b;
  const float* wg_t;         // [width, width] output gate, transposed
  const float* bg;           // [width]
  const float* wo_t;         // [width, width] output projection, transposed
  const float* bo;           // [width]
  const float* mn_w;         // [width] MLP norm
  const float* mn_b;
  const float* w1_t;         // [width, hidden]
  const float* w2_t;         // [hidden, width]
  float* out;                // [B*T, width]
  int64_t time;
  float rn_eps, mn_eps;
  int32_t width, heads, hidden;
};

size_t readout_smem_floats(int width, int hidden, int heads) {
  return static_cast<size_t>(8) * width + hidden + 2 * (width / heads) + kGemvWarps * kGemvMaxPass + kGemvWarps;
}

__global__ void __launch_bounds__(kReadoutThreads) cow_readout_kernel(const __grid_constant__ ReadoutLaunch P) {
  extern __shared__ float4 smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok = blockIdx.x;  // b * T + t
  const int64_t b = tok / P.time, t = tok % P.time;
  const int W = P.width, H = P.heads, hw = W / H, HD = P.hidden;
  float* s_n = reinterpret_cast<float*>(smem_raw);  // [W] controller input, later the MLP's normalised t1
  float* s_r = s_n + W;                              // [W] readings (heads side by side), normalised; later t1
  float* s_t = s_r + W;                              // [W] gated readings
  float* s_tok = s_t + W;                            // [W] residual input
  float* s_bg = s_tok + W;                           // [W] gate bias
  float* s_bo = s_bg + W;                            // [W] output bias
  float* s_mnw = s_bo + W;                           // [W] MLP norm
  float* s_mnb = s_mnw + W;
  float* s_rnw = s_mnb + W;                          // [hw] readings norm
  float* s_rnb = s_rnw + hw;
  float* s_h = s_rnb + hw;                           // [HD]
  float* s_part = s_h + HD;                          // [kGemvWarps * kGemvMaxPass]
  float* s_red = s_part + kGemvWarps * kGemvMaxPass;  // [kGemvWarps]
  // every small operand in one batch of independent loads (one L2 round trip),
  // instead of one dependent round trip per epilogue
  for (int k = tid; k < W; k += kReadoutThreads) {
    const int h = k / hw, d = k % hw;
    s_n[k] = P.normalized[tok * W + k];
    s_r[k] = P.readings[((b * H + h) * P.time + t) * hw + d];
    s_tok[k] = P.tokens[tok * W + k];
    s_bg[k] = P.bg[k];
    s_bo[k] = P.bo[k];
    s_mnw[k] = P.mn_w[k];
    s_mnb[k] = P.mn_b[k];
  }
  for (int k = tid; k < hw; k += kReadoutThreads) {
    s_rnw[k] = P.rn_w[k];
    s_rnb[k] = P.rn_b[k];
  }
  __syncthreads();
  // readings norm in place, one warp per head
  for (int h = warp; h < H; h += kReadoutThreads / 32) {
    float* row = s_r + h * hw;
    float sum = 0.f;
    for (int k = lane; k < hw; k += 32) sum += row[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    const float mean = sum / static_cast<float>(hw);
    float q = 0.f;
    for (int k = lane; k < hw; k += 32) {
      const float d = row[k] - mean;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(kFull, q, o);
    const float rstd = rsqrtf(q / static_cast<float>(hw) + P.rn_eps);
    for (int k = lane; k < hw; k += 32) row[k] = (row[k] - mean) * rstd * s_rnw[k] + s_rnb[k];
  }
  __syncthreads();
  // gated readings: sigmoid(W_g n + b_g) * r
  gemv<4, 4>(s_n, W, P.wg_t, W, s_part, [&](int o, float g) { s_t[o] = s_r[o] / (1.f + expf(-(g + s_bg[o]))); });
  // t1 = tokens + W_o (gated) + b_o
  gemv<4, 4>(s_t, W, P.wo_t, W, s_part, [&](int o, float v) { s_r[o] = s_tok[o] + (v + s_bo[o]); });
  // the MLP block over t1 (held in s_r)
  mlp_residual(s_r, s_n, s_h, s_part, s_red, W, HD, s_mnw, s_mnb, P.mn_eps, P.w1_t, P.w2_t, P.out + tok * W);
}

}  // namespace

extern "C" {

int cow_readout_mlp_step(const float* tokens, const float* normalized, const float* readings, const float* rn_weight,
                         const float* rn_bias, float rn_eps, const float* gate_weight_t, const float* gate_bias,
                         const float* out_weight_t, const float* out_bias, const float* mlp_norm_weight,
                         const float* mlp_norm_bias, float mlp_eps, const float* mlp_in_weight_t,
                         const float* mlp_out_weight_t, int64_t batch, int64_t time, int32_t width, int32_t heads,
                         int32_t hidden, float* out, void* stream) {
  if (!tokens || !normalized || !readings || !rn_weight || !rn_bias || !gate_weight_t || !gate_bias ||
      !out_weight_t || !out_bias || !mlp_norm_weight || !mlp_norm_bias || !mlp_in_weight_t || !mlp_out_weight_t ||
      !out || batch < 0 || time < 0 || heads < 1 || width < 1 || width % heads || hidden < 1)
    return COW_ERR_INVALID;
  if (width > kReadoutMaxWidth || hidden > kReadoutMaxHidden || heads > 64) return COW_ERR_UNSUPPORTED;
  const int64_t rows = batch * time;
  if (rows == 0) return COW_OK;
  ReadoutLaunch P{tokens, normalized, readings, rn_weight, rn_bias, gate_weight_t, gate_bias, out_weight_t,
                  out_bias, mlp_norm_weight, mlp_norm_bias, mlp_in_weight_t, mlp_out_weight_t, out, time,
                  rn_eps, mlp_eps, width, heads, hidden};
  const size_t smem = sizeof(float) * readout_smem_floats(width, hidden, heads);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return COW_ERR_CUDA;
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return COW_ERR_UNSUPPORTED;
  if (!configured[dev]) {
    const int most = static_cast<int>(sizeof(float) * readout_smem_floats(kReadoutMaxWidth, kReadoutMaxHidden, 1));
    if (cudaFuncSetAttribute(cow_readout_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, most) != cudaSuccess)
      return COW_ERR_CUDA;
    configured[dev] = true;
  }
  cow_readout_kernel<<<static_cast<unsigned>(rows), kReadoutThreads, smem, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
