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

__global__ void __launch_bounds__(kReadoutThreads) cow_readout_kernel(const __grid_constant__ ReadoutLaunch P) {
  __shared__ float s_n[kReadoutMaxWidth];    // normalised controller input, later the MLP's normalised t1
  __shared__ float s_r[kReadoutMaxWidth];    // normalised readings (heads -> width), later t1
  __shared__ float s_t[kReadoutMaxWidth];    // gated readings
  __shared__ float s_h[kReadoutMaxHidden];   // MLP hidden activations
  __shared__ float s_part[kReadoutThreads / 32 * 256];  // partials of passes up to 256 outputs
  __shared__ float s_red[kReadoutThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok = blockIdx.x;  // b * T + t
  const int64_t b = tok / P.time, t = tok % P.time;
  const int W = P.width, H = P.heads, hw = W / H;
  for (int k = tid; k < W; k += kReadoutThreads) s_n[k] = P.normalized[tok * W + k];
  // readings norm, one warp per head
  for (int h = warp; h < H; h += kReadoutThreads / 32) {
    const float* row = P.readings + ((b * H + h) * P.time + t) * hw;
    float s = 0.f;
    for (int k = lane; k < hw; k += 32) s += row[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
    const float mean = s / static_cast<float>(hw);
    float q = 0.f;
    for (int k = lane; k < hw; k += 32) {
      const float d = row[k] - mean;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(kFull, q, o);
    const float rstd = rsqrtf(q / static_cast<float>(hw) + P.rn_eps);
    for (int k = lane; k < hw; k += 32) s_r[h * hw + k] = (row[k] - mean) * rstd * P.rn_w[k] + P.rn_b[k];
  }
  __syncthreads();
  // gated readings: sigmoid(W_g n + b_g) * r
  gemv<4, 8>(s_n, W, P.wg_t, W, s_part, [&](int o, float g) { s_t[o] = s_r[o] / (1.f + expf(-(g + P.bg[o]))); });
  // t1 = tokens + W_o (gated) + b_o
  gemv<4, 8>(s_t, W, P.wo_t, W, s_part, [&](int o, float v) { s_r[o] = P.tokens[tok * W + o] + (v + P.bo[o]); });
  // the MLP block over t1 (held in s_r)
  mlp_residual(s_r, s_n, s_h, s_part, s_red, W, P.hidden, P.mn_w, P.mn_b, P.mn_eps, P.w1_t, P.w2_t,
               P.out + tok * W);
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
  cow_readout_kernel<<<static_cast<unsigned>(rows), kReadoutThreads, 0, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
