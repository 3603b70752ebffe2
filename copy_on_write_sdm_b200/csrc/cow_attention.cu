// cow_attention.cu -- one decode token through a dense attention block, fused.
//
// The dense ("A") layers of the reference's decode stack (copy_on_write_sdm/
// inference.py:640-651 with model.py:47-190 CausalSelfAttention.decode_with_cache
// and model.py:25-45 ResidualMLP, eval mode) run for every request
//   n     = LayerNorm(tokens)                     q, k, v = split(W_qkv n)   (no bias)
//   cache[b, :, pos] = k, v                      (the fixed-capacity K/V cache)
//   o_h   = softmax(q_h . K_h[0..pos] / sqrt(hw)) V_h[0..pos]   per head h
//   t1    = tokens + W_out o                     (no bias)
//   out   = t1 + W_2 GELU(W_1 LayerNorm(t1))
// as about 25 PyTorch kernels.  Here one 1024-thread block per request does all
// of it; positions come from a device array, so a CUDA graph replays it at every
// step.  Weights are transposed ([in, out], row-major).

#include "cow_common.cuh"
#include "cow_gemv.cuh"

namespace {

constexpr int kAttnMaxWidth = 512;
constexpr int kAttnMaxHidden = 2048;
constexpr int kAttnMaxSmem = 200 * 1024;

struct AttentionLaunch {
  const float* tokens;     // [B, width]
  const int64_t* pos;      // [B] cache slot this token is written to
  const float* ln_w;       // [width] attention norm
  const float* ln_b;
  const float* qkv_t;      // [width, 3 width]: q | k | v, each heads x hw
  const float* out_t;      // [width, width]
  float* key_cache;        // [B, heads, capacity, hw]
  float* value_cache;
  const float* mn_w;       // [width] MLP norm
  const float* mn_b;
  const float* w1_t;       // [width, hidden]
  const float* w2_t;       // [hidden, width]
  float* out;              // [B, width]
  int64_t capacity;
  float ln_eps, mn_eps;
  int32_t width, heads, hidden;
  int32_t vec;  // cache rows read as float4 words: head width a multiple of 4, caches 16-byte aligned
};

size_t attention_smem_floats(int width, int heads, int hidden, int64_t capacity) {
  return static_cast<size_t>(11) * width + hidden + static_cast<size_t>(heads) * capacity + kGemvWarps * kGemvMaxPass +
         kGemvWarps + heads;
}

__global__ void __launch_bounds__(kGemvThreads) cow_attention_kernel(const __grid_constant__ AttentionLaunch P) {
  extern __shared__ float4 smem_raw[];
  const int W = P.width, H = P.heads, hw = W / H, HD = P.hidden;
  const int64_t cap = P.capacity;
  float* s_x = reinterpret_cast<float*>(smem_raw);  // [W] block input
  float* s_n = s_x + W;                              // [W] normalised input, later the MLP's
  float* s_qkv = s_n + W;                            // [3W]
  float* s_o = s_qkv + 3 * W;                        // [W] attention output (heads side by side)
  float* s_t1 = s_o + W;                             // [W]
  float* s_h = s_t1 + W;                             // [HD]
  float* s_part = s_h + HD;                          // [kGemvWarps * kGemvMaxPass]
  float* s_red = s_part + kGemvWarps * kGemvMaxPass;  // [kGemvWarps]
  float* s_inv = s_red + kGemvWarps;                 // [H] 1 / softmax denominator
  float* s_lnw = s_inv + H;                          // [W] attention norm
  float* s_lnb = s_lnw + W;
  float* s_mnw = s_lnb + W;                          // [W] MLP norm
  float* s_mnb = s_mnw + W;
  float* s_sc = s_mnb + W;                           // [H][L] scores, then probabilities
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.x;
  const int64_t pos = P.pos[b];
  if (pos < 0 || pos >= cap) {  // the host checks positions; a bad one yields NaN, not a stray write
    for (int k = tid; k < W; k += kGemvThreads) P.out[b * W + k] = __int_as_float(0x7fc00000);
    return;
  }
  const int L = static_cast<int>(pos) + 1;
  // attention norm
  float acc = 0.f;
  for (int k = tid; k < W; k += kGemvThreads) {  // the token and the norms' weights in one batch of loads
    const float v = P.tokens[b * W + k];
    s_lnw[k] = P.ln_w[k];
    s_lnb[k] = P.ln_b[k];
    s_mnw[k] = P.mn_w[k];
    s_mnb[k] = P.mn_b[k];
    s_x[k] = v;
    acc += v;
  }
  const float mean = block_sum(acc, s_red, tid) / static_cast<float>(W);
  acc = 0.f;
  for (int k = tid; k < W; k += kGemvThreads) {
    const float d = s_x[k] - mean;
    acc += d * d;
  }
  const float rstd = rsqrtf(block_sum(acc, s_red, tid) / static_cast<float>(W) + P.ln_eps);
  for (int k = tid; k < W; k += kGemvThreads) s_n[k] = (s_x[k] - mean) * rstd * s_lnw[k] + s_lnb[k];
  __syncthreads();
  gemv<8, 4>(s_n, W, P.qkv_t, 3 * W, s_part, [&](int o, float v) { s_qkv[o] = v; });
  // this token's key and value into the cache
  for (int i = tid; i < 2 * W; i += kGemvThreads) {
    const int which = i / W, hd = i % W, h = hd / hw, d = hd % hw;
    float* cache = which ? P.value_cache : P.key_cache;
    cache[((b * H + h) * cap + pos) * hw + d] = s_qkv[(1 + which) * W + hd];
  }
  __syncthreads();  // the block's cache stores are visible to its own loads below
  // scores, one thread per (head, position); a key row is read as float4 words,
  // all issued before the dot product so one row costs one round trip
  const float scale = 1.f / sqrtf(static_cast<float>(hw));
  const bool vec = P.vec != 0;
  for (int i = tid; i < H * L; i += kGemvThreads) {
    const int h = i / L, j = i % L;
    const float* kr = P.key_cache + ((b * H + h) * cap + j) * hw;
    const float* q = s_qkv + h * hw;
    float dot = 0.f;
    if (vec) {
      for (int d0 = 0; d0 < hw; d0 += 32) {
        float4 kv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          kv[u] = d0 + 4 * u < hw ? __ldg(reinterpret_cast<const float4*>(kr + d0) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (d0 + 4 * u < hw) {
            const float* qq = q + d0 + 4 * u;
            dot = fmaf(qq[0], kv[u].x, dot);
            dot = fmaf(qq[1], kv[u].y, dot);
            dot = fmaf(qq[2], kv[u].z, dot);
            dot = fmaf(qq[3], kv[u].w, dot);
          }
        }
      }
    } else {
      for (int d = 0; d < hw; ++d) dot = fmaf(q[d], kr[d], dot);
    }
    s_sc[i] = dot * scale;
  }
  __syncthreads();
  // softmax per head, one warp per head
  for (int h = warp; h < H; h += kGemvWarps) {
    float* sc = s_sc + h * L;
    float m = -INFINITY;
    for (int j = lane; j < L; j += 32) m = fmaxf(m, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) {
      const float e = expf(sc[j] - m);
      sc[j] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    if (lane == 0) s_inv[h] = 1.f / sum;
  }
  __syncthreads();
  // o[h, d] = sum_j p[h, j] V[h, j, d]: strands of threads split j; with hw a
  // multiple of 4 a thread owns four dimensions (float4 loads, 32 strands at width
  // 128), each strand issuing its value rows eight at a time
  {
    const int cols = vec ? W / 4 : W;  // threads per strand
    const int strands = kGemvThreads / cols;
    const int c = tid % cols, st = tid / cols;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (st < strands) {
      const int hd = vec ? 4 * c : c, h = hd / hw, d = hd % hw;
      const float* vr = P.value_cache + (b * H + h) * cap * hw + d;
      const float* p = s_sc + h * L;
      for (int j0 = st; j0 < L; j0 += 8 * strands) {
        float4 x[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u * strands;
          if (j < L)
            x[u] = vec ? __ldg(reinterpret_cast<const float4*>(vr + static_cast<int64_t>(j) * hw))
                       : make_float4(__ldg(vr + static_cast<int64_t>(j) * hw), 0.f, 0.f, 0.f);
          else
            x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u * strands;
          const float pj = j < L ? p[j] : 0.f;
          v.x = fmaf(pj, x[u].x, v.x);
          v.y = fmaf(pj, x[u].y, v.y);
          v.z = fmaf(pj, x[u].z, v.z);
          v.w = fmaf(pj, x[u].w, v.w);
        }
      }
      // partials reuse the gemv scratch: strands * W <= kGemvThreads * 4 floats
      float* pp = s_part + st * W + hd;
      pp[0] = v.x;
      if (vec) {
        pp[1] = v.y;
        pp[2] = v.z;
        pp[3] = v.w;
      }
    }
    __syncthreads();
    for (int o = tid; o < W; o += kGemvThreads) {
      float sum = 0.f;
      for (int k = 0; k < strands; ++k) sum += s_part[k * W + o];
      s_o[o] = sum * s_inv[o / hw];
    }
    __syncthreads();
  }
  gemv<4, 4>(s_o, W, P.out_t, W, s_part, [&](int o, float v) { s_t1[o] = s_x[o] + v; });
  mlp_residual(s_t1, s_n, s_h, s_part, s_red, W, HD, s_mnw, s_mnb, P.mn_eps, P.w1_t, P.w2_t, P.out + b * W);
}

}  // namespace

extern "C" {

int cow_attention_mlp_decode(const float* tokens, const int64_t* positions, const float* ln_weight,
                             const float* ln_bias, float ln_eps, const float* qkv_weight_t,
                             const float* out_weight_t, float* key_cache, float* value_cache, int64_t capacity,
                             const float* mlp_norm_weight, const float* mlp_norm_bias, float mlp_eps,
                             const float* mlp_in_weight_t, const float* mlp_out_weight_t, int64_t batch,
                             int32_t width, int32_t heads, int32_t hidden, float* out, void* stream) {
  if (!tokens || !positions || !ln_weight || !ln_bias || !qkv_weight_t || !out_weight_t || !key_cache ||
      !value_cache || !mlp_norm_weight || !mlp_norm_bias || !mlp_in_weight_t || !mlp_out_weight_t || !out ||
      out == tokens || batch < 0 || capacity < 1 || heads < 1 || width < 1 || width % heads || hidden < 1)
    return COW_ERR_INVALID;
  if (width > kAttnMaxWidth || hidden > kAttnMaxHidden) return COW_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * attention_smem_floats(width, heads, hidden, capacity);
  if (smem > static_cast<size_t>(kAttnMaxSmem)) return COW_ERR_UNSUPPORTED;
  if (batch == 0) return COW_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return COW_ERR_CUDA;
  static bool configured[64] = {};
  if (dev < 0 || dev >= 64) return COW_ERR_UNSUPPORTED;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(cow_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnMaxSmem) !=
        cudaSuccess)
      return COW_ERR_CUDA;
    configured[dev] = true;
  }
  AttentionLaunch P{tokens, positions, ln_weight, ln_bias, qkv_weight_t, out_weight_t, key_cache, value_cache,
                    mlp_norm_weight, mlp_norm_bias, mlp_in_weight_t, mlp_out_weight_t, out, capacity, ln_eps,
                    mlp_eps, width, heads, hidden,
                    ((width / heads) % 4 == 0 && (reinterpret_cast<uintptr_t>(key_cache) |
                                                  reinterpret_cast<uintptr_t>(value_cache)) % 16 == 0) ? 1 : 0};
  cow_attention_kernel<<<static_cast<unsigned>(batch), kGemvThreads, smem, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
