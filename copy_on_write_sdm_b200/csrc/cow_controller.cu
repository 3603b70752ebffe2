// cow_controller.cu -- fused route selection of the SDM controller.
//
// After the controller's projections, the reference selects each bank's read
// and write addresses with product keys (sdm.py:96-159): the best
// min(k, sqrt(N)) entries of each of the two codebook score halves, the
// Cartesian sums of the two shortlists, the best k pair sums, addresses
// first * sqrt(N) + second sorted ascending, softmax weights of the selected
// sums; and the gates: forget = -exp(A_log) * softplus(f + dt_bias), input =
// sigmoid(i) (inference.py:459-519).  In PyTorch that is about thirty small
// kernels per SDM layer and token.  Here one warp does all of it for one
// (bank, position) row.

#include "cow_common.cuh"

namespace {

constexpr int kRouteMaxShort = 32;   // shortlist length per codebook half
constexpr int kRouteMaxRoot = 256;   // sqrt(N) <= 256, i.e. N <= 65,536
constexpr float kNegInf = -3.402823466e38f;  // below every finite score; marks taken entries

struct RouteLaunch {
  const float* read_proj;    // [B, T, H * 2 * root]
  const float* write_proj;
  const float* forget_proj;  // [B, T, H]
  const float* input_proj;
  const float* a_log;        // [H]
  const float* dt_bias;      // [H]
  int64_t* read_indices;     // [B*H, T, R]
  float* read_weights;
  int64_t* write_indices;    // [B*H, T, W]
  float* write_weights;
  float* input_gate;         // [B*H, T]
  float* forget_log_gate;
  int64_t batch, time;
  int32_t heads, root, reads, writes;
};

// Warp-wide arg-max of (value, index) pairs; ties go to the smaller index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(kFull, v, o);
    const int oi = __shfl_xor_sync(kFull, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// Top-`count` of `n` scores held lane-strided (element e on lane e % 32, slot e / 32),
// best first, into shared memory.
template <int SLOTS>
__device__ __forceinline__ void warp_topk(float (&x)[SLOTS], int n, int count, float* out_v, int* out_i, int lane) {
  for (int s = 0; s < count; ++s) {
    float v = kNegInf;
    int i = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
      const int e = j * 32 + lane;
      if (e < n && (x[j] > v || (x[j] == v && e < i))) {
        v = x[j];
        i = e;
      }
    }
    warp_argmax(v, i);
    if (lane == 0) {
      out_v[s] = v;
      out_i[s] = i;
    }
    if (i % 32 == lane) {
#pragma unroll
      for (int j = 0; j < SLOTS; ++j)
        if (j == i / 32) x[j] = kNegInf;
    }
    __syncwarp();
  }
}

// Candidate pairs (i+1)(j+1) <= k for k <= 32: sum over i of floor(32 / (i+1)) = 119.
constexpr int kRouteMaxCand = 128;

struct RouteSmem {
  float av[kRouteMaxShort], bv[kRouteMaxShort];
  int ai[kRouteMaxShort], bi[kRouteMaxShort];
  float pv[kRouteMaxShort];
  int pi[kRouteMaxShort];
  int cp[kRouteMaxCand];  // candidate pairs, i * kRouteMaxShort + j
};

// Shortlist of one codebook half: its best `short_len` entries, best first.
// Halves of at most 32 entries take one rank per lane (every lane counts the
// entries ahead of its own: larger, or equal at a smaller index); longer
// halves take `short_len` arg-max rounds.
template <int HALF_SLOTS>
__device__ __forceinline__ void shortlist(const float* scores, int root, int short_len, float* out_v, int* out_i,
                                          int lane) {
  if (root <= 32) {
    const float x = lane < root ? scores[lane] : kNegInf;
    int rank = 0;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const float v = __shfl_sync(kFull, x, j);
      rank += (j < root && (v > x || (v == x && j < lane))) ? 1 : 0;
    }
    if (lane < root && rank < short_len) {
      out_v[rank] = x;
      out_i[rank] = lane;
    }
    __syncwarp();
    return;
  }
  float half[HALF_SLOTS];
#pragma unroll
  for (int j = 0; j < HALF_SLOTS; ++j) {
    const int e = j * 32 + lane;
    half[j] = e < root ? scores[e] : kNegInf;
  }
  warp_topk<HALF_SLOTS>(half, root, short_len, out_v, out_i, lane);
}

// Product-key selection of `k` addresses for one row of scores (2*root values).
// With both shortlists sorted best first, pair (i, j) has at least
// (i+1)(j+1) - 1 pairs at least as good ahead of it, so only pairs with
// (i+1)(j+1) <= k can be among the best k: at most ~4k candidates instead of
// short^2 (ties between equal sums aside, the same selection).
__device__ __forceinline__ void select_routes(const float* scores, int root, int k, RouteSmem& sm, int lane,
                                              int64_t* out_idx, float* out_w) {
  constexpr int kHalfSlots = kRouteMaxRoot / 32;  // 8 values per lane at most
  const int short_len = k < root ? k : root;
  shortlist<kHalfSlots>(scores, root, short_len, sm.av, sm.ai, lane);
  shortlist<kHalfSlots>(scores + root, root, short_len, sm.bv, sm.bi, lane);
  // candidates: lane i < short_len owns pairs (i, j), j < min(short, k / (i+1)),
  // written to sm.cp at that lane's exclusive prefix
  const int lim = lane < short_len ? min(short_len, k / (lane + 1)) : 0;
  int incl = lim;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += y;
  }
  const int total = __shfl_sync(kFull, incl, 31);
  for (int j = 0; j < lim; ++j) sm.cp[incl - lim + j] = lane * kRouteMaxShort + j;
  __syncwarp();
  constexpr int kCandSlots = kRouteMaxCand / 32;
  float ps[kCandSlots];
  int pp[kCandSlots];
#pragma unroll
  for (int j = 0; j < kCandSlots; ++j) {
    const int c = j * 32 + lane;
    pp[j] = c < total ? sm.cp[c] : 0;
    ps[j] = c < total ? sm.av[pp[j] / kRouteMaxShort] + sm.bv[pp[j] % kRouteMaxShort] : kNegInf;
  }
  const int take = k < total ? k : total;
  // `take` arg-max rounds over the candidates; a tie goes to the smaller (i, j)
  for (int s = 0; s < take; ++s) {
    float v = kNegInf;
    int key = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kCandSlots; ++j) {
      const int c = j * 32 + lane;
      if (c < total && (ps[j] > v || (ps[j] == v && pp[j] < key))) {
        v = ps[j];
        key = pp[j];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(kFull, v, o);
      const int ok = __shfl_xor_sync(kFull, key, o);
      if (ov > v || (ov == v && ok < key)) {
        v = ov;
        key = ok;
      }
    }
    if (lane == 0) {
      sm.pv[s] = v;
      sm.pi[s] = key;
    }
#pragma unroll
    for (int j = 0; j < kCandSlots; ++j)
      if (j * 32 + lane < total && pp[j] == key) ps[j] = kNegInf;
  }
  __syncwarp();
  // lane s < take holds selected pair s; addresses ascending, softmax weights
  int addr = 0x7fffffff;
  float v = kNegInf;
  if (lane < take) {
    const int p = sm.pi[lane];
    addr = sm.ai[p / kRouteMaxShort] * root + sm.bi[p % kRouteMaxShort];
    v = sm.pv[lane];
  }
  float m = v;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  const float ex = lane < take ? expf(v - m) : 0.f;
  float sum = ex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  int rank = 0;
  for (int j = 0; j < take; ++j) {
    const int other = __shfl_sync(kFull, addr, j);
    rank += other < addr ? 1 : 0;
  }
  if (lane < take) {
    out_idx[rank] = addr;
    out_w[rank] = ex / sum;
  }
}

__global__ void __launch_bounds__(128) cow_route_kernel(const __grid_constant__ RouteLaunch P) {
  __shared__ RouteSmem s_sm[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + warp;  // (bank, t) = (b*H + h) * T + t
  const int64_t rows = P.batch * P.heads * P.time;
  if (row >= rows) return;
  const int H = P.heads;
  const int64_t t = row % P.time;
  const int64_t bank = row / P.time;
  const int64_t b = bank / H;
  const int h = static_cast<int>(bank % H);
  const int64_t tok = b * P.time + t;  // row of the [B, T, ...] projections
  const int key_w = 2 * P.root;
  auto& sm = s_sm[warp];
  auto select = [&](const float* scores, int k, int64_t* idx, float* w) {
    select_routes(scores, P.root, k, sm, lane, idx, w);
    __syncwarp();
  };
  select(P.read_proj + (tok * H + h) * key_w, P.reads, P.read_indices + row * P.reads, P.read_weights + row * P.reads);
  select(P.write_proj + (tok * H + h) * key_w, P.writes, P.write_indices + row * P.writes,
         P.write_weights + row * P.writes);
  if (lane == 0) {
    const float x = P.forget_proj[tok * H + h] + P.dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, threshold 20
    P.forget_log_gate[row] = -expf(P.a_log[h]) * sp;
    P.input_gate[row] = 1.f / (1.f + expf(-P.input_proj[tok * H + h]));
  }
}

// Whole controller for one token row (b, t): layer norm, the read / write /
// value / forget / input projections (weights concatenated and transposed to
// [width, Ntot] so that consecutive threads read consecutive outputs), then
// per bank h the route selection, the gates and the value slice.
struct ControllerLaunch {
  const float* tokens;      // [B*T, width]
  const float* ln_w;        // [width]
  const float* ln_b;
  const float* wt;          // [width, Ntot]: read H*2root | write H*2root | value width | forget H | input H
  const float* bias;        // [Ntot]
  const float* a_log;       // [H]
  const float* dt_bias;     // [H]
  float* normalized;        // [B*T, width]
  int64_t* read_indices;    // [B*H, T, R]
  float* read_weights;
  int64_t* write_indices;   // [B*H, T, W]
  float* write_weights;
  float* values;            // [B*H, T, width / H]
  float* input_gate;        // [B*H, T]
  float* forget_log_gate;
  int64_t batch, time;
  float eps;
  int32_t width, heads, root, reads, writes, ntot;
};

constexpr int kCtrlThreads = 512;
constexpr int kCtrlMaxWidth = 512;
constexpr int kCtrlMaxOut = 4096;
constexpr int kCtrlWarps = kCtrlThreads / 32;
constexpr int kCtrlJ = 4, kCtrlU = 8, kCtrlPass = 32 * kCtrlJ;  // projection pass: 128 outputs
static_assert(kCtrlMaxWidth <= kCtrlThreads, "the prologue loads one element per thread");
constexpr int kCtrlGateHeads = 64;  // gate parameters of the first 64 banks staged in shared memory

__global__ void __launch_bounds__(kCtrlThreads) cow_controller_kernel(const __grid_constant__ ControllerLaunch P) {
  __shared__ float s_x[kCtrlMaxWidth];
  __shared__ float s_out[kCtrlMaxOut];
  __shared__ float s_red[2][kCtrlWarps];
  __shared__ float s_part[kCtrlWarps * kCtrlPass];
  __shared__ RouteSmem s_sm[kCtrlWarps];
  __shared__ float s_al[kCtrlGateHeads], s_dt[kCtrlGateHeads];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t tok = blockIdx.x;  // b * T + t
  const int width = P.width, H = P.heads, key_w = 2 * P.root;
  // every small operand in one batch of independent loads: the token, the norm's
  // weights (width <= kCtrlThreads, so one element per thread), the projection
  // bias (into s_out, where the projection adds to it) and the gate parameters
  float sum = 0.f, lw = 0.f, lb = 0.f;
  if (tid < width) {
    const float v = P.tokens[tok * width + tid];
    lw = P.ln_w[tid];
    lb = P.ln_b[tid];
    s_x[tid] = v;
    sum = v;
  }
  for (int o = tid; o < P.ntot; o += kCtrlThreads) s_out[o] = P.bias[o];
  if (tid < H && tid < kCtrlGateHeads) {
    s_al[tid] = P.a_log[tid];
    s_dt[tid] = P.dt_bias[tid];
  }
  // layer norm: mean, then variance of the centred values (two passes over shared memory)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  if (lane == 0) s_red[0][warp] = sum;
  __syncthreads();
  float mean = 0.f;
#pragma unroll
  for (int w = 0; w < kCtrlWarps; ++w) mean += s_red[0][w];
  mean /= static_cast<float>(width);
  float sq = 0.f;
  for (int k = tid; k < width; k += kCtrlThreads) {
    const float d = s_x[k] - mean;
    sq += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(kFull, sq, o);
  if (lane == 0) s_red[1][warp] = sq;
  __syncthreads();
  float var = 0.f;
#pragma unroll
  for (int w = 0; w < kCtrlWarps; ++w) var += s_red[1][w];
  const float rstd = rsqrtf(var / static_cast<float>(width) + P.eps);
  if (tid < width) {
    const float nv = (s_x[tid] - mean) * rstd * lw + lb;
    P.normalized[tok * width + tid] = nv;
    s_x[tid] = nv;
  }
  __syncthreads();
  // projections: passes of 128 outputs (4 per lane); the warps split k (warp w
  // takes k = w, w + 16, ...) with up to 32 weight loads in flight per lane, and
  // their partial sums meet in shared memory
  const int N = P.ntot;
  for (int o0 = 0; o0 < N; o0 += kCtrlPass) {
    float acc[kCtrlJ] = {0.f, 0.f, 0.f, 0.f};
    int k = warp;
    if (o0 + kCtrlPass <= N) {
      for (; k + (kCtrlU - 1) * kCtrlWarps < width; k += kCtrlU * kCtrlWarps) {
        float w[kCtrlU][kCtrlJ];
#pragma unroll
        for (int u = 0; u < kCtrlU; ++u) {
          const float* row = P.wt + static_cast<int64_t>(k + u * kCtrlWarps) * N + o0 + lane;
#pragma unroll
          for (int j = 0; j < kCtrlJ; ++j) w[u][j] = __ldg(row + 32 * j);
        }
#pragma unroll
        for (int u = 0; u < kCtrlU; ++u) {
          const float x = s_x[k + u * kCtrlWarps];
#pragma unroll
          for (int j = 0; j < kCtrlJ; ++j) acc[j] = fmaf(x, w[u][j], acc[j]);
        }
      }
    }
    for (; k < width; k += kCtrlWarps) {
      const float x = s_x[k];
      const float* row = P.wt + static_cast<int64_t>(k) * N + o0 + lane;
#pragma unroll
      for (int j = 0; j < kCtrlJ; ++j)
        if (o0 + lane + 32 * j < N) acc[j] = fmaf(x, __ldg(row + 32 * j), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < kCtrlJ; ++j) s_part[warp * kCtrlPass + lane + 32 * j] = acc[j];
    __syncthreads();
    {  // four threads per output, each adding a quarter of the warps' partials
      const int o = tid >> 2, r = tid & 3;
      float v = 0.f;
#pragma unroll
      for (int w = r; w < kCtrlWarps; w += 4) v += s_part[w * kCtrlPass + o];
      v += __shfl_xor_sync(kFull, v, 1);
      v += __shfl_xor_sync(kFull, v, 2);
      if (r == 0 && o0 + o < N) s_out[o0 + o] += v;
    }
    __syncthreads();
  }
  const int64_t b = tok / P.time, t = tok % P.time;
  const int hw = width / H;
  const float* rproj = s_out;
  const float* wproj = s_out + H * key_w;
  const float* vproj = wproj + H * key_w;
  const float* fproj = vproj + width;
  const float* iproj = fproj + H;
  // one warp per (bank, read or write) route selection; the read warp also
  // writes the bank's value slice and gates
  for (int item = warp; item < 2 * H; item += kCtrlWarps) {
    const int h = item >> 1;
    const int64_t row = (b * H + h) * P.time + t;
    auto& sm = s_sm[warp];
    __syncwarp();  // the warp's previous selection is done with sm
    if (item & 1) {
      select_routes(wproj + h * key_w, P.root, P.writes, sm, lane, P.write_indices + row * P.writes,
                    P.write_weights + row * P.writes);
      continue;
    }
    select_routes(rproj + h * key_w, P.root, P.reads, sm, lane, P.read_indices + row * P.reads,
                  P.read_weights + row * P.reads);
    for (int k = lane; k < hw; k += 32) P.values[row * hw + k] = vproj[h * hw + k];
    if (lane == 0) {
      const float x = fproj[h] + (h < kCtrlGateHeads ? s_dt[h] : P.dt_bias[h]);
      const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, threshold 20
      P.forget_log_gate[row] = -expf(h < kCtrlGateHeads ? s_al[h] : P.a_log[h]) * sp;
      P.input_gate[row] = 1.f / (1.f + expf(-iproj[h]));
    }
  }
}

}  // namespace

extern "C" {

int cow_route_controller(const float* read_proj, const float* write_proj, const float* forget_proj,
                         const float* input_proj, const float* a_log, const float* dt_bias, int64_t batch,
                         int64_t time, int32_t heads, int32_t root, int32_t reads, int32_t writes,
                         int64_t* read_indices, float* read_weights, int64_t* write_indices, float* write_weights,
                         float* input_gate, float* forget_log_gate, void* stream) {
  if (!read_proj || !write_proj || !forget_proj || !input_proj || !a_log || !dt_bias || !read_indices ||
      !read_weights || !write_indices || !write_weights || !input_gate || !forget_log_gate || batch < 0 ||
      time < 0 || heads < 1)
    return COW_ERR_INVALID;
  if (root < 1 || root > kRouteMaxRoot || reads < 1 || writes < 1 || reads > root * root ||
      writes > root * root || (reads < root ? reads : root) > kRouteMaxShort ||
      (writes < root ? writes : root) > kRouteMaxShort || reads > 32 || writes > 32)
    return COW_ERR_UNSUPPORTED;
  const int64_t rows = batch * heads * time;
  if (rows == 0) return COW_OK;
  RouteLaunch P{read_proj, write_proj, forget_proj, input_proj, a_log, dt_bias, read_indices, read_weights,
                write_indices, write_weights, input_gate, forget_log_gate, batch, time, heads, root, reads, writes};
  cow_route_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, as_stream(stream)>>>(P);
  return launch_status();
}

int cow_controller_step(const float* tokens, const float* ln_weight, const float* ln_bias, float eps,
                        const float* weights_t, const float* bias, const float* a_log, const float* dt_bias,
                        int64_t batch, int64_t time, int32_t width, int32_t heads, int32_t root, int32_t reads,
                        int32_t writes, float* normalized, int64_t* read_indices, float* read_weights,
                        int64_t* write_indices, float* write_weights, float* values, float* input_gate,
                        float* forget_log_gate, void* stream) {
  if (!tokens || !ln_weight || !ln_bias || !weights_t || !bias || !a_log || !dt_bias || !normalized ||
      !read_indices || !read_weights || !write_indices || !write_weights || !values || !input_gate ||
      !forget_log_gate || batch < 0 || time < 0 || heads < 1 || width < 1 || width % heads)
    return COW_ERR_INVALID;
  const int64_t ntot = 4LL * heads * root + width + 2LL * heads;
  if (width > kCtrlMaxWidth || ntot > kCtrlMaxOut || root < 1 || root > kRouteMaxRoot || reads < 1 || writes < 1 ||
      reads > root * root || writes > root * root || reads > 32 || writes > 32)
    return COW_ERR_UNSUPPORTED;
  const int64_t rows = batch * time;
  if (rows == 0) return COW_OK;
  ControllerLaunch P{tokens, ln_weight, ln_bias, weights_t, bias, a_log, dt_bias, normalized, read_indices,
                     read_weights, write_indices, write_weights, values, input_gate, forget_log_gate, batch, time,
                     eps, width, heads, root, reads, writes, static_cast<int32_t>(ntot)};
  cow_controller_kernel<<<static_cast<unsigned>(rows), kCtrlThreads, 0, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
