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

struct RouteSmem {
  float av[kRouteMaxShort], bv[kRouteMaxShort];
  int ai[kRouteMaxShort], bi[kRouteMaxShort];
  float pv[kRouteMaxShort];
  int pi[kRouteMaxShort];
};

// Product-key selection of `k` addresses for one row of scores (2*root values).
__device__ __forceinline__ void select_routes(const float* scores, int root, int k, RouteSmem& sm, int lane,
                                              int64_t* out_idx, float* out_w) {
  constexpr int kSlots = 2 * kRouteMaxRoot / 32;  // 16 values per lane at most
  const int short_len = k < root ? k : root;
  float half[kSlots / 2];
  // first codebook half
#pragma unroll
  for (int j = 0; j < kSlots / 2; ++j) {
    const int e = j * 32 + lane;
    half[j] = e < root ? scores[e] : kNegInf;
  }
  warp_topk<kSlots / 2>(half, root, short_len, sm.av, sm.ai, lane);
#pragma unroll
  for (int j = 0; j < kSlots / 2; ++j) {
    const int e = j * 32 + lane;
    half[j] = e < root ? scores[root + e] : kNegInf;
  }
  warp_topk<kSlots / 2>(half, root, short_len, sm.bv, sm.bi, lane);
  // pair (i, j) at flat position i * short + j, score a_i + b_j
  const int pairs = short_len * short_len;
  constexpr int kPairSlots = kRouteMaxShort * kRouteMaxShort / 32;
  float ps[kPairSlots];
#pragma unroll
  for (int j = 0; j < kPairSlots; ++j) {
    const int p = j * 32 + lane;
    ps[j] = p < pairs ? sm.av[p / short_len] + sm.bv[p % short_len] : kNegInf;
  }
  const int take = k < pairs ? k : pairs;
  warp_topk<kPairSlots>(ps, pairs, take, sm.pv, sm.pi, lane);
  // lane s < take holds selected pair s; addresses ascending, softmax weights
  int addr = 0x7fffffff;
  float v = kNegInf;
  if (lane < take) {
    const int p = sm.pi[lane];
    addr = sm.ai[p / short_len] * root + sm.bi[p % short_len];
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
  select_routes(P.read_proj + (tok * H + h) * key_w, P.root, P.reads, sm, lane, P.read_indices + row * P.reads,
                P.read_weights + row * P.reads);
  __syncwarp();
  select_routes(P.write_proj + (tok * H + h) * key_w, P.root, P.writes, sm, lane,
                P.write_indices + row * P.writes, P.write_weights + row * P.writes);
  if (lane == 0) {
    const float x = P.forget_proj[tok * H + h] + P.dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));  // softplus, threshold 20
    P.forget_log_gate[row] = -expf(P.a_log[h]) * sp;
    P.input_gate[row] = 1.f / (1.f + expf(-P.input_proj[tok * H + h]));
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

}  // extern "C"
