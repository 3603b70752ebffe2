// cow_prefill.cu -- sparse prefill handoff kernels.

#include <cstdlib>

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// sparse prefill recurrence (rows already materialised, map complete)
// --------------------------------------------------------------------------

struct PrefillLayer {
  const float* m0;
  const int64_t* templates;
  void* slab;
  const int32_t* map;
  int32_t* status;
  cow_step step;
  int64_t banks, template_count, block_begin;
};

// Several independent pools (layers) walk their prefixes in one launch; block
// b belongs to the last layer whose block_begin <= b.
struct PrefillLaunch {
  PrefillLayer layer[COW_MAX_LAYERS];
  int64_t slots, time;
  int32_t layers, width, writes, reads, idx64, act_dt;
};

// One token's gates and value row.
template <int CH>
struct PrefillToken {
  float fl, in_g, er_g;
  float4 val[CH];
};

template <int CH>
__device__ __forceinline__ void load_prefill_token(PrefillToken<CH>& k, const cow_step& st, int64_t row, int D,
                                                   int adt, int lane) {
  k.fl = ld1_rt(st.forget_log_gate, row, adt);
  k.in_g = ld1_rt(st.input_gate, row, adt);
  k.er_g = ld1_rt(st.erase_gate, row, adt);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 4;
    k.val[c] = col < D ? ld4_rt(st.values, row * D + col, adt) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// One warp walks one bank's T tokens.  The map is fixed during the walk (all
// written slots were placed beforehand), so only the row contents carry the
// token-to-token dependence: token t+1's routes, gates and values are loaded
// a token ahead and its map lookups run while token t's rows are in flight,
// leaving one dependent round trip (the rows) per token.
template <int SDT, int CH, int WMAX, int RC>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_prefill_kernel(const __grid_constant__ PrefillLaunch P) {
  __shared__ WarpMetaT<32 * RC> s_meta[kBanksPerCta][2];  // per warp: metadata of tokens t and t+1
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int l = 0;
  while (l + 1 < P.layers && static_cast<int64_t>(blockIdx.x) >= P.layer[l + 1].block_begin) ++l;
  const PrefillLayer& Ly = P.layer[l];
  const int64_t bank = (static_cast<int64_t>(blockIdx.x) - Ly.block_begin) * kBanksPerCta + warp;
  if (bank >= Ly.banks) return;
  const int D = P.width, W = P.writes, R = P.reads;
  const int64_t N = P.slots, T = P.time;
  const int64_t tmpl = Ly.templates[bank];
  if (tmpl < 0 || tmpl >= Ly.template_count) {
    if (lane == 0) atomicOr(Ly.status, COW_ST_TEMPLATE_RANGE);
    return;
  }
  const int64_t m0_base = tmpl * N;
  const cow_step& st = Ly.step;
  const float* m0 = Ly.m0;
  void* slab = Ly.slab;
  const int32_t* mrow = Ly.map + bank * N;
  // Token t of bank b is row b*T + t of every [banks,T,...] input.
  RouteRaw<RC> raw;
  PrefillToken<CH> cur, next;
  load_route_raw<RC>(raw, st, bank * T, W, R, P.idx64, P.act_dt, lane);
  load_prefill_token<CH>(cur, st, bank * T, D, P.act_dt, lane);
  {
    unsigned first_mask;
    int route_bits;
    const bool bad = finish_routes<false, RC>(s_meta[warp][0], raw, mrow, nullptr, 0, N, W, R, lane, first_mask,
                                              route_bits);
    // Every written slot was placed before the walk, so an unmapped write
    // slot means the mark pass and the routes disagree.
    if (bad || first_mask != 0u) {
      if (lane == 0) atomicOr(Ly.status, route_bits ? route_bits : COW_ST_INDEX_RANGE);
      return;
    }
  }
  if (T > 1) {
    load_route_raw<RC>(raw, st, bank * T + 1, W, R, P.idx64, P.act_dt, lane);
    load_prefill_token<CH>(next, st, bank * T + 1, D, P.act_dt, lane);
  }
  for (int64_t t = 0; t < T; ++t) {
    const int64_t row = bank * T + t;
    auto& sm = s_meta[warp][t & 1];
    // This token's rows: write rows and the first read group in flight ...
    float4 upd[WMAX][CH];
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          upd[w][c] = col < D ? Elem<SDT>::ld4(slab, static_cast<int64_t>(phys) * D + col)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    float4 v0[ReadGroup<CH>::G][CH];
    float wt0[ReadGroup<CH>::G];
    load_read_group<SDT, CH>(v0, wt0, sm, 0, R, slab, 0, m0, m0_base, lane, D);
    // ... while the next token's map lookups resolve, and the token after
    // that has its routes, gates and value row requested.
    int next_bits = 0;
    bool next_bad = false;
    if (t + 1 < T) {
      unsigned first_mask;
      next_bad = finish_routes<false, RC>(s_meta[warp][(t + 1) & 1], raw, mrow, nullptr, 0, N, W, R, lane,
                                          first_mask, next_bits);
      next_bad = next_bad || first_mask != 0u;
    }
    PrefillToken<CH> after = next;
    if (t + 2 < T) {
      load_route_raw<RC>(raw, st, row + 2, W, R, P.idx64, P.act_dt, lane);
      load_prefill_token<CH>(after, st, row + 2, D, P.act_dt, lane);
    }
    gated_delta<SDT, CH, WMAX>(upd, sm, W, expf(cur.fl), cur.in_g, cur.er_g, cur.val, lane, D);
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          if (col < D) Elem<SDT>::st4(slab, static_cast<int64_t>(phys) * D + col, upd[w][c]);
        }
      }
    }
    float4 acc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    accumulate_group<CH>(acc, v0, wt0);
    read_remaining<SDT, CH>(acc, sm, R, slab, 0, m0, m0_base, lane, D);
    add_forwarded<CH, WMAX>(acc, upd, sm, W);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) st4_rt(st.output, row * D + col, acc[c], P.act_dt);
    }
    __syncwarp();
    if (next_bad) {
      if (lane == 0) atomicOr(Ly.status, next_bits ? next_bits : COW_ST_INDEX_RANGE);
      return;
    }
    cur = next;
    next = after;
  }
}

// --------------------------------------------------------------------------
// resolved-route prefill: a parallel route pass, then the recurrence
// --------------------------------------------------------------------------
//
// The map is fixed for the whole walk, so every token's route resolution
// (index checks, map lookups, repeated-write check, read-after-write folding)
// is independent of the row contents.  cow_prefill_meta_kernel resolves the
// tokens of a time chunk for all banks at once, one warp per (bank, token),
// into compact records; cow_prefill_walk_kernel then walks the chunk with one
// warp per bank, fetching each record a token ahead by cp.async, so a token's
// serial chain is its rows and arithmetic only.  Floating-point operations and
// their order are those of cow_prefill_kernel.
//
// Record of one (bank, token), 32-bit words: [0] error bits (0 = usable),
// [1..3] unused, then wphys[W], ww[W], fwt[W], ridx[R], rsrc[R], rw[R];
// padded to a multiple of 4 words.
inline int prefill_record_words(int writes, int reads) { return (4 + 3 * writes + 3 * reads + 3) & ~3; }

struct RecordView {
  const int* wphys;
  const float* ww;
  const float* fwt;
  const int* ridx;
  const int* rsrc;
  const float* rw;
  __device__ RecordView(const int* base, int W, int R)
      : wphys(base + 4),
        ww(reinterpret_cast<const float*>(base + 4 + W)),
        fwt(reinterpret_cast<const float*>(base + 4 + 2 * W)),
        ridx(base + 4 + 3 * W),
        rsrc(base + 4 + 3 * W + R),
        rw(reinterpret_cast<const float*>(base + 4 + 3 * W + 2 * R)) {}
};

struct PrefillChunk {
  int32_t* records;  // [total banks, tc, rec_words]
  int64_t t0, tc;
  int32_t rec_words;
  int64_t bank_begin[COW_MAX_LAYERS];  // first flattened bank of each pool
};

__device__ __forceinline__ int chunk_layer(const PrefillLaunch& P, const PrefillChunk& C, int64_t gbank) {
  int l = 0;
  while (l + 1 < P.layers && gbank >= C.bank_begin[l + 1]) ++l;
  return l;
}

template <int WMAX, int RC>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_prefill_meta_kernel(const __grid_constant__ PrefillLaunch P, const __grid_constant__ PrefillChunk C,
                            int64_t total_banks) {
  __shared__ WarpMetaT<32 * RC> s_meta[kBanksPerCta];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * kBanksPerCta + warp;
  if (g >= total_banks * C.tc) return;
  const int64_t gbank = g / C.tc, tt = g - gbank * C.tc;
  const int l = chunk_layer(P, C, gbank);
  const PrefillLayer& Ly = P.layer[l];
  const int64_t bank = gbank - C.bank_begin[l];
  const int W = P.writes, R = P.reads;
  const int64_t N = P.slots, T = P.time;
  auto& sm = s_meta[warp];
  unsigned first_mask;
  int route_bits;
  const bool bad = load_routes<false, RC>(sm, Ly.step, Ly.map, bank * T + C.t0 + tt, bank, N, W, R, P.idx64,
                                          P.act_dt, lane, first_mask, route_bits);
  int32_t* rec = C.records + g * C.rec_words;
  // Every written slot was placed before the walk, so an unmapped write slot
  // means the mark pass and the routes disagree.
  if (lane == 0) rec[0] = (bad || first_mask != 0u) ? (route_bits ? route_bits : COW_ST_INDEX_RANGE) : 0;
  if (lane < W) {
    rec[4 + lane] = sm.wphys[lane];
    reinterpret_cast<float*>(rec)[4 + W + lane] = sm.ww[lane];
    reinterpret_cast<float*>(rec)[4 + 2 * W + lane] = sm.fwt[lane];
  }
  for (int r = lane; r < R; r += 32) {
    rec[4 + 3 * W + r] = sm.ridx[r];
    rec[4 + 3 * W + R + r] = sm.rsrc[r];
    reinterpret_cast<float*>(rec)[4 + 3 * W + 2 * R + r] = sm.rw[r];
  }
}

__device__ __forceinline__ void fetch_record(int32_t* dst, const int32_t* src, int rec_words, int lane) {
  for (int i = lane; i < (rec_words >> 2); i += 32) cp_async16(dst + 4 * i, src + 4 * i);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <int SDT, int CH, int WMAX, int RC>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_prefill_walk_kernel(const __grid_constant__ PrefillLaunch P, const __grid_constant__ PrefillChunk C) {
  extern __shared__ __align__(16) int32_t s_rec[];  // per warp: records of tokens t and t+1
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int l = 0;
  while (l + 1 < P.layers && static_cast<int64_t>(blockIdx.x) >= P.layer[l + 1].block_begin) ++l;
  const PrefillLayer& Ly = P.layer[l];
  const int64_t bank = (static_cast<int64_t>(blockIdx.x) - Ly.block_begin) * kBanksPerCta + warp;
  if (bank >= Ly.banks) return;
  const int D = P.width, W = P.writes, R = P.reads;
  const int64_t N = P.slots, T = P.time;
  const int64_t tmpl = Ly.templates[bank];
  if (tmpl < 0 || tmpl >= Ly.template_count) {
    if (lane == 0) atomicOr(Ly.status, COW_ST_TEMPLATE_RANGE);
    return;
  }
  const int64_t m0_base = tmpl * N;
  const cow_step& st = Ly.step;
  const float* m0 = Ly.m0;
  void* slab = Ly.slab;
  const int RW = C.rec_words;
  int32_t* buf[2] = {s_rec + static_cast<int64_t>(warp) * 2 * RW, s_rec + (static_cast<int64_t>(warp) * 2 + 1) * RW};
  const int32_t* recs = C.records + (C.bank_begin[l] + bank) * C.tc * RW;
  PrefillToken<CH> cur, next;
  const int64_t t_end = C.t0 + C.tc;
  fetch_record(buf[0], recs, RW, lane);
  load_prefill_token<CH>(cur, st, bank * T + C.t0, D, P.act_dt, lane);
  if (C.t0 + 1 < t_end) load_prefill_token<CH>(next, st, bank * T + C.t0 + 1, D, P.act_dt, lane);
  for (int64_t t = C.t0; t < t_end; ++t) {
    const int64_t row = bank * T + t;
    const int cb = static_cast<int>((t - C.t0) & 1);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncwarp();
    const int32_t* rec = buf[cb];
    if (rec[0] != 0) {
      if (lane == 0) atomicOr(Ly.status, rec[0]);
      return;
    }
    const RecordView sm(rec, W, R);
    // This token's rows: write rows and the first read group in flight ...
    float4 upd[WMAX][CH];
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          upd[w][c] = col < D ? Elem<SDT>::ld4(slab, static_cast<int64_t>(phys) * D + col)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    float4 v0[ReadGroup<CH>::G][CH];
    float wt0[ReadGroup<CH>::G];
    load_read_group<SDT, CH>(v0, wt0, sm, 0, R, slab, 0, m0, m0_base, lane, D);
    // ... while the next token's record, gates and value row are requested.
    if (t + 1 < t_end) fetch_record(buf[cb ^ 1], recs + (t + 1 - C.t0) * RW, RW, lane);
    PrefillToken<CH> after = next;
    if (t + 2 < t_end) load_prefill_token<CH>(after, st, row + 2, D, P.act_dt, lane);
    gated_delta<SDT, CH, WMAX>(upd, sm, W, expf(cur.fl), cur.in_g, cur.er_g, cur.val, lane, D);
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          if (col < D) Elem<SDT>::st4(slab, static_cast<int64_t>(phys) * D + col, upd[w][c]);
        }
      }
    }
    float4 acc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    accumulate_group<CH>(acc, v0, wt0);
    read_remaining<SDT, CH>(acc, sm, R, slab, 0, m0, m0_base, lane, D);
    add_forwarded<CH, WMAX>(acc, upd, sm, W);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) st4_rt(st.output, row * D + col, acc[c], P.act_dt);
    }
    __syncwarp();  // every lane has read this token's record before it is refilled
    cur = next;
    next = after;
  }
}



// Few banks (a serving cohort): each bank's walk is one warp's serial chain of
// about five hundred instructions per token, and a handful of warps cannot
// fill the GPU.  This variant gives each bank a block of kWalkSplit warps (f32
// rows, width <= 128, W <= 4, R <= 32): every warp loads the W write rows and
// computes the same gated-delta update (identical rows in every warp), warp k
// stores write row k and reads rows r == k (mod kWalkSplit), and the partial
// readouts meet in shared memory, where warp 0 sums them in warp order.  Rows
// and maps are bit-identical to the one-warp walk; readings differ only by
// the order of that sum.  Two block barriers per token: after every warp
// has loaded the write rows (so they may be overwritten), and at the top of
// the next token (the stores are visible, the next record has landed and the
// partials are complete; they alternate between two buffers by token parity,
// so warp 0 reads one token's partials while the others write the next).
constexpr int kWalkSplit = 4;
constexpr int64_t kWalkSplitMaxBanks = 2048;

__global__ void __launch_bounds__(kWalkSplit * 32)
    cow_prefill_split_walk_kernel(const __grid_constant__ PrefillLaunch P, const __grid_constant__ PrefillChunk C) {
  extern __shared__ __align__(16) int32_t s_rec[];  // records of tokens t and t+1
  __shared__ __align__(16) float4 s_part[2][kWalkSplit][32];  // by token parity
  const int k = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t gbank = blockIdx.x;
  const int l = chunk_layer(P, C, gbank);
  const PrefillLayer& Ly = P.layer[l];
  const int64_t bank = gbank - C.bank_begin[l];
  const int D = P.width, W = P.writes, R = P.reads;
  const int64_t N = P.slots, T = P.time;
  const int64_t tmpl = Ly.templates[bank];
  if (tmpl < 0 || tmpl >= Ly.template_count) {
    if (k == 0 && lane == 0) atomicOr(Ly.status, COW_ST_TEMPLATE_RANGE);
    return;
  }
  const int64_t m0_base = tmpl * N;
  const cow_step& st = Ly.step;
  const float* m0 = Ly.m0;
  float* slab = static_cast<float*>(Ly.slab);
  const int RW = C.rec_words;
  const int32_t* recs = C.records + gbank * C.tc * RW;
  const bool col_ok = lane * 4 < D;
  const int64_t t_end = C.t0 + C.tc;
  PrefillToken<1> cur, next;
  load_prefill_token<1>(cur, st, bank * T + C.t0, D, P.act_dt, lane);
  if (C.t0 + 1 < t_end) load_prefill_token<1>(next, st, bank * T + C.t0 + 1, D, P.act_dt, lane);
  if (k == 0) {
    fetch_record(s_rec, recs, RW, lane);
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  }
  for (int64_t t = C.t0; t <= t_end; ++t) {
    __syncthreads();
    if (k == 0 && t > C.t0) {
      // The previous token's readout: partials summed in warp order.
      const int pb = static_cast<int>((t - 1 - C.t0) & 1);
      float4 sum = s_part[pb][0][lane];
#pragma unroll
      for (int j = 1; j < kWalkSplit; ++j) {
        const float4 x = s_part[pb][j][lane];
        sum = make_float4(sum.x + x.x, sum.y + x.y, sum.z + x.z, sum.w + x.w);
      }
      if (col_ok) st4_rt(st.output, (bank * T + t - 1) * D + lane * 4, sum, P.act_dt);
    }
    if (t == t_end) break;
    const int32_t* rec = s_rec + ((t - C.t0) & 1) * RW;
    if (rec[0] != 0) {
      if (k == 0 && lane == 0) atomicOr(Ly.status, rec[0]);
      return;
    }
    const RecordView sm(rec, W, R);
    float4 upd[4][1];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W) upd[w][0] = col_ok ? Elem<COW_F32>::ld4(slab, static_cast<int64_t>(sm.wphys[w]) * D + lane * 4)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 v[32 / kWalkSplit];
    float wt[32 / kWalkSplit];
#pragma unroll
    for (int j = 0; j < 32 / kWalkSplit; ++j) {
      const int r = k + kWalkSplit * j;
      const int src = r < R ? sm.rsrc[r] : -2;
      wt[j] = src >= -1 ? sm.rw[r] : 0.f;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col_ok) {
        if (src >= 0) x = Elem<COW_F32>::ld4(slab, static_cast<int64_t>(src) * D + lane * 4);
        else if (src == -1) x = ld4_m0(m0, (m0_base + sm.ridx[r]) * D + lane * 4);
      }
      v[j] = x;
    }
    if (k == 0 && t + 1 < t_end) fetch_record(s_rec + ((t + 1 - C.t0) & 1) * RW, recs + (t + 1 - C.t0) * RW, RW, lane);
    PrefillToken<1> after = next;
    if (t + 2 < t_end) load_prefill_token<1>(after, st, bank * T + t + 2, D, P.act_dt, lane);
    gated_delta<COW_F32, 1, 4>(upd, sm, W, expf(cur.fl), cur.in_g, cur.er_g, cur.val, lane, D);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 32 / kWalkSplit; ++j) acc = f4_axpy(wt[j], v[j], acc);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W && w == k) acc = f4_axpy(sm.fwt[w], upd[w][0], acc);
    }
    s_part[(t - C.t0) & 1][k][lane] = acc;
    // Every warp has loaded this token's write rows (and read rows) before
    // any of them is overwritten.
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W && w == k && col_ok) Elem<COW_F32>::st4(slab, static_cast<int64_t>(sm.wphys[w]) * D + lane * 4, upd[w][0]);
    }
    if (k == 0) asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    cur = next;
    next = after;
  }
}

// Fills the launch descriptor shared by both prefill walks and the number of
// 4-warp blocks (0 = nothing to do); returns a COW_* status.
int prefill_setup(PrefillLaunch& P, const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                  int64_t time, int32_t writes, int32_t reads, int32_t index_dtype, int32_t act_dtype,
                  int64_t* bank_begin, int64_t& blocks) {
  blocks = 0;
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!pools || !prefixes || layers < 1 || layers > COW_MAX_LAYERS || time < 0 || !valid_dtype(act_dtype))
    return COW_ERR_INVALID;
  const cow_pool& p0 = pools[0];
  if (!check_step_shape(p0.width, writes, reads)) return COW_ERR_UNSUPPORTED;
  int64_t banks = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& pool = pools[l];
    if (pool.width != p0.width || pool.slots != p0.slots || pool.slab_dtype != p0.slab_dtype ||
        !valid_dtype(pool.slab_dtype) || pool.banks < 0)
      return COW_ERR_INVALID;
    if (!check_step_ptrs(prefixes[l], act_dtype) || !pool.slab || !pool.map || !pool.m0 || !pool.templates ||
        !row_aligned(pool.slab, pool.slab_dtype) || !aligned16(pool.m0))
      return COW_ERR_INVALID;
    PrefillLayer& L = P.layer[l];
    L.m0 = pool.m0;
    L.templates = pool.templates;
    L.slab = pool.slab;
    L.map = pool.map;
    L.status = pool.status;
    L.step = prefixes[l];
    L.banks = pool.banks;
    L.template_count = pool.template_count;
    L.block_begin = blocks;
    if (bank_begin) bank_begin[l] = banks;
    blocks += (pool.banks + kBanksPerCta - 1) / kBanksPerCta;
    banks += pool.banks;
  }
  P.slots = p0.slots;
  P.time = time;
  P.layers = layers;
  P.width = static_cast<int32_t>(p0.width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  if (time == 0) blocks = 0;
  return COW_OK;
}

// COW_PREFILL_SPLIT=0 in the environment keeps cohorts on the one-warp walk
// (for comparisons).
bool split_walk_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("COW_PREFILL_SPLIT");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Records of one chunk are capped at this many bytes; longer prefixes are
// walked in several chunks.
constexpr int64_t kPrefillRecordCap = int64_t(256) << 20;

int64_t total_banks_of(const cow_pool* pools, int32_t layers) {
  int64_t b = 0;
  for (int l = 0; l < layers; ++l) b += pools[l].banks > 0 ? pools[l].banks : 0;
  return b;
}

}  // namespace

extern "C" {

int cow_prefill_recurrence_layers(const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                                  int64_t time, int32_t writes, int32_t reads, int32_t index_dtype,
                                  int32_t act_dtype, void* stream) {
  PrefillLaunch P{};
  int64_t blocks = 0;
  const int status = prefill_setup(P, pools, prefixes, layers, time, writes, reads, index_dtype, act_dtype, nullptr,
                                   blocks);
  if (status != COW_OK || blocks == 0) return status;
  void (*fn)(PrefillLaunch) = nullptr;
  const int ch = width_chunks(pools[0].width);
  COW_SELECT_KERNEL(cow_prefill_kernel, pools[0].slab_dtype, ch, route_variant(writes, reads), fn);
  fn<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, 0, as_stream(stream)>>>(P);
  return launch_status();
}

int64_t cow_prefill_workspace_bytes(const cow_pool* pools, int32_t layers, int64_t time, int32_t writes,
                                    int32_t reads) {
  if (!pools || layers < 1 || layers > COW_MAX_LAYERS || time < 0 || writes < 1 || writes > COW_MAX_WRITES ||
      reads < 1 || reads > COW_MAX_READS)
    return -1;
  const int64_t banks = total_banks_of(pools, layers);
  const int64_t per_token = banks * prefill_record_words(writes, reads) * 4;
  if (per_token == 0 || time == 0 || banks > kWalkSplitMaxBanks) return 16;
  int64_t tc = kPrefillRecordCap / per_token;
  if (tc < 1) tc = 1;
  if (tc > time) tc = time;
  return tc * per_token;
}

int cow_prefill_recurrence_layers_ws(const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                                     int64_t time, int32_t writes, int32_t reads, int32_t index_dtype,
                                     int32_t act_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  PrefillLaunch P{};
  PrefillChunk C{};
  int64_t blocks = 0;
  const int status = prefill_setup(P, pools, prefixes, layers, time, writes, reads, index_dtype, act_dtype,
                                   C.bank_begin, blocks);
  if (status != COW_OK || blocks == 0) return status;
  const int64_t banks = total_banks_of(pools, layers);
  if (banks > kWalkSplitMaxBanks) {
    // Thousands of banks fill the GPU with one-warp walks and are bound by
    // row bandwidth: the walk that resolves each token's routes a token ahead
    // costs no route records (about 10 % less time there).
    void (*fn)(PrefillLaunch) = nullptr;
    COW_SELECT_KERNEL(cow_prefill_kernel, pools[0].slab_dtype, width_chunks(pools[0].width),
                      route_variant(writes, reads), fn);
    fn<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, 0, as_stream(stream)>>>(P);
    return launch_status();
  }
  C.rec_words = prefill_record_words(writes, reads);
  const int64_t per_token = banks * C.rec_words * 4;
  if (!workspace || !aligned16(workspace) || workspace_bytes < per_token) return COW_ERR_INVALID;
  int64_t tc = workspace_bytes / per_token;
  if (tc > kPrefillRecordCap / per_token) tc = kPrefillRecordCap / per_token;
  if (tc < 1) tc = 1;
  if (tc > time) tc = time;
  C.records = static_cast<int32_t*>(workspace);
  const int rv = route_variant(writes, reads);
  void (*meta)(PrefillLaunch, PrefillChunk, int64_t) =
      rv == 0 ? cow_prefill_meta_kernel<4, 1> : (rv == 1 ? cow_prefill_meta_kernel<8, 1> : cow_prefill_meta_kernel<32, 8>);
  void (*walk)(PrefillLaunch, PrefillChunk) = nullptr;
  COW_SELECT_KERNEL(cow_prefill_walk_kernel, pools[0].slab_dtype, width_chunks(pools[0].width), rv, walk);
  const bool split = pools[0].slab_dtype == COW_F32 && pools[0].width <= 128 && rv == 0 && reads <= 32 &&
                     split_walk_enabled();
  const size_t smem = static_cast<size_t>(split ? 1 : kBanksPerCta) * 2 * C.rec_words * 4;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(split ? reinterpret_cast<const void*>(cow_prefill_split_walk_kernel)
                                 : reinterpret_cast<const void*>(walk), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return launch_status();
  cudaStream_t s = as_stream(stream);
  for (int64_t t0 = 0; t0 < time; t0 += tc) {
    C.t0 = t0;
    C.tc = time - t0 < tc ? time - t0 : tc;
    const int64_t warps = banks * C.tc;
    meta<<<static_cast<unsigned>((warps + kBanksPerCta - 1) / kBanksPerCta), kBanksPerCta * 32, 0, s>>>(P, C, banks);
    if (split)
      cow_prefill_split_walk_kernel<<<static_cast<unsigned>(banks), kWalkSplit * 32, smem, s>>>(P, C);
    else
      walk<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, smem, s>>>(P, C);
    const int st = launch_status();
    if (st != COW_OK) return st;
  }
  return COW_OK;
}

int cow_prefill_recurrence(const cow_pool* pool, const cow_step* prefix, int64_t time, int32_t writes,
                           int32_t reads, int32_t index_dtype, int32_t act_dtype, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  return cow_prefill_recurrence_layers(pool, prefix, 1, time, writes, reads, index_dtype, act_dtype, stream);
}

}  // extern "C"
