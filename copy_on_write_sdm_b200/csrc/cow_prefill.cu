// cow_prefill.cu -- sparse prefill handoff kernels.

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

}  // namespace

extern "C" {

int cow_prefill_recurrence_layers(const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                                  int64_t time, int32_t writes, int32_t reads, int32_t index_dtype,
                                  int32_t act_dtype, void* stream) {
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!pools || !prefixes || layers < 1 || layers > COW_MAX_LAYERS || time < 0 || !valid_dtype(act_dtype))
    return COW_ERR_INVALID;
  const cow_pool& p0 = pools[0];
  if (!check_step_shape(p0.width, writes, reads)) return COW_ERR_UNSUPPORTED;
  PrefillLaunch P{};
  int64_t blocks = 0;
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
    blocks += (pool.banks + kBanksPerCta - 1) / kBanksPerCta;
  }
  if (time == 0 || blocks == 0) return COW_OK;
  P.slots = p0.slots;
  P.time = time;
  P.layers = layers;
  P.width = static_cast<int32_t>(p0.width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  void (*fn)(PrefillLaunch) = nullptr;
  const int ch = width_chunks(p0.width);
  COW_SELECT_KERNEL(cow_prefill_kernel, p0.slab_dtype, ch, route_variant(writes, reads), fn);
  fn<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, 0, as_stream(stream)>>>(P);
  return launch_status();
}

int cow_prefill_recurrence(const cow_pool* pool, const cow_step* prefix, int64_t time, int32_t writes,
                           int32_t reads, int32_t index_dtype, int32_t act_dtype, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  return cow_prefill_recurrence_layers(pool, prefix, 1, time, writes, reads, index_dtype, act_dtype, stream);
}

}  // extern "C"
