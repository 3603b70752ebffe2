// cow_prefill.cu -- sparse prefill handoff kernels.

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// sparse prefill recurrence (rows already materialised, map complete)
// --------------------------------------------------------------------------

struct PrefillLaunch {
  const float* m0;
  const int64_t* templates;
  void* slab;
  const int32_t* map;
  int32_t* status;
  cow_step step;
  int64_t banks, slots, time, template_count;
  int32_t width, writes, reads, idx64, act_dt, _pad;
};

template <int SDT, int CH, int WMAX, int RC>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_prefill_kernel(const __grid_constant__ PrefillLaunch P) {
  __shared__ WarpMetaT<32 * RC> s_meta[kBanksPerCta];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t bank = static_cast<int64_t>(blockIdx.x) * kBanksPerCta + warp;
  if (bank >= P.banks) return;
  const int D = P.width, W = P.writes, R = P.reads;
  const int64_t N = P.slots, T = P.time;
  auto& sm = s_meta[warp];
  const int64_t tmpl = P.templates[bank];
  if (tmpl < 0 || tmpl >= P.template_count) {
    if (lane == 0) atomicOr(P.status, COW_ST_TEMPLATE_RANGE);
    return;
  }
  const int64_t m0_base = tmpl * N;
  const cow_step& st = P.step;
  for (int64_t t = 0; t < T; ++t) {
    // Token t of bank b is row b*T + t of every [banks,T,...] input.  The map
    // is fixed during the walk (all written slots were placed beforehand), so
    // only the row contents carry the token-to-token dependence.
    const int64_t row = bank * T + t;
    const float fl = ld1_rt(st.forget_log_gate, row, P.act_dt);
    const float in_g = ld1_rt(st.input_gate, row, P.act_dt);
    const float er_g = ld1_rt(st.erase_gate, row, P.act_dt);
    float4 val[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      val[c] = col < D ? ld4_rt(st.values, row * D + col, P.act_dt) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    unsigned first_mask;
    int route_bits;
    const bool bad = load_routes<false, RC>(sm, st, P.map, row, bank, N, W, R, P.idx64, P.act_dt, lane,
                                            first_mask, route_bits);
    // Every written slot was placed before the walk, so an unmapped write
    // slot means the mark pass and the routes disagree.
    if (bad || first_mask != 0u) {
      if (lane == 0) atomicOr(P.status, route_bits ? route_bits : COW_ST_INDEX_RANGE);
      return;
    }
    const float alpha = expf(fl);
    float4 upd[WMAX][CH];
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          upd[w][c] = col < D ? Elem<SDT>::ld4(P.slab, static_cast<int64_t>(phys) * D + col)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    float4 v0[ReadGroup<CH>::G][CH];
    float wt0[ReadGroup<CH>::G];
    load_read_group<SDT, CH>(v0, wt0, sm, 0, R, P.slab, 0, P.m0, m0_base, lane, D);
    gated_delta<SDT, CH, WMAX>(upd, sm, W, alpha, in_g, er_g, val, lane, D);
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          if (col < D) Elem<SDT>::st4(P.slab, static_cast<int64_t>(phys) * D + col, upd[w][c]);
        }
      }
    }
    float4 acc[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    accumulate_group<CH>(acc, v0, wt0);
    read_remaining<SDT, CH>(acc, sm, R, P.slab, 0, P.m0, m0_base, lane, D);
    add_forwarded<CH, WMAX>(acc, upd, sm, W);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) st4_rt(st.output, row * D + col, acc[c], P.act_dt);
    }
    __syncwarp();
  }
}

}  // namespace

extern "C" {

int cow_prefill_recurrence(const cow_pool* pool, const cow_step* prefix, int64_t time, int32_t writes,
                           int32_t reads, int32_t index_dtype, int32_t act_dtype, void* stream) {
  if (!pool || !prefix || time < 0 || !valid_dtype(act_dtype) || !valid_dtype(pool->slab_dtype)) return COW_ERR_INVALID;
  if (!check_step_shape(pool->width, writes, reads)) return COW_ERR_UNSUPPORTED;
  if (!check_step_ptrs(*prefix, act_dtype) || !pool->slab || !pool->map || !pool->m0 || !pool->templates ||
      !row_aligned(pool->slab, pool->slab_dtype) || !aligned16(pool->m0))
    return COW_ERR_INVALID;
  if (time == 0 || pool->banks == 0) return COW_OK;
  PrefillLaunch P{};
  P.m0 = pool->m0;
  P.templates = pool->templates;
  P.slab = pool->slab;
  P.map = pool->map;
  P.status = pool->status;
  P.step = *prefix;
  P.banks = pool->banks;
  P.slots = pool->slots;
  P.time = time;
  P.template_count = pool->template_count;
  P.width = static_cast<int32_t>(pool->width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  void (*fn)(PrefillLaunch) = nullptr;
  const int ch = width_chunks(pool->width);
  COW_SELECT_KERNEL(cow_prefill_kernel, pool->slab_dtype, ch, route_variant(writes, reads), fn);
  const int64_t blocks = (pool->banks + kBanksPerCta - 1) / kBanksPerCta;
  fn<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, 0, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
