// cow_decode.cu -- fused packed decode step (the hot path).
//
// Hot path: one fused decode launch covers every bank of up to COW_MAX_LAYERS
// independent SDM pools.  One warp owns one bank; lane l owns columns
// [4l, 4l+4) (+128 per chunk) of every row, so each row moves as 32 x 16-byte
// coalesced accesses and the whole gated-delta update and weighted read are
// lane-local (no cross-lane reductions, no block barriers between the write
// and the read: the lane that stores a column is the lane that reads it back).
//
// Determinism: the reference's CPU path pops free rows in the flattened
// [banks, W] order (allocator.py:1467-1481).  The kernel reproduces that order
// exactly with a single-pass decoupled look-back scan over tiles of banks,
// ordered by a dynamic ticket so a tile only ever waits on tiles that already
// started.  First touches depend only on the pre-step map, so every row load
// and all arithmetic run before the scan resolves; only the placement of the
// first-touch rows waits for it.  Every wait is bounded and reports
// COW_ST_WAIT_TIMEOUT instead of hanging.


#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// fused packed decode step
// --------------------------------------------------------------------------

template <int SDT, int CH, int WMAX>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_decode_kernel(const __grid_constant__ DecodeLaunch P) {
  __shared__ WarpMeta s_meta[kBanksPerCta];
  __shared__ int s_cnt[kBanksPerCta];
  __shared__ uint32_t s_ticket, s_epoch;
  __shared__ int s_layer, s_old_free, s_tile_excl;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = P.width, W = P.writes, R = P.reads;

  if (threadIdx.x == 0) {
    const uint32_t t = atomicAdd(&P.header[0], 1u);
    int l = 0;
    while (l + 1 < P.layers && static_cast<int>(t) >= P.layer[l].tile_begin + P.layer[l].tiles) ++l;
    s_ticket = t;
    s_layer = l;
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&P.header[2]);
    s_old_free = *reinterpret_cast<volatile int32_t*>(P.layer[l].free_count);
  }
  __syncthreads();
  const DecodeLayer& L = P.layer[s_layer];
  const int tile = static_cast<int>(s_ticket) - L.tile_begin;
  const int64_t bank = static_cast<int64_t>(tile) * kBanksPerCta + warp;
  const bool live = bank < L.banks;
  const int64_t N = L.slots;
  WarpMeta& sm = s_meta[warp];

  unsigned first_mask = 0;
  bool bad = false;
  int route_bits = 0;
  int64_t tmpl = 0;
  if (live) {
    const bool bad_route = load_routes<false>(sm, L.step, L.map, bank, bank, N, W, R, P.idx64,
                                              P.act_dt, lane, first_mask, route_bits);
    tmpl = L.templates[bank];
    const bool bad_tmpl = tmpl < 0 || tmpl >= L.template_count;
    bad = bad_route || bad_tmpl;
    if (bad && lane == 0) {
      atomicOr(L.status, route_bits | (bad_tmpl ? COW_ST_TEMPLATE_RANGE : 0));
    }
    if (bad) first_mask = 0;
  }
  if (lane == 0) s_cnt[warp] = __popc(first_mask);
  __syncthreads();

  // Publish this tile's first-touch aggregate as early as possible.
  int tile_agg = 0;
#pragma unroll
  for (int w = 0; w < kBanksPerCta; ++w) tile_agg += s_cnt[w];
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t st = tile == 0 ? kFlagInclusive : kFlagAggregate;
    *reinterpret_cast<volatile uint64_t*>(&P.flags[s_ticket]) =
        pack_flag(s_epoch, st, static_cast<uint32_t>(tile_agg));
  }

  // Row traffic and arithmetic: independent of where first touches land.
  float4 upd[WMAX][CH];
  if (live && !bad) {
    const float alpha = expf(ld1_rt(L.step.forget_log_gate, bank, P.act_dt));
    const float in_g = ld1_rt(L.step.input_gate, bank, P.act_dt);
    const float er_g = ld1_rt(L.step.erase_gate, bank, P.act_dt);
    const int64_t m0_base = tmpl * N;
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
        const int slot = sm.widx[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (col < D) {
            x = phys < 0 ? ld4_m0(L.m0, (m0_base + slot) * D + col)
                         : Elem<SDT>::ld4(L.slab, static_cast<int64_t>(phys) * D + col);
          }
          upd[w][c] = x;
        }
      }
    }
    float4 val[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      val[c] = col < D ? ld4_rt(L.step.values, bank * D + col, P.act_dt) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    gated_delta<SDT, CH, WMAX>(upd, sm, W, alpha, in_g, er_g, val, lane, D);
    // Rows that already had a private copy are written back in place now.
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
        if (phys >= 0) {
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int col = (c * 32 + lane) * 4;
            if (col < D) Elem<SDT>::st4(L.slab, static_cast<int64_t>(phys) * D + col, upd[w][c]);
          }
        }
      }
    }
    float4 acc[CH];
    sparse_read<SDT, CH, WMAX>(acc, upd, sm, W, R, L.slab, 0, L.m0, m0_base, lane, D);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) st4_rt(L.step.output, bank * D + col, acc[c], P.act_dt);
    }
  } else if (live) {
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      if (col < D) st4_rt(L.step.output, bank * D + col, make_float4(0.f, 0.f, 0.f, 0.f), P.act_dt);
    }
  }

  // Decoupled look-back over the preceding tiles of this pool (warp 0).
  if (warp == 0) {
    int excl = 0;
    if (tile > 0) {
      int64_t pred = static_cast<int64_t>(s_ticket) - 1;
      const int64_t first_ticket = L.tile_begin;
      bool timed_out = false;
      while (true) {
        const int64_t idx = pred - lane;
        uint32_t st = kFlagInclusive, v = 0;
        if (idx >= first_ticket) {
          int spins = 0;
          while (true) {
            const uint64_t f = ld_volatile_u64(&P.flags[idx]);
            st = (static_cast<uint32_t>(f >> 32) == s_epoch) ? static_cast<uint32_t>((f >> 30) & 3u) : 0u;
            v = static_cast<uint32_t>(f & 0x3fffffffu);
            if (st != 0u) break;
            if (++spins > kSpinLimit) {
              timed_out = true;
              st = kFlagInclusive;
              v = 0;
              break;
            }
            __nanosleep(spins < 64 ? 32 : 256);
          }
        }
        __threadfence();
        const unsigned incl = __ballot_sync(kFull, st == kFlagInclusive);
        const int stop = incl ? __ffs(incl) - 1 : 31;
        excl += warp_sum(lane <= stop ? static_cast<int>(v) : 0);
        if (incl) break;
        pred -= 32;
      }
      if (__any_sync(kFull, timed_out) && lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
    }
    if (lane == 0) {
      s_tile_excl = excl;
      const int inclusive = excl + tile_agg;
      if (tile > 0) {
        __threadfence();
        *reinterpret_cast<volatile uint64_t*>(&P.flags[s_ticket]) =
            pack_flag(s_epoch, kFlagInclusive, static_cast<uint32_t>(inclusive));
      }
      if (tile == L.tiles - 1) {
        const int remaining = s_old_free - inclusive;
        *L.free_count = remaining > 0 ? remaining : 0;
      }
    }
  }
  __syncthreads();

  // Place the first touches: pop free_rows[old_free - 1 - rank].
  if (live && !bad) {
    int bank_excl = 0;
    for (int w = 0; w < warp; ++w) bank_excl += s_cnt[w];
    int newp = -1;
    const bool first = lane < W && ((first_mask >> lane) & 1u);
    if (first) {
      const int rank = s_tile_excl + bank_excl + __popc(first_mask & ((1u << lane) - 1u));
      const int pos = s_old_free - 1 - rank;
      if (pos >= 0) {
        newp = L.free_rows[pos];
        L.map[bank * N + sm.widx[lane]] = newp;
      } else {
        atomicOr(L.status, COW_ST_SLAB_EXHAUSTED);
      }
    }
    if (L.step.first_touch != nullptr && lane < W) L.step.first_touch[bank * W + lane] = (first && newp >= 0) ? 1 : 0;
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W && ((first_mask >> w) & 1u)) {
        const int p = __shfl_sync(kFull, newp, w);
        if (p >= 0) {
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int col = (c * 32 + lane) * 4;
            if (col < D) Elem<SDT>::st4(L.slab, static_cast<int64_t>(p) * D + col, upd[w][c]);
          }
        }
      }
    }
  } else if (live && L.step.first_touch != nullptr && lane < W) {
    L.step.first_touch[bank * W + lane] = 0;
  }

  // Recycle the scan header once every tile of this launch is finished.
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t d = atomicAdd(&P.header[1], 1u);
    if (d == static_cast<uint32_t>(P.total_tiles) - 1u) {
      P.header[0] = 0u;
      P.header[1] = 0u;
      __threadfence();
      P.header[2] = s_epoch + 1u;
    }
  }
}

}  // namespace

namespace cowrt {
thread_local int last_cuda_error = 0;
}  // namespace cowrt

extern "C" {

int cow_abi_version(void) { return COW_ABI_VERSION; }

const char* cow_last_error(void) {
  return cudaGetErrorString(static_cast<cudaError_t>(cowrt::last_cuda_error));
}

int64_t cow_decode_scratch_bytes(int64_t total_banks, int32_t layers) {
  const int64_t tiles = (total_banks + kBanksPerCta - 1) / kBanksPerCta + (layers > 0 ? layers : 1);
  return 16 + 8 * tiles;
}

int cow_decode_step(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes, int32_t reads,
                    int32_t index_dtype, int32_t act_dtype, void* scan_scratch, int64_t scratch_bytes,
                    void* stream) {
  if (!pools || !steps || layers < 1 || layers > COW_MAX_LAYERS || !scan_scratch) return COW_ERR_INVALID;
  if (!valid_dtype(act_dtype) || (index_dtype != COW_I32 && index_dtype != COW_I64)) return COW_ERR_INVALID;
  const int64_t width = pools[0].width;
  const int sdt = pools[0].slab_dtype;
  if (!valid_dtype(sdt)) return COW_ERR_INVALID;
  if (!check_step_shape(width, writes, reads)) return COW_ERR_UNSUPPORTED;
  if (!aligned16(scan_scratch)) return COW_ERR_INVALID;
  DecodeLaunch P{};
  int32_t tiles = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& p = pools[l];
    if (p.width != width || p.slab_dtype != sdt || p.banks < 0 || p.slots < 1 || !p.m0 || !p.templates ||
        !p.slab || !p.map || !p.free_rows || !p.free_count || !p.status || !aligned16(p.m0) ||
        !row_aligned(p.slab, sdt) || !check_step_ptrs(steps[l], act_dtype))
      return COW_ERR_INVALID;
    if (p.banks * writes >= (int64_t(1) << 30) || p.capacity >= (int64_t(1) << 31)) return COW_ERR_UNSUPPORTED;
    DecodeLayer& L = P.layer[l];
    L.m0 = p.m0;
    L.templates = p.templates;
    L.slab = p.slab;
    L.map = p.map;
    L.free_rows = p.free_rows;
    L.free_count = p.free_count;
    L.status = p.status;
    L.step = steps[l];
    L.banks = p.banks;
    L.slots = p.slots;
    L.capacity = p.capacity;
    L.template_count = p.template_count;
    L.tile_begin = tiles;
    L.tiles = static_cast<int32_t>((p.banks + kBanksPerCta - 1) / kBanksPerCta);
    tiles += L.tiles;
  }
  if (tiles == 0) return COW_OK;
  if (scratch_bytes < 16 + 8 * static_cast<int64_t>(tiles)) return COW_ERR_INVALID;
  P.header = static_cast<uint32_t*>(scan_scratch);
  P.flags = reinterpret_cast<uint64_t*>(static_cast<char*>(scan_scratch) + 16);
  P.layers = layers;
  P.width = static_cast<int32_t>(width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  P.total_tiles = tiles;
  void (*fn)(DecodeLaunch) = nullptr;
  const int ch = width_chunks(width);
  COW_SELECT_KERNEL(cow_decode_kernel, sdt, ch, writes <= 8, fn);
  fn<<<tiles, kBanksPerCta * 32, 0, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
