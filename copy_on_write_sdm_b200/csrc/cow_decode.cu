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
// is in flight before the scan resolves, and banks without first touches
// (other than the banks that publish group totals) never wait on it; only the
// placement of first-touch rows needs it.  The pool's free count and scan
// epoch are advanced by the bank that arrives last (an atomic arrival count),
// so closing a pool waits on nobody either.  Every wait is bounded and reports
// COW_ST_WAIT_TIMEOUT instead of hanging.


#include <cstdlib>
#include <mutex>

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// fused packed decode step
// --------------------------------------------------------------------------

// Single-pass launches close each pool by arrival count: header word 0 of the
// pool counts arrived banks above bit kCloseShift and their first touches
// below it (the host enables this when both fields fit).
constexpr int kCloseShift = 18;

// kF32I64: activations f32 and indices int64 at compile time (the common
// serving case; the launcher picks it for the f32 / W <= 4 / R <= 32 variant).
template <int SDT, int CH, int WMAX, int RC, bool kF32I64 = false>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_decode_kernel(const __grid_constant__ DecodeLaunch P) {
  const int act_dt = kF32I64 ? COW_F32 : P.act_dt;
  const int idx64 = kF32I64 ? 1 : P.idx64;
  // Common shapes (f32 rows, R <= 32, width <= 128) copy their read rows into
  // shared memory with bulk copies (one per row, on a per-warp mbarrier)
  // rather than holding them in registers.
  constexpr bool kStageReads = RC == 1 && CH == 1 && SDT == COW_F32;
  __shared__ WarpMetaT<32 * RC> s_meta[kBanksPerCta];
  __shared__ uint64_t s_bar[kBanksPerCta];  // per warp: the read-row copies' barrier
  __shared__ int s_tile;
  // dynamic: [read rows, per warp R x D floats (kStageReads)] [map rows, per warp N ints (P.stage_map)]
  extern __shared__ __align__(16) unsigned char dyn_smem[];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = P.width, W = P.writes, R = P.reads;

  // Pool of this block: contiguous block ranges, pool-major.
  int l = 0;
  while (l + 1 < P.layers && static_cast<int>(blockIdx.x) >= P.layer[l].tile_begin + P.layer[l].tiles) ++l;
  const DecodeLayer& L = P.layer[l];
  uint32_t* hdr = P.header + l;  // this pool's ticket / arrival word
  int tile;
  if (P.dynamic_tiles && !P.two_pass) {
    // More blocks than can be resident at once: a ticket orders the tiles by
    // start time, so a warp only ever waits on warps that are running.
    if (threadIdx.x == 0) s_tile = static_cast<int>(atomicAdd(&hdr[0], 1u));
    __syncthreads();
    tile = s_tile;
  } else {
    tile = static_cast<int>(blockIdx.x) - L.tile_begin;
  }
  // One warp = one bank = one scan element; nothing below synchronises the block.
  const int64_t bank = static_cast<int64_t>(tile) * kBanksPerCta + warp;
  if (bank >= L.banks) return;
  const int64_t N = L.slots;
  auto& sm = s_meta[warp];
  float* const s_reads = reinterpret_cast<float*>(dyn_smem) + static_cast<int64_t>(warp) * R * D;
  int32_t* const s_mapw = reinterpret_cast<int32_t*>(dyn_smem + P.read_stage_bytes) + static_cast<int64_t>(warp) * N;
  uint64_t* const flags = P.flags + static_cast<int64_t>(L.tile_begin) * kBanksPerCta;

  // Round 1: everything that does not depend on the routes.  The epoch and
  // the free count are read before this warp publishes or arrives; the bank
  // that closes the pool rewrites them only after every bank has done so, so
  // all banks see the launch's starting values.
  uint32_t epoch = 0;
  int old_free = 0, excl_given = 0;
  if (lane == 0) {
    if (!P.two_pass) {
      epoch = *reinterpret_cast<volatile uint32_t*>(&P.header[kEpochWord]);
      old_free = *reinterpret_cast<volatile int32_t*>(L.free_count);
    }
  }
  const int64_t tmpl = L.templates[bank];
  const float fl = ld1_rt(L.step.forget_log_gate, bank, act_dt);
  const float in_g = ld1_rt(L.step.input_gate, bank, act_dt);
  const float er_g = ld1_rt(L.step.erase_gate, bank, act_dt);
  float4 val[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 4;
    val[c] = col < D ? ld4_rt(L.step.values, bank * D + col, act_dt) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  unsigned first_mask = 0;
  int route_bits = 0;
  const bool bad_route = load_routes<false, RC>(sm, L.step, L.map, bank, bank, N, W, R, idx64, act_dt, lane,
                                                first_mask, route_bits, P.stage_map ? s_mapw : nullptr, L.log_t);
  const bool bad_tmpl = tmpl < 0 || tmpl >= L.template_count;
  const bool bad = bad_route || bad_tmpl;
  if (bad) {
    if (lane == 0) atomicOr(L.status, route_bits | (bad_tmpl ? COW_ST_TEMPLATE_RANGE : 0));
    first_mask = 0;
  }
  epoch = __shfl_sync(kFull, epoch, 0);
  old_free = __shfl_sync(kFull, old_free, 0);
  const int count = __popc(first_mask);
  uint32_t arrived = 0;
  if (lane == 0 && !P.two_pass) {
    *reinterpret_cast<volatile uint64_t*>(flags + bank) =
        pack_flag(epoch, kFlagAggregate, static_cast<uint32_t>(count));
    // Arrival: this bank has read the pool's starting epoch and free count (the
    // values were consumed by the shuffles above, so the reads are complete).
    if (P.counter_close) arrived = atomicAdd(&hdr[0], (1u << kCloseShift) + static_cast<uint32_t>(count));
  }

  // Row traffic: every read row (shared memory) or the first read group
  // (registers) and the write rows are requested together; the prefix scan
  // then runs while they are in flight.
  float4 upd[WMAX][CH];
  float4 v0[kStageReads ? 1 : ReadGroup<CH>::G][CH];
  float wt0[kStageReads ? 1 : ReadGroup<CH>::G];
  const int64_t m0_base = tmpl * N;
  if (!bad) {
    // Write rows first (registers), then the read rows (shared memory): the
    // issue loop of the read copies runs under the write rows' latency.
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
    if constexpr (kStageReads) {
      // Lane r requests read row r as one bulk copy (R <= 32); the warp's
      // barrier completes when all the bytes have landed.
      uint64_t* bar = &s_bar[warp];
      const int src = lane < R ? sm.rsrc[lane] : -2;
      const bool copy = src >= -1;
      const unsigned n_rows = __popc(__ballot_sync(kFull, copy));
      if (lane == 0) {
        mbar_init(bar, 1);
        mbar_arrive_expect_tx(bar, n_rows * static_cast<unsigned>(D) * 4u);
      }
      __syncwarp();
      if (copy) {
        const float* row = src >= 0 ? static_cast<const float*>(L.slab) + static_cast<int64_t>(src) * D
                                    : L.m0 + (m0_base + sm.ridx[lane]) * D;
        bulk_row_copy(s_reads + lane * D, row, static_cast<unsigned>(D) * 4u, bar);
      }
    }
    if constexpr (!kStageReads) load_read_group<SDT, CH>(v0, wt0, sm, 0, R, L.slab, 0, L.m0, m0_base, lane, D);
  }

  // The bank that arrived last closes the pool: every other bank has read the
  // starting epoch and free count, and the arrivals carried their first
  // touches.  Its stores depend on the atomic's result, so they cannot be
  // performed before the other banks' reads; no fence (which would also wait
  // for this warp's row loads) is needed.
  if (lane == 0 && P.counter_close && static_cast<int64_t>(arrived >> kCloseShift) == L.banks - 1) {
    const int total = static_cast<int>(arrived & ((1u << kCloseShift) - 1u)) + count;
    const int remaining = old_free - total > 0 ? old_free - total : 0;
    if (total > 0) *L.free_count = remaining;
    mirror_free(L, epoch, remaining);
    hdr[0] = 0u;
    close_pool_epoch(P.header, P.active_pools, epoch);
  }

  // Exclusive prefix of first touches over the preceding banks of this pool
  // (two-level scan, about one round trip), overlapped with the row loads
  // above.  Only banks that place rows, close the pool by look-back or
  // publish a scan group's total need it.
  int excl;
  if (P.two_pass) {
    // cow_count_kernel produced this bank's prefix and the pool's starting free
    // count.  This grid may start while that kernel still runs (programmatic
    // dependent launch): everything above touches nothing it writes, and the
    // wait below returns once its memory operations are visible.  The map
    // stores of the placement come after it, through the shuffled values.
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      excl_given = reinterpret_cast<const int32_t*>(P.flags)[static_cast<int64_t>(L.tile_begin) * kBanksPerCta + bank];
      old_free = reinterpret_cast<const int32_t*>(P.flags)[static_cast<int64_t>(P.total_tiles) * kBanksPerCta + l];
    }
    excl = __shfl_sync(kFull, excl_given, 0);
    old_free = __shfl_sync(kFull, old_free, 0);
  } else if (count == 0 && (P.counter_close || bank != L.banks - 1) && bank % kScanGroup != kScanGroup - 1) {
    // Nothing to place, not the bank that closes the pool and not the bank
    // that publishes its scan group's total: the prefix is not needed.
    excl = 0;
  } else {
    bool timed_out = false;
    excl = pool_prefix(flags, P.group_flags + L.group_begin, bank, count, epoch, lane, timed_out);
    if (__any_sync(kFull, timed_out) && lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
    if (lane == 0 && !P.counter_close) {
      const int inclusive = excl + count;
      if (bank == L.banks - 1) {
        // Every bank of this pool has published, hence has read the starting
        // epoch and free count: close the launch for this pool.
        const int remaining = old_free - inclusive > 0 ? old_free - inclusive : 0;
        if (inclusive > 0) *L.free_count = remaining;
        mirror_free(L, epoch, remaining);
        if (P.dynamic_tiles) hdr[0] = 0u;
        close_pool_epoch(P.header, P.active_pools, epoch);
      }
    }
  }

  // Arithmetic, write-back of rows that were already private, readout.
  float4 acc[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (!bad) {
    gated_delta<SDT, CH, WMAX>(upd, sm, W, expf(fl), in_g, er_g, val, lane, D);
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
    if constexpr (kStageReads) {
      if (!mbar_wait(&s_bar[warp], 0, kSpinLimit)) {
        // Report, then wait (bounded again) so no copy lands after the warp exits.
        if (lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
        mbar_wait(&s_bar[warp], 0, kSpinLimit);
      }
      if (lane * 4 < D) {
        for (int r = 0; r < R; ++r) {
          if (sm.rsrc[r] >= -1) acc[0] = f4_axpy(sm.rw[r], *reinterpret_cast<const float4*>(s_reads + r * D + lane * 4), acc[0]);
        }
      }
    } else {
      accumulate_group<CH>(acc, v0, wt0);
      read_remaining<SDT, CH>(acc, sm, R, L.slab, 0, L.m0, m0_base, lane, D);
    }
    add_forwarded<CH, WMAX>(acc, upd, sm, W);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < D) st4_rt(L.step.output, bank * D + col, acc[c], act_dt);
  }

  // Place the first touches: pop free_rows[old_free - 1 - rank].
  int newp = -1;
  const bool first = lane < W && ((first_mask >> lane) & 1u);
  if (first) {
    const int rank = excl + __popc(first_mask & ((1u << lane) - 1u));
    const int pos = old_free - 1 - rank;
    if (pos >= 0) {
      newp = L.free_rows[pos];
      if (L.log_t == 0) {
        L.map[bank * N + sm.widx[lane]] = newp;
      } else if (!hash_insert(reinterpret_cast<unsigned long long*>(L.map) + (bank << L.log_t), L.log_t,
                              sm.widx[lane], newp)) {
        atomicOr(L.status, COW_ST_MAP_FULL);
      }
    } else {
      atomicOr(L.status, COW_ST_SLAB_EXHAUSTED);
    }
  }
  if (L.step.first_touch != nullptr && lane < W) L.step.first_touch[bank * W + lane] = (first && newp >= 0) ? 1 : 0;
  if (first_mask != 0u) {
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
  }
}

// --------------------------------------------------------------------------
// small launches: one bank per block, split over kSplit warps
// --------------------------------------------------------------------------
//
// With a few hundred banks per launch each SM sub-partition holds about one
// warp, and the step is bound by the serial instruction chain of that warp
// (about a thousand dependent instructions for f32 rows, W <= 4, R <= 32,
// width <= 128), not by memory.  This variant gives each bank a block of
// kSplit warps.  Every warp resolves the bank's routes (identical metadata,
// no barrier) and holds all W write rows (the gated-delta update needs all of
// them for the retrieved vector); warp k stores write rows w == k (mod kSplit)
// and reads rows r == k (mod kSplit) into registers (kBulk: bulk-copied into
// shared memory instead, rows read after a write this step then copied from
// M0 with weight 0); rows read after a write this step are fed from the
// updated registers.
// The kSplit partial readouts meet in shared memory.  Warp 0 alone takes
// part in the pool's scan and close and places the first touches, exactly as
// cow_decode_kernel does (same flags, same epoch, same pop order).  Its
// activations are f32 and its indices int64 at compile time (the common
// serving case), which removes the per-load dtype dispatch.
// Warps per bank (a compile-time choice; measured on the batch-64 screen: 2 warps
// 7.3 us, 4 warps 5.8 us, 8 warps 6.2 us per step).
#ifndef COW_SPLIT_WARPS
#define COW_SPLIT_WARPS 4
#endif
constexpr int kSplit = COW_SPLIT_WARPS;
constexpr int kSplitRows = 32 / kSplit;  // read rows per warp (R <= 32)

template <bool kBulk>
__global__ void __launch_bounds__(kSplit * 32)
    cow_decode_split_kernel(const __grid_constant__ DecodeLaunch P) {
  __shared__ WarpMetaT<32> s_meta[kSplit];
  __shared__ uint64_t s_bar[kSplit];
  __shared__ __align__(16) float s_rows[kSplit][kSplitRows][128];
  __shared__ __align__(16) float s_rw[kSplit][kSplitRows];
  __shared__ __align__(16) float4 s_part[kSplit][32];
  extern __shared__ __align__(16) unsigned char dyn_smem[];  // staged map rows, N ints per warp

  const int k = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int D = P.width, W = P.writes, R = P.reads;
  int l = 0;
  while (l + 1 < P.layers && static_cast<int>(blockIdx.x) >= P.layer[l + 1].split_begin) ++l;
  const DecodeLayer& L = P.layer[l];
  uint32_t* hdr = P.header + l;
  const int64_t bank = static_cast<int64_t>(blockIdx.x) - L.split_begin;
  const int64_t N = L.slots;
  auto& sm = s_meta[k];
  int32_t* const s_mapw = reinterpret_cast<int32_t*>(dyn_smem) + static_cast<int64_t>(k) * N;
  uint64_t* const flags = P.flags + static_cast<int64_t>(L.tile_begin) * kBanksPerCta;

  uint32_t epoch = 0;
  int old_free = 0;
  if (k == 0 && lane == 0) {
    epoch = *reinterpret_cast<volatile uint32_t*>(&P.header[kEpochWord]);
    old_free = *reinterpret_cast<volatile int32_t*>(L.free_count);
  }
  const int64_t tmpl = L.templates[bank];
  const float fl = ld1_rt(L.step.forget_log_gate, bank, COW_F32);
  const float in_g = ld1_rt(L.step.input_gate, bank, COW_F32);
  const float er_g = ld1_rt(L.step.erase_gate, bank, COW_F32);
  float4 val[1];
  val[0] = lane * 4 < D ? ld4_rt(L.step.values, bank * D + lane * 4, COW_F32) : make_float4(0.f, 0.f, 0.f, 0.f);
  unsigned first_mask = 0;
  int route_bits = 0;
  const bool bad_route = load_routes<false, 1>(sm, L.step, L.map, bank, bank, N, W, R, 1, COW_F32, lane,
                                               first_mask, route_bits, s_mapw);
  const bool bad_tmpl = tmpl < 0 || tmpl >= L.template_count;
  const bool bad = bad_route || bad_tmpl;
  if (bad) {
    if (k == 0 && lane == 0) atomicOr(L.status, route_bits | (bad_tmpl ? COW_ST_TEMPLATE_RANGE : 0));
    first_mask = 0;
  }
  const int count = __popc(first_mask);
  uint32_t arrived = 0;
  if (k == 0) {
    epoch = __shfl_sync(kFull, epoch, 0);
    old_free = __shfl_sync(kFull, old_free, 0);
    if (lane == 0) {
      *reinterpret_cast<volatile uint64_t*>(flags + bank) = pack_flag(epoch, kFlagAggregate, static_cast<uint32_t>(count));
      arrived = atomicAdd(&hdr[0], (1u << kCloseShift) + static_cast<uint32_t>(count));
    }
  }

  // This warp's read rows r = k + kSplit*j: one bulk copy per row (lane j),
  // slab rows for private slots, M0 rows otherwise (weight 0 when the slot
  // was written this step: its updated row is added from registers).
  const int64_t m0_base = tmpl * N;
  const int my_rows = R > k ? (R - k + kSplit - 1) / kSplit : 0;
  float4 upd[4][1];
  float4 rrow[kBulk ? 1 : kSplitRows];
  float rwt[kBulk ? 1 : kSplitRows];
  if (!bad) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W) {
        const int phys = sm.wphys[w];
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane * 4 < D) {
          x = phys < 0 ? ld4_m0(L.m0, (m0_base + sm.widx[w]) * D + lane * 4)
                       : Elem<COW_F32>::ld4(L.slab, static_cast<int64_t>(phys) * D + lane * 4);
        }
        upd[w][0] = x;
      }
    }
    if constexpr (kBulk) {
      uint64_t* bar = &s_bar[k];
      if (lane == 0) {
        mbar_init(bar, 1);
        mbar_arrive_expect_tx(bar, static_cast<unsigned>(my_rows) * static_cast<unsigned>(D) * 4u);
      }
      __syncwarp();
      if (lane < my_rows) {
        const int r = k + kSplit * lane;
        const int src = sm.rsrc[r];
        s_rw[k][lane] = src >= -1 ? sm.rw[r] : 0.f;
        const float* row = src >= 0 ? static_cast<const float*>(L.slab) + static_cast<int64_t>(src) * D
                                    : L.m0 + (m0_base + sm.ridx[r]) * D;
        bulk_row_copy(&s_rows[k][lane][0], row, static_cast<unsigned>(D) * 4u, bar);
      }
    } else {
      // Read rows straight into registers (a warp has at most kSplitRows):
      // rows written this step are skipped (their updated value is added from
      // registers), so the weights and the sum order match the bulk variant.
#pragma unroll
      for (int j = 0; j < kSplitRows; ++j) {
        const int r = k + kSplit * j;
        const int src = r < R ? sm.rsrc[r] : -2;
        rwt[j] = src >= -1 ? sm.rw[r] : 0.f;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane * 4 < D) {
          if (src >= 0) x = Elem<COW_F32>::ld4(L.slab, static_cast<int64_t>(src) * D + lane * 4);
          else if (src == -1) x = ld4_m0(L.m0, (m0_base + sm.ridx[r]) * D + lane * 4);
        }
        rrow[j] = x;
      }
    }
  }

  int excl = 0;
  if (k == 0) {
    if (lane == 0 && static_cast<int64_t>(arrived >> kCloseShift) == L.banks - 1) {
      const int total = static_cast<int>(arrived & ((1u << kCloseShift) - 1u)) + count;
      const int remaining = old_free - total > 0 ? old_free - total : 0;
      if (total > 0) *L.free_count = remaining;
      mirror_free(L, epoch, remaining);
      hdr[0] = 0u;
      close_pool_epoch(P.header, P.active_pools, epoch);
    }
    if (count > 0 || bank % kScanGroup == kScanGroup - 1) {
      bool timed_out = false;
      excl = pool_prefix(flags, P.group_flags + L.group_begin, bank, count, epoch, lane, timed_out);
      if (__any_sync(kFull, timed_out) && lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
    }
  }

  float4 acc[1] = {make_float4(0.f, 0.f, 0.f, 0.f)};
  if (!bad) {
    gated_delta<COW_F32, 1, 4>(upd, sm, W, expf(fl), in_g, er_g, val, lane, D);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W && w % kSplit == k) acc[0] = f4_axpy(sm.fwt[w], upd[w][0], acc[0]);
    }
    if constexpr (kBulk) {
      if (my_rows > 0 && !mbar_wait(&s_bar[k], 0, kSpinLimit)) {
        if (lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
        mbar_wait(&s_bar[k], 0, kSpinLimit);
      }
      if (lane * 4 < D) {
        for (int j = 0; j < my_rows; ++j)
          acc[0] = f4_axpy(s_rw[k][j], *reinterpret_cast<const float4*>(&s_rows[k][j][lane * 4]), acc[0]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < kSplitRows; ++j) {
        if (j < my_rows) acc[0] = f4_axpy(rwt[j], rrow[j], acc[0]);
      }
    }
  }
  s_part[k][lane] = acc[0];
  // Every warp has consumed its copies of the write rows (the update used
  // them), so the private rows may now be overwritten in place.
  __syncthreads();
  if (!bad) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W && w % kSplit == k) {
        const int phys = sm.wphys[w];
        if (phys >= 0 && lane * 4 < D) Elem<COW_F32>::st4(L.slab, static_cast<int64_t>(phys) * D + lane * 4, upd[w][0]);
      }
    }
  }
  if (k != 0) return;
  float4 sum = s_part[0][lane];
#pragma unroll
  for (int j = 1; j < kSplit; ++j) {
    const float4 x = s_part[j][lane];
    sum = make_float4(sum.x + x.x, sum.y + x.y, sum.z + x.z, sum.w + x.w);
  }
  if (lane * 4 < D) st4_rt(L.step.output, bank * D + lane * 4, sum, COW_F32);

  // Place the first touches: pop free_rows[old_free - 1 - rank].
  int newp = -1;
  const bool first = lane < W && ((first_mask >> lane) & 1u);
  if (first) {
    const int rank = excl + __popc(first_mask & ((1u << lane) - 1u));
    const int pos = old_free - 1 - rank;
    if (pos >= 0) {
      newp = L.free_rows[pos];
      L.map[bank * N + sm.widx[lane]] = newp;
    } else {
      atomicOr(L.status, COW_ST_SLAB_EXHAUSTED);
    }
  }
  if (L.step.first_touch != nullptr && lane < W) L.step.first_touch[bank * W + lane] = (first && newp >= 0) ? 1 : 0;
  if (first_mask != 0u) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      if (w < W && ((first_mask >> w) & 1u)) {
        const int p = __shfl_sync(kFull, newp, w);
        if (p >= 0 && lane * 4 < D) Elem<COW_F32>::st4(L.slab, static_cast<int64_t>(p) * D + lane * 4, upd[w][0]);
      }
    }
  }
}

// --------------------------------------------------------------------------
// first-touch prefix pass for large launches
// --------------------------------------------------------------------------
//
// With thousands of banks per pool, warps of the fused kernel would wait on one
// another's first-touch counts with their rows already loaded.  Large launches
// therefore compute every bank's exclusive prefix first: one thread per bank
// reads only its route indices and W map entries (same validity rules as the
// decode kernel: an out-of-range index, a repeated write address or a bad
// template makes the bank allocate nothing), a block scan covers 128 banks, and
// each block adds the aggregates of the pool's earlier blocks.  Results: the
// prefix of every bank slot and the pool's starting free count (in the scan
// flag region, read as int32), and the pool's new free count.

constexpr int kCountThreads = kScanGroup;  // one count block per 128-bank scan group (reuses its flag)
constexpr int kCountUnroll = 8;  // route elements a thread loads per round

__global__ void __launch_bounds__(kCountThreads) cow_count_kernel(const __grid_constant__ DecodeLaunch P) {
  __shared__ int s_warp[kCountThreads / 32];
  __shared__ int s_blk, s_base;
  __shared__ uint32_t s_epoch;
  __shared__ int s_old;
  __shared__ int s_wi[kCountThreads * COW_MAX_WRITES];  // the block's write slots, bank-major
  __shared__ int s_bad[kCountThreads];
  const int tid = threadIdx.x, lane = tid & 31;
  int l = 0;
  while (l + 1 < P.layers && static_cast<int>(blockIdx.x) >= P.layer[l].count_block_begin + P.layer[l].count_blocks) ++l;
  const DecodeLayer& L = P.layer[l];
  uint32_t* hdr = P.header + l;  // this pool's block ticket
  // The decode pass may start now: it waits for this grid only where it reads
  // the prefixes.
  asm volatile("griddepcontrol.launch_dependents;");
  int blk;
  if (P.dynamic_tiles) {
    if (tid == 0) s_blk = static_cast<int>(atomicAdd(&hdr[0], 1u));
    __syncthreads();
    blk = s_blk;
  } else {
    blk = static_cast<int>(blockIdx.x) - L.count_block_begin;
  }
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile uint32_t*>(&P.header[kEpochWord]);
    s_old = *reinterpret_cast<volatile int32_t*>(L.free_count);
  }
  s_bad[tid] = 0;
  const int64_t bank0 = static_cast<int64_t>(blk) * kCountThreads;
  const int64_t bank = bank0 + tid;
  const int64_t N = L.slots;
  const int W = P.writes, R = P.reads;
  const int nb = static_cast<int>(L.banks - bank0 < kCountThreads ? L.banks - bank0 : kCountThreads);
  const cow_step& st = L.step;
  // Route indices of the block's banks are contiguous: the whole block reads
  // them with consecutive threads on consecutive elements.  The first round of
  // write and read indices and the templates go out together, before anything
  // waits (one memory round trip for the common W <= 8, R <= 16).
  constexpr int kReadUnroll = 16;
  int64_t wraw[kCountUnroll], rraw[kReadUnroll];
#pragma unroll
  for (int u = 0; u < kCountUnroll; ++u) {
    const int e = u * kCountThreads + tid;
    wraw[u] = e < nb * W ? ld_index(st.write_indices, bank0 * W + e, P.idx64) : 0;
  }
#pragma unroll
  for (int u = 0; u < kReadUnroll; ++u) {
    const int e = u * kCountThreads + tid;
    rraw[u] = e < nb * R ? ld_index(st.read_indices, bank0 * R + e, P.idx64) : 0;
  }
  int64_t tmpl = 0;
  if (tid < nb) tmpl = L.templates[bank];
  __syncthreads();  // s_bad cleared, epoch and free count read
  const uint32_t epoch = s_epoch;
  auto take_write = [&](int e, int64_t raw) {
    if (e < nb * W) {
      const bool ok = raw >= 0 && raw < N;
      s_wi[e] = ok ? static_cast<int>(raw) : -1 - (e % W);  // distinct sentinels never count as repeats
      if (!ok) s_bad[e / W] = 1;
    }
  };
  auto take_read = [&](int e, int64_t raw) {
    if (e < nb * R && (raw < 0 || raw >= N)) s_bad[e / R] = 1;
  };
#pragma unroll
  for (int u = 0; u < kCountUnroll; ++u) take_write(u * kCountThreads + tid, wraw[u]);
#pragma unroll
  for (int u = 0; u < kReadUnroll; ++u) take_read(u * kCountThreads + tid, rraw[u]);
  // Further rounds (W > 8 or R > 16 with full blocks).
  for (int e0 = kCountThreads * kCountUnroll; e0 < nb * W; e0 += kCountThreads * kCountUnroll) {
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) {
      const int e = e0 + u * kCountThreads + tid;
      wraw[u] = e < nb * W ? ld_index(st.write_indices, bank0 * W + e, P.idx64) : 0;
    }
#pragma unroll
    for (int u = 0; u < kCountUnroll; ++u) take_write(e0 + u * kCountThreads + tid, wraw[u]);
  }
  for (int e0 = kCountThreads * kReadUnroll; e0 < nb * R; e0 += kCountThreads * kReadUnroll) {
#pragma unroll
    for (int u = 0; u < kReadUnroll; ++u) {
      const int e = e0 + u * kCountThreads + tid;
      rraw[u] = e < nb * R ? ld_index(st.read_indices, bank0 * R + e, P.idx64) : 0;
    }
#pragma unroll
    for (int u = 0; u < kReadUnroll; ++u) take_read(e0 + u * kCountThreads + tid, rraw[u]);
  }
  __syncthreads();
  int count = 0;
  if (tid < nb) {
    const int* wi = s_wi + tid * W;
    bool bad = s_bad[tid] != 0 || tmpl < 0 || tmpl >= L.template_count;
    for (int a = 1; a < W; ++a)
      for (int b = 0; b < a; ++b) bad |= wi[a] == wi[b];
    if (!bad) {
      for (int w0 = 0; w0 < W; w0 += 8) {
        int32_t m[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (w0 + u >= W) {
            m[u] = 0;
          } else if (L.log_t == 0) {
            m[u] = L.map[bank * N + wi[w0 + u]];
          } else {
            m[u] = hash_find(reinterpret_cast<const unsigned long long*>(L.map) + (bank << L.log_t), L.log_t,
                             wi[w0 + u]);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) count += m[u] < 0 ? 1 : 0;
      }
    }
  }
  int total;
  const int local = block_exclusive_scan_n<kCountThreads>(count, s_warp, total);
  uint64_t* const bflags = P.group_flags + L.group_begin;  // one aggregate per count block
  if (tid == 0) *reinterpret_cast<volatile uint64_t*>(bflags + blk) = pack_flag(epoch, kFlagAggregate, total);
  if (tid < 32) {
    bool timed_out = false;
    const int base = sum_flags(bflags, 0, blk, epoch, lane, timed_out);
    if (__any_sync(kFull, timed_out) && lane == 0) atomicOr(L.status, COW_ST_WAIT_TIMEOUT);
    if (lane == 0) s_base = base;
  }
  __syncthreads();
  int32_t* const excl = reinterpret_cast<int32_t*>(P.flags);
  if (bank < L.banks) excl[static_cast<int64_t>(L.tile_begin) * kBanksPerCta + bank] = s_base + local;
  if (tid == 0 && blk == L.count_blocks - 1) {
    // Every block of this pool has published, hence has read the starting
    // epoch and free count: record it for the decode pass and close the pool.
    const int inclusive = s_base + total;
    excl[static_cast<int64_t>(P.total_tiles) * kBanksPerCta + l] = s_old;
    const int remaining = s_old - inclusive > 0 ? s_old - inclusive : 0;
    *L.free_count = remaining;
    mirror_free(L, epoch, remaining);
    if (P.dynamic_tiles) hdr[0] = 0u;
    close_pool_epoch(P.header, P.active_pools, epoch);
  }
}

}  // namespace

namespace cowrt {
thread_local int last_cuda_error = 0;
}  // namespace cowrt

// Look-back scratch of cow_decode_step_noalloc.  Static device memory starts
// zeroed when the module loads (tickets 0, epoch 0, every flag "not
// published").  Each launch resets the tickets it used and advances the one
// launch epoch, so the array is ready for the next call whatever pool layout
// that call has.  In host code the name is only a stand-in: the device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[COW_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, resolved once
// per device.
int noalloc_scratch(void** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    cowrt::last_cuda_error = static_cast<int>(e);
    return COW_ERR_CUDA;
  }
  if (device < 0 || device >= kMaxDevices) return COW_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return COW_OK;
}

}  // namespace

namespace {

// Blocks of `fn` that fit on the current device at once (cached per device
// and kernel).  A launch within this bound runs its tiles in block order;
// beyond it the kernel orders tiles by a ticket instead.
constexpr int64_t kStageMaxBanks = 148 * 16;
// Launches with at least this many banks compute the first-touch prefix in a
// separate pass (cow_count_kernel) before the decode pass.
constexpr int64_t kTwoPassMinBanks = 12288;
// Launches of at most this many banks (and a shape the split kernel covers)
// run one bank per block of kSplit warps.
constexpr int64_t kSplitMaxBanks = 2048;

// COW_DECODE_SPLIT=0 in the environment turns the split kernel off (for
// comparisons); read once per process.
// COW_DECODE_SPLIT_BULK=1 stages the split kernel's read rows by bulk copies
// into shared memory instead of loading them into registers (comparisons).
bool split_bulk_rows() {
  static const bool on = [] {
    const char* v = std::getenv("COW_DECODE_SPLIT_BULK");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

bool split_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("COW_DECODE_SPLIT");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}



}  // namespace

extern "C" {

int cow_abi_version(void) { return COW_ABI_VERSION; }


const char* cow_last_error(void) {
  return cudaGetErrorString(static_cast<cudaError_t>(cowrt::last_cuda_error));
}

int64_t cow_decode_scratch_bytes(int64_t total_banks, int32_t layers) {
  // one 8-byte scan flag per bank slot (pools padded to whole 4-bank tiles),
  // then one per group of kScanGroup banks
  const int64_t pools = layers > 0 ? layers : 1;
  const int64_t tiles = (total_banks + kBanksPerCta - 1) / kBanksPerCta + pools;
  return kScanHeaderBytes + 8 * (kBanksPerCta * tiles + total_banks / kScanGroup + pools);
}

}  // extern "C"

namespace {

// cow_decode_step's launch logic.  `allow_split` is off when the step's inputs
// live in host memory: the split kernel reads every bank's routes once per
// warp, which costs four PCIe round trips where one suffices.
int decode_step_impl(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes, int32_t reads,
                     int32_t index_dtype, int32_t act_dtype, void* scan_scratch, int64_t scratch_bytes, void* stream,
                     bool allow_split) {
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
    L.free_mirror = reinterpret_cast<unsigned long long*>(p.free_mirror);
    L.log_t = 0;
    if (p.map_kind == COW_MAP_HASH) {
      const int64_t t = p.table_slots;
      if (t < 4 || t > (int64_t(1) << 30) || (t & (t - 1)) != 0 || p.slots >= (int64_t(1) << 31)) return COW_ERR_INVALID;
      while ((int64_t(1) << L.log_t) < t) ++L.log_t;
    } else if (p.map_kind != COW_MAP_DENSE) {
      return COW_ERR_INVALID;
    }
    L.tile_begin = tiles;
    L.tiles = static_cast<int32_t>((p.banks + kBanksPerCta - 1) / kBanksPerCta);
    tiles += L.tiles;
  }
  if (tiles == 0) return COW_OK;
  for (int l = 0; l < layers; ++l) P.active_pools += pools[l].banks > 0 ? 1 : 0;
  int64_t groups = 0;
  for (int l = 0; l < layers; ++l) {
    P.layer[l].group_begin = groups;
    groups += (pools[l].banks + kScanGroup - 1) / kScanGroup;
  }
  if (scratch_bytes < kScanHeaderBytes + 8 * (kBanksPerCta * static_cast<int64_t>(tiles) + groups)) return COW_ERR_INVALID;
  P.header = static_cast<uint32_t*>(scan_scratch);
  P.flags = reinterpret_cast<uint64_t*>(static_cast<char*>(scan_scratch) + kScanHeaderBytes);
  P.group_flags = P.flags + kBanksPerCta * static_cast<int64_t>(tiles);
  P.layers = layers;
  P.width = static_cast<int32_t>(width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  P.total_tiles = tiles;
  void (*fn)(DecodeLaunch) = nullptr;
  const int ch = width_chunks(width);
  const int rv = route_variant(writes, reads);
  COW_SELECT_KERNEL(cow_decode_kernel, sdt, ch, rv, fn);
  if (sdt == COW_F32 && ch == 1 && rv == 0 && act_dtype == COW_F32 && index_dtype == COW_I64)
    fn = cow_decode_kernel<COW_F32, 1, 4, 1, true>;
  // Latency-bound launches (at most ~16 warps per SM) with small tables stage
  // each bank's map row in shared memory: N*4 extra bytes per bank buy one
  // dependent memory round trip less.
  bool stage = true;
  int64_t total_banks = 0;
  for (int l = 0; l < layers; ++l) {
    stage = stage && pools[l].map_kind == COW_MAP_DENSE && pools[l].slots <= kStageSlots && pools[l].slots % 4 == 0 &&
            aligned16(pools[l].map);
    total_banks += pools[l].banks;
  }
  P.stage_map = stage && total_banks <= kStageMaxBanks ? 1 : 0;
  P.read_stage_bytes = static_cast<int32_t>(read_stage_bytes(reads, width, ch, rv, sdt));
  int64_t max_slots = 0;
  for (int l = 0; l < layers; ++l) max_slots = pools[l].slots > max_slots ? pools[l].slots : max_slots;
  const size_t smem = P.read_stage_bytes + (P.stage_map ? kBanksPerCta * max_slots * sizeof(int32_t) : 0);
  const int resident = resident_blocks(reinterpret_cast<const void*>(fn), kBanksPerCta * 32, smem);
  if (resident <= 0) return COW_ERR_UNSUPPORTED;
  if (total_banks >= kTwoPassMinBanks) {
    // Large launch: prefix pass first, then the decode pass with no waits.
    int32_t blocks = 0;
    for (int l = 0; l < layers; ++l) {
      P.layer[l].count_block_begin = blocks;
      P.layer[l].count_blocks = static_cast<int32_t>((pools[l].banks + kCountThreads - 1) / kCountThreads);
      blocks += P.layer[l].count_blocks;
    }
    const int count_resident = resident_blocks(reinterpret_cast<const void*>(cow_count_kernel), kCountThreads, 0);
    if (count_resident <= 0) return COW_ERR_UNSUPPORTED;
    P.dynamic_tiles = blocks > count_resident ? 1 : 0;
    cow_count_kernel<<<blocks, kCountThreads, 0, as_stream(stream)>>>(P);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
    P.two_pass = 1;
    P.dynamic_tiles = 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles));
    cfg.blockDim = dim3(kBanksPerCta * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, P);
    if (e != cudaSuccess) {
      cudaGetLastError();
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
    return launch_status();
  } else {
    P.dynamic_tiles = tiles > resident ? 1 : 0;
    // The arrival count shares header word 0 with the tile ticket; it serves
    // launches without dynamic tiles whose banks and first touches per pool
    // fit its two fields.  Otherwise the pool's last bank closes it by look-back.
    bool fits = !P.dynamic_tiles;
    for (int l = 0; l < layers; ++l)
      fits = fits && pools[l].banks < (int64_t(1) << (32 - kCloseShift)) &&
             pools[l].banks * writes < (int64_t(1) << kCloseShift);
    P.counter_close = fits ? 1 : 0;
    if (fits && allow_split && split_enabled() && sdt == COW_F32 && act_dtype == COW_F32 && index_dtype == COW_I64 && ch == 1 && rv == 0 && P.stage_map && width <= 128 &&
        total_banks <= kSplitMaxBanks) {
      // Small launch: one bank per block of kSplit warps (cow_decode_split_kernel).
      const size_t split_smem = static_cast<size_t>(kSplit) * max_slots * sizeof(int32_t);
      void (*split_fn)(DecodeLaunch) = split_bulk_rows() ? cow_decode_split_kernel<true> : cow_decode_split_kernel<false>;
      const int split_resident = resident_blocks(reinterpret_cast<const void*>(split_fn), kSplit * 32, split_smem);
      if (static_cast<int64_t>(split_resident) >= total_banks) {
        int32_t begin = 0;
        for (int l = 0; l < layers; ++l) {
          P.layer[l].split_begin = begin;
          begin += static_cast<int32_t>(pools[l].banks);
        }
        split_fn<<<static_cast<unsigned>(total_banks), kSplit * 32, split_smem, as_stream(stream)>>>(P);
        return launch_status();
      }
    }
  }
  fn<<<tiles, kBanksPerCta * 32, smem, as_stream(stream)>>>(P);
  return launch_status();
}

// Page-locked host ranges registered for zero-copy steps: host address, bytes
// and the device's address of the same bytes.
struct HostRange {
  const char* host;
  int64_t bytes;
  char* device;
};
constexpr int kMaxHostRanges = 64;
std::mutex g_host_mutex;
HostRange g_host_ranges[kMaxHostRanges];
int g_host_count = 0;

// Device address of [q, q + bytes) when it lies in page-locked host memory:
// a registered range first (no runtime call), else cudaPointerGetAttributes.
char* mapped_address(const void* q, int64_t bytes) {
  const char* c = static_cast<const char*>(q);
  {
    std::lock_guard<std::mutex> lock(g_host_mutex);
    for (int i = 0; i < g_host_count; ++i) {
      const HostRange& r = g_host_ranges[i];
      if (c >= r.host && c + bytes <= r.host + r.bytes) return r.device + (c - r.host);
    }
  }
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) return nullptr;
  return static_cast<char*>(a.devicePointer);
}

}  // namespace

extern "C" {

int cow_decode_step(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes, int32_t reads,
                    int32_t index_dtype, int32_t act_dtype, void* scan_scratch, int64_t scratch_bytes,
                    void* stream) {
  return decode_step_impl(pools, steps, layers, writes, reads, index_dtype, act_dtype, scan_scratch, scratch_bytes,
                          stream, true);
}

int cow_register_host_range(const void* host, int64_t bytes) {
  if (!host || bytes <= 0) return COW_ERR_INVALID;
  cudaPointerAttributes first{}, last{};
  const char* c = static_cast<const char*>(host);
  if (cudaPointerGetAttributes(&first, host) != cudaSuccess ||
      cudaPointerGetAttributes(&last, c + bytes - 1) != cudaSuccess) {
    cudaGetLastError();
    return COW_ERR_INVALID;
  }
  if (first.type != cudaMemoryTypeHost || last.type != cudaMemoryTypeHost || !first.devicePointer ||
      static_cast<char*>(last.devicePointer) - static_cast<char*>(first.devicePointer) != bytes - 1)
    return COW_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_host_mutex);
  if (g_host_count == kMaxHostRanges) return COW_ERR_UNSUPPORTED;
  g_host_ranges[g_host_count++] = HostRange{c, bytes, static_cast<char*>(first.devicePointer)};
  return COW_OK;
}

int cow_unregister_host_range(const void* host) {
  std::lock_guard<std::mutex> lock(g_host_mutex);
  for (int i = 0; i < g_host_count; ++i) {
    if (g_host_ranges[i].host == host) {
      g_host_ranges[i] = g_host_ranges[--g_host_count];
      return COW_OK;
    }
  }
  return COW_ERR_INVALID;
}

int cow_decode_step_checked(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes,
                            int32_t reads, int32_t index_dtype, int32_t act_dtype, void* scan_scratch,
                            int64_t scratch_bytes, void* stream, int32_t* status_out) {
  const int rc = cow_decode_step(pools, steps, layers, writes, reads, index_dtype, act_dtype, scan_scratch,
                                 scratch_bytes, stream);
  if (rc != COW_OK) return rc;
  cudaStream_t st = as_stream(stream);
  int32_t words[COW_MAX_LAYERS] = {};
  for (int l = 0; l < layers; ++l) {
    const cudaError_t e = cudaMemcpyAsync(&words[l], pools[l].status, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) {
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
  }
  const cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    cowrt::last_cuda_error = static_cast<int>(e);
    return COW_ERR_CUDA;
  }
  int32_t any = 0;
  for (int l = 0; l < layers; ++l) any |= words[l];
  if (status_out) *status_out = any;
  return any != 0 ? COW_ERR_DEVICE : COW_OK;
}

int cow_decode_step_host(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes, int32_t reads,
                         int32_t index_dtype, int32_t act_dtype, void* scan_scratch, int64_t scratch_bytes,
                         void* device_inputs, const void* host_inputs, int64_t input_bytes, void* host_outputs,
                         const void* device_outputs, int64_t output_bytes, void* stream) {
  if (input_bytes < 0 || output_bytes < 0 || (input_bytes > 0 && (!device_inputs || !host_inputs)) ||
      (output_bytes > 0 && (!host_outputs || !device_outputs)))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (input_bytes > 0) {
    const cudaError_t e = cudaMemcpyAsync(device_inputs, host_inputs, static_cast<size_t>(input_bytes),
                                          cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
  }
  const int rc = cow_decode_step(pools, steps, layers, writes, reads, index_dtype, act_dtype, scan_scratch,
                                 scratch_bytes, stream);
  if (rc != COW_OK) return rc;
  if (output_bytes > 0) {
    const cudaError_t e = cudaMemcpyAsync(host_outputs, device_outputs, static_cast<size_t>(output_bytes),
                                          cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) {
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
  }
  return COW_OK;
}

int cow_decode_step_host_overlapped(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes,
                                    int32_t reads, int32_t index_dtype, int32_t act_dtype, void* scan_scratch,
                                    int64_t scratch_bytes, void* device_inputs, const void* host_inputs,
                                    int64_t input_bytes, void* host_outputs, const void* device_outputs,
                                    int64_t output_bytes, void* compute_stream, void* h2d_stream, void* d2h_stream,
                                    void* h2d_done, void* computed, void* d2h_done) {
  if (input_bytes <= 0 || output_bytes <= 0 || !device_inputs || !host_inputs || !host_outputs || !device_outputs ||
      !h2d_done || !computed || !d2h_done)
    return COW_ERR_INVALID;
  cudaStream_t cs = as_stream(compute_stream), hs = as_stream(h2d_stream), ds = as_stream(d2h_stream);
  cudaEvent_t e_h2d = static_cast<cudaEvent_t>(h2d_done), e_comp = static_cast<cudaEvent_t>(computed),
              e_d2h = static_cast<cudaEvent_t>(d2h_done);
  // The buffers of this step were last used by the step that recorded this
  // pair's events: its decode read the inputs and its readout copy, which
  // itself waited for that decode, read the outputs.  One wait on that readout
  // copy (e_d2h) therefore frees both buffers; the decode then waits only for
  // this step's input copy, which follows it on the copy stream.  Waiting on
  // an event that was never recorded returns at once.
  cudaError_t e = cudaStreamWaitEvent(hs, e_d2h, 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(device_inputs, host_inputs, static_cast<size_t>(input_bytes),
                                            cudaMemcpyHostToDevice, hs);
  if (e == cudaSuccess) e = cudaEventRecord(e_h2d, hs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, e_h2d, 0);
  if (e != cudaSuccess) {
    cowrt::last_cuda_error = static_cast<int>(e);
    return COW_ERR_CUDA;
  }
  const int rc = cow_decode_step(pools, steps, layers, writes, reads, index_dtype, act_dtype, scan_scratch,
                                 scratch_bytes, compute_stream);
  if (rc != COW_OK) return rc;
  e = cudaEventRecord(e_comp, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ds, e_comp, 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(host_outputs, device_outputs, static_cast<size_t>(output_bytes),
                                            cudaMemcpyDeviceToHost, ds);
  if (e == cudaSuccess) e = cudaEventRecord(e_d2h, ds);
  if (e != cudaSuccess) {
    cowrt::last_cuda_error = static_cast<int>(e);
    return COW_ERR_CUDA;
  }
  return COW_OK;
}

int cow_decode_step_host_piped(const cow_host_pipeline* p, const void* host_inputs, void* compute_stream) {
  if (!p) return COW_ERR_INVALID;
  return cow_decode_step_host_overlapped(p->pools, p->steps, p->layers, p->writes, p->reads, p->index_dtype,
                                         p->act_dtype, p->scan_scratch, p->scratch_bytes, p->device_inputs,
                                         host_inputs, p->input_bytes, p->host_outputs, p->device_outputs,
                                         p->output_bytes, compute_stream, p->h2d_stream, p->d2h_stream, p->h2d_done,
                                         p->computed, p->d2h_done);
}

int cow_decode_step_host_mapped(const cow_host_pipeline* p, const void* host_inputs, void* host_outputs,
                                void* stream) {
  if (!p || !host_inputs || !host_outputs || !p->steps || !p->device_inputs || !p->device_outputs ||
      p->layers < 1 || p->layers > COW_MAX_LAYERS)
    return COW_ERR_INVALID;
  // Both host buffers must be page-locked and mapped for the device: the
  // kernel dereferences them.  Pageable memory is refused before any launch.
  char* mapped[2] = {mapped_address(host_inputs, p->input_bytes), mapped_address(host_outputs, p->output_bytes)};
  if (!mapped[0] || !mapped[1]) return COW_ERR_INVALID;
  // The step descriptors point into the device buffers; the same offsets into
  // the caller's pinned host buffers give the kernel's inputs and outputs.
  const char* in0 = static_cast<const char*>(p->device_inputs);
  const char* out0 = static_cast<const char*>(p->device_outputs);
  const char* hin = static_cast<const char*>(mapped[0]);
  char* hout = static_cast<char*>(mapped[1]);
  auto rebase_in = [&](const void* q) -> const void* {
    return q == nullptr ? nullptr : hin + (static_cast<const char*>(q) - in0);
  };
  cow_step steps[COW_MAX_LAYERS];
  for (int l = 0; l < p->layers; ++l) {
    const cow_step& s = p->steps[l];
    steps[l].write_indices = rebase_in(s.write_indices);
    steps[l].write_weights = rebase_in(s.write_weights);
    steps[l].values = rebase_in(s.values);
    steps[l].input_gate = rebase_in(s.input_gate);
    steps[l].erase_gate = rebase_in(s.erase_gate);
    steps[l].forget_log_gate = rebase_in(s.forget_log_gate);
    steps[l].read_indices = rebase_in(s.read_indices);
    steps[l].read_weights = rebase_in(s.read_weights);
    steps[l].output = hout + (static_cast<const char*>(s.output) - out0);
    steps[l].first_touch = nullptr;
  }
  const int rc = decode_step_impl(p->pools, steps, p->layers, p->writes, p->reads, p->index_dtype, p->act_dtype,
                                  p->scan_scratch, p->scratch_bytes, stream, false);
  if (rc != COW_OK) return rc;
  if (p->d2h_done) {
    const cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(p->d2h_done), as_stream(stream));
    if (e != cudaSuccess) {
      cowrt::last_cuda_error = static_cast<int>(e);
      return COW_ERR_CUDA;
    }
  }
  return COW_OK;
}

int cow_decode_step_noalloc(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes,
                            int32_t reads, int32_t index_dtype, int32_t act_dtype, void* stream) {
  if (!pools || !steps || layers < 1 || layers > COW_MAX_LAYERS) return COW_ERR_INVALID;
  int64_t total_banks = 0;
  for (int l = 0; l < layers; ++l) {
    if (pools[l].banks < 0) return COW_ERR_INVALID;
    total_banks += pools[l].banks;
  }
  if (cow_decode_scratch_bytes(total_banks, layers) > COW_NOALLOC_SCRATCH_BYTES) return COW_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != COW_OK) return rc;
  return cow_decode_step(pools, steps, layers, writes, reads, index_dtype, act_dtype, scratch,
                         COW_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
