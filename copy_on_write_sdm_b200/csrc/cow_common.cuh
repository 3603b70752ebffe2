// cow_common.cuh -- shared device helpers of the packed copy-on-write SDM kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "cow_sdm.h"

#define COW_ABI_VERSION 1

namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kBanksPerCta = 4;  // warps per decode CTA
constexpr int kSpinLimit = 1 << 21;
constexpr int kLookbackPerLane = 4;  // scan flags each lane reads per look-back probe
// Scan scratch header (32-bit words): one ticket / arrival word per pool slot,
// then the launch epoch and the count of pools closed in the running launch.
// Every flag a launch writes carries the launch epoch, which the last pool to
// close advances once; flags left by any earlier launch, whatever its pool
// layout, therefore carry an older epoch and never read as published.
constexpr int kScanHeaderBytes = 8 * COW_MAX_LAYERS;
constexpr int kEpochWord = COW_MAX_LAYERS;
constexpr int kClosedWord = COW_MAX_LAYERS + 1;
static_assert(4 * (kClosedWord + 1) <= kScanHeaderBytes, "scan header too small");

// --------------------------------------------------------------------------
// element access
// --------------------------------------------------------------------------

__device__ __forceinline__ float4 f4_axpy(float a, float4 x, float4 y) {
  return make_float4(fmaf(a, x.x, y.x), fmaf(a, x.y, y.y), fmaf(a, x.z, y.z), fmaf(a, x.w, y.w));
}
__device__ __forceinline__ float4 f4_scale(float a, float4 x) {
  return make_float4(a * x.x, a * x.y, a * x.z, a * x.w);
}

template <int DT>
struct Elem;

template <>
struct Elem<COW_F32> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t e) {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + e);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t e, float4 v) {
    *reinterpret_cast<float4*>(static_cast<float*>(p) + e) = v;
  }
  static __device__ __forceinline__ float4 round4(float4 v) { return v; }
  static __device__ __forceinline__ float ld1(const void* p, int64_t i) {
    return static_cast<const float*>(p)[i];
  }
};

template <>
struct Elem<COW_BF16> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t e) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(p) + e);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t e, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<unsigned*>(&a);
    u.y = *reinterpret_cast<unsigned*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p) + e) = u;
  }
  static __device__ __forceinline__ float r1(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ float4 round4(float4 v) {
    return make_float4(r1(v.x), r1(v.y), r1(v.z), r1(v.w));
  }
  static __device__ __forceinline__ float ld1(const void* p, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
};

template <>
struct Elem<COW_F16> {
  static __device__ __forceinline__ float4 ld4(const void* p, int64_t e) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(p) + e);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  static __device__ __forceinline__ void st4(void* p, int64_t e, float4 v) {
    __half2 a = __floats2half2_rn(v.x, v.y);
    __half2 b = __floats2half2_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<unsigned*>(&a);
    u.y = *reinterpret_cast<unsigned*>(&b);
    *reinterpret_cast<uint2*>(static_cast<__half*>(p) + e) = u;
  }
  static __device__ __forceinline__ float r1(float x) { return __half2float(__float2half_rn(x)); }
  static __device__ __forceinline__ float4 round4(float4 v) {
    return make_float4(r1(v.x), r1(v.y), r1(v.z), r1(v.w));
  }
  static __device__ __forceinline__ float ld1(const void* p, int64_t i) {
    return __half2float(static_cast<const __half*>(p)[i]);
  }
};

// Activation tensors (weights, values, gates, readouts) carry a runtime dtype:
// the branch is warp-uniform and off the row-traffic critical path.
__device__ __forceinline__ float ld1_rt(const void* p, int64_t i, int dt) {
  if (dt == COW_F32) return Elem<COW_F32>::ld1(p, i);
  if (dt == COW_BF16) return Elem<COW_BF16>::ld1(p, i);
  return Elem<COW_F16>::ld1(p, i);
}
__device__ __forceinline__ float4 ld4_rt(const void* p, int64_t e, int dt) {
  if (dt == COW_F32) return Elem<COW_F32>::ld4(p, e);
  if (dt == COW_BF16) return Elem<COW_BF16>::ld4(p, e);
  return Elem<COW_F16>::ld4(p, e);
}
__device__ __forceinline__ void st4_rt(void* p, int64_t e, float4 v, int dt) {
  if (dt == COW_F32) Elem<COW_F32>::st4(p, e, v);
  else if (dt == COW_BF16) Elem<COW_BF16>::st4(p, e, v);
  else Elem<COW_F16>::st4(p, e, v);
}
__device__ __forceinline__ int64_t ld_index(const void* p, int64_t i, int idx64) {
  return idx64 ? static_cast<const long long*>(p)[i] : static_cast<const int*>(p)[i];
}
__device__ __forceinline__ float4 ld4_m0(const float* m0, int64_t e) {
  return __ldg(reinterpret_cast<const float4*>(m0 + e));
}

// 16-byte global -> shared copies that bypass L1 and need no registers.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Bulk (TMA engine) copies of whole rows into shared memory, completed on an
// mbarrier: one instruction moves one row, whichever its length.
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// dst, src 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_row_copy(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)) : "memory");
}
// Bounded wait for phase `parity` of the barrier; false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int limit) {
  for (int i = 0; i < limit; ++i) {
    unsigned done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    if (done) return true;
  }
  return false;
}

// --------------------------------------------------------------------------
// hashed logical maps (cow_pool.map_kind == COW_MAP_HASH)
// --------------------------------------------------------------------------
//
// A bank's private slots live in an open-addressing table of T = 2^log_t
// 64-bit entries, (slot << 32) | physical row, all ones when empty.  Entries
// form buckets of four (32 bytes, one memory sector); a slot is looked for from
// its home bucket (a multiplicative hash of the slot) onwards, bucket by
// bucket, each bucket read with two 16-byte loads.  Only one warp touches a
// bank's table during a decode step, lookups of a step precede its inserts,
// and entries are never deleted inside a step, so a lookup stops at the first
// empty entry.  T >= 4.
constexpr unsigned long long kHashEmpty = ~0ull;

__device__ __forceinline__ uint32_t hash_home(int slot, int log_buckets) {
  return log_buckets == 0 ? 0u : (static_cast<uint32_t>(slot) * 2654435761u) >> (32 - log_buckets);
}

// Physical row of `slot` in the bank's table, -1 when the slot is shared.
__device__ __forceinline__ int hash_find(const unsigned long long* table, int log_t, int slot) {
  const uint32_t mask = (1u << (log_t - 2)) - 1u;
  uint32_t b = hash_home(slot, log_t - 2);
  for (uint32_t n = 0; n <= mask; ++n) {
    const ulonglong2* q = reinterpret_cast<const ulonglong2*>(table + 4 * static_cast<int64_t>(b));
    const ulonglong2 lo = q[0], hi = q[1];
    const unsigned long long e[4] = {lo.x, lo.y, hi.x, hi.y};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (e[k] == kHashEmpty) return -1;
      if (static_cast<int>(e[k] >> 32) == slot) return static_cast<int>(static_cast<uint32_t>(e[k]));
    }
    b = (b + 1u) & mask;
  }
  return -1;
}

// Claim the first empty entry from `slot`'s home bucket on; false when the
// table is full.
__device__ __forceinline__ bool hash_insert(unsigned long long* table, int log_t, int slot, int phys) {
  const uint32_t mask = (1u << (log_t - 2)) - 1u;
  const unsigned long long entry =
      (static_cast<unsigned long long>(static_cast<uint32_t>(slot)) << 32) | static_cast<uint32_t>(phys);
  uint32_t b = hash_home(slot, log_t - 2);
  for (uint32_t n = 0; n <= mask; ++n) {
    unsigned long long* q = table + 4 * static_cast<int64_t>(b);
    for (int k = 0; k < 4; ++k)
      if (q[k] == kHashEmpty && atomicCAS(q + k, kHashEmpty, entry) == kHashEmpty) return true;
    b = (b + 1u) & mask;
  }
  return false;
}

// Largest logical table whose map row a decode warp may stage in shared memory.
constexpr int kStageSlots = 1024;

// --------------------------------------------------------------------------
// per-warp route metadata (shared memory, broadcast reads)
// --------------------------------------------------------------------------

template <int RMAX>
struct WarpMetaT {
  int widx[COW_MAX_WRITES];
  int wphys[COW_MAX_WRITES];  // map entry before the step (-1 = shared M0)
  float ww[COW_MAX_WRITES];
  float fwt[COW_MAX_WRITES];  // summed read weight of reads that hit write slot w this step
  int ridx[RMAX];
  int rsrc[RMAX];  // >= 0 slab row, -1 M0 row, <= -2 forwarded write slot -(w+2)
  float rw[RMAX];
};
using WarpMeta = WarpMetaT<COW_MAX_READS>;

struct DecodeLayer {
  const float* m0;
  const int64_t* templates;
  void* slab;
  int32_t* map;
  const int32_t* free_rows;
  int32_t* free_count;
  int32_t* status;
  cow_step step;
  int64_t banks, slots, capacity, template_count, group_begin;
  int32_t tile_begin, tiles;
  int32_t count_block_begin, count_blocks;  // two-pass launches: blocks of cow_count_kernel
  int32_t split_begin;                      // split launches: first block (= bank 0) of this pool
  unsigned long long* free_mirror;          // optional host word: (launch epoch << 32) | free count
  int32_t log_t;                            // hashed map: log2 entries per bank's table (0: dense map)
};

// Free count of a closed pool, mirrored to the pool's host word (if any).
__device__ __forceinline__ void mirror_free(const DecodeLayer& L, uint32_t epoch, int free_rows) {
  if (L.free_mirror != nullptr)
    *reinterpret_cast<volatile unsigned long long*>(L.free_mirror) =
        (static_cast<unsigned long long>(epoch) << 32) | static_cast<uint32_t>(free_rows);
}

struct DecodeLaunch {
  DecodeLayer layer[COW_MAX_LAYERS];
  uint32_t* header;    // [ticket per pool slot] + launch epoch + closed-pool count
  uint64_t* flags;        // one per bank slot, pool-major (tile_begin * 4 + bank)
  uint64_t* group_flags;  // one per group of kScanGroup banks, pool-major (group_begin + group)
  int32_t layers, width, writes, reads, idx64, act_dt, total_tiles, dynamic_tiles, stage_map, read_stage_bytes;
  int32_t two_pass, counter_close;  // counter_close: pools close by arrival count (cow_decode_kernel)
  int32_t active_pools;             // pools with at least one bank (each closes once per launch)
};

constexpr uint32_t kFlagAggregate = 1u;
constexpr uint32_t kFlagInclusive = 2u;

__device__ __forceinline__ uint64_t pack_flag(uint32_t epoch, uint32_t st, uint32_t v) {
  return (static_cast<uint64_t>(epoch) << 32) | (static_cast<uint64_t>(st) << 30) | (v & 0x3fffffffu);
}

// Called once per pool and launch, after every bank of that pool has read the
// launch epoch.  The last pool to close resets the count and advances the
// epoch, so every pool of the launch read the same epoch and no later launch
// can mistake one of this launch's flags for its own.
__device__ __forceinline__ void close_pool_epoch(uint32_t* header, int active_pools, uint32_t epoch) {
  const uint32_t closed = atomicAdd(&header[kClosedWord], 1u);
  if (static_cast<int>(closed) == active_pools - 1) {
    header[kClosedWord] = 0u;
    *reinterpret_cast<volatile uint32_t*>(&header[kEpochWord]) = epoch + 1u;
  }
}

__device__ __forceinline__ uint64_t ld_volatile_u64(const uint64_t* p) {
  return *reinterpret_cast<const volatile uint64_t*>(p);
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// --------------------------------------------------------------------------
// ordered prefix of first-touch counts across the banks of one pool
// --------------------------------------------------------------------------
//
// Every bank publishes its count (an epoch-tagged "aggregate" flag) as soon as
// its routes are resolved.  Banks form groups of kScanGroup; the last bank of
// a group publishes the group total.  A bank's exclusive prefix is the sum of
// the earlier aggregates of its own group plus the earlier group totals: two
// probes issued together, about one memory round trip, however many banks run
// at once (no chain of inclusive prefixes).
constexpr int kScanGroup = 128;

__device__ __forceinline__ uint32_t wait_flag(const uint64_t* p, uint32_t epoch, bool& timed_out) {
  int spins = 0;
  while (true) {
    const uint64_t f = ld_volatile_u64(p);
    if (static_cast<uint32_t>(f >> 32) == epoch && ((f >> 30) & 3u) != 0u) return static_cast<uint32_t>(f & 0x3fffffffu);
    if (++spins > kSpinLimit) {
      timed_out = true;
      return 0u;
    }
    __nanosleep(spins < 64 ? 20 : 200);
  }
}

// Sum of the flags [lo, hi) (hi - lo <= 32 * kLookbackPerLane per probe),
// each lane waiting on its own flags; the first loads of all lanes go out
// together.
__device__ __forceinline__ int sum_flags(const uint64_t* f, int64_t lo, int64_t hi, uint32_t epoch, int lane,
                                         bool& timed_out) {
  int total = 0;
  for (int64_t base = lo; base < hi; base += 32 * kLookbackPerLane) {
    uint64_t first[kLookbackPerLane];
#pragma unroll
    for (int j = 0; j < kLookbackPerLane; ++j) {
      const int64_t i = base + kLookbackPerLane * lane + j;
      first[j] = i < hi ? ld_volatile_u64(f + i) : 0;
    }
    int part = 0;
#pragma unroll
    for (int j = 0; j < kLookbackPerLane; ++j) {
      const int64_t i = base + kLookbackPerLane * lane + j;
      if (i < hi) {
        const uint64_t x = first[j];
        const bool ready = static_cast<uint32_t>(x >> 32) == epoch && ((x >> 30) & 3u) != 0u;
        part += static_cast<int>(ready ? static_cast<uint32_t>(x & 0x3fffffffu) : wait_flag(f + i, epoch, timed_out));
      }
    }
    total += warp_sum(part);
  }
  return total;
}

// Block-wide exclusive prefix sum of one int per thread (kThreads threads,
// multiple of 32, at most 1024); `total` receives the block sum.
template <int kThreads>
__device__ __forceinline__ int block_exclusive_scan_n(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kThreads / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kThreads / 32) s_warp[lane] = w;
  }
  __syncthreads();
  total = s_warp[kThreads / 32 - 1];
  const int before = warp > 0 ? s_warp[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

// Exclusive prefix for `bank` (warp-uniform result).  `bank_flags` / `group_flags`
// are this pool's regions; the bank's own aggregate must already be published.
__device__ __forceinline__ int pool_prefix(const uint64_t* bank_flags, uint64_t* group_flags, int64_t bank, int count,
                                           uint32_t epoch, int lane, bool& timed_out) {
  const int64_t group = bank / kScanGroup, gstart = group * kScanGroup;
  const int in_group = sum_flags(bank_flags, gstart, bank, epoch, lane, timed_out);
  if (bank - gstart == kScanGroup - 1 && lane == 0) {
    *reinterpret_cast<volatile uint64_t*>(group_flags + group) =
        pack_flag(epoch, kFlagInclusive, static_cast<uint32_t>(in_group + count));
  }
  return in_group + sum_flags(group_flags, 0, group, epoch, lane, timed_out);
}

// Load the W write routes and R read routes of one bank into the warp's
// metadata.  Returns a warp-uniform "bad" flag (an index out of range or a
// repeated write address); `first_mask` has bit w set for first touches.
//
// `row` indexes the [rows, W] / [rows, R] route tensors; `map_row` selects the
// bank's map row (they differ in the prefill, whose routes are [banks*T, ...]).
// Every index and weight is loaded in one round, every map entry in a second:
// two dependent memory round trips in all.  Lane l holds write slot l and read
// slots l, l+32, ... (R <= 32*RC).
//
// With `staged` (a per-warp shared buffer of N <= kStageSlots ints, N % 4 == 0)
// the bank's whole map row is copied into shared memory in the first round,
// so the map lookups cost no second dependent trip to memory.
// A token's raw routes, loaded into registers (lane w: write slot w; lane l:
// read slots l, l+32, ...) before anything depends on them.
template <int RC>
struct RouteRaw {
  int64_t wraw;
  float wwv;
  int64_t rraw[RC];
  float rwv[RC];
};

template <int RC>
__device__ __forceinline__ void load_route_raw(RouteRaw<RC>& q, const cow_step& st, int64_t row, int W, int R,
                                               int idx64, int adt, int lane) {
  q.wraw = 0;
  q.wwv = 0.f;
  if (lane < W) {
    q.wraw = ld_index(st.write_indices, row * W + lane, idx64);
    q.wwv = ld1_rt(st.write_weights, row * W + lane, adt);
  }
#pragma unroll
  for (int c = 0; c < RC; ++c) {
    const int r = c * 32 + lane;
    q.rraw[c] = 0;
    q.rwv[c] = 0.f;
    if (r < R) {
      q.rraw[c] = ld_index(st.read_indices, row * R + r, idx64);
      q.rwv[c] = ld1_rt(st.read_weights, row * R + r, adt);
    }
  }
}

// Validate raw routes, look their slots up in the map (`mrow`: the bank's
// dense map row, global or staged; `table`: its hashed table when log_t > 0)
// and write the warp's metadata.  Returns a warp-uniform "bad" flag (an index
// out of range or a repeated write address); `first_mask` has bit w set for
// first touches.
template <bool kDense, int RC, class M>
__device__ __forceinline__ bool finish_routes(M& sm, const RouteRaw<RC>& q, const int32_t* mrow,
                                              const unsigned long long* table, int log_t, int64_t N, int W, int R,
                                              int lane, unsigned& first_mask, int& error_bits) {
  const bool wok = lane < W && q.wraw >= 0 && q.wraw < N;
  bool bad = lane < W && !wok;
  const int wi = wok ? static_cast<int>(q.wraw) : 0;
  int wp = -1;
  if (!kDense && lane < W) wp = log_t ? hash_find(table, log_t, wi) : mrow[wi];
  int ri[RC], rp[RC];
#pragma unroll
  for (int c = 0; c < RC; ++c) {
    const int r = c * 32 + lane;
    const bool ok = q.rraw[c] >= 0 && q.rraw[c] < N;
    ri[c] = ok ? static_cast<int>(q.rraw[c]) : 0;
    rp[c] = -1;
    if (r < R) {
      bad |= !ok;
      if (!kDense) rp[c] = log_t ? hash_find(table, log_t, ri[c]) : mrow[ri[c]];
    }
  }
  // Out-of-range lanes get a unique sentinel so they never count as repeats.
  const unsigned same = __match_any_sync(kFull, wok ? wi : -1 - lane);
  const bool dup = wok && __popc(same) > 1;
  first_mask = __ballot_sync(kFull, lane < W && wp < 0 && !kDense);
  sm.widx[lane] = lane < W ? wi : -1;
  sm.wphys[lane] = wp;
  sm.ww[lane] = q.wwv;
  sm.fwt[lane] = 0.f;
  __syncwarp();
  // Reads of a slot written this step see the updated row (read-after-write,
  // allocator.py:1503-1517); its value is still in registers, so those reads
  // are folded into one weight per write slot (fwt) instead of reloading it.
  // Write slot of each read slot, if any: write slot w's address comes from
  // lane w by shuffle.
  int fwv[RC];
#pragma unroll
  for (int c = 0; c < RC; ++c) fwv[c] = -1;
  for (int w = 0; w < W; ++w) {
    const int waddr = __shfl_sync(kFull, wi, w);
#pragma unroll
    for (int c = 0; c < RC; ++c) fwv[c] = waddr == ri[c] ? w : fwv[c];
  }
#pragma unroll
  for (int c = 0; c < RC; ++c) {
    const int r = c * 32 + lane;
    if (r < R) {
      const int fw = fwv[c];
      sm.ridx[r] = ri[c];
      sm.rsrc[r] = fw >= 0 ? -(fw + 2) : (rp[c] >= 0 ? rp[c] : -1);
      sm.rw[r] = q.rwv[c];
      if (fw >= 0) atomicAdd(&sm.fwt[fw], q.rwv[c]);
    }
  }
  const bool any_dup = __any_sync(kFull, dup);
  const bool any_oob = __any_sync(kFull, bad);
  error_bits = (any_dup ? COW_ST_DUPLICATE_WRITE : 0) | (any_oob ? COW_ST_INDEX_RANGE : 0);
  __syncwarp();
  return any_dup || any_oob;
}

template <bool kDense, int RC, class M>
__device__ __forceinline__ bool load_routes(M& sm, const cow_step& st, const int32_t* map,
                                            int64_t row, int64_t map_row, int64_t N, int W, int R,
                                            int idx64, int adt, int lane, unsigned& first_mask,
                                            int& error_bits, int32_t* staged = nullptr, int log_t = 0) {
  // Hashed maps: `map` points at the pool's [banks, 2^log_t] uint64 tables.
  const unsigned long long* table =
      log_t ? reinterpret_cast<const unsigned long long*>(map) + (map_row << log_t) : nullptr;
  // The first 256 map entries come through registers (their latency is the
  // route loads' latency), any further ones through cp.async.
  constexpr int kRegStage = 2;
  int4 mtmp[kRegStage];
  if (!kDense && staged != nullptr) {
    const int4* src = reinterpret_cast<const int4*>(map + map_row * N);
#pragma unroll
    for (int k = 0; k < kRegStage; ++k) {
      const int i = lane + 32 * k;
      if (i < static_cast<int>(N >> 2)) mtmp[k] = __ldcg(src + i);
    }
    for (int i = lane + 32 * kRegStage; i < static_cast<int>(N >> 2); i += 32) cp_async16(staged + 4 * i, src + i);
  }
  RouteRaw<RC> q;
  load_route_raw<RC>(q, st, row, W, R, idx64, adt, lane);
  const int32_t* mrow = map + map_row * N;
  if (!kDense && staged != nullptr) {
#pragma unroll
    for (int k = 0; k < kRegStage; ++k) {
      const int i = lane + 32 * k;
      if (i < static_cast<int>(N >> 2)) reinterpret_cast<int4*>(staged)[i] = mtmp[k];
    }
    if (N > 128 * kRegStage) cp_async_wait_all();
    __syncwarp();
    mrow = staged;
  }
  return finish_routes<kDense, RC>(sm, q, mrow, table, log_t, N, W, R, lane, first_mask, error_bits);
}

// Gated-delta update of the W write rows (allocator.py:1489-1501): the rows
// arrive in `upd` (already loaded), leave as the updated values rounded to
// the slab dtype.
template <int SDT, int CH, int WMAX, class M>
__device__ __forceinline__ void gated_delta(float4 (&upd)[WMAX][CH], const M& sm, int W,
                                            float alpha, float in_g, float er_g,
                                            const float4 (&val)[CH], int lane, int D) {
  float4 ret[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) ret[c] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < WMAX; ++w) {
    if (w < W) {
      const float wt = sm.ww[w];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        upd[w][c] = f4_scale(alpha, upd[w][c]);
        ret[c] = f4_axpy(wt, upd[w][c], ret[c]);
      }
    }
  }
  float4 delta[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    delta[c] = make_float4(in_g * val[c].x - er_g * ret[c].x, in_g * val[c].y - er_g * ret[c].y,
                           in_g * val[c].z - er_g * ret[c].z, in_g * val[c].w - er_g * ret[c].w);
  }
#pragma unroll
  for (int w = 0; w < WMAX; ++w) {
    if (w < W) {
      const float wt = sm.ww[w];
#pragma unroll
      for (int c = 0; c < CH; ++c) upd[w][c] = Elem<SDT>::round4(f4_axpy(wt, delta[c], upd[w][c]));
    }
  }
  (void)lane;
  (void)D;
}

// Weighted sparse read after the write (allocator.py:1507-1517), in pieces so
// the first group of read rows can be requested together with the write rows.
// Rows of slots written this step come from registers (add_forwarded); the
// rest from the slab / dense table (src >= 0) or M0 (src == -1).
template <int CH>
struct ReadGroup {
  static constexpr int G = CH >= 4 ? 4 : 16 / CH;
};

template <int SDT, int CH, class M>
__device__ __forceinline__ void load_read_group(float4 (&v)[ReadGroup<CH>::G][CH], float (&wt)[ReadGroup<CH>::G],
                                                const M& sm, int r0, int R, const void* rows,
                                                int64_t row_base, const float* m0, int64_t m0_base, int lane,
                                                int D) {
  constexpr int G = ReadGroup<CH>::G;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int r = r0 + j;
    const int src = r < R ? sm.rsrc[r] : -2;
    wt[j] = src >= -1 ? sm.rw[r] : 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int col = (c * 32 + lane) * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col < D) {
        if (src >= 0) x = Elem<SDT>::ld4(rows, (row_base + src) * D + col);
        else if (src == -1) x = ld4_m0(m0, (m0_base + sm.ridx[r]) * D + col);
      }
      v[j][c] = x;
    }
  }
}

template <int CH>
__device__ __forceinline__ void accumulate_group(float4 (&acc)[CH], const float4 (&v)[ReadGroup<CH>::G][CH],
                                                 const float (&wt)[ReadGroup<CH>::G]) {
#pragma unroll
  for (int j = 0; j < ReadGroup<CH>::G; ++j) {
#pragma unroll
    for (int c = 0; c < CH; ++c) acc[c] = f4_axpy(wt[j], v[j][c], acc[c]);
  }
}

// Groups after the first: load and accumulate in turn.
template <int SDT, int CH, class M>
__device__ __forceinline__ void read_remaining(float4 (&acc)[CH], const M& sm, int R, const void* rows,
                                               int64_t row_base, const float* m0, int64_t m0_base, int lane,
                                               int D) {
  constexpr int G = ReadGroup<CH>::G;
  for (int r0 = G; r0 < R; r0 += G) {
    float4 v[G][CH];
    float wt[G];
    load_read_group<SDT, CH>(v, wt, sm, r0, R, rows, row_base, m0, m0_base, lane, D);
    accumulate_group<CH>(acc, v, wt);
  }
}

template <int CH, int WMAX, class M>
__device__ __forceinline__ void add_forwarded(float4 (&acc)[CH], const float4 (&upd)[WMAX][CH], const M& sm,
                                              int W) {
#pragma unroll
  for (int w = 0; w < WMAX; ++w) {
    if (w < W) {
      const float f = sm.fwt[w];
#pragma unroll
      for (int c = 0; c < CH; ++c) acc[c] = f4_axpy(f, upd[w][c], acc[c]);
    }
  }
}

// --------------------------------------------------------------------------
// host helpers
// --------------------------------------------------------------------------

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

// Last CUDA error seen by an entry point on this host thread (cow_last_error).
namespace cowrt {
extern thread_local int last_cuda_error;
}  // namespace cowrt

namespace {

inline int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return COW_OK;
  cowrt::last_cuda_error = static_cast<int>(e);
  return COW_ERR_CUDA;
}

inline int grid_for(int64_t n, int threads, int max_blocks = 148 * 16) {
  int64_t b = (n + threads - 1) / threads;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool valid_dtype(int dt) { return dt == COW_F32 || dt == COW_BF16 || dt == COW_F16; }
inline int elem_size(int dt) { return dt == COW_F32 ? 4 : 2; }
inline bool row_aligned(const void* p, int dt) {
  // 4-element row vectors need 16-byte (f32) or 8-byte (16-bit) alignment.
  return (reinterpret_cast<uintptr_t>(p) & static_cast<uintptr_t>(4 * elem_size(dt) - 1)) == 0;
}

inline int width_chunks(int64_t width) {
  if (width <= 128) return 1;
  if (width <= 256) return 2;
  return 4;
}

inline bool check_step_shape(int64_t width, int writes, int reads) {
  return width > 0 && width % 4 == 0 && width <= COW_MAX_WIDTH && writes >= 1 && writes <= COW_MAX_WRITES &&
         reads >= 1 && reads <= COW_MAX_READS;
}

// Entry points other than the decode step work on dense [banks, slots] maps.
inline bool dense_maps(const cow_pool* p, int64_t n) {
  for (int64_t i = 0; p != nullptr && i < n; ++i)
    if (p[i].map_kind != COW_MAP_DENSE) return false;
  return true;
}

inline bool check_step_ptrs(const cow_step& s, int adt) {
  return s.write_indices && s.write_weights && s.values && s.input_gate && s.erase_gate && s.forget_log_gate &&
         s.read_indices && s.read_weights && s.output && row_aligned(s.values, adt) && row_aligned(s.output, adt);
}

// Kernel variants: slab dtype x row chunks (width <= 128/256/512) x route
// capacity (W <= 4 and R <= 32; W <= 8 and R <= 32; W <= 32 and R <= 256).
#define COW_VARIANT(KERNEL, SDT_, CH_, RV) \
  (RV == 0 ? KERNEL<SDT_, CH_, 4, 1> : (RV == 1 ? KERNEL<SDT_, CH_, 8, 1> : KERNEL<SDT_, CH_, 32, 8>))
#define COW_SELECT_KERNEL(KERNEL, SDT, CH, RV, FN)                                                            \
  do {                                                                                                       \
    if (SDT == COW_F32) {                                                                                    \
      FN = CH == 1 ? COW_VARIANT(KERNEL, COW_F32, 1, RV)                                                     \
                   : (CH == 2 ? COW_VARIANT(KERNEL, COW_F32, 2, RV) : COW_VARIANT(KERNEL, COW_F32, 4, RV));  \
    } else if (SDT == COW_BF16) {                                                                            \
      FN = CH == 1 ? COW_VARIANT(KERNEL, COW_BF16, 1, RV)                                                    \
                   : (CH == 2 ? COW_VARIANT(KERNEL, COW_BF16, 2, RV) : COW_VARIANT(KERNEL, COW_BF16, 4, RV)); \
    } else {                                                                                                 \
      FN = CH == 1 ? COW_VARIANT(KERNEL, COW_F16, 1, RV)                                                     \
                   : (CH == 2 ? COW_VARIANT(KERNEL, COW_F16, 2, RV) : COW_VARIANT(KERNEL, COW_F16, 4, RV));  \
    }                                                                                                        \
  } while (0)

// Route variant: 0 (W <= 4, R <= 32), 1 (W <= 8, R <= 32), 2 (W <= 32, R <= 256).
inline int route_variant(int writes, int reads) { return reads > 32 || writes > 8 ? 2 : (writes > 4 ? 1 : 0); }

// The common shapes (f32 rows, R <= 32, width <= 128) stage their read rows in shared
// memory with cp.async instead of registers: dynamic shared memory bytes per
// block for that staging (0 for other shapes).
inline size_t read_stage_bytes(int reads, int64_t width, int ch, int rv, int dtype) {
  return (rv <= 1 && ch == 1 && dtype == COW_F32) ? static_cast<size_t>(kBanksPerCta) * reads * width * sizeof(float) : 0;
}

// Blocks of `fn` (with `smem` dynamic shared memory) that fit on the current
// device at once, cached per device / kernel / size; raises the kernel's
// dynamic shared memory limit when it needs more than the default 48 KiB.
inline int resident_blocks(const void* fn, int threads, size_t smem) {
  struct Entry {
    int device;
    const void* fn;
    size_t smem;
    int blocks;
  };
  static Entry cache[128];
  static int used = 0;
  static std::mutex mu;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].device == device && cache[i].fn == fn && cache[i].smem == smem) return cache[i].blocks;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  const int blocks = sms * per_sm;
  if (used < 128) cache[used++] = Entry{device, fn, smem, blocks};
  return blocks;
}

}  // namespace
