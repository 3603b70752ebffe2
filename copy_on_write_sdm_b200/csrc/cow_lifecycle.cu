// cow_lifecycle.cu -- allocator lifecycle kernels: init, pack, grow, release, repack,
// append, retain, validate, materialize.
//
// Every multi-step operation runs for up to COW_MAX_LAYERS independent pools in
// one set of launches: grid.y (or grid.x for the one-CTA-per-pool kernels) is
// the pool, and the per-pool arguments travel in a __grid_constant__ array.
// The single-pool entry points are the same code with one pool.

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// ordered prefix-count machinery for the lifecycle operations
// --------------------------------------------------------------------------

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanSeg = kScanThreads * kScanItems;
constexpr int kScanHeader = 8;  // int32 slots before the per-block offsets

enum ScanOp : int { kOpPack = 0, kOpRepack = 1, kOpAppend = 2, kOpRelease = 3, kOpAdmit = 4 };

struct ScanCtx {
  int op;
  int64_t n, slots;
  const int32_t* map;        // pack / repack / append: the map being scanned
  const int64_t* bank_idx;   // release: selected banks, in the caller's order
  int32_t* pool_map;         // release: map rows to clear
  int32_t* out_map;          // pack: in place; repack: new map; append: admitted map
  int32_t* src_rows;
  int32_t* dst_rows;
  int32_t* free_rows;
  int32_t* free_count;       // release / append: updated; pack: only read into free_out
  const int32_t* gate_status;  // release: skip everything when the bank list was bad
  int32_t* scratch;            // [0]=total, [1]=old free count, [kScanHeader..] block offsets
  int32_t* total_out;          // optional copy of the total
  int32_t* free_out;           // optional copy of the free count before the operation
};

struct ScanLaunch {
  ScanCtx c[COW_MAX_LAYERS];
  int32_t layers;
};

__host__ __device__ inline int64_t scan_blocks_of(int64_t n) { return (n + kScanSeg - 1) / kScanSeg; }

__device__ __forceinline__ bool scan_flag(const ScanCtx& c, int64_t i) {
  if (c.op == kOpRelease) {
    if (c.gate_status != nullptr && (*c.gate_status & COW_ST_BAD_BANK_LIST)) return false;
    const int64_t b = c.bank_idx[i / c.slots];
    return c.pool_map[b * c.slots + i % c.slots] >= 0;
  }
  return c.map[i] >= 0;
}

__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
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
    int w = lane < (kScanThreads / 32) ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, w, o);
      if (lane >= o) w += y;
    }
    if (lane < (kScanThreads / 32)) s_warp[lane] = w;
  }
  __syncthreads();
  total = s_warp[kScanThreads / 32 - 1];
  const int before = warp > 0 ? s_warp[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

// grid (max blocks over pools, pools); a block past its pool's extent exits whole.
__global__ void __launch_bounds__(kScanThreads) scan_count_kernel(const __grid_constant__ ScanLaunch L) {
  const ScanCtx& c = L.c[blockIdx.y];
  if (static_cast<int64_t>(blockIdx.x) >= scan_blocks_of(c.n)) return;
  __shared__ int s_warp[kScanThreads / 32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanSeg + static_cast<int64_t>(threadIdx.x) * kScanItems;
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + k;
    if (i < c.n && scan_flag(c, i)) ++cnt;
  }
  int total;
  block_exclusive_scan(cnt, s_warp, total);
  if (threadIdx.x == 0) c.scratch[kScanHeader + blockIdx.x] = total;
}

// One CTA per pool: exclusive scan of the per-block counts, total, and the
// free count bookkeeping of release (push) / append (pop).
__global__ void __launch_bounds__(1024) scan_blocks_kernel(const __grid_constant__ ScanLaunch L) {
  const ScanCtx& c = L.c[blockIdx.x];
  const int64_t nblocks = scan_blocks_of(c.n);
  __shared__ int s_part[1024];
  const int64_t per = (nblocks + 1023) / 1024;
  const int64_t b0 = threadIdx.x * per;
  int sum = 0;
  for (int64_t b = b0; b < b0 + per && b < nblocks; ++b) sum += c.scratch[kScanHeader + b];
  s_part[threadIdx.x] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int v = threadIdx.x >= o ? s_part[threadIdx.x - o] : 0;
    __syncthreads();
    s_part[threadIdx.x] += v;
    __syncthreads();
  }
  int run = s_part[threadIdx.x] - sum;
  for (int64_t b = b0; b < b0 + per && b < nblocks; ++b) {
    const int v = c.scratch[kScanHeader + b];
    c.scratch[kScanHeader + b] = run;
    run += v;
  }
  if (threadIdx.x == 1023) {
    const int total = s_part[1023];
    c.scratch[0] = total;
    if (c.total_out != nullptr) *c.total_out = total;
    if (c.free_count != nullptr) {
      const int old = *c.free_count;
      c.scratch[1] = old;
      if (c.free_out != nullptr) *c.free_out = old;
      if (c.op == kOpRelease) *c.free_count = old + total;
      if (c.op == kOpAppend || c.op == kOpAdmit) *c.free_count = old - total;
    }
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const __grid_constant__ ScanLaunch L) {
  const ScanCtx& c = L.c[blockIdx.y];
  if (static_cast<int64_t>(blockIdx.x) >= scan_blocks_of(c.n)) return;
  __shared__ int s_warp[kScanThreads / 32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanSeg + static_cast<int64_t>(threadIdx.x) * kScanItems;
  bool f[kScanItems];
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + k;
    f[k] = i < c.n && scan_flag(c, i);
    cnt += f[k];
  }
  int total;
  int rank = block_exclusive_scan(cnt, s_warp, total) + c.scratch[kScanHeader + blockIdx.x];
  const int old_free = c.scratch[1];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int64_t i = base + k;
    if (i >= c.n) break;
    switch (c.op) {
      case kOpPack:
        c.out_map[i] = f[k] ? rank : -1;
        if (f[k]) c.src_rows[rank] = static_cast<int32_t>(i);
        break;
      case kOpRepack:
        if (f[k]) c.src_rows[rank] = c.map[i];
        c.out_map[i] = f[k] ? rank : -1;
        break;
      case kOpAppend:
        if (f[k]) {
          const int dst = c.free_rows[old_free - 1 - rank];
          c.src_rows[rank] = c.map[i];
          c.dst_rows[rank] = dst;
          c.out_map[i] = dst;
        } else {
          c.out_map[i] = -1;
        }
        break;
      case kOpAdmit:  // append's pops, rows to come from M0 (source = flat bank*slots+slot)
        if (f[k]) {
          const int dst = c.free_rows[old_free - 1 - rank];
          c.src_rows[rank] = static_cast<int32_t>(i);
          c.dst_rows[rank] = dst;
          c.out_map[i] = dst;
        } else {
          c.out_map[i] = -1;
        }
        break;
      case kOpRelease: {
        if (c.gate_status != nullptr && (*c.gate_status & COW_ST_BAD_BANK_LIST)) break;
        const int64_t b = c.bank_idx[i / c.slots];
        int32_t* e = &c.pool_map[b * c.slots + i % c.slots];
        if (f[k]) c.free_rows[old_free + rank] = *e;
        *e = -1;
        break;
      }
    }
    rank += f[k];
  }
}

// --------------------------------------------------------------------------
// per-pool argument arrays of the small kernels
// --------------------------------------------------------------------------

template <typename T>
struct Layers {
  T c[COW_MAX_LAYERS];
  int32_t layers;
};

struct FillFreeCtx {  // free_rows[:cap - A] = arange(A, cap), A = *live
  int32_t* free_rows;
  int64_t cap;
  int32_t* free_count;
  int32_t* status;
  const int32_t* live;
};

struct CopyCtx {  // see copy_rows_kernel
  void* dst;
  const int32_t* dst_rows;
  const void* src;
  const int32_t* src_rows;
  const int32_t* count_dev;  // when set, rows [*count_dev, count) are skipped
  const float* m0;
  const int64_t* templates;
  int64_t count, width, slots;
  int32_t dst_dt, src_dt, mode, _pad;
};

struct MarkCtx {
  const void* widx;
  int32_t* map;
  int32_t* status;
  const void* ridx;  // read routes [banks,T,R] checked for range (may be null)
};

struct BankListCtx {
  const int64_t* idx;
  int64_t count, banks;
  int32_t* mask;
  int32_t* status;
};

struct StatusOrCtx {
  int32_t* status;
  const int32_t* bits;
};

struct RetainCtx {
  const int32_t* map;
  const int64_t* templates;
  const int64_t* idx;
  int64_t count, slots, banks;
  const int32_t* mask;
  int32_t* new_map;
  int64_t* new_templates;
  int32_t* status;
};

struct ValidateCtx {
  const int32_t* map;
  int64_t map_n, cap;
  const int32_t* free_rows;
  const int32_t* free_count;
  int32_t* counts;
  int32_t* status;       // validate bits
  const int32_t* pool_status;
  int32_t* out;          // [pool status, validate bits, free count]
};

#define COW_GRID_STRIDE(i, n)                                                                      \
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,                    \
               i##_stride = static_cast<int64_t>(gridDim.x) * blockDim.x;                          \
       i < (n); i += i##_stride)

// --------------------------------------------------------------------------
// small kernels (grid.y = pool)
// --------------------------------------------------------------------------

__global__ void init_pool_kernel(int32_t* map, int64_t map_n, int32_t* free_rows, int64_t cap,
                                 int32_t* free_count, int32_t* status) {
  const int64_t m = map_n > cap ? map_n : cap;
  COW_GRID_STRIDE(i, m) {
    if (i < map_n) map[i] = -1;
    if (i < cap) free_rows[i] = static_cast<int32_t>(i);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *free_count = static_cast<int32_t>(cap);
    *status = 0;
  }
}

__global__ void fill_free_kernel(const __grid_constant__ Layers<FillFreeCtx> L) {
  const FillFreeCtx& c = L.c[blockIdx.y];
  const int64_t a = *c.live;
  COW_GRID_STRIDE(j, c.cap - a) { c.free_rows[j] = static_cast<int32_t>(a + j); }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *c.free_count = static_cast<int32_t>(c.cap - a);
    if (c.status != nullptr) *c.status = 0;
  }
}

__global__ void mask_to_map_kernel(const uint8_t* active, int64_t n, int32_t* map) {
  COW_GRID_STRIDE(i, n) { map[i] = active[i] ? 0 : -1; }
}

__global__ void prefill_mark_kernel(const __grid_constant__ Layers<MarkCtx> L, int idx64, int64_t banks, int64_t time,
                                    int writes, int64_t slots, int reads) {
  const MarkCtx& c = L.c[blockIdx.y];
  if (c.ridx != nullptr) {
    COW_GRID_STRIDE(i, banks * time * reads) {
      const int64_t r = ld_index(c.ridx, i, idx64);
      if (r < 0 || r >= slots) atomicOr(c.status, COW_ST_INDEX_RANGE);
    }
  }
  COW_GRID_STRIDE(i, banks * time * writes) {
    const int64_t bank = i / (time * writes);
    const int64_t s = ld_index(c.widx, i, idx64);
    if (s < 0 || s >= slots) {
      atomicOr(c.status, COW_ST_INDEX_RANGE);
      continue;
    }
    // A token that writes one slot twice is refused before anything is placed.
    const int w = static_cast<int>(i % writes);
    for (int j = 0; j < w; ++j) {
      if (ld_index(c.widx, i - w + j, idx64) == s) atomicOr(c.status, COW_ST_DUPLICATE_WRITE);
    }
    c.map[bank * slots + s] = 0;
  }
}

// One warp per row; 16-byte vectors when both dtypes allow it.  mode 0: row
// src_rows[k] of src; mode 1: src_rows[k] is a flat bank*slots+slot index and
// the row comes from m0[templates[bank], slot].
constexpr int kCopyRowsPerWarp = 4;  // rows a warp moves per iteration, their loads in flight together

__global__ void copy_rows_kernel(const __grid_constant__ Layers<CopyCtx> L) {
  const CopyCtx& c = L.c[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const int64_t count = c.count_dev != nullptr ? min(c.count, static_cast<int64_t>(*c.count_dev)) : c.count;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t width = c.width;
  const void* sbase = c.mode == 1 ? static_cast<const void*>(c.m0) : c.src;
  const int sdt = c.mode == 1 ? static_cast<int>(COW_F32) : c.src_dt;
  const bool small = c.slots > 0 && c.slots < (int64_t{1} << 31);
  for (int64_t k0 = (blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5)) * kCopyRowsPerWarp;
       k0 < count; k0 += warps * kCopyRowsPerWarp) {
    int64_t d[kCopyRowsPerWarp], s[kCopyRowsPerWarp];
#pragma unroll
    for (int u = 0; u < kCopyRowsPerWarp; ++u) {
      const int64_t k = k0 + u < count ? k0 + u : count - 1;  // a clamped duplicate rewrites the same row
      d[u] = c.dst_rows ? c.dst_rows[k] : k;
      if (c.mode == 1) {
        const int64_t flat = c.src_rows[k];
        int64_t bank, slot;
        if (small && flat >= 0 && flat < (int64_t{1} << 31)) {
          const uint32_t f = static_cast<uint32_t>(flat), n = static_cast<uint32_t>(c.slots);
          bank = f / n;
          slot = f - static_cast<uint32_t>(bank) * n;
        } else {
          bank = flat / c.slots;
          slot = flat % c.slots;
        }
        s[u] = c.templates[bank] * c.slots + slot;
      } else {
        s[u] = c.src_rows ? c.src_rows[k] : k;
      }
    }
    if ((width & 3) == 0) {
      for (int64_t e = lane * 4; e < width; e += 128) {
        float4 v[kCopyRowsPerWarp];
#pragma unroll
        for (int u = 0; u < kCopyRowsPerWarp; ++u) v[u] = ld4_rt(sbase, s[u] * width + e, sdt);
#pragma unroll
        for (int u = 0; u < kCopyRowsPerWarp; ++u) st4_rt(c.dst, d[u] * width + e, v[u], c.dst_dt);
      }
    } else {
#pragma unroll
      for (int u = 0; u < kCopyRowsPerWarp; ++u) {
        for (int64_t e = lane; e < width; e += 32) {
          const float v = ld1_rt(sbase, s[u] * width + e, sdt);
          if (c.dst_dt == COW_F32) static_cast<float*>(c.dst)[d[u] * width + e] = v;
          else if (c.dst_dt == COW_BF16) static_cast<__nv_bfloat16*>(c.dst)[d[u] * width + e] = __float2bfloat16_rn(v);
          else static_cast<__half*>(c.dst)[d[u] * width + e] = __float2half_rn(v);
        }
      }
    }
  }
}

__global__ void grow_kernel(const void* old_slab, const int32_t* old_free_rows, int64_t old_cap, void* new_slab,
                            int32_t* new_free_rows, int64_t new_cap, int64_t row_bytes, int32_t* free_count,
                            int32_t* status) {
  // Byte copy of the old slab (16-byte words; row_bytes*old_cap is a multiple
  // of 16 whenever width*elem is), then the free stack.
  const int64_t bytes = row_bytes * old_cap;
  if ((bytes & 15) == 0) {
    const int4* s = static_cast<const int4*>(old_slab);
    int4* d = static_cast<int4*>(new_slab);
    COW_GRID_STRIDE(i, bytes / 16) { d[i] = s[i]; }
  } else {
    const uint8_t* s = static_cast<const uint8_t*>(old_slab);
    uint8_t* d = static_cast<uint8_t*>(new_slab);
    COW_GRID_STRIDE(i, bytes) { d[i] = s[i]; }
  }
  const int64_t old_free = *free_count;
  const int64_t added = new_cap - old_cap;
  COW_GRID_STRIDE(i, old_free + added) {
    new_free_rows[i] = i < old_free ? old_free_rows[i] : static_cast<int32_t>(old_cap + (i - old_free));
  }
}

// Growth inside reserved storage: the slab rows old_cap..new_cap-1 already exist,
// so only their ids are pushed above the current free entries, in the order the
// copying growth gives them.
__global__ void grow_append_kernel(int32_t* free_rows, int64_t old_cap, int64_t new_cap, const int32_t* free_count) {
  const int64_t old_free = *free_count;
  COW_GRID_STRIDE(i, new_cap - old_cap) { free_rows[old_free + i] = static_cast<int32_t>(old_cap + i); }
}

__global__ void grow_finish_kernel(int32_t* free_count, int64_t added, int32_t* status) {
  *free_count += static_cast<int32_t>(added);
  *status = 0;
}

__global__ void bank_list_kernel(const __grid_constant__ Layers<BankListCtx> L) {
  const BankListCtx& c = L.c[blockIdx.y];
  COW_GRID_STRIDE(s, c.count) {
    const int64_t b = c.idx[s];
    if (b < 0 || b >= c.banks) {
      atomicOr(c.status, COW_ST_BAD_BANK_LIST);
      continue;
    }
    if (atomicAdd(&c.mask[b], 1) != 0) atomicOr(c.status, COW_ST_BAD_BANK_LIST);
  }
}

__global__ void status_or_kernel(const __grid_constant__ Layers<StatusOrCtx> L) {
  const StatusOrCtx& c = L.c[blockIdx.y];
  if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(c.status, *c.bits);
}

// One warp per bank row of the map.  Rows of 16-byte multiples (slots % 4 == 0,
// the map 16-byte aligned) move as int4 words, four in flight per lane.
__device__ __forceinline__ bool map_row_vec(const int32_t* map, int64_t slots) {
  return (slots & 3) == 0 && (reinterpret_cast<uintptr_t>(map) & 15) == 0;
}

// A bank that is not retained must hold no live rows (release cleared them);
// retained banks are not read at all.
__global__ void retain_check_kernel(const __grid_constant__ Layers<RetainCtx> L) {
  const RetainCtx& c = L.c[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const bool vec = map_row_vec(c.map, c.slots);
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); b < c.banks;
       b += warps) {
    if (c.mask[b]) continue;
    const int32_t* row = c.map + b * c.slots;
    bool live = false;
    if (vec) {
      const int4* r4 = reinterpret_cast<const int4*>(row);
#pragma unroll 4
      for (int64_t j = lane; j < c.slots / 4; j += 32) {
        const int4 v = r4[j];
        live |= (v.x >= 0) | (v.y >= 0) | (v.z >= 0) | (v.w >= 0);
      }
    } else {
      for (int64_t j = lane; j < c.slots; j += 32) live |= row[j] >= 0;
    }
    if (__any_sync(kFull, live) && lane == 0) atomicOr(c.status, COW_ST_DISCARD_LIVE);
  }
}

// Survivor s takes bank idx[s]'s map row and template, in list order.
__global__ void retain_gather_kernel(const __grid_constant__ Layers<RetainCtx> L) {
  const RetainCtx& c = L.c[blockIdx.y];
  if (c.banks == 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const bool vec = map_row_vec(c.map, c.slots) && map_row_vec(c.new_map, c.slots);
  for (int64_t s = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); s < c.count;
       s += warps) {
    int64_t b = c.idx[s];
    b = b < 0 ? 0 : (b >= c.banks ? c.banks - 1 : b);
    const int32_t* src = c.map + b * c.slots;
    int32_t* dst = c.new_map + s * c.slots;
    if (vec) {
      const int4* s4 = reinterpret_cast<const int4*>(src);
      int4* d4 = reinterpret_cast<int4*>(dst);
#pragma unroll 4
      for (int64_t j = lane; j < c.slots / 4; j += 32) d4[j] = s4[j];
    } else {
      for (int64_t j = lane; j < c.slots; j += 32) dst[j] = src[j];
    }
    if (lane == 0) c.new_templates[s] = c.templates[b];
  }
}

__global__ void validate_count_kernel(const __grid_constant__ Layers<ValidateCtx> L) {
  const ValidateCtx& c = L.c[blockIdx.y];
  const int64_t fc = *c.free_count;
  if (blockIdx.x == 0 && threadIdx.x == 0 && (fc < 0 || fc > c.cap)) atomicOr(c.status, COW_ST_ROW_RANGE);
  COW_GRID_STRIDE(i, c.map_n) {
    const int32_t v = c.map[i];
    if (v < 0) continue;
    if (v >= c.cap) {
      atomicOr(c.status, COW_ST_ROW_RANGE);
      continue;
    }
    atomicAdd(&c.counts[v], 1);
  }
  const int64_t fcl = fc < 0 ? 0 : (fc > c.cap ? c.cap : fc);
  COW_GRID_STRIDE(i, fcl) {
    const int32_t v = c.free_rows[i];
    if (v < 0 || v >= c.cap) {
      atomicOr(c.status, COW_ST_ROW_RANGE);
      continue;
    }
    atomicAdd(&c.counts[v], 1 << 16);
  }
}

__global__ void validate_check_kernel(const __grid_constant__ Layers<ValidateCtx> L) {
  const ValidateCtx& c = L.c[blockIdx.y];
  int bits = 0;
  COW_GRID_STRIDE(i, c.cap) {
    const int v = c.counts[i];
    const int a = v & 0xffff, f = v >> 16;
    if (a > 1) bits |= COW_ST_MULTI_OWNER;
    if (f > 1) bits |= COW_ST_FREE_DUPLICATE;
    if (a + f == 0) bits |= COW_ST_NOT_COVERED;
    if (a >= 1 && f >= 1) bits |= COW_ST_NOT_COVERED;
  }
  if (bits) atomicOr(c.status, bits);
}

// After the checks: [pool status, validate bits, free count] per pool.
__global__ void validate_report_kernel(const __grid_constant__ Layers<ValidateCtx> L) {
  if (threadIdx.x >= L.layers) return;
  const ValidateCtx& c = L.c[threadIdx.x];
  if (c.out != nullptr) {
    c.out[0] = *c.pool_status;
    c.out[1] = *c.status;
    c.out[2] = *c.free_count;
  }
}

__global__ void materialize_kernel(const float* m0, const int64_t* templates, const void* slab, int slab_dt,
                                   const int32_t* map, int64_t banks, int64_t slots, int64_t width, void* out,
                                   int out_dt) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = banks * slots;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); k < rows; k += warps) {
    const int32_t p = map[k];
    const int64_t b = k / slots, s = k % slots;
    for (int64_t e = lane * 4; e < width; e += 128) {
      float4 v = p >= 0 ? ld4_rt(slab, static_cast<int64_t>(p) * width + e, slab_dt)
                        : ld4_m0(m0, (templates[b] * slots + s) * width + e);
      st4_rt(out, k * width + e, v, out_dt);
    }
  }
}

// --------------------------------------------------------------------------
// launch helpers
// --------------------------------------------------------------------------

dim3 layer_grid(int64_t max_n, int threads, int layers) {
  return dim3(static_cast<unsigned>(grid_for(max_n, threads)), static_cast<unsigned>(layers));
}

int run_scan_count(const ScanLaunch& L, cudaStream_t st) {
  int64_t nb = 0;
  for (int l = 0; l < L.layers; ++l) nb = std::max<int64_t>(nb, scan_blocks_of(L.c[l].n));
  if (nb > 0) {
    scan_count_kernel<<<dim3(static_cast<unsigned>(nb), L.layers), kScanThreads, 0, st>>>(L);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  scan_blocks_kernel<<<L.layers, 1024, 0, st>>>(L);
  return launch_status();
}

int run_scan_apply(const ScanLaunch& L, cudaStream_t st) {
  int64_t nb = 0;
  for (int l = 0; l < L.layers; ++l) nb = std::max<int64_t>(nb, scan_blocks_of(L.c[l].n));
  if (nb == 0) return COW_OK;
  scan_apply_kernel<<<dim3(static_cast<unsigned>(nb), L.layers), kScanThreads, 0, st>>>(L);
  return launch_status();
}

int run_copy_rows(const Layers<CopyCtx>& L, cudaStream_t st) {
  int64_t m = 0;
  for (int l = 0; l < L.layers; ++l) m = std::max<int64_t>(m, L.c[l].count);
  if (m == 0) return COW_OK;
  copy_rows_kernel<<<layer_grid(m * 32, 256, L.layers), 256, 0, st>>>(L);
  return launch_status();
}

bool copy_args_ok(const CopyCtx& c) {
  if (c.count == 0) return true;
  if (!c.dst || c.count < 0 || c.width < 1 || !valid_dtype(c.dst_dt)) return false;
  if (c.mode == 1)
    return c.m0 && c.templates && c.src_rows && c.slots >= 1 && c.width % 4 == 0 && aligned16(c.m0);
  if (c.mode != 0 || !c.src || !valid_dtype(c.src_dt)) return false;
  return c.width % 4 != 0 || (row_aligned(c.src, c.src_dt) && row_aligned(c.dst, c.dst_dt));
}

// Workspace layouts, in int32 words, every region rounded up to 16 bytes.
inline int64_t words16(int64_t words) { return (words + 3) / 4 * 4; }
inline int64_t scan_words(int64_t n) { return words16(scan_blocks_of(n) + kScanHeader); }

bool layers_ok(const cow_pool* pools, int32_t layers) {
  if (!pools || layers < 1 || layers > COW_MAX_LAYERS) return false;
  for (int l = 0; l < layers; ++l)
    if (pools[l].banks < 0 || pools[l].slots < 1 || pools[l].capacity < 0) return false;
  return true;
}

bool workspace_ok(const void* ws, int64_t have, int64_t need) {
  return ws != nullptr && aligned16(ws) && have >= need;
}

}  // namespace

extern "C" {

int64_t cow_scan_blocks(int64_t n) { return scan_blocks_of(n) + kScanHeader; }

int cow_init_pool(const cow_pool* p, void* stream) {
  if (!dense_maps(p, 1)) return COW_ERR_UNSUPPORTED;
  if (!p || !p->map || !p->free_rows || !p->free_count || !p->status || p->capacity < 0 || p->banks < 0)
    return COW_ERR_INVALID;
  const int64_t n = p->banks * p->slots;
  const int64_t m = n > p->capacity ? n : p->capacity;
  init_pool_kernel<<<grid_for(m, 256), 256, 0, as_stream(stream)>>>(p->map, n, p->free_rows, p->capacity,
                                                                   p->free_count, p->status);
  return launch_status();
}

int cow_prefill_mark(const void* write_indices, int32_t index_dtype, int64_t banks, int64_t time, int32_t writes,
                     int64_t slots, int32_t* map, int32_t* status, void* stream) {
  if (!write_indices || !map || !status || banks < 0 || time < 0 || writes < 1 || slots < 1) return COW_ERR_INVALID;
  const int64_t n = banks * time * writes;
  if (n == 0) return COW_OK;
  Layers<MarkCtx> L{};
  L.c[0] = MarkCtx{write_indices, map, status, nullptr};
  L.layers = 1;
  prefill_mark_kernel<<<layer_grid(n, 256, 1), 256, 0, as_stream(stream)>>>(L, index_dtype == COW_I64, banks, time,
                                                                         writes, slots, 0);
  return launch_status();
}

int cow_mask_to_map(const uint8_t* active, int64_t n, int32_t* map, void* stream) {
  if ((!active || !map) && n > 0) return COW_ERR_INVALID;
  if (n == 0) return COW_OK;
  mask_to_map_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(active, n, map);
  return launch_status();
}

int cow_pack_count(const int32_t* map, int64_t n, int32_t* flags_scratch, void* stream) {
  if ((!map && n > 0) || !flags_scratch || n < 0) return COW_ERR_INVALID;
  ScanLaunch L{};
  L.layers = 1;
  ScanCtx& c = L.c[0];
  c.op = kOpPack;
  c.n = n;
  c.slots = 1;
  c.map = map;
  c.scratch = flags_scratch;
  return run_scan_count(L, as_stream(stream));
}

int cow_pack_apply(int32_t* map, int64_t n, int32_t* src_index, const cow_pool* pool, int32_t* flags_scratch,
                   void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if ((!map && n > 0) || !pool || !flags_scratch || !src_index) return COW_ERR_INVALID;
  ScanLaunch L{};
  L.layers = 1;
  ScanCtx& c = L.c[0];
  c.op = kOpPack;
  c.n = n;
  c.slots = 1;
  c.map = map;
  c.out_map = map;
  c.src_rows = src_index;
  c.scratch = flags_scratch;
  cudaStream_t st = as_stream(stream);
  int rc = run_scan_apply(L, st);
  if (rc != COW_OK) return rc;
  Layers<FillFreeCtx> F{};
  F.c[0] = FillFreeCtx{pool->free_rows, pool->capacity, pool->free_count, pool->status, flags_scratch};
  F.layers = 1;
  fill_free_kernel<<<layer_grid(pool->capacity, 256, 1), 256, 0, st>>>(F);
  return launch_status();
}

int cow_copy_rows(void* dst, int32_t dst_dtype, const int32_t* dst_rows, const void* src, int32_t src_dtype,
                  const int32_t* src_rows, int64_t count, int64_t width, int32_t mode, const float* m0,
                  const int64_t* templates, int64_t slots, void* stream) {
  Layers<CopyCtx> L{};
  L.c[0] = CopyCtx{dst, dst_rows, src, src_rows, nullptr, m0, templates, count, width, slots,
                   dst_dtype, src_dtype, mode, 0};
  L.layers = 1;
  if (!copy_args_ok(L.c[0])) return COW_ERR_INVALID;
  return run_copy_rows(L, as_stream(stream));
}

int cow_grow(const void* old_slab, const int32_t* old_free_rows, int64_t old_capacity, void* new_slab,
             int32_t* new_free_rows, int64_t new_capacity, int64_t width, int32_t slab_dtype, int32_t* free_count,
             int32_t* status, void* stream) {
  if (!old_slab || !old_free_rows || !new_slab || !new_free_rows || !free_count || !status ||
      new_capacity < old_capacity || !valid_dtype(slab_dtype) || width < 1)
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  const int64_t row_bytes = width * elem_size(slab_dtype);
  const int64_t work = (row_bytes * old_capacity) / 16 > new_capacity ? (row_bytes * old_capacity) / 16 : new_capacity;
  grow_kernel<<<grid_for(work, 256), 256, 0, st>>>(old_slab, old_free_rows, old_capacity, new_slab, new_free_rows,
                                                 new_capacity, row_bytes, free_count, status);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  grow_finish_kernel<<<1, 1, 0, st>>>(free_count, new_capacity - old_capacity, status);
  return launch_status();
}

int cow_grow_in_place(int32_t* free_rows, int64_t old_capacity, int64_t new_capacity, int32_t* free_count,
                      int32_t* status, void* stream) {
  if (!free_rows || !free_count || !status || old_capacity < 0 || new_capacity < old_capacity ||
      new_capacity > INT32_MAX)
    return COW_ERR_INVALID;
  if (new_capacity == old_capacity) return COW_OK;
  cudaStream_t st = as_stream(stream);
  grow_append_kernel<<<grid_for(new_capacity - old_capacity, 256), 256, 0, st>>>(free_rows, old_capacity,
                                                                                  new_capacity, free_count);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  grow_finish_kernel<<<1, 1, 0, st>>>(free_count, new_capacity - old_capacity, status);
  return launch_status();
}

// ---- release ---------------------------------------------------------------

int64_t cow_release_workspace_bytes(const cow_pool* pools, const int64_t* counts, int32_t layers) {
  if (!layers_ok(pools, layers) || !counts) return -1;
  int64_t words = 0;
  for (int l = 0; l < layers; ++l)
    words += words16(pools[l].banks > 0 ? pools[l].banks : 1) + scan_words(counts[l] * pools[l].slots);
  return words * 4;
}

int cow_release_layers(const cow_pool* pools, const int64_t* const* bank_indices, const int64_t* counts,
                       int32_t layers, void* workspace, int64_t workspace_bytes, int32_t* released, void* stream) {
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(pools, layers) || !bank_indices || !counts || !released) return COW_ERR_INVALID;
  const int64_t need = cow_release_workspace_bytes(pools, counts, layers);
  if (!workspace_ok(workspace, workspace_bytes, need)) return COW_ERR_INVALID;
  for (int l = 0; l < layers; ++l)
    if (counts[l] < 0 || (counts[l] > 0 && !bank_indices[l])) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  // Zero the masks and scan headers; flags[2] of each pool gates its release
  // (a bad bank list releases nothing).
  if (cudaMemsetAsync(workspace, 0, static_cast<size_t>(need), st) != cudaSuccess) return COW_ERR_CUDA;
  Layers<BankListCtx> B{};
  Layers<StatusOrCtx> S{};
  ScanLaunch C{};
  B.layers = S.layers = C.layers = layers;
  int32_t* w = static_cast<int32_t*>(workspace);
  int64_t max_count = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& p = pools[l];
    int32_t* mask = w;
    w += words16(p.banks > 0 ? p.banks : 1);
    int32_t* flags = w;
    w += scan_words(counts[l] * p.slots);
    B.c[l] = BankListCtx{bank_indices[l], counts[l], p.banks, mask, flags + 2};
    S.c[l] = StatusOrCtx{p.status, flags + 2};
    ScanCtx& c = C.c[l];
    c.op = kOpRelease;
    c.n = counts[l] * p.slots;
    c.slots = p.slots;
    c.bank_idx = bank_indices[l];
    c.pool_map = p.map;
    c.free_rows = p.free_rows;
    c.free_count = p.free_count;
    c.gate_status = flags + 2;
    c.scratch = flags;
    c.total_out = released + l;
    max_count = std::max(max_count, counts[l]);
  }
  if (max_count > 0) {
    bank_list_kernel<<<layer_grid(max_count, 256, layers), 256, 0, st>>>(B);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
    status_or_kernel<<<dim3(1, layers), 32, 0, st>>>(S);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  int rc = run_scan_count(C, st);
  if (rc != COW_OK) return rc;
  return run_scan_apply(C, st);
}

int cow_release(const cow_pool* pool, const int64_t* bank_indices, int64_t count, int32_t* bank_mask,
                int32_t* flags_scratch, int32_t* released, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if (!pool || !bank_mask || !flags_scratch || !released || count < 0 || (count > 0 && !bank_indices))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(bank_mask, 0, sizeof(int32_t) * (pool->banks > 0 ? pool->banks : 1), st) != cudaSuccess ||
      cudaMemsetAsync(flags_scratch, 0, sizeof(int32_t) * kScanHeader, st) != cudaSuccess)
    return COW_ERR_CUDA;
  if (count > 0) {
    Layers<BankListCtx> B{};
    B.c[0] = BankListCtx{bank_indices, count, pool->banks, bank_mask, flags_scratch + 2};
    B.layers = 1;
    bank_list_kernel<<<layer_grid(count, 256, 1), 256, 0, st>>>(B);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
    Layers<StatusOrCtx> S{};
    S.c[0] = StatusOrCtx{pool->status, flags_scratch + 2};
    S.layers = 1;
    status_or_kernel<<<1, 32, 0, st>>>(S);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  ScanLaunch C{};
  C.layers = 1;
  ScanCtx& c = C.c[0];
  c.op = kOpRelease;
  c.n = count * pool->slots;
  c.slots = pool->slots;
  c.bank_idx = bank_indices;
  c.pool_map = pool->map;
  c.free_rows = pool->free_rows;
  c.free_count = pool->free_count;
  c.gate_status = flags_scratch + 2;
  c.scratch = flags_scratch;
  c.total_out = released;
  int rc = run_scan_count(C, st);
  if (rc != COW_OK) return rc;
  return run_scan_apply(C, st);
}

// ---- trim ------------------------------------------------------------------

int cow_repack(const cow_pool* pool, int32_t* new_map, void* new_slab, int32_t* new_free_rows, int64_t new_capacity,
               int32_t* src_rows, int32_t* flags_scratch, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if (!pool || !new_map || !new_slab || !new_free_rows || !src_rows || !flags_scratch) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanLaunch C{};
  C.layers = 1;
  ScanCtx& c = C.c[0];
  c.op = kOpRepack;
  c.n = pool->banks * pool->slots;
  c.slots = pool->slots;
  c.map = pool->map;
  c.out_map = new_map;
  c.src_rows = src_rows;
  c.scratch = flags_scratch;
  int rc = run_scan_apply(C, st);
  if (rc != COW_OK) return rc;
  Layers<FillFreeCtx> F{};
  F.c[0] = FillFreeCtx{new_free_rows, new_capacity, pool->free_count, pool->status, flags_scratch};
  F.layers = 1;
  fill_free_kernel<<<layer_grid(new_capacity, 256, 1), 256, 0, st>>>(F);
  return launch_status();
}

// ---- admission ---------------------------------------------------------------

int cow_append(const cow_pool* dst, const cow_pool* other, int32_t* admitted_map, int32_t* src_rows,
               int32_t* dst_rows, int32_t* flags_scratch, void* stream) {
  if (!dense_maps(dst, 1) || !dense_maps(other, 1)) return COW_ERR_UNSUPPORTED;
  if (!dst || !other || !admitted_map || !src_rows || !dst_rows || !flags_scratch) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanLaunch C{};
  C.layers = 1;
  ScanCtx& c = C.c[0];
  c.op = kOpAppend;
  c.n = other->banks * other->slots;
  c.slots = other->slots;
  c.map = other->map;
  c.out_map = admitted_map;
  c.src_rows = src_rows;
  c.dst_rows = dst_rows;
  c.free_rows = dst->free_rows;
  c.free_count = dst->free_count;
  c.scratch = flags_scratch;
  // The count phase (run by the caller through cow_pack_count) did not touch
  // free_count; redo it here with the append bookkeeping.
  int rc = run_scan_count(C, st);
  if (rc != COW_OK) return rc;
  return run_scan_apply(C, st);
}

int64_t cow_append_workspace_bytes(const cow_pool* others, int32_t layers) {
  if (!layers_ok(others, layers)) return -1;
  int64_t words = 0;
  for (int l = 0; l < layers; ++l) {
    const int64_t n = others[l].banks * others[l].slots;
    words += scan_words(n) + 2 * words16(n > 0 ? n : 1);
  }
  return words * 4;
}

int cow_append_count_layers(const cow_pool* dsts, const cow_pool* others, int32_t layers, void* workspace,
                            int64_t workspace_bytes, int32_t* counts, void* stream) {
  if (!dense_maps(dsts, layers) || !dense_maps(others, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(dsts, layers) || !layers_ok(others, layers) || !counts) return COW_ERR_INVALID;
  if (!workspace_ok(workspace, workspace_bytes, cow_append_workspace_bytes(others, layers))) return COW_ERR_INVALID;
  ScanLaunch C{};
  C.layers = layers;
  int32_t* w = static_cast<int32_t*>(workspace);
  for (int l = 0; l < layers; ++l) {
    const int64_t n = others[l].banks * others[l].slots;
    if (!dsts[l].free_count || (n > 0 && !others[l].map)) return COW_ERR_INVALID;
    ScanCtx& c = C.c[l];
    c.op = kOpPack;  // counting only; free_count is read, not changed
    c.n = n;
    c.slots = others[l].slots;
    c.map = others[l].map;
    c.free_count = dsts[l].free_count;
    c.scratch = w;
    c.total_out = counts + 2 * l;
    c.free_out = counts + 2 * l + 1;
    w += scan_words(n) + 2 * words16(n > 0 ? n : 1);
  }
  return run_scan_count(C, as_stream(stream));
}

int cow_append_layers(const cow_pool* dsts, const cow_pool* others, int32_t layers, int32_t* const* admitted_maps,
                      void* workspace, int64_t workspace_bytes, void* stream) {
  if (!dense_maps(dsts, layers) || !dense_maps(others, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(dsts, layers) || !layers_ok(others, layers) || !admitted_maps) return COW_ERR_INVALID;
  if (!workspace_ok(workspace, workspace_bytes, cow_append_workspace_bytes(others, layers))) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanLaunch C{};
  Layers<CopyCtx> K{};
  C.layers = K.layers = layers;
  int32_t* w = static_cast<int32_t*>(workspace);
  for (int l = 0; l < layers; ++l) {
    const cow_pool& d = dsts[l];
    const cow_pool& o = others[l];
    const int64_t n = o.banks * o.slots;
    if (o.slots != d.slots || o.width != d.width || o.slab_dtype != d.slab_dtype || !d.free_rows ||
        !d.free_count || !d.slab || (n > 0 && (!o.map || !o.slab || !admitted_maps[l])))
      return COW_ERR_INVALID;
    int32_t* flags = w;
    int32_t* src_rows = flags + scan_words(n);
    int32_t* dst_rows = src_rows + words16(n > 0 ? n : 1);
    w = dst_rows + words16(n > 0 ? n : 1);
    ScanCtx& c = C.c[l];
    c.op = kOpAppend;
    c.n = n;
    c.slots = o.slots;
    c.map = o.map;
    c.out_map = admitted_maps[l];
    c.src_rows = src_rows;
    c.dst_rows = dst_rows;
    c.free_rows = d.free_rows;
    c.free_count = d.free_count;
    c.scratch = flags;
    K.c[l] = CopyCtx{d.slab, dst_rows, o.slab, src_rows, flags, nullptr, nullptr, n, d.width, d.slots,
                     d.slab_dtype, o.slab_dtype, 0, 0};
    if (!copy_args_ok(K.c[l])) return COW_ERR_INVALID;
  }
  int rc = run_scan_count(C, st);
  if (rc != COW_OK) return rc;
  rc = run_scan_apply(C, st);
  if (rc != COW_OK) return rc;
  return run_copy_rows(K, st);
}

// ---- compaction --------------------------------------------------------------

int cow_retain(const cow_pool* pool, const int64_t* bank_indices, int64_t count, int32_t* new_map,
               int64_t* new_templates, int32_t* selected, int32_t* status, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if (!pool || !selected || !status || count < 0 || (count > 0 && (!bank_indices || !new_map || !new_templates)))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(selected, 0, sizeof(int32_t) * (pool->banks > 0 ? pool->banks : 1), st) != cudaSuccess)
    return COW_ERR_CUDA;
  Layers<BankListCtx> B{};
  Layers<RetainCtx> R{};
  B.layers = R.layers = 1;
  B.c[0] = BankListCtx{bank_indices, count, pool->banks, selected, status};
  R.c[0] = RetainCtx{pool->map, pool->templates, bank_indices, count, pool->slots, pool->banks, selected,
                     new_map, new_templates, status};
  if (count > 0) {
    bank_list_kernel<<<layer_grid(count, 256, 1), 256, 0, st>>>(B);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  if (pool->banks * pool->slots > 0) {
    retain_check_kernel<<<layer_grid(pool->banks * 32, 256, 1), 256, 0, st>>>(R);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  if (count > 0 && pool->banks > 0) {
    retain_gather_kernel<<<layer_grid(count * 32, 256, 1), 256, 0, st>>>(R);
    return launch_status();
  }
  return COW_OK;
}

int64_t cow_retain_workspace_bytes(const cow_pool* pools, int32_t layers) {
  if (!layers_ok(pools, layers)) return -1;
  int64_t words = 0;
  for (int l = 0; l < layers; ++l) words += words16(pools[l].banks > 0 ? pools[l].banks : 1);
  return words * 4;
}

int cow_retain_layers(const cow_pool* pools, const int64_t* const* bank_indices, const int64_t* counts, int32_t layers,
                      int32_t* const* new_maps, int64_t* const* new_templates, void* workspace,
                      int64_t workspace_bytes, int32_t* status, void* stream) {
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(pools, layers) || !bank_indices || !counts || !new_maps || !new_templates || !status)
    return COW_ERR_INVALID;
  const int64_t need = cow_retain_workspace_bytes(pools, layers);
  if (!workspace_ok(workspace, workspace_bytes, need)) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(workspace, 0, static_cast<size_t>(need), st) != cudaSuccess ||
      cudaMemsetAsync(status, 0, sizeof(int32_t) * layers, st) != cudaSuccess)
    return COW_ERR_CUDA;
  Layers<BankListCtx> B{};
  Layers<RetainCtx> R{};
  B.layers = R.layers = layers;
  int32_t* w = static_cast<int32_t*>(workspace);
  int64_t max_count = 0, max_map = 0, max_gather = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& p = pools[l];
    const int64_t cnt = counts[l];
    if (cnt < 0 || (cnt > 0 && (!bank_indices[l] || !new_maps[l] || !new_templates[l]))) return COW_ERR_INVALID;
    B.c[l] = BankListCtx{bank_indices[l], cnt, p.banks, w, status + l};
    R.c[l] = RetainCtx{p.map, p.templates, bank_indices[l], cnt, p.slots, p.banks, w, new_maps[l],
                       new_templates[l], status + l};
    w += words16(p.banks > 0 ? p.banks : 1);
    max_count = std::max(max_count, cnt);
    if (p.slots > 0) max_map = std::max(max_map, p.banks);  // one warp per bank row
    if (p.banks > 0 && p.slots > 0) max_gather = std::max(max_gather, cnt);
  }
  if (max_count > 0) {
    bank_list_kernel<<<layer_grid(max_count, 256, layers), 256, 0, st>>>(B);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  if (max_map > 0) {
    retain_check_kernel<<<layer_grid(max_map * 32, 256, layers), 256, 0, st>>>(R);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  if (max_gather > 0) {
    retain_gather_kernel<<<layer_grid(max_gather * 32, 256, layers), 256, 0, st>>>(R);
    return launch_status();
  }
  return COW_OK;
}

// ---- prefill packing ---------------------------------------------------------

int64_t cow_pack_workspace_bytes(int64_t n, int32_t layers) {
  if (n < 0 || layers < 1 || layers > COW_MAX_LAYERS) return -1;
  return (scan_words(n) + words16(n > 0 ? n : 1)) * 4 * static_cast<int64_t>(layers);
}

int cow_prefill_mark_count_layers(const void* const* write_indices, const void* const* read_indices,
                                  int32_t index_dtype, int64_t banks, int64_t time, int32_t writes, int32_t reads,
                                  int64_t slots, int32_t* const* maps, int32_t layers, void* workspace,
                                  int64_t workspace_bytes, int32_t* out, void* stream) {
  if (!write_indices || !maps || !out || layers < 1 || layers > COW_MAX_LAYERS || banks < 0 || time < 0 ||
      writes < 1 || slots < 1 || reads < 0 || (reads > 0 && !read_indices))
    return COW_ERR_INVALID;
  const int64_t n = banks * slots;
  if (!workspace_ok(workspace, workspace_bytes, cow_pack_workspace_bytes(n, layers))) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(out, 0, sizeof(int32_t) * 2 * layers, st) != cudaSuccess) return COW_ERR_CUDA;
  Layers<MarkCtx> M{};
  ScanLaunch C{};
  M.layers = C.layers = layers;
  const int64_t stride = scan_words(n) + words16(n > 0 ? n : 1);
  for (int l = 0; l < layers; ++l) {
    if ((n > 0 && !maps[l]) || (banks * time > 0 && !write_indices[l])) return COW_ERR_INVALID;
    if (n > 0 && cudaMemsetAsync(maps[l], 0xff, sizeof(int32_t) * n, st) != cudaSuccess) return COW_ERR_CUDA;
    if (reads > 0 && banks * time > 0 && !read_indices[l]) return COW_ERR_INVALID;
    M.c[l] = MarkCtx{write_indices[l], maps[l], out + 2 * l, reads > 0 ? read_indices[l] : nullptr};
    ScanCtx& c = C.c[l];
    c.op = kOpPack;
    c.n = n;
    c.slots = 1;
    c.map = maps[l];
    c.scratch = static_cast<int32_t*>(workspace) + stride * l;
    c.total_out = out + 2 * l + 1;
  }
  const int64_t elems = banks * time * (writes > reads ? writes : reads);
  if (elems > 0) {
    prefill_mark_kernel<<<layer_grid(elems, 256, layers), 256, 0, st>>>(M, index_dtype == COW_I64, banks, time, writes,
                                                                       slots, reads);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  return run_scan_count(C, st);
}

int64_t cow_admit_prefix_workspace_bytes(int64_t cohort_banks, int64_t slots, int32_t layers) {
  if (cohort_banks < 0 || slots < 1 || layers < 1 || layers > COW_MAX_LAYERS) return -1;
  const int64_t n = cohort_banks * slots;
  return (scan_words(n) + 2 * words16(n > 0 ? n : 1)) * 4 * layers;
}

int cow_admit_prefix_layers(const cow_pool* dsts, int32_t* const* marks, const int64_t* cohort_templates,
                            int64_t cohort_banks, int32_t layers, int32_t* const* admitted_maps, void* workspace,
                            int64_t workspace_bytes, void* stream) {
  if (!dense_maps(dsts, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(dsts, layers) || !marks || !admitted_maps || cohort_banks < 0 ||
      (cohort_banks > 0 && !cohort_templates))
    return COW_ERR_INVALID;
  if (!workspace_ok(workspace, workspace_bytes, cow_admit_prefix_workspace_bytes(cohort_banks, dsts[0].slots, layers)))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanLaunch C{};
  Layers<CopyCtx> K{};
  C.layers = K.layers = layers;
  const int64_t n = cohort_banks * dsts[0].slots;
  int32_t* w = static_cast<int32_t*>(workspace);
  for (int l = 0; l < layers; ++l) {
    const cow_pool& d = dsts[l];
    if (d.slots != dsts[0].slots || !d.free_rows || !d.free_count || !d.slab || !d.m0 ||
        (n > 0 && (!marks[l] || !admitted_maps[l])))
      return COW_ERR_INVALID;
    int32_t* flags = w;
    int32_t* src_rows = flags + scan_words(n);
    int32_t* dst_rows = src_rows + words16(n > 0 ? n : 1);
    w = dst_rows + words16(n > 0 ? n : 1);
    ScanCtx& c = C.c[l];
    c.op = kOpAdmit;
    c.n = n;
    c.slots = d.slots;
    c.map = marks[l];
    c.out_map = admitted_maps[l];
    c.src_rows = src_rows;
    c.dst_rows = dst_rows;
    c.free_rows = d.free_rows;
    c.free_count = d.free_count;
    c.scratch = flags;
    K.c[l] = CopyCtx{d.slab, dst_rows, nullptr, src_rows, flags, d.m0, cohort_templates, n, d.width, d.slots,
                     d.slab_dtype, COW_F32, 1, 0};
    if (!copy_args_ok(K.c[l])) return COW_ERR_INVALID;
  }
  if (n == 0) return COW_OK;
  int rc = run_scan_count(C, st);
  if (rc != COW_OK) return rc;
  rc = run_scan_apply(C, st);
  if (rc != COW_OK) return rc;
  return run_copy_rows(K, st);
}

int cow_pack_apply_layers(const cow_pool* pools, int32_t layers, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(pools, layers)) return COW_ERR_INVALID;
  const int64_t n = pools[0].banks * pools[0].slots;
  if (!workspace_ok(workspace, workspace_bytes, cow_pack_workspace_bytes(n, layers))) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanLaunch C{};
  Layers<FillFreeCtx> F{};
  Layers<CopyCtx> K{};
  C.layers = F.layers = K.layers = layers;
  const int64_t stride = scan_words(n) + words16(n > 0 ? n : 1);
  int64_t max_cap = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& p = pools[l];
    if (p.banks * p.slots != n || !p.map || !p.free_rows || !p.free_count || !p.slab || !p.m0 || !p.templates)
      return COW_ERR_INVALID;
    int32_t* flags = static_cast<int32_t*>(workspace) + stride * l;
    int32_t* src_index = flags + scan_words(n);
    ScanCtx& c = C.c[l];
    c.op = kOpPack;
    c.n = n;
    c.slots = 1;
    c.map = p.map;
    c.out_map = p.map;
    c.src_rows = src_index;
    c.scratch = flags;
    F.c[l] = FillFreeCtx{p.free_rows, p.capacity, p.free_count, p.status, flags};
    K.c[l] = CopyCtx{p.slab, nullptr, nullptr, src_index, flags, p.m0, p.templates, std::min(n, p.capacity),
                     p.width, p.slots, p.slab_dtype, COW_F32, 1, 0};
    if (!copy_args_ok(K.c[l])) return COW_ERR_INVALID;
    max_cap = std::max(max_cap, p.capacity);
  }
  int rc = run_scan_apply(C, st);
  if (rc != COW_OK) return rc;
  fill_free_kernel<<<layer_grid(max_cap, 256, layers), 256, 0, st>>>(F);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  return run_copy_rows(K, st);
}

// ---- validation --------------------------------------------------------------

int cow_validate(const cow_pool* pool, int32_t* counts, int32_t* status, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if (!pool || !counts || !status) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (pool->capacity > 0 &&
      cudaMemsetAsync(counts, 0, sizeof(int32_t) * pool->capacity, st) != cudaSuccess)
    return COW_ERR_CUDA;
  Layers<ValidateCtx> V{};
  V.layers = 1;
  const int64_t n = pool->banks * pool->slots;
  V.c[0] = ValidateCtx{pool->map, n, pool->capacity, pool->free_rows, pool->free_count, counts, status,
                       pool->status, nullptr};
  validate_count_kernel<<<layer_grid(std::max(n, pool->capacity), 256, 1), 256, 0, st>>>(V);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  if (pool->capacity > 0) {
    validate_check_kernel<<<layer_grid(pool->capacity, 256, 1), 256, 0, st>>>(V);
    return launch_status();
  }
  return COW_OK;
}

int64_t cow_validate_workspace_bytes(const cow_pool* pools, int32_t layers) {
  if (!layers_ok(pools, layers)) return -1;
  int64_t words = 0;
  for (int l = 0; l < layers; ++l) words += words16(pools[l].capacity + 1);
  return words * 4;
}

int cow_validate_layers(const cow_pool* pools, int32_t layers, void* workspace, int64_t workspace_bytes, int32_t* out,
                        void* stream) {
  if (!dense_maps(pools, layers)) return COW_ERR_UNSUPPORTED;
  if (!layers_ok(pools, layers) || !out) return COW_ERR_INVALID;
  const int64_t need = cow_validate_workspace_bytes(pools, layers);
  if (!workspace_ok(workspace, workspace_bytes, need)) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(workspace, 0, static_cast<size_t>(need), st) != cudaSuccess) return COW_ERR_CUDA;
  Layers<ValidateCtx> V{};
  V.layers = layers;
  int32_t* w = static_cast<int32_t*>(workspace);
  int64_t max_work = 0, max_cap = 0;
  for (int l = 0; l < layers; ++l) {
    const cow_pool& p = pools[l];
    if (!p.map || !p.free_rows || !p.free_count || !p.status) return COW_ERR_INVALID;
    const int64_t n = p.banks * p.slots;
    // the last word of each region holds that pool's validate bits
    V.c[l] = ValidateCtx{p.map, n, p.capacity, p.free_rows, p.free_count, w, w + p.capacity, p.status, out + 3 * l};
    w += words16(p.capacity + 1);
    max_work = std::max(max_work, std::max(n, p.capacity));
    max_cap = std::max(max_cap, p.capacity);
  }
  validate_count_kernel<<<layer_grid(max_work, 256, layers), 256, 0, st>>>(V);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  if (max_cap > 0) {
    validate_check_kernel<<<layer_grid(max_cap, 256, layers), 256, 0, st>>>(V);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  validate_report_kernel<<<1, 32, 0, st>>>(V);
  return launch_status();
}

int cow_materialize(const cow_pool* pool, void* out, int32_t out_dtype, void* stream) {
  if (!dense_maps(pool, 1)) return COW_ERR_UNSUPPORTED;
  if (!pool || !out || !valid_dtype(out_dtype) || pool->width % 4 != 0) return COW_ERR_INVALID;
  const int64_t rows = pool->banks * pool->slots;
  if (rows == 0) return COW_OK;
  materialize_kernel<<<grid_for(rows * 32, 256), 256, 0, as_stream(stream)>>>(
      pool->m0, pool->templates, pool->slab, pool->slab_dtype, pool->map, pool->banks, pool->slots, pool->width, out,
      out_dtype);
  return launch_status();
}

}  // extern "C"
