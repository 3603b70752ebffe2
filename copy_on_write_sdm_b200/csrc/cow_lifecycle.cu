// cow_lifecycle.cu -- allocator lifecycle kernels: init, pack, grow, release, repack,
// append, retain, validate, materialize.

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// ordered prefix-count machinery for the lifecycle operations
// --------------------------------------------------------------------------

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanSeg = kScanThreads * kScanItems;
constexpr int kScanHeader = 8;  // int32 slots before the per-block offsets

enum ScanOp : int { kOpPack = 0, kOpRepack = 1, kOpAppend = 2, kOpRelease = 3 };

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
  int32_t* free_count;
  const int32_t* gate_status;  // release: skip everything when the bank list was bad
  int32_t* scratch;            // [0]=total, [1]=old free count, [kScanHeader..] block offsets
};

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

__global__ void __launch_bounds__(kScanThreads) scan_count_kernel(const __grid_constant__ ScanCtx c) {
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

// Single CTA: exclusive scan of the per-block counts, total, and the free
// count bookkeeping of release (push) / append (pop).
__global__ void __launch_bounds__(1024) scan_blocks_kernel(const __grid_constant__ ScanCtx c, int64_t nblocks) {
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
    if (c.free_count != nullptr) {
      const int old = *c.free_count;
      c.scratch[1] = old;
      if (c.op == kOpRelease) *c.free_count = old + total;
      if (c.op == kOpAppend) *c.free_count = old - total;
    }
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const __grid_constant__ ScanCtx c) {
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
// small utility kernels
// --------------------------------------------------------------------------

__global__ void init_pool_kernel(int32_t* map, int64_t map_n, int32_t* free_rows, int64_t cap,
                                 int32_t* free_count, int32_t* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < map_n || i < cap; i += stride) {
    if (i < map_n) map[i] = -1;
    if (i < cap) free_rows[i] = static_cast<int32_t>(i);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *free_count = static_cast<int32_t>(cap);
    *status = 0;
  }
}

__global__ void fill_free_kernel(int32_t* free_rows, int64_t cap, int32_t* free_count, int32_t* status,
                                 const int32_t* scratch) {
  // free_rows[:cap - A] = arange(A, cap), A = scratch[0] (the live row count)
  const int64_t a = scratch[0];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < cap - a; j += stride) {
    free_rows[j] = static_cast<int32_t>(a + j);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *free_count = static_cast<int32_t>(cap - a);
    if (status != nullptr) *status = 0;
  }
}

__global__ void mask_to_map_kernel(const uint8_t* active, int64_t n, int32_t* map) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    map[i] = active[i] ? 0 : -1;
}

__global__ void prefill_mark_kernel(const void* widx, int idx64, int64_t banks, int64_t time, int writes,
                                    int64_t slots, int32_t* map, int32_t* status) {
  const int64_t n = banks * time * writes;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const int64_t bank = i / (time * writes);
    const int64_t s = ld_index(widx, i, idx64);
    if (s < 0 || s >= slots) {
      atomicOr(status, COW_ST_INDEX_RANGE);
      continue;
    }
    map[bank * slots + s] = 0;
  }
}

// One warp per row; 16-byte vectors when both dtypes allow it.
__global__ void copy_rows_kernel(void* dst, int dst_dt, const int32_t* dst_rows, const void* src, int src_dt,
                                 const int32_t* src_rows, int64_t count, int64_t width, int mode,
                                 const float* m0, const int64_t* templates, int64_t slots) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); k < count; k += warps) {
    const int64_t d = dst_rows ? dst_rows[k] : k;
    const void* sbase = src;
    int sdt = src_dt;
    int64_t s;
    if (mode == 1) {
      const int64_t flat = src_rows[k];
      s = templates[flat / slots] * slots + flat % slots;
      sbase = m0;
      sdt = COW_F32;
    } else {
      s = src_rows ? src_rows[k] : k;
    }
    if ((width & 3) == 0) {
      for (int64_t e = lane * 4; e < width; e += 128) {
        st4_rt(dst, d * width + e, ld4_rt(sbase, s * width + e, sdt), dst_dt);
      }
    } else {
      for (int64_t e = lane; e < width; e += 32) {
        const float v = ld1_rt(sbase, s * width + e, sdt);
        if (dst_dt == COW_F32) static_cast<float*>(dst)[d * width + e] = v;
        else if (dst_dt == COW_BF16) static_cast<__nv_bfloat16*>(dst)[d * width + e] = __float2bfloat16_rn(v);
        else static_cast<__half*>(dst)[d * width + e] = __float2half_rn(v);
      }
    }
  }
}

__global__ void grow_kernel(const void* old_slab, const int32_t* old_free_rows, int64_t old_cap, void* new_slab,
                            int32_t* new_free_rows, int64_t new_cap, int64_t row_bytes, int32_t* free_count,
                            int32_t* status) {
  // Byte copy of the old slab (16-byte words; row_bytes*old_cap is a multiple
  // of 16 whenever width*elem is), then the free stack.
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t bytes = row_bytes * old_cap;
  if ((bytes & 15) == 0) {
    const int4* s = static_cast<const int4*>(old_slab);
    int4* d = static_cast<int4*>(new_slab);
    for (int64_t i = tid; i < bytes / 16; i += stride) d[i] = s[i];
  } else {
    const uint8_t* s = static_cast<const uint8_t*>(old_slab);
    uint8_t* d = static_cast<uint8_t*>(new_slab);
    for (int64_t i = tid; i < bytes; i += stride) d[i] = s[i];
  }
  const int64_t old_free = *free_count;
  const int64_t added = new_cap - old_cap;
  for (int64_t i = tid; i < old_free + added; i += stride) {
    new_free_rows[i] = i < old_free ? old_free_rows[i] : static_cast<int32_t>(old_cap + (i - old_free));
  }
}

__global__ void grow_finish_kernel(int32_t* free_count, int64_t added, int32_t* status) {
  *free_count += static_cast<int32_t>(added);
  *status = 0;
}

__global__ void bank_list_kernel(const int64_t* idx, int64_t count, int64_t banks, int32_t* mask, int32_t* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < count; s += stride) {
    const int64_t b = idx[s];
    if (b < 0 || b >= banks) {
      atomicOr(status, COW_ST_BAD_BANK_LIST);
      continue;
    }
    if (atomicAdd(&mask[b], 1) != 0) atomicOr(status, COW_ST_BAD_BANK_LIST);
  }
}

__global__ void status_or_kernel(int32_t* status, const int32_t* bits) { atomicOr(status, *bits); }

__global__ void retain_check_kernel(const int32_t* map, int64_t banks, int64_t slots, const int32_t* mask,
                                    int32_t* status) {
  const int64_t n = banks * slots;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    if (map[i] >= 0 && mask[i / slots] == 0) atomicOr(status, COW_ST_DISCARD_LIVE);
  }
}

__global__ void retain_gather_kernel(const int32_t* map, const int64_t* templates, const int64_t* idx, int64_t count,
                                     int64_t slots, int64_t banks, int32_t* new_map, int64_t* new_templates) {
  const int64_t n = count * slots;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const int64_t s = i / slots;
    int64_t b = idx[s];
    b = b < 0 ? 0 : (b >= banks ? banks - 1 : b);
    new_map[i] = map[b * slots + i % slots];
    if (i % slots == 0) new_templates[s] = templates[b];
  }
}

__global__ void validate_count_kernel(const int32_t* map, int64_t map_n, const int32_t* free_rows,
                                      const int32_t* free_count, int64_t cap, int32_t* counts, int32_t* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t fc = *free_count;
  if (blockIdx.x == 0 && threadIdx.x == 0 && (fc < 0 || fc > cap)) atomicOr(status, COW_ST_ROW_RANGE);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < map_n; i += stride) {
    const int32_t v = map[i];
    if (v < 0) continue;
    if (v >= cap) {
      atomicOr(status, COW_ST_ROW_RANGE);
      continue;
    }
    atomicAdd(&counts[v], 1);
  }
  const int64_t fcl = fc < 0 ? 0 : (fc > cap ? cap : fc);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < fcl; i += stride) {
    const int32_t v = free_rows[i];
    if (v < 0 || v >= cap) {
      atomicOr(status, COW_ST_ROW_RANGE);
      continue;
    }
    atomicAdd(&counts[v], 1 << 16);
  }
}

__global__ void validate_check_kernel(const int32_t* counts, int64_t cap, int32_t* status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int bits = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < cap; i += stride) {
    const int c = counts[i];
    const int a = c & 0xffff, f = c >> 16;
    if (a > 1) bits |= COW_ST_MULTI_OWNER;
    if (f > 1) bits |= COW_ST_FREE_DUPLICATE;
    if (a + f == 0) bits |= COW_ST_NOT_COVERED;
    if (a >= 1 && f >= 1) bits |= COW_ST_NOT_COVERED;
  }
  if (bits) atomicOr(status, bits);
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

int run_scan_count(ScanCtx& c, cudaStream_t st) {
  const int64_t nb = (c.n + kScanSeg - 1) / kScanSeg;
  if (nb > 0) {
    scan_count_kernel<<<static_cast<unsigned>(nb), kScanThreads, 0, st>>>(c);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  scan_blocks_kernel<<<1, 1024, 0, st>>>(c, nb);
  return launch_status();
}

int run_scan_apply(ScanCtx& c, cudaStream_t st) {
  const int64_t nb = (c.n + kScanSeg - 1) / kScanSeg;
  if (nb == 0) return COW_OK;
  scan_apply_kernel<<<static_cast<unsigned>(nb), kScanThreads, 0, st>>>(c);
  return launch_status();
}

}  // namespace

extern "C" {

int64_t cow_scan_blocks(int64_t n) { return (n + kScanSeg - 1) / kScanSeg + kScanHeader; }

int cow_init_pool(const cow_pool* p, void* stream) {
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
  prefill_mark_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(write_indices, index_dtype == COW_I64, banks,
                                                                      time, writes, slots, map, status);
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
  ScanCtx c{};
  c.op = kOpPack;
  c.n = n;
  c.slots = 1;
  c.map = map;
  c.scratch = flags_scratch;
  return run_scan_count(c, as_stream(stream));
}

int cow_pack_apply(int32_t* map, int64_t n, int32_t* src_index, const cow_pool* pool, int32_t* flags_scratch,
                   void* stream) {
  if ((!map && n > 0) || !pool || !flags_scratch || !src_index) return COW_ERR_INVALID;
  ScanCtx c{};
  c.op = kOpPack;
  c.n = n;
  c.slots = 1;
  c.map = map;
  c.out_map = map;
  c.src_rows = src_index;
  c.scratch = flags_scratch;
  cudaStream_t st = as_stream(stream);
  int rc = run_scan_apply(c, st);
  if (rc != COW_OK) return rc;
  fill_free_kernel<<<grid_for(pool->capacity, 256), 256, 0, st>>>(pool->free_rows, pool->capacity,
                                                                 pool->free_count, pool->status, flags_scratch);
  return launch_status();
}

int cow_copy_rows(void* dst, int32_t dst_dtype, const int32_t* dst_rows, const void* src, int32_t src_dtype,
                  const int32_t* src_rows, int64_t count, int64_t width, int32_t mode, const float* m0,
                  const int64_t* templates, int64_t slots, void* stream) {
  if (count == 0) return COW_OK;
  if (!dst || count < 0 || width < 1 || !valid_dtype(dst_dtype)) return COW_ERR_INVALID;
  if (mode == 1) {
    if (!m0 || !templates || !src_rows || slots < 1 || width % 4 != 0 || !aligned16(m0)) return COW_ERR_INVALID;
  } else if (mode == 0) {
    if (!src || !valid_dtype(src_dtype)) return COW_ERR_INVALID;
    if (width % 4 == 0 && (!row_aligned(src, src_dtype) || !row_aligned(dst, dst_dtype))) return COW_ERR_INVALID;
  } else {
    return COW_ERR_INVALID;
  }
  copy_rows_kernel<<<grid_for(count * 32, 256), 256, 0, as_stream(stream)>>>(
      dst, dst_dtype, dst_rows, src, src_dtype, src_rows, count, width, mode, m0, templates, slots);
  return launch_status();
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

int cow_release(const cow_pool* pool, const int64_t* bank_indices, int64_t count, int32_t* bank_mask,
                int32_t* flags_scratch, int32_t* released, void* stream) {
  if (!pool || !bank_mask || !flags_scratch || !released || count < 0 || (count > 0 && !bank_indices))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(bank_mask, 0, sizeof(int32_t) * (pool->banks > 0 ? pool->banks : 1), st) != cudaSuccess ||
      cudaMemsetAsync(flags_scratch, 0, sizeof(int32_t) * kScanHeader, st) != cudaSuccess)
    return COW_ERR_CUDA;
  // flags_scratch[2] gates the release: a bad bank list releases nothing.
  if (count > 0) {
    bank_list_kernel<<<grid_for(count, 256), 256, 0, st>>>(bank_indices, count, pool->banks, bank_mask,
                                                         flags_scratch + 2);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
    status_or_kernel<<<1, 1, 0, st>>>(pool->status, flags_scratch + 2);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  ScanCtx c{};
  c.op = kOpRelease;
  c.n = count * pool->slots;
  c.slots = pool->slots;
  c.bank_idx = bank_indices;
  c.pool_map = pool->map;
  c.free_rows = pool->free_rows;
  c.free_count = pool->free_count;
  c.gate_status = flags_scratch + 2;
  c.scratch = flags_scratch;
  int rc = run_scan_count(c, st);
  if (rc != COW_OK) return rc;
  rc = run_scan_apply(c, st);
  if (rc != COW_OK) return rc;
  return cudaMemcpyAsync(released, flags_scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) == cudaSuccess
             ? COW_OK
             : COW_ERR_CUDA;
}

int cow_repack(const cow_pool* pool, int32_t* new_map, void* new_slab, int32_t* new_free_rows, int64_t new_capacity,
               int32_t* src_rows, int32_t* flags_scratch, void* stream) {
  if (!pool || !new_map || !new_slab || !new_free_rows || !src_rows || !flags_scratch) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanCtx c{};
  c.op = kOpRepack;
  c.n = pool->banks * pool->slots;
  c.slots = pool->slots;
  c.map = pool->map;
  c.out_map = new_map;
  c.src_rows = src_rows;
  c.scratch = flags_scratch;
  int rc = run_scan_apply(c, st);
  if (rc != COW_OK) return rc;
  fill_free_kernel<<<grid_for(new_capacity, 256), 256, 0, st>>>(new_free_rows, new_capacity, pool->free_count,
                                                               pool->status, flags_scratch);
  return launch_status();
}

int cow_append(const cow_pool* dst, const cow_pool* other, int32_t* admitted_map, int32_t* src_rows,
               int32_t* dst_rows, int32_t* flags_scratch, void* stream) {
  if (!dst || !other || !admitted_map || !src_rows || !dst_rows || !flags_scratch) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  ScanCtx c{};
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
  int rc = run_scan_count(c, st);
  if (rc != COW_OK) return rc;
  return run_scan_apply(c, st);
}

int cow_retain(const cow_pool* pool, const int64_t* bank_indices, int64_t count, int32_t* new_map,
               int64_t* new_templates, int32_t* selected, int32_t* status, void* stream) {
  if (!pool || !selected || !status || count < 0 || (count > 0 && (!bank_indices || !new_map || !new_templates)))
    return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(selected, 0, sizeof(int32_t) * (pool->banks > 0 ? pool->banks : 1), st) != cudaSuccess)
    return COW_ERR_CUDA;
  if (count > 0) {
    bank_list_kernel<<<grid_for(count, 256), 256, 0, st>>>(bank_indices, count, pool->banks, selected, status);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  const int64_t n = pool->banks * pool->slots;
  if (n > 0) {
    retain_check_kernel<<<grid_for(n, 256), 256, 0, st>>>(pool->map, pool->banks, pool->slots, selected, status);
    if (launch_status() != COW_OK) return COW_ERR_CUDA;
  }
  if (count > 0 && pool->banks > 0) {
    retain_gather_kernel<<<grid_for(count * pool->slots, 256), 256, 0, st>>>(
        pool->map, pool->templates, bank_indices, count, pool->slots, pool->banks, new_map, new_templates);
    return launch_status();
  }
  return COW_OK;
}

int cow_validate(const cow_pool* pool, int32_t* counts, int32_t* status, void* stream) {
  if (!pool || !counts || !status) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (pool->capacity > 0 &&
      cudaMemsetAsync(counts, 0, sizeof(int32_t) * pool->capacity, st) != cudaSuccess)
    return COW_ERR_CUDA;
  const int64_t n = pool->banks * pool->slots;
  const int64_t m = n > pool->capacity ? n : pool->capacity;
  validate_count_kernel<<<grid_for(m, 256), 256, 0, st>>>(pool->map, n, pool->free_rows, pool->free_count,
                                                        pool->capacity, counts, status);
  if (launch_status() != COW_OK) return COW_ERR_CUDA;
  if (pool->capacity > 0) {
    validate_check_kernel<<<grid_for(pool->capacity, 256), 256, 0, st>>>(counts, pool->capacity, status);
    return launch_status();
  }
  return COW_OK;
}

int cow_materialize(const cow_pool* pool, void* out, int32_t out_dtype, void* stream) {
  if (!pool || !out || !valid_dtype(out_dtype) || pool->width % 4 != 0) return COW_ERR_INVALID;
  const int64_t rows = pool->banks * pool->slots;
  if (rows == 0) return COW_OK;
  materialize_kernel<<<grid_for(rows * 32, 256), 256, 0, as_stream(stream)>>>(
      pool->m0, pool->templates, pool->slab, pool->slab_dtype, pool->map, pool->banks, pool->slots, pool->width, out,
      out_dtype);
  return launch_status();
}

}  // extern "C"
