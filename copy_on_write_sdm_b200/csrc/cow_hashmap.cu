// cow_hashmap.cu -- hashed logical maps: conversion to and from the dense map.
//
// The reference keeps a dense int32 logical-to-physical map of [banks, slots]
// (allocator.py:496-504), Theta(banks * N) bytes whatever the number of
// private slots; at N = 65,536 that is 256 KiB per bank and layer.  A hashed
// pool keeps, per bank, an open-addressing table of T = 2^k 64-bit entries
// ((slot << 32) | physical row, all ones when empty; see cow_common.cuh), so
// the map costs 8 T bytes per bank with T sized to the bank's private slots.
// The fused decode step reads and extends the tables directly.  The lifecycle
// operations (release, compaction, admission, trim, validation) work on the
// dense form: the host expands a pool's tables into a dense map for the
// operation and rebuilds them afterwards with these kernels.  Row placement
// never depends on where an entry sits in a table, so maps, free stacks and
// physical rows stay exactly those of the dense pool.

#include "cow_common.cuh"

namespace {

constexpr int kHashThreads = 256;

int hash_log2(int64_t t) {
  if (t < 4 || t > (int64_t(1) << 30) || (t & (t - 1)) != 0) return -1;
  int k = 0;
  while ((int64_t(1) << k) < t) ++k;
  return k;
}

int memset_status(cudaError_t e) {
  if (e == cudaSuccess) return COW_OK;
  cudaGetLastError();
  cowrt::last_cuda_error = static_cast<int>(e);
  return COW_ERR_CUDA;
}

int64_t hash_grid(int64_t n) {
  const int64_t blocks = (n + kHashThreads - 1) / kHashThreads;
  return blocks < 148 * 64 ? (blocks > 0 ? blocks : 1) : 148 * 64;
}

// Every private slot of the dense map goes into its bank's table.
__global__ void __launch_bounds__(kHashThreads)
    hash_from_dense_kernel(const int32_t* map, int64_t banks, int64_t slots, unsigned long long* tables, int log_t,
                           int32_t* status) {
  const int64_t n = banks * slots;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t phys = map[i];
    if (phys < 0) continue;
    const int64_t bank = i / slots;
    const int slot = static_cast<int>(i - bank * slots);
    if (!hash_insert(tables + (bank << log_t), log_t, slot, phys)) atomicOr(status, COW_ST_MAP_FULL);
  }
}

// Every table entry goes back to its dense map position (the map starts at -1).
__global__ void __launch_bounds__(kHashThreads)
    hash_to_dense_kernel(const unsigned long long* tables, int64_t banks, int log_t, int32_t* map, int64_t slots,
                         int32_t* status) {
  const int64_t n = banks << log_t;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const unsigned long long e = tables[i];
    if (e == kHashEmpty) continue;
    const int64_t bank = i >> log_t;
    const int64_t slot = static_cast<int64_t>(e >> 32);
    if (slot >= slots) {
      atomicOr(status, COW_ST_ROW_RANGE);
      continue;
    }
    map[bank * slots + slot] = static_cast<int32_t>(static_cast<uint32_t>(e));
  }
}

// Largest number of occupied entries in any bank's table.
__global__ void __launch_bounds__(kHashThreads)
    hash_max_live_kernel(const unsigned long long* tables, int64_t banks, int log_t, int32_t* out) {
  __shared__ int s_warp[kHashThreads / 32];
  const int64_t t = int64_t(1) << log_t;
  for (int64_t bank = blockIdx.x; bank < banks; bank += gridDim.x) {
    const unsigned long long* tb = tables + (bank << log_t);
    int live = 0;
    for (int64_t i = threadIdx.x; i < t; i += blockDim.x) live += tb[i] != kHashEmpty ? 1 : 0;
    int total;
    block_exclusive_scan_n<kHashThreads>(live, s_warp, total);
    if (threadIdx.x == 0) atomicMax(out, total);
  }
}

}  // namespace

extern "C" {

int cow_hash_from_dense(const int32_t* map, int64_t banks, int64_t slots, void* tables, int64_t table_slots,
                        int32_t* status, void* stream) {
  const int log_t = hash_log2(table_slots);
  if (banks < 0 || slots < 1 || slots >= (int64_t(1) << 31) || log_t < 0 || !status || (banks > 0 && (!map || !tables)))
    return COW_ERR_INVALID;
  if (banks == 0) return COW_OK;
  cudaStream_t st = as_stream(stream);
  if (const int rc = memset_status(cudaMemsetAsync(tables, 0xff, static_cast<size_t>(banks << log_t) * 8u, st))) return rc;
  hash_from_dense_kernel<<<static_cast<unsigned>(hash_grid(banks * slots)), kHashThreads, 0, st>>>(
      map, banks, slots, static_cast<unsigned long long*>(tables), log_t, status);
  return launch_status();
}

int cow_hash_to_dense(const void* tables, int64_t banks, int64_t table_slots, int32_t* map, int64_t slots,
                      int32_t* status, void* stream) {
  const int log_t = hash_log2(table_slots);
  if (banks < 0 || slots < 1 || log_t < 0 || !status || (banks > 0 && (!map || !tables))) return COW_ERR_INVALID;
  if (banks == 0) return COW_OK;
  cudaStream_t st = as_stream(stream);
  if (const int rc = memset_status(cudaMemsetAsync(map, 0xff, static_cast<size_t>(banks * slots) * 4u, st))) return rc;
  hash_to_dense_kernel<<<static_cast<unsigned>(hash_grid(banks << log_t)), kHashThreads, 0, st>>>(
      static_cast<const unsigned long long*>(tables), banks, log_t, map, slots, status);
  return launch_status();
}

int cow_hash_max_live(const void* tables, int64_t banks, int64_t table_slots, int32_t* out, void* stream) {
  const int log_t = hash_log2(table_slots);
  if (banks < 0 || log_t < 0 || !out || (banks > 0 && !tables)) return COW_ERR_INVALID;
  cudaStream_t st = as_stream(stream);
  if (const int rc = memset_status(cudaMemsetAsync(out, 0, sizeof(int32_t), st))) return rc;
  if (banks == 0) return COW_OK;
  const int64_t blocks = banks < 148 * 16 ? banks : 148 * 16;
  hash_max_live_kernel<<<static_cast<unsigned>(blocks), kHashThreads, 0, st>>>(
      static_cast<const unsigned long long*>(tables), banks, log_t, out);
  return launch_status();
}

}  // extern "C"
