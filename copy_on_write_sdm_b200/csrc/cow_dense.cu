// cow_dense.cu -- dense-table control kernel (the latency reference).

#include "cow_common.cuh"

namespace {

// --------------------------------------------------------------------------
// dense-table control
// --------------------------------------------------------------------------

struct DenseLayer {
  void* memory;
  cow_step step;
  int64_t banks, bank_begin;
};
struct DenseLaunch {
  DenseLayer layer[COW_MAX_LAYERS];
  int64_t slots, total_banks;
  int32_t layers, width, writes, reads, idx64, act_dt;
};

template <int SDT, int CH, int WMAX, int RC>
__global__ void __launch_bounds__(kBanksPerCta * 32)
    cow_dense_kernel(const __grid_constant__ DenseLaunch P) {
  constexpr bool kStageReads = RC == 1 && CH == 1 && SDT == COW_F32;
  __shared__ WarpMetaT<32 * RC> s_meta[kBanksPerCta];
  extern __shared__ __align__(16) unsigned char dyn_smem[];  // read rows, per warp R x D floats
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * kBanksPerCta + warp;
  if (g >= P.total_banks) return;
  int l = 0;
  while (l + 1 < P.layers && g >= P.layer[l].bank_begin + P.layer[l].banks) ++l;
  const DenseLayer& L = P.layer[l];
  const int64_t bank = g - L.bank_begin;
  const int D = P.width, W = P.writes, R = P.reads;
  const int64_t N = P.slots;
  auto& sm = s_meta[warp];
  float* const s_reads = reinterpret_cast<float*>(dyn_smem) + static_cast<int64_t>(warp) * R * D;
  const float fl = ld1_rt(L.step.forget_log_gate, bank, P.act_dt);
  const float in_g = ld1_rt(L.step.input_gate, bank, P.act_dt);
  const float er_g = ld1_rt(L.step.erase_gate, bank, P.act_dt);
  float4 val[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 4;
    val[c] = col < D ? ld4_rt(L.step.values, bank * D + col, P.act_dt) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  unsigned first_mask;
  int route_bits;
  const bool bad = load_routes<true, RC>(sm, L.step, nullptr, bank, bank, N, W, R, P.idx64, P.act_dt, lane,
                                         first_mask, route_bits);
  float4 acc[CH];
#pragma unroll
  for (int c = 0; c < CH; ++c) acc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (!bad) {
    // In the dense table every slot is its own row: rsrc = slot.
    for (int r = lane; r < R; r += 32) {
      if (sm.rsrc[r] == -1) sm.rsrc[r] = sm.ridx[r];
    }
    __syncwarp();
    const float alpha = expf(fl);
    float4 upd[WMAX][CH];
    const int64_t base = bank * N;
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int slot = sm.widx[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          upd[w][c] = col < D ? Elem<SDT>::ld4(L.memory, (base + slot) * D + col) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
    float4 v0[kStageReads ? 1 : ReadGroup<CH>::G][CH];
    float wt0[kStageReads ? 1 : ReadGroup<CH>::G];
    if constexpr (kStageReads) {
      if (lane * 4 < D) {
        for (int r = 0; r < R; ++r) {
          const int src = sm.rsrc[r];
          if (src >= 0)
            cp_async16(s_reads + r * D + lane * 4, static_cast<const float*>(L.memory) + (base + src) * D + lane * 4);
        }
      }
    } else {
      load_read_group<SDT, CH>(v0, wt0, sm, 0, R, L.memory, base, nullptr, 0, lane, D);
    }
    gated_delta<SDT, CH, WMAX>(upd, sm, W, alpha, in_g, er_g, val, lane, D);
#pragma unroll
    for (int w = 0; w < WMAX; ++w) {
      if (w < W) {
        const int slot = sm.widx[w];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
          const int col = (c * 32 + lane) * 4;
          if (col < D) Elem<SDT>::st4(L.memory, (base + slot) * D + col, upd[w][c]);
        }
      }
    }
    if constexpr (kStageReads) {
      cp_async_wait_all();
      if (lane * 4 < D) {
        for (int r = 0; r < R; ++r) {
          if (sm.rsrc[r] >= 0) acc[0] = f4_axpy(sm.rw[r], *reinterpret_cast<const float4*>(s_reads + r * D + lane * 4), acc[0]);
        }
      }
    } else {
      accumulate_group<CH>(acc, v0, wt0);
      read_remaining<SDT, CH>(acc, sm, R, L.memory, base, nullptr, 0, lane, D);
    }
    add_forwarded<CH, WMAX>(acc, upd, sm, W);
  }
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 4;
    if (col < D) st4_rt(L.step.output, bank * D + col, acc[c], P.act_dt);
  }
}

}  // namespace

extern "C" {

int cow_dense_step(void* const* memories, const int64_t* banks, const cow_step* steps, int32_t layers, int64_t slots,
                   int64_t width, int32_t mem_dtype, int32_t writes, int32_t reads, int32_t index_dtype,
                   int32_t act_dtype, void* stream) {
  if (!memories || !banks || !steps || layers < 1 || layers > COW_MAX_LAYERS || slots < 1) return COW_ERR_INVALID;
  if (!valid_dtype(act_dtype) || !valid_dtype(mem_dtype) || (index_dtype != COW_I32 && index_dtype != COW_I64))
    return COW_ERR_INVALID;
  if (!check_step_shape(width, writes, reads)) return COW_ERR_UNSUPPORTED;
  DenseLaunch P{};
  int64_t total = 0;
  for (int l = 0; l < layers; ++l) {
    if (!memories[l] || banks[l] < 0 || !row_aligned(memories[l], mem_dtype) || !check_step_ptrs(steps[l], act_dtype))
      return COW_ERR_INVALID;
    P.layer[l].memory = memories[l];
    P.layer[l].step = steps[l];
    P.layer[l].banks = banks[l];
    P.layer[l].bank_begin = total;
    total += banks[l];
  }
  if (total == 0) return COW_OK;
  P.slots = slots;
  P.total_banks = total;
  P.layers = layers;
  P.width = static_cast<int32_t>(width);
  P.writes = writes;
  P.reads = reads;
  P.idx64 = index_dtype == COW_I64;
  P.act_dt = act_dtype;
  void (*fn)(DenseLaunch) = nullptr;
  const int ch = width_chunks(width);
  const int rv = route_variant(writes, reads);
  COW_SELECT_KERNEL(cow_dense_kernel, mem_dtype, ch, rv, fn);
  const size_t smem = read_stage_bytes(reads, width, ch, rv, mem_dtype);
  if (resident_blocks(reinterpret_cast<const void*>(fn), kBanksPerCta * 32, smem) <= 0) return COW_ERR_UNSUPPORTED;
  const int64_t blocks = (total + kBanksPerCta - 1) / kBanksPerCta;
  fn<<<static_cast<unsigned>(blocks), kBanksPerCta * 32, smem, as_stream(stream)>>>(P);
  return launch_status();
}

}  // extern "C"
