/*
 * cow_sdm.h -- C ABI of the B200 (sm_100a) packed copy-on-write SDM library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, cast to cudaStream_t inside), allocates nothing and
 * returns an int status (COW_OK on success).  Device-side failures that can
 * only be detected while a kernel runs (slab exhaustion, bad route indices,
 * duplicate writes, a bounded wait that gave up) are OR-ed into the state's
 * 32-bit device status word (COW_ST_* bits); the host reads it at its next
 * synchronisation point.  Nothing traps or asserts on the device.
 *
 * Storage conventions are those of the reference's PackedSDMCopyOnWriteState
 * (copy_on_write_sdm/allocator.py:477-505):
 *   m0         [templates, slots, width]  shared initial memory (float32 here)
 *   templates  [banks] int64              template of each bank (bank = request*H + head)
 *   slab       [capacity, width]          pooled private rows (f32 / bf16 / f16)
 *   map        [banks, slots] int32       logical -> physical row, -1 = shared M0
 *   free_rows  [capacity] int32           free stack, top at free_rows[free_count-1]
 *   free_count int32 (device scalar)
 *   status     int32 (device scalar)      the reference's overflow_flag, widened to bits
 */
#ifndef COW_SDM_H
#define COW_SDM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------- */
#define COW_OK 0
#define COW_ERR_INVALID 1      /* bad argument (null pointer, size, alignment) */
#define COW_ERR_UNSUPPORTED 2  /* shape outside the compiled kernels (see each entry) */
#define COW_ERR_CUDA 3         /* a CUDA runtime call or launch failed */
#define COW_ERR_DEVICE 4       /* cow_decode_step_checked found status bits set */

/* ---- element / index type codes -------------------------------------- */
#define COW_F32 0
#define COW_BF16 1
#define COW_F16 2
#define COW_I32 0
#define COW_I64 1

/* ---- device status bits ---------------------------------------------- */
#define COW_ST_SLAB_EXHAUSTED 0x1     /* a first touch found the free stack empty */
#define COW_ST_INDEX_RANGE 0x2        /* a route index lies outside [0, slots) */
#define COW_ST_DUPLICATE_WRITE 0x4    /* one step wrote one logical slot twice */
#define COW_ST_WAIT_TIMEOUT 0x8       /* a bounded inter-CTA wait gave up */
#define COW_ST_TEMPLATE_RANGE 0x10    /* a template index lies outside m0 */
#define COW_ST_BAD_BANK_LIST 0x20     /* released/retained bank index invalid or duplicated */
#define COW_ST_DISCARD_LIVE 0x40      /* retain_banks would drop a bank that still owns rows */
#define COW_ST_MULTI_OWNER 0x100      /* validate: a physical row has several owners */
#define COW_ST_FREE_DUPLICATE 0x200   /* validate: free stack holds a row twice */
#define COW_ST_NOT_COVERED 0x400      /* validate: a row is neither live nor free */
#define COW_ST_ROW_RANGE 0x800        /* validate: a map / stack entry lies outside capacity */
#define COW_ST_MAP_FULL 0x1000        /* a hashed map's bank table had no empty entry for a first touch */

#define COW_MAX_LAYERS 8
#define COW_MAX_WRITES 32
#define COW_MAX_READS 256
#define COW_MAX_WIDTH 512

/* One packed pool: the reference's PackedSDMCopyOnWriteState fields. */
typedef struct cow_pool {
  const float* m0;
  const int64_t* templates;
  void* slab;
  int32_t* map;
  int32_t* free_rows;
  int32_t* free_count;
  int32_t* status;
  int64_t banks, slots, width, capacity, template_count;
  int32_t slab_dtype; /* COW_F32 / COW_BF16 / COW_F16 */
  int32_t map_kind;   /* COW_MAP_DENSE (0): map is [banks, slots] int32;
                         COW_MAP_HASH (1): map is [banks, table_slots] uint64
                         open-addressing tables (see cow_hash_from_dense) */
  int64_t table_slots; /* hashed maps: entries per bank, a power of two >= 4 (0 for dense maps) */
  /* Optional (may be NULL): a page-locked host word the decode step writes
   * once per launch after the pool's free count is settled:
   * (launch epoch << 32) | free count.  The launch epoch is the scan
   * scratch's launch counter (0 for the first launch on zero-filled scratch,
   * +1 per launch), so a runtime that owns its scratch knows which step a
   * value belongs to and can renew its capacity proof without reading the
   * device. */
  uint64_t* free_mirror;
} cow_pool;

#define COW_MAP_DENSE 0
#define COW_MAP_HASH 1

/* One decode step's routes for one pool (the arguments of
 * packed_sdm_cow_step, allocator.py:1382-1396).  Index tensors are [banks,W] /
 * [banks,R] in index_dtype; weights, values, gates and output share act_dtype.
 * erase_gate may equal input_gate (the reference's default, allocator.py:1439).
 * first_touch (optional, may be NULL) receives uint8 [banks,W]. */
typedef struct cow_step {
  const void* write_indices;
  const void* write_weights;
  const void* values;
  const void* input_gate;
  const void* erase_gate;
  const void* forget_log_gate;
  const void* read_indices;
  const void* read_weights;
  void* output;
  uint8_t* first_touch;
} cow_step;

/* Library / ABI version and the bytes of decode scan scratch a launch of
 * `layers` pools with `total_banks` banks needs.  The scratch is zero-filled
 * before first use and can then be reused by any sequence of launches on one
 * stream, whatever their pool layouts: every launch tags its scan flags with
 * one launch epoch and advances it once all its pools are closed, so flags
 * left by an earlier launch never read as published.  (The 32-bit epoch
 * repeats after 2^32 launches on one buffer; a flag would have to survive
 * untouched for that long to be misread.)  Calls that overlap on the GPU must
 * use distinct scratch. */
int cow_abi_version(void);
/* Text of the last CUDA error an entry point of this thread returned
 * COW_ERR_CUDA for ("no error" if none). */
const char* cow_last_error(void);
int64_t cow_decode_scratch_bytes(int64_t total_banks, int32_t layers);

/* Fused packed decode step over `layers` independent pools in ONE launch.
 * Replaces packed_sdm_cow_step's Triton path (allocator.py:1179-1262, kernel
 * allocator.py:74-229) and its torch path (allocator.py:1467-1526), with the
 * torch path's deterministic pop order: pop free_rows[old_free-1-rank], rank
 * = prefix count of first touches over the flattened [banks,W] order.
 * Limits: width % 4 == 0, width <= 512, W <= 32, R <= 256, layers <= 8; all
 * pools share width, W, R, slab dtype, act dtype and index dtype. */
int cow_decode_step(const cow_pool* pools, const cow_step* steps, int32_t layers,
                    int32_t writes, int32_t reads, int32_t index_dtype, int32_t act_dtype,
                    void* scan_scratch, int64_t scratch_bytes, void* stream);

/* No counterpart in the reference.  cow_decode_step for callers that cannot
 * allocate device memory when they call in: a host binding this C ABI from
 * another language or runtime (cgo, JNI, a C++ server) that does not own the
 * allocator managing the GPU's memory -- a cudaMalloc behind that allocator's
 * back would escape its accounting and can synchronise the device -- or a
 * serving loop that must not allocate while it decodes.  Same arguments and
 * results as cow_decode_step, minus the scratch: the look-back flags live in a
 * fixed COW_NOALLOC_SCRATCH_BYTES (1 MiB) array compiled into the library,
 * which every GPU that loads the library holds until the process exits.
 * - Limit: cow_decode_scratch_bytes(total banks, layers) must not exceed
 *   COW_NOALLOC_SCRATCH_BYTES (about 131,000 banks per call); larger calls
 *   return COW_ERR_SCRATCH_LIMIT and launch nothing.
 * - The first call on a device resolves the array's address for that device
 *   (cudaGetSymbolAddress, with the caller's current device); make that first
 *   call before any stream capture.  `stream` must belong to the current device.
 * - Every call on a device shares the one array and keeps what the last call
 *   left there.  Any sequence of calls that do not overlap may use it,
 *   whatever their pool layouts (the launch epoch described at
 *   cow_decode_scratch_bytes).  Calls that overlap on the GPU (e.g. on two streams)
 *   race on it.
 * - The resolved address is cached per device for the life of the process:
 *   do not keep using the library across a cudaDeviceReset.
 * Calls no cudaMalloc, cudaFree or other allocating routine. */
#define COW_ERR_SCRATCH_LIMIT 5
#define COW_NOALLOC_SCRATCH_BYTES (1 << 20)
int cow_decode_step_noalloc(const cow_pool* pools, const cow_step* steps, int32_t layers,
                            int32_t writes, int32_t reads, int32_t index_dtype, int32_t act_dtype,
                            void* stream);

/* cow_decode_step followed by a synchronisation of `stream` and a read of
 * every pool's status word: the reference's unproven / diagnostic path
 * (allocator.py:1263-1319, whose _device_assert raises on overflow and bad
 * indices).  Returns COW_ERR_DEVICE when any pool's status has bits set
 * (the pools' statuses are OR-ed into *status_out when it is not NULL),
 * COW_OK otherwise.  Blocks the calling thread; not for stream capture. */
int cow_decode_step_checked(const cow_pool* pools, const cow_step* steps, int32_t layers,
                            int32_t writes, int32_t reads, int32_t index_dtype, int32_t act_dtype,
                            void* scan_scratch, int64_t scratch_bytes, void* stream, int32_t* status_out);

/* Host-to-host decode step on `stream`: one cudaMemcpyAsync of `input_bytes`
 * from pinned `host_inputs` to `device_inputs` (the buffer the step
 * descriptors point into), the fused decode step, one cudaMemcpyAsync of
 * `output_bytes` from `device_outputs` back to pinned `host_outputs`.  The
 * serving runtime's per-token call (DecodeSession.step_host), one C call per
 * token instead of three runtime calls from the host language. */
int cow_decode_step_host(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes, int32_t reads,
                         int32_t index_dtype, int32_t act_dtype, void* scan_scratch, int64_t scratch_bytes,
                         void* device_inputs, const void* host_inputs, int64_t input_bytes, void* host_outputs,
                         const void* device_outputs, int64_t output_bytes, void* stream);

/* cow_decode_step_host with the copies on their own streams, for a runtime
 * that rotates through several input / output buffer pairs: the input copy
 * runs on `h2d_stream` once the readout copy that last read this pair's
 * `device_outputs` is done (`d2h_done`; that copy waited for the decode that
 * read `device_inputs`, so both buffers are free), the decode on
 * `compute_stream` after the input copy (`h2d_done`), the readout copy on
 * `d2h_stream` after the decode (`computed`).  All three events
 * (cudaEvent_t) belong to this buffer pair and are recorded again here.
 * Decode steps stay in call order on `compute_stream`; the copies of
 * neighbouring steps overlap them.  Nine runtime calls per step. */
int cow_decode_step_host_overlapped(const cow_pool* pools, const cow_step* steps, int32_t layers, int32_t writes,
                                    int32_t reads, int32_t index_dtype, int32_t act_dtype, void* scan_scratch,
                                    int64_t scratch_bytes, void* device_inputs, const void* host_inputs,
                                    int64_t input_bytes, void* host_outputs, const void* device_outputs,
                                    int64_t output_bytes, void* compute_stream, void* h2d_stream, void* d2h_stream,
                                    void* h2d_done, void* computed, void* d2h_done);

/* The constant arguments of cow_decode_step_host_overlapped for one buffer pair,
 * built once by a runtime that streams many steps through the same pools and
 * buffers (rebuilt whenever a pool's tensors are replaced). */
typedef struct cow_host_pipeline {
  const cow_pool* pools;
  const cow_step* steps;
  int32_t layers, writes, reads, index_dtype, act_dtype, _pad;
  void* scan_scratch;
  int64_t scratch_bytes;
  void* device_inputs;
  int64_t input_bytes;
  void* host_outputs;
  const void* device_outputs;
  int64_t output_bytes;
  void* h2d_stream;
  void* d2h_stream;
  void* h2d_done;
  void* computed;
  void* d2h_done;
} cow_host_pipeline;

/* cow_decode_step_host_overlapped with the arguments of `pipe`, for the step
 * whose pinned input bytes are `host_inputs`, decoded on `compute_stream`.
 * Same ordering and error behaviour; three arguments cross the binding per
 * step instead of twenty-one. */
int cow_decode_step_host_piped(const cow_host_pipeline* pipe, const void* host_inputs, void* compute_stream);

/* Host-to-host decode step with no copy calls: the fused decode kernel reads
 * the step's inputs straight from `host_inputs` and writes the readouts
 * straight into `host_outputs` (zero-copy access to page-locked host memory
 * over PCIe; both buffers must be pinned with cudaHostAlloc / cudaHostRegister
 * and laid out like `pipe`'s device buffers: every step pointer of `pipe`
 * is rebased from device_inputs / device_outputs onto them).  One kernel
 * launch per token and no runtime copy calls; when `pipe->d2h_done` is not
 * NULL it is recorded on `stream` after the launch and marks the readouts'
 * arrival.  Decode steps stay in call order on `stream`.  The caller must not
 * touch `host_inputs` / `host_outputs` until that event has completed. */
int cow_decode_step_host_mapped(const cow_host_pipeline* pipe, const void* host_inputs, void* host_outputs,
                                void* stream);

/* Register / forget a page-locked host range for cow_decode_step_host_mapped:
 * steps whose host buffers lie inside a registered range skip the per-call
 * pointer query (two runtime calls per token).  Registration checks that the
 * whole range is page-locked and mapped for the current device; the caller
 * keeps the memory alive and unregisters it before freeing it.  At most 64
 * ranges per process.  No counterpart in the reference (host-side serving
 * plumbing). */
int cow_register_host_range(const void* host, int64_t bytes);
int cow_unregister_host_range(const void* host);

/* Hashed logical maps (cow_pool.map_kind == COW_MAP_HASH).  No counterpart
 * in the reference, which keeps only the dense [banks, slots] int32 map
 * (allocator.py:496-504) and names a sparse map as future work.  Each bank
 * owns an open-addressing table of table_slots (a power of two, >= 4) uint64
 * entries, (slot << 32) | physical row, all ones when empty, probed in
 * 32-byte buckets of four from a multiplicative hash of the slot.
 * cow_decode_step reads and extends hashed pools directly (a first touch
 * that finds its bank's table full sets COW_ST_MAP_FULL and maps nothing);
 * every other entry point taking a cow_pool needs a dense map and returns
 * COW_ERR_UNSUPPORTED for a hashed one.
 *   cow_hash_from_dense: tables [banks, table_slots] <- every map entry >= 0
 *                        (the tables are cleared first)
 *   cow_hash_to_dense:   map [banks, slots] <- -1 everywhere, then every entry
 *   cow_hash_max_live:   *out <- the largest number of entries in one bank */
int cow_hash_from_dense(const int32_t* map, int64_t banks, int64_t slots, void* tables, int64_t table_slots,
                        int32_t* status, void* stream);
int cow_hash_to_dense(const void* tables, int64_t banks, int64_t table_slots, int32_t* map, int64_t slots,
                      int32_t* status, void* stream);
int cow_hash_max_live(const void* tables, int64_t banks, int64_t table_slots, int32_t* out, void* stream);

/* Dense-table control (dense_sdm_sparse_step, allocator.py:1529-1633, kernel
 * allocator.py:368-460): the same math on dense [banks,slots,width] tables.
 * memories[l] has dtype mem_dtype; same limits as cow_decode_step. */
int cow_dense_step(void* const* memories, const int64_t* banks, const cow_step* steps,
                   int32_t layers, int64_t slots, int64_t width, int32_t mem_dtype,
                   int32_t writes, int32_t reads, int32_t index_dtype, int32_t act_dtype,
                   void* stream);

/* Fill a fresh pool: map = -1, free_rows = arange(capacity), free_count =
 * capacity, status = 0 (PackedSDMCopyOnWriteState.allocate, allocator.py:507-586). */
int cow_init_pool(const cow_pool* pool, void* stream);

/* Prefix-count helpers shared by the lifecycle operations.  `flags_scratch`
 * is int32 [cow_scan_blocks(n) + 8].  Phase 1 counts (and, for release /
 * append, updates free_count on the device); the total lands in
 * flags_scratch[0] so the host can size new buffers before phase 2. */
int64_t cow_scan_blocks(int64_t n);

/* Prefill handoff, sparse form.  Marks the union of hard-written addresses
 * of a [banks,T,W] route list (the active mask of inference.py:334-347):
 * map[bank, slot] = 0 for every written slot.  `map` must hold -1 elsewhere
 * (the caller fills it).  Out-of-range indices set COW_ST_INDEX_RANGE. */
int cow_prefill_mark(const void* write_indices, int32_t index_dtype, int64_t banks, int64_t time,
                     int32_t writes, int64_t slots, int32_t* map, int32_t* status, void* stream);

/* map[i] = active[i] ? 0 : -1 for a uint8/bool [banks,slots] mask. */
int cow_mask_to_map(const uint8_t* active, int64_t n, int32_t* map, void* stream);

/* nonzero()-order layout, phase 1: count the entries of `map` that are >= 0.
 * The total lands in flags_scratch[0] (device int32), which the host reads
 * to size the slab before phase 2. */
int cow_pack_count(const int32_t* map, int64_t n, int32_t* flags_scratch, void* stream);
/* from_dense_overlay layout (allocator.py:589-690), phase 2: map[i] = rank in
 * nonzero() order (or -1), src_index[rank] = i, free_rows[:cap-A] = arange(A,
 * cap), free_count = cap - A, status = 0.  Rows are copied by cow_copy_rows. */
int cow_pack_apply(int32_t* map, int64_t n, int32_t* src_index, const cow_pool* pool,
                   int32_t* flags_scratch, void* stream);

/* Copy rows into a slab.  mode 0: dst[dst_rows ? dst_rows[k] : k] =
 * src[src_rows ? src_rows[k] : k]; mode 1: src_rows[k] is a flat (bank*slots+slot)
 * index and the row comes from m0[templates[bank], slot] (first-touch copy). */
int cow_copy_rows(void* dst, int32_t dst_dtype, const int32_t* dst_rows, const void* src,
                  int32_t src_dtype, const int32_t* src_rows, int64_t count, int64_t width,
                  int32_t mode, const float* m0, const int64_t* templates, int64_t slots,
                  void* stream);

/* Sparse prefix recurrence on a packed pool whose touched rows are already
 * materialised from m0: one warp per bank walks the T tokens, applying the
 * gated-delta write (sdm.py:474-529 restricted to written rows) and the
 * read-after-write readout.  Inputs [banks,T,...]; readings [banks,T,width]. */
int cow_prefill_recurrence(const cow_pool* pool, const cow_step* prefix, int64_t time,
                           int32_t writes, int32_t reads, int32_t index_dtype,
                           int32_t act_dtype, void* stream);
/* The same recurrence for `layers` independent pools (one prefix per pool,
 * same width, slots, W, R and dtypes) in one launch, so the serial token walks
 * of every SDM layer of a prefilled cohort run side by side
 * (prefill_faithful_sdm_stack, inference.py:369-456, prefills all layers). */
int cow_prefill_recurrence_layers(const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                                  int64_t time, int32_t writes, int32_t reads, int32_t index_dtype,
                                  int32_t act_dtype, void* stream);
/* The same recurrence in two passes per time chunk: a parallel pass resolves
 * the routes of every (bank, token) of the chunk against the fixed map into
 * records in `workspace` (index checks, map lookups, repeated-write check,
 * read-after-write folding), then the walk runs the chunk's tokens on those
 * records, so a token's serial chain holds only its rows and arithmetic.
 * Same rows, maps and status bits as cow_prefill_recurrence_layers (same
 * operations in the same order).  Cohorts of f32 rows, width <= 128, W <= 4
 * and R <= 32 walk with four warps per bank, whose partial readouts are
 * summed in another order: readings agree within rounding.  The workspace
 * (16-byte aligned) must hold the records of at least one token of every
 * bank; the walk covers T in chunks of as many tokens as fit (at most
 * 256 MiB of records per chunk).  cow_prefill_workspace_bytes gives the size
 * that covers the longest chunk (-1 for invalid arguments).  Launches of more
 * than 2,048 banks, which fill the GPU and are bound by row bandwidth, run
 * the per-token walk of cow_prefill_recurrence_layers and need no workspace
 * (the size is then 16).  Replaces the dense prefix recurrence of
 * sdm.py:474-529 as used by prefill_faithful_sdm_stack (inference.py:369-456). */
int64_t cow_prefill_workspace_bytes(const cow_pool* pools, int32_t layers, int64_t time, int32_t writes,
                                    int32_t reads);
int cow_prefill_recurrence_layers_ws(const cow_pool* pools, const cow_step* prefixes, int32_t layers,
                                     int64_t time, int32_t writes, int32_t reads, int32_t index_dtype,
                                     int32_t act_dtype, void* workspace, int64_t workspace_bytes, void* stream);

/* grow_capacity (allocator.py:692-744): copy rows [0,old_cap) into the new
 * slab, the old free stack below arange(old_cap,new_cap) in the new stack,
 * free_count += new_cap-old_cap, status = 0. */
int cow_grow(const void* old_slab, const int32_t* old_free_rows, int64_t old_capacity,
             void* new_slab, int32_t* new_free_rows, int64_t new_capacity, int64_t width,
             int32_t slab_dtype, int32_t* free_count, int32_t* status, void* stream);

/* grow_capacity (allocator.py:692-744) when the slab and free stack already have
 * storage for new_capacity rows (a reserve behind the current capacity): the
 * same resulting stack and free_count as cow_grow, with no row copy.  free_rows
 * must hold new_capacity entries. */
int cow_grow_in_place(int32_t* free_rows, int64_t old_capacity, int64_t new_capacity, int32_t* free_count,
                      int32_t* status, void* stream);

/* release (allocator.py:1019-1068): push every live row of the selected banks
 * at old_free + rank over the flattened [S,slots] order given; clear their map
 * rows.  `released` receives the count (device int32).  `bank_mask` is int32
 * [banks] scratch used to reject out-of-range or repeated bank indices
 * (COW_ST_BAD_BANK_LIST in the pool status; nothing is released then). */
int cow_release(const cow_pool* pool, const int64_t* bank_indices, int64_t count,
                int32_t* bank_mask, int32_t* flags_scratch, int32_t* released, void* stream);

/* trim_capacity (allocator.py:776-840), phase 2 after cow_pack_count on the
 * pool's map: new_map = rank in nonzero() order, rows gathered into
 * new_slab[0..A), new_free_rows[:new_cap-A] = arange(A,new_cap). */
int cow_repack(const cow_pool* pool, int32_t* new_map, void* new_slab, int32_t* new_free_rows,
               int64_t new_capacity, int32_t* src_rows, int32_t* flags_scratch, void* stream);

/* append_banks_from (allocator.py:842-915), after cow_pack_count on other's
 * map: pop A rows from the top of dst's stack in other's nonzero() order, copy
 * the rows, write the admitted map rows into admitted_map [other.banks,slots]
 * and decrement dst's free_count. */
int cow_append(const cow_pool* dst, const cow_pool* other, int32_t* admitted_map,
               int32_t* src_rows, int32_t* dst_rows, int32_t* flags_scratch, void* stream);

/* retain_banks (allocator.py:917-943): new_map[s] = map[idx[s]], new_templates[s]
 * = templates[idx[s]]; sets COW_ST_BAD_BANK_LIST / COW_ST_DISCARD_LIVE in
 * `status` (a scratch status word, not the pool's) instead of raising.
 * `selected` is int32 [banks] scratch. */
int cow_retain(const cow_pool* pool, const int64_t* bank_indices, int64_t count,
               int32_t* new_map, int64_t* new_templates, int32_t* selected, int32_t* status,
               void* stream);

/* validate_invariants (allocator.py:1070-1096) on the device: `counts` is
 * int32 [capacity] scratch; result bits are OR-ed into `status`. */
int cow_validate(const cow_pool* pool, int32_t* counts, int32_t* status, void* stream);

/* ---- several pools per call ---------------------------------------------
 * The SDM layers of one serving batch change together: release, compaction,
 * admission and prefill touch every layer's pool.  These entry points do one
 * operation for up to COW_MAX_LAYERS pools with one set of launches (the pool
 * is a grid dimension), writing every per-pool result the host needs into one
 * small device array so that a single synchronisation reads them all.  Each
 * takes a caller-owned, 16-byte aligned `workspace` of at least the matching
 * *_workspace_bytes() (a negative size means the arguments are invalid); the
 * workspace is free again when the call's work has run on `stream`.
 * Per-pool pointer arguments are host arrays of device pointers. */

/* release for each pool l of counts[l] banks bank_indices[l][*]; released[l]
 * (device int32) receives pool l's count. */
int64_t cow_release_workspace_bytes(const cow_pool* pools, const int64_t* counts, int32_t layers);
int cow_release_layers(const cow_pool* pools, const int64_t* const* bank_indices, const int64_t* counts,
                       int32_t layers, void* workspace, int64_t workspace_bytes, int32_t* released, void* stream);

/* retain_banks for each pool; status[l] (device int32) receives pool l's
 * COW_ST_BAD_BANK_LIST / COW_ST_DISCARD_LIVE bits (zero = the new map and
 * templates in new_maps[l] / new_templates[l] are valid). */
int64_t cow_retain_workspace_bytes(const cow_pool* pools, int32_t layers);
int cow_retain_layers(const cow_pool* pools, const int64_t* const* bank_indices, const int64_t* counts, int32_t layers,
                      int32_t* const* new_maps, int64_t* const* new_templates, void* workspace,
                      int64_t workspace_bytes, int32_t* status, void* stream);

/* append_banks_from for each pair (dsts[l], others[l]).  Phase 1 writes
 * counts[2l] = live rows of others[l] and counts[2l+1] = free rows of dsts[l]
 * (device int32) so that the host can grow dsts[l] first; phase 2 (same
 * workspace, untouched in between) pops, copies the rows and writes the
 * admitted map rows into admitted_maps[l] [others[l].banks, slots]. */
int64_t cow_append_workspace_bytes(const cow_pool* others, int32_t layers);
int cow_append_count_layers(const cow_pool* dsts, const cow_pool* others, int32_t layers, void* workspace,
                            int64_t workspace_bytes, int32_t* counts, void* stream);
int cow_append_layers(const cow_pool* dsts, const cow_pool* others, int32_t layers, int32_t* const* admitted_maps,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* Sparse prefill layout for each pool.  Phase 1 sets maps[l] [banks,slots] to
 * -1, marks the written slots of write_indices[l] [banks,T,W] and counts them:
 * out[2l] = status bits (COW_ST_INDEX_RANGE for a write route, or a read
 * route of read_indices[l] [banks,T,R] when reads > 0, outside the slots;
 * COW_ST_DUPLICATE_WRITE for a token that writes one slot twice),
 * out[2l+1] = live rows.  Phase 2
 * (same workspace; pools[l].map = maps[l], slab and stack sized by the host)
 * assigns rows 0..A-1 in nonzero() order, fills the free stack with
 * arange(A, capacity) and copies each live row from m0.  n = banks*slots. */
int64_t cow_pack_workspace_bytes(int64_t n, int32_t layers);
int cow_prefill_mark_count_layers(const void* const* write_indices, const void* const* read_indices,
                                  int32_t index_dtype, int64_t banks, int64_t time, int32_t writes, int32_t reads,
                                  int64_t slots, int32_t* const* maps, int32_t layers, void* workspace,
                                  int64_t workspace_bytes, int32_t* out, void* stream);
int cow_pack_apply_layers(const cow_pool* pools, int32_t layers, void* workspace, int64_t workspace_bytes,
                          void* stream);

/* A prefilled cohort admitted straight into live pools: the same result as
 * packing the cohort into pools of its own (cow_pack_apply_layers) and then
 * appending them (cow_append_layers, allocator.py:842-915), without the
 * cohort's slab.  `marks[l]` [cohort_banks, slots] holds the marks of
 * cow_prefill_mark_count_layers (0 written, -1 not); every marked entry, in
 * nonzero() order, pops dsts[l]'s free stack (free_rows[free_count-1-rank]),
 * its row is filled from m0[cohort_templates[bank], slot] and
 * admitted_maps[l] [cohort_banks, slots] receives the popped rows (-1
 * elsewhere); free_count drops by the live count.  The caller proves the
 * free rows beforehand (growing the pool as append does), then extends the
 * pool's map and templates with admitted_maps / cohort_templates and runs the
 * prefix walk (cow_prefill_recurrence_layers_ws) on the admitted banks.  No
 * counterpart in the reference as one call (it is prefill_faithful_sdm_stack
 * followed by FaithfulSDMDecodeState.admit, inference.py:161-206, 369-456). */
int64_t cow_admit_prefix_workspace_bytes(int64_t cohort_banks, int64_t slots, int32_t layers);
int cow_admit_prefix_layers(const cow_pool* dsts, int32_t* const* marks, const int64_t* cohort_templates,
                            int64_t cohort_banks, int32_t layers, int32_t* const* admitted_maps, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* validate_invariants for each pool: out[3l..3l+2] (device int32) = the
 * pool's status word, the partition bits (COW_ST_MULTI_OWNER,
 * COW_ST_FREE_DUPLICATE, COW_ST_NOT_COVERED, COW_ST_ROW_RANGE), free count. */
int64_t cow_validate_workspace_bytes(const cow_pool* pools, int32_t layers);
int cow_validate_layers(const cow_pool* pools, int32_t layers, void* workspace, int64_t workspace_bytes, int32_t* out,
                        void* stream);

/* Controller route selection (sdm.py:96-159, inference.py:459-519), FP32: from
 * the read / write codebook projections [B,T,H*2*root] and the forget / input
 * gate projections [B,T,H], one warp per (bank = b*H+h, position t) writes the
 * product-key addresses (sorted ascending) and softmax weights [B*H,T,R|W],
 * forget_log_gate = -exp(A_log[h]) * softplus(f + dt_bias[h]) and
 * input_gate = sigmoid(i) [B*H,T].  root = sqrt(N) <= 256, R, W <= 32. */
int cow_route_controller(const float* read_proj, const float* write_proj, const float* forget_proj,
                         const float* input_proj, const float* a_log, const float* dt_bias, int64_t batch,
                         int64_t time, int32_t heads, int32_t root, int32_t reads, int32_t writes,
                         int64_t* read_indices, float* read_weights, int64_t* write_indices, float* write_weights,
                         float* input_gate, float* forget_log_gate, void* stream);

/* The whole SDM controller for a [B,T,width] token block, FP32: layer norm
 * (ln_weight, ln_bias, eps), the read / write / value / forget / input
 * projections as one matrix weights_t [width, Ntot] (columns: read H*2*root,
 * write H*2*root, value width, forget H, input H; bias [Ntot]), then per bank
 * the route selection and gates of cow_route_controller and the value slice
 * [B*H,T,width/H].  normalized [B,T,width] is written for the readout.
 * width <= 512, Ntot <= 4096, root <= 256, R, W <= 32. */
int cow_controller_step(const float* tokens, const float* ln_weight, const float* ln_bias, float eps,
                        const float* weights_t, const float* bias, const float* a_log, const float* dt_bias,
                        int64_t batch, int64_t time, int32_t width, int32_t heads, int32_t root, int32_t reads,
                        int32_t writes, float* normalized, int64_t* read_indices, float* read_weights,
                        int64_t* write_indices, float* write_weights, float* values, float* input_gate,
                        float* forget_log_gate, void* stream);

/* The SDM layer's readout, its residual add and the MLP block after it, for a
 * [B,T,width] token block, FP32 (replaces copy_on_write_sdm/inference.py:523-536
 * _finish_faithful_sdm_step with the adds at inference.py:660-661 and
 * model.py:25-45 ResidualMLP in eval mode):
 *   r   = LayerNorm_hw(readings [B*H,T,hw]; rn_weight, rn_bias, rn_eps), heads -> width
 *   t1  = tokens + out_weight (sigmoid(gate_weight normalized + gate_bias) * r) + out_bias
 *   out = t1 + mlp_out_weight GELU_erf(mlp_in_weight LayerNorm(t1; mlp_norm_*, mlp_eps))
 * Matrices are passed transposed ([in, out], row-major).  width <= 512,
 * hidden <= 2048, heads <= 64; out must not alias tokens. */
int cow_readout_mlp_step(const float* tokens, const float* normalized, const float* readings, const float* rn_weight,
                         const float* rn_bias, float rn_eps, const float* gate_weight_t, const float* gate_bias,
                         const float* out_weight_t, const float* out_bias, const float* mlp_norm_weight,
                         const float* mlp_norm_bias, float mlp_eps, const float* mlp_in_weight_t,
                         const float* mlp_out_weight_t, int64_t batch, int64_t time, int32_t width, int32_t heads,
                         int32_t hidden, float* out, void* stream);

/* One decode token per request through a dense attention block and the MLP after
 * it, FP32 (replaces copy_on_write_sdm/inference.py:640-651: model.py
 * CausalSelfAttention.decode_with_cache, the residual adds and ResidualMLP, eval
 * mode): LayerNorm(ln_*), q|k|v = qkv_weight n (no bias), k and v stored at
 * positions[b] of key_cache / value_cache [batch, heads, capacity, width/heads],
 * softmax(q.K/sqrt(hw)) V over slots 0..positions[b] per head, t1 = tokens +
 * out_weight o, out = t1 + mlp_out GELU_erf(mlp_in LayerNorm(t1; mlp_norm_*)).
 * positions is a device int64 [batch]; a position outside [0, capacity) gives a
 * NaN row and writes nothing.  Matrices are transposed ([in, out], row-major).
 * width <= 512, hidden <= 2048, heads * capacity bounded by shared memory
 * (COW_ERR_UNSUPPORTED beyond); out must not alias tokens. */
int cow_attention_mlp_decode(const float* tokens, const int64_t* positions, const float* ln_weight,
                             const float* ln_bias, float ln_eps, const float* qkv_weight_t,
                             const float* out_weight_t, float* key_cache, float* value_cache, int64_t capacity,
                             const float* mlp_norm_weight, const float* mlp_norm_bias, float mlp_eps,
                             const float* mlp_in_weight_t, const float* mlp_out_weight_t, int64_t batch,
                             int32_t width, int32_t heads, int32_t hidden, float* out, void* stream);

/* materialize_dense (allocator.py:1004-1017): dense [banks,slots,width] in out_dtype. */
int cow_materialize(const cow_pool* pool, void* out, int32_t out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* COW_SDM_H */
