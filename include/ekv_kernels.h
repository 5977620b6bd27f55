/*
 * ekv_kernels.h — C ABI of libekv_b200.so, the sm_100a data path for sparse-KV
 * residency: lookup, Top-K row gather, demote/promote row migration and the
 * per-chunk freeable bitmap with its cross-rank AND.
 *
 * Conventions (same as the reference's ev_* ABI, native/elastic_vmm.cpp:289-369):
 *   - every function returns int: 0 on success, -1 on error;
 *   - ekv_error() returns the calling thread's last error message ("" if none);
 *   - pointers are plain device addresses (or mapped pinned-host addresses where
 *     a parameter says so); strides and sizes are int64 element counts unless a
 *     name ends in _bytes;
 *   - index arrays carry their element size (4 = int32, 8 = int64) in the
 *     matching *_esize argument; values are read as signed integers;
 *   - `device` is the CUDA ordinal that owns `stream` and every buffer; the call
 *     makes it current for the calling thread before launching;
 *   - work is launched asynchronously on `stream` (a cudaStream_t, NULL = the
 *     legacy default stream); no call synchronizes, allocates device memory, or
 *     retains a pointer after it returns.
 * Threading: calls may come from any thread; concurrent calls that write the
 * same buffers race exactly as two kernels on different streams would.
 */
#ifndef EKV_KERNELS_H
#define EKV_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Largest number of planes (K/V tensors of individual layers) one call takes. */
#define EKV_MAX_PLANES 256
/* Most requests whose host-side shared-prefix metadata fits the launch parameters. */
#define EKV_SHARED_INLINE_MAX 512
/* Most layers one logical-shadow migration check or reset covers in a launch. */
#define EKV_SHADOW_MAX_LAYERS 128

/* Thread-local message of the last failed call on this thread. */
const char* ekv_error(void);

/* ABI version of this library (bumped on any signature change). */
#define EKV_ABI_VERSION 2
int ekv_abi_version(void);

/*
 * R1 — resident lookup.  Replaces the Triton `_resolve` launch of
 * resolve_resident (adaptive_sparse/resident_lookup.py:6-40).
 * For every s < n_selected, row = selected[s], and every column j < width
 * (width = topk_width * block_size):
 *     block = topk[row, j / block_size];  pos = block * block_size + j % block_size
 *     out[row, j] = (block >= 0 && pos < lengths[row])
 *                   ? (int32) mapping[table[rows[row], pos]] : -1
 * Rows not listed in `selected` are not written.  All arrays are strided.
 */
int ekv_resolve_resident(
    const void* topk, int topk_esize, int64_t topk_row_stride, int64_t topk_col_stride,
    int64_t topk_width,
    const void* table, int table_esize, int64_t table_row_stride, int64_t table_col_stride,
    const void* mapping, int mapping_esize, int64_t mapping_stride,
    const void* rows, int rows_esize, int64_t rows_stride,
    const void* lengths, int lengths_esize, int64_t lengths_stride,
    const void* selected, int selected_esize, int64_t selected_stride, int64_t n_selected,
    int32_t* out, int64_t out_row_stride, int64_t out_col_stride,
    int64_t block_size, int device, void* stream);

/*
 * R2 — logical-token -> hot-slot lookup with miss detection and compaction.
 * No single reference symbol: R1 with `mapping` replaced by a per-request
 * residency map (-1 = not resident), plus the hit/miss contract of the swap
 * kernel exercised by tests/smoke_minimax_swap.py:28-62.
 * For b < batch, i < k:  t = topk[b, i]; n = min(lengths[b], map_width)
 *     valid = 0 <= t < n;  slot = valid ? res_map[b, t] : -1
 *     slots[b, i] = slot;  miss[b, i] = valid && slot < 0
 * miss_list[b, :] holds the token ids t of row b's misses in ascending i order,
 * followed by -1 up to k; miss_count[b] is their number.  lengths may be NULL
 * (n = map_width); miss, miss_list and miss_count may each be NULL.
 */
int ekv_lookup_slots(
    const void* res_map, int map_esize, int64_t map_row_stride, int64_t map_width,
    const void* topk, int topk_esize, int64_t topk_row_stride,
    const void* lengths, int lengths_esize,
    int64_t batch, int64_t k,
    int32_t* slots, int64_t slots_row_stride,
    uint8_t* miss, int64_t miss_row_stride,
    int32_t* miss_list, int64_t miss_list_row_stride,
    int32_t* miss_count,
    int device, void* stream);

/*
 * R3 — Top-K row gather.  Replaces the Triton `_gather` launch of gather_rows
 * (experimental/sparse_read.py:11-51).  For b < batch, i < selected:
 *     pos = positions[b*selected + i], req = request_ids[b]
 *     valid = 0 <= pos < lengths[b]
 *     off = indirect == 1 ? slot_offsets[request_table[req*table_width + pos]]
 *         : indirect == 2 ? sink_elements + req*request_stride + s*width
 *                           with s = request_table[req*table_width + pos]  (valid only if s >= 0)
 *         :                 sink_elements + req*request_stride + pos*width
 *     out[(b*selected + i)*width + c] = valid ? raw[off + c] : 0,  c < width
 * Modes 0 and 1 are the reference's direct and software-table addressing; mode
 * 2 ("mapped", new) reads a residency map (token -> slot in the request's fixed
 * region, -1 = absent) so a lookup and its gather are one launch; there a position
 * must also be below table_width (the map's row width) to be valid.
 * Offsets, strides and width are counted in elements of `itemsize` bytes; the
 * payload is copied bit for bit.  Index arrays are contiguous.
 *
 * `indirect` may carry EKV_GATHER_INDICES_READY (ORed onto the mode): the caller
 * promises that the kernel launched immediately before this one in `stream` does
 * not write positions, request_ids, lengths, request_table or slot_offsets.  The
 * gather then walks its first index chain while that kernel drains (programmatic
 * dependent launch) instead of after it; payload reads and every store still wait
 * for it.  Results are identical either way; only a broken promise can differ.
 */
#define EKV_GATHER_INDICES_READY 16
/*
 * `indirect` may also carry EKV_GATHER_DISJOINT: the caller promises that no kernel
 * that may still run when this gather starts -- the kernels before it in `stream`
 * back to the last one launched without this flag -- writes anything the gather
 * reads or reads or writes anything it writes (e.g. the back-to-back per-layer
 * gathers of a decode step: disjoint planes, index inputs and outputs).  The gather
 * then copies at once, while those kernels drain, and waits for them only before
 * it completes, so the stream's order of completion is kept.
 */
#define EKV_GATHER_DISJOINT 32
int ekv_gather_rows(
    const void* raw, void* out, int64_t itemsize,
    const void* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* request_table, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream);

/*
 * R3, batched over planes — the same row selection applied to n_planes
 * source planes at once (all layers' K and V in one launch; the index chain is
 * resolved once per row).  src_planes / dst_planes are HOST arrays of n_planes
 * device addresses (n_planes <= EKV_MAX_PLANES); plane p's row comes from
 * src_planes[p] + off*itemsize and lands at dst_planes[p] + (b*selected+i)*width*itemsize.
 */
int ekv_gather_rows_planes(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
    const void* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* request_table, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream);

/*
 * R2 + R3 fused — one layer's lookup_slots and its mapped gather in one launch,
 * so each residency-map entry is read once per layer instead of once by the
 * lookup and again by the gather.  No reference counterpart: the reference
 * resolves a layer's Top-K (request_residency.py:819-826) and then reads the
 * rows (sparse_read.py:33-51) in separate launches.  res_map is [batch', map_width]
 * contiguous; request_ids[b] picks row b's map row and region; for b < batch, i < k:
 *     t = topk[b*k + i];  n = min(lengths[b], map_width);  valid = 0 <= t < n
 *     s = valid ? res_map[request_ids[b]*map_width + t] : -1
 *     slots[b*k + i] = s (int32);  miss[b*k + i] = valid && s < 0
 * and plane p's output row (b, i) is ekv_gather_rows_planes in mapped mode (2)
 * with positions = topk, request_table = res_map, table_width = map_width.  With
 * request_ids = 0..batch-1, slots and miss equal ekv_lookup_slots' on the same
 * map, Top-K and lengths; ekv_compact_misses then gives its miss list and count.
 * slots and miss are contiguous [batch, k].  flags: EKV_GATHER_INDICES_READY and/or
 * EKV_GATHER_DISJOINT.
 */
int ekv_lookup_gather_planes(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_planes, int64_t itemsize,
    const void* topk, int topk_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const void* res_map, int map_esize, int64_t map_width,
    int64_t batch, int64_t k, int64_t width,
    int64_t request_stride, int64_t sink_elements,
    int32_t* slots, uint8_t* miss,
    int flags, int device, void* stream);

/*
 * R2's miss-list compaction from a miss mask already written (by
 * ekv_lookup_gather_planes): miss_list[b, :] holds topk[b, i] for every i with
 * miss[b, i] != 0 in ascending i order, then -1 up to k; miss_count[b] (may be
 * NULL) is their number -- ekv_lookup_slots' miss_list and miss_count for the
 * same mask.  No reference counterpart (a part of R2).
 */
int ekv_compact_misses(
    const uint8_t* miss, int64_t miss_row_stride,
    const void* topk, int topk_esize, int64_t topk_row_stride,
    int64_t batch, int64_t k,
    int32_t* miss_list, int64_t miss_list_row_stride,
    int32_t* miss_count,
    int device, void* stream);

/*
 * R3, batched over layers — every layer's own row selection in one launch: layer
 * l (l < n_layers <= EKV_MAX_LAYERS) is ekv_gather_rows_planes over planes
 * l*planes_per_layer .. (l+1)*planes_per_layer - 1 of src_planes / dst_planes
 * with positions[l] and request_tables[l] (HOST arrays of n_layers device
 * addresses; request_tables may be NULL in direct mode).  request_ids, lengths,
 * slot_offsets and the geometry are shared by all layers;
 * n_layers * planes_per_layer <= EKV_MAX_PLANES.  No flag bits.  For a decode
 * step whose every layer's Top-K is known when the step starts: the same bytes
 * as n_layers per-layer calls, without a launch boundary between layers.  The
 * per-layer entry points above replace the reference's per-layer calls; this one
 * has no reference counterpart.
 */
#define EKV_MAX_LAYERS 128
int ekv_gather_layers(
    const uint64_t* src_planes, const uint64_t* dst_planes, int n_layers, int planes_per_layer,
    int64_t itemsize,
    const uint64_t* positions, int positions_esize,
    const void* request_ids, int request_ids_esize,
    const void* lengths, int lengths_esize,
    const uint64_t* request_tables, int table_esize,
    const void* slot_offsets, int offsets_esize,
    int64_t batch, int64_t selected, int64_t width,
    int64_t table_width, int64_t request_stride, int64_t sink_elements,
    int indirect, int device, void* stream);

/*
 * R5 — migration row copies between KV planes and a staging buffer.  Replaces
 * the data movement of HostKVCache.backup_from_device_all_layer /
 * load_to_device_per_layer called at adaptive_sparse/migration.py:109-111 and
 * :231-237.  `staging` may be device memory or pinned host memory that is
 * mapped into the device address space (cudaHostAlloc / cudaHostRegister).
 *
 * Task list: n_tasks rows.  Task t copies row_bytes between
 *     plane  planes[p] + slot*row_bytes   and   staging + soff
 * where
 *   plane_index != NULL ("list" form):
 *       p = plane_index[t] (int32), slot = slots[t], soff = stage_rows ? stage_rows[t]*row_bytes
 *                                                                       : t*row_bytes
 *   plane_index == NULL ("cross" form, n_tasks = n_planes * n_slots):
 *       p = t / n_slots, j = t % n_slots, slot = slots[j],
 *       soff = p*stage_plane_stride_bytes + (stage_rows ? stage_rows[j] : j)*row_bytes
 * ekv_pack_rows copies plane -> staging, ekv_unpack_rows staging -> plane.
 * planes is a HOST array of n_planes device addresses.
 */
int ekv_pack_rows(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const void* stage_rows, int stage_rows_esize,
    void* staging, int64_t stage_plane_stride_bytes, int64_t n_tasks,
    int device, void* stream);

int ekv_unpack_rows(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const void* stage_rows, int stage_rows_esize,
    const void* staging, int64_t stage_plane_stride_bytes, int64_t n_tasks,
    int device, void* stream);

/*
 * R5, staged through the copy engines — the same task list (plane_index /
 * slots / n_slots / n_tasks as above; no stage_rows) moved between the planes
 * and PINNED host memory `host_staging` through a ring of four device slots cut
 * from the caller's `scratch` device buffer (scratch_bytes >= 4 * 256-aligned
 * slots of at least one row): the row-copy kernel packs / unpacks one slot on
 * `stream` while `copy_stream` (NULL = an internal per-device stream) moves
 * another across the host link with cudaMemcpyAsync.
 * `segments` is a HOST array of n_segments triples (first_task, count,
 * host_byte_offset): tasks [first_task, first_task + count) occupy consecutive
 * rows of host_staging starting at host_byte_offset; segments are in task order
 * and cover [0, n_tasks).  When `stream` completes, the transfer is complete.
 * Calls on one device must not overlap.  Replaces the same reference call sites
 * as ekv_pack_rows / ekv_unpack_rows.
 */
int ekv_pack_rows_staged(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    void* host_staging, int64_t n_tasks,
    void* scratch, int64_t scratch_bytes,
    int device, void* stream, void* copy_stream);

int ekv_unpack_rows_staged(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    const void* host_staging, int64_t n_tasks,
    void* scratch, int64_t scratch_bytes,
    int device, void* stream, void* copy_stream);

/*
 * Staged demotion that allocates nothing.  No counterpart in the reference.
 * Same arguments and result as ekv_pack_rows_staged without `scratch`: the
 * ring is the library's own 8 MiB device array (4 slots of 2 MiB), held by
 * every GPU that loads the library until the process exits.  For callers that
 * cannot allocate device memory when they demote (an engine that reserved all
 * of HBM for its KV pool, a host without a device allocator).  Rows must be at
 * most 2 MiB (larger ones are rejected with an error).  The first call on a
 * device looks up the ring's address with that device current: make it before
 * any stream capture.  That address (and the copy stream and events the staged
 * path keeps per device) is cached for the life of the process, so resetting
 * the device (cudaDeviceReset) after the first call is not supported.  Calls
 * share the ring: calls that overlap on the GPU race.  Calls no cudaMalloc /
 * cudaFree.
 */
int ekv_pack_rows_staged_noalloc(
    const uint64_t* planes, int n_planes, int64_t row_bytes,
    const int32_t* plane_index, const void* slots, int slots_esize, int64_t n_slots,
    const int64_t* segments, int64_t n_segments,
    void* host_staging, int64_t n_tasks,
    int device, void* stream, void* copy_stream);

/*
 * Hot-buffer swap-in, step 1: victim selection.  Replaces the LRU half of the
 * block swap kernel the reference calls through SGLang's coordinator
 * (adaptive_sparse/request_residency.py:805-809, :829-832).  One block per row b:
 * hot slots referenced by this step's hits (slots[b, :] >= 0, from
 * ekv_lookup_slots) are pinned; misses r < miss_count[b] (miss_list[b, r]) take
 * the first unreferenced slots in ring order starting at hand[b], written to
 * promo_slot[b, r] (-1 for r >= the number assigned); then
 * res_map[b, evicted token] = -1, res_map[b, miss token] = slot,
 * slot_token[b, slot] = miss token, hand[b] = last victim + 1 (mod hot_capacity).
 * All arrays int32; hot_capacity <= 65536.  Top-K token ids must be unique per row.
 */
int ekv_swap_select(
    int32_t* res_map, int64_t map_row_stride, int64_t map_width,
    int32_t* slot_token, int64_t token_row_stride, int64_t hot_capacity,
    int32_t* hand,
    const int32_t* slots, int64_t slots_row_stride, int64_t k,
    const int32_t* miss_list, int64_t list_row_stride, const int32_t* miss_count,
    int32_t* promo_slot, int64_t promo_row_stride,
    int64_t batch, int device, void* stream);

/*
 * Hot-buffer swap-in, step 2: promotion copies.  Replaces the host -> hot-buffer
 * loads of the same swap kernel.  For every row b, r < miss_count[b] with
 * promo_slot[b, r] = s >= 0 and token t = miss_list[b, r], and every plane p:
 *     hot_planes[p] + sink_bytes + b*request_bytes + s*row_bytes
 *         <- history_planes[p] + (b*history_rows_per_request + t)*row_bytes
 * history_planes may be pinned host memory (read through unified addressing)
 * or device memory; both plane arrays are HOST arrays of n_planes addresses.
 */
int ekv_promote_rows(
    const uint64_t* history_planes, const uint64_t* hot_planes, int n_planes, int64_t row_bytes,
    int64_t history_rows_per_request, int64_t sink_bytes, int64_t request_bytes,
    const int32_t* miss_list, int64_t list_row_stride, const int32_t* miss_count,
    const int32_t* promo_slot, int64_t promo_row_stride,
    int64_t batch, int64_t k, int device, void* stream);

/*
 * R4/R6 — page -> chunk projection counts.  Restates PhysicalPages.chunks
 * (adaptive_sparse/minimax_vmm.py:40-52) and _chunk_release_counts
 * (adaptive_sparse/scheduler_budget.py:155-156): for each page and plane p,
 * the chunks plane_chunk[p] + [page*page_size*row_bytes[p] / chunk_bytes,
 * (page*page_size*row_bytes[p] + page_size*row_bytes[p] - 1) / chunk_bytes]
 * each get +1 in counts[0:n_chunks] (int32).  Pages must be distinct.  When
 * `accumulate` is 0 counts is cleared first.  plane_chunk / plane_row_bytes are
 * HOST arrays of n_planes values.  Chunks >= n_chunks are counted in
 * *overflow (device int32, may be NULL) instead of being written.
 */
int ekv_chunk_counts(
    const void* pages, int pages_esize, int64_t n_pages,
    const int64_t* plane_chunk, const int64_t* plane_row_bytes, int n_planes,
    int64_t page_size, int64_t chunk_bytes,
    int32_t* counts, int64_t n_chunks, int accumulate, int32_t* overflow,
    int device, void* stream);

/*
 * R6 — freeable bitmap.  Restates _releasable_counts
 * (adaptive_sparse/scheduler_budget.py:159-162): bit c of out_bits is set iff
 *     counts[c] > 0 && counts[c] == refs[c] && bit c of mapped_bits is set.
 * Bitmaps are uint64 words, chunk c at word c/64, bit c%64; bits >= n_chunks
 * of the last word are 0.
 */
int ekv_freeable_bitmap(
    const int32_t* counts, const int32_t* refs, const uint64_t* mapped_bits,
    int64_t n_chunks, uint64_t* out_bits, int device, void* stream);

/*
 * R6 — cross-rank combine: out[w] = AND over r < n_ranks of gathered[r*n_words + w].
 * Replaces the candidate-key intersection of rank_demotions
 * (adaptive_sparse/runtime_value.py:180-185) over the exchange() of
 * adaptive_sparse/scheduler_budget.py:1447-1452 for the joint chunk set;
 * `gathered` is the NCCL all-gather of every rank's bitmap.
 */
int ekv_bitmap_and(
    const uint64_t* gathered, int n_ranks, int64_t n_words, uint64_t* out,
    int device, void* stream);

/*
 * R6 — freeable bitmap and its AND over the tensor-parallel ranks in ONE kernel,
 * over peer memory instead of an NCCL all-gather (same result as
 * ekv_freeable_bitmap + all-gather + ekv_bitmap_and).  Every rank launches it with
 * the same `epoch` (a call counter starting at 1).  peer_buffers is a HOST array
 * of n_ranks device addresses (rank r's peer-visible buffer, e.g. symmetric
 * memory; 256 + 16 * n_words bytes, zeroed once before the first call);
 * peer_buffers[rank] is this rank's own.  The local bitmap is either built from
 * counts / refs / mapped_bits or taken from local_bits.  A rank waits at most
 * max_polls polls (~64 ns apart) for each peer; if one does not arrive, *status
 * (device uint32, may be NULL) gets bit 0 and `out` is not written.
 * local_out (may be NULL) receives this rank's own bitmap.
 */
int ekv_freeable_and_peers(
    const int32_t* counts, const int32_t* refs, const uint64_t* mapped_bits, const uint64_t* local_bits,
    int64_t n_chunks, const uint64_t* peer_buffers, int n_ranks, int rank, uint32_t epoch,
    uint32_t max_polls, uint64_t* out, uint64_t* local_out, uint32_t* status, int device, void* stream);

/*
 * Shared-prefix donor-slot resolution, batched — replaces
 * resolve_shared_block_locations_batched (adaptive_sparse/shared_prefix.py:122-204;
 * the scalar form :70-119 is requests = 1) called at
 * adaptive_sparse/request_residency.py:210-218.
 *
 * block_ids [requests, per_request] (int32/int64, strides block_row / block_col
 * elements).  source_rows / shared_tokens: int64 [requests] in device memory, or
 * NULL to use the scalar source_row / shared_count for every request; with
 * meta_on_host != 0 both are HOST arrays of at most EKV_SHARED_INLINE_MAX
 * entries, copied into the launch parameters (no device copy; reusable as soon
 * as the call returns).  seq_len
 * [requests] (stride len_stride; 0 broadcasts one value).  request_table
 * [table_rows, table_width] with strides table_row / table_col; device_mapping
 * [map_len] with stride map_stride.  Outputs: valid uint8 [requests, per_request]
 * and physical int32 [requests, per_request, block_size] (contiguous).
 * masked_blocks (may be NULL, may alias block_ids, same esize and strides)
 * receives -1 where the block is valid and the block id elsewhere, the caller's
 * masked_fill (request_residency.py:231).  exclude_newest != 0 also requires
 * (block + 1) * block_size < seq_len (request_residency.py:220).
 * Source rows must lie in [0, table_rows) (the Python API checks this, as the
 * reference does); a row outside resolves to slot 0 and an invalid block.
 */
int ekv_resolve_shared_blocks(
    const void* block_ids, int block_esize, int64_t requests, int64_t per_request, int64_t block_row,
    int64_t block_col, const int64_t* source_rows, int64_t source_row, const int64_t* shared_tokens,
    int64_t shared_count, const void* seq_len, int len_esize, int64_t len_stride, int64_t block_size,
    const void* request_table, int table_esize, int64_t table_rows, int64_t table_width, int64_t table_row,
    int64_t table_col, const void* device_mapping, int map_esize, int64_t map_len, int64_t map_stride,
    int meta_on_host, uint8_t* valid, int32_t* physical, void* masked_blocks, int exclude_newest, int device,
    void* stream);

/*
 * Logical-shadow checker (diagnostic bitwise validation of KV rows) — replaces
 * the torch bodies of LogicalShadow (adaptive_sparse/logical_shadow.py:14-140).
 * Rows are bf16 (any even byte length); every stride below is in BYTES between
 * consecutive slots of a [slots, ...] buffer whose rows are contiguous.
 *
 * ekv_shadow_check — LogicalShadow.check (:45-86) for one decode step of one
 * layer.  blocks [1, batch, n_blocks] (strides blocks_row / blocks_col
 * elements of dims 1 and 2), lengths / rows [batch], request_table
 * [.., table_width]; physical [1, batch, n_blocks * block_size] int32 (strides
 * phys_row / phys_col of dims 1 and 2) or NULL (physical = logical);
 * live_pages [live_len] uint8 or NULL (every in-range slot backed).  Caches
 * hold cache_rows slots; the shadow holds capacity slots with an initialized
 * flag each.  Writes clean_blocks [1, batch, n_blocks] (contiguous, blocks'
 * element size) and physical_out [1, batch, n_blocks * block_size] int32, and
 * ADDS to counts[7] (uint64 on the device): checked tokens, checked bytes,
 * uninitialized logical tokens, invalid physical tokens, mismatched tokens,
 * calls (+1), malformed Top-K blocks.  batch <= 65535.
 */
int ekv_shadow_check(
    const void* blocks, int blocks_esize, int64_t batch, int64_t n_blocks, int64_t blocks_row, int64_t blocks_col,
    const void* lengths, int len_esize, int64_t len_stride, const void* rows, int rows_esize, int64_t rows_stride,
    const void* request_table, int table_esize, int64_t table_width, int64_t table_row, int64_t table_col,
    const int32_t* physical, int64_t phys_row, int64_t phys_col, const uint8_t* live_pages, int64_t live_len,
    const void* k_cache, const void* v_cache, int64_t cache_rows, int64_t k_cache_stride, int64_t v_cache_stride,
    const void* k_shadow, const void* v_shadow, const uint8_t* initialized, int64_t capacity,
    int64_t k_shadow_stride, int64_t v_shadow_stride, int64_t k_row_bytes, int64_t v_row_bytes,
    int64_t block_size, int64_t page_size, void* clean_blocks, int32_t* physical_out, uint64_t* counts,
    int device, void* stream);

/*
 * ekv_shadow_check_complete — LogicalShadow.check_complete (:88-123): for every
 * layer and every (logical[i], physical[i]) pair, compare the pool's K/V rows
 * at physical[i] with the shadow's at logical[i].  pool_k / pool_v / shadow_k /
 * shadow_v / initialized are HOST arrays of n_layers device addresses (at most
 * EKV_SHADOW_MAX_LAYERS); pool buffers hold pool_size + page_size slots.
 * live_pages [live_len] uint8.  ADDS to counts[4]: checked tokens, checked
 * bytes, invalid tokens, mismatched tokens (summed over the layers).
 */
int ekv_shadow_check_complete(
    const void* logical, int logical_esize, const void* physical, int physical_esize, int64_t n,
    int64_t page_size, int64_t pool_size, int64_t capacity, const uint8_t* live_pages, int64_t live_len,
    const uint64_t* pool_k, const uint64_t* pool_v, const uint64_t* shadow_k, const uint64_t* shadow_v,
    const uint64_t* initialized, int n_layers, int64_t pool_k_stride, int64_t pool_v_stride,
    int64_t shadow_k_stride, int64_t shadow_v_stride, int64_t k_row_bytes, int64_t v_row_bytes, uint64_t* counts,
    int device, void* stream);

/*
 * ekv_shadow_write — LogicalShadow.write (:30-43): shadow rows at
 * locations[r] = key / value row r, initialized[locations[r]] = 1.  Negative
 * locations count from the end; locations outside [-capacity, capacity) are
 * skipped.
 */
int ekv_shadow_write(
    void* k_shadow, void* v_shadow, uint8_t* initialized, int64_t capacity, int64_t k_shadow_stride,
    int64_t v_shadow_stride, const void* key, const void* value, int64_t key_stride, int64_t value_stride,
    int64_t k_row_bytes, int64_t v_row_bytes, const void* locations, int loc_esize, int64_t n, int device,
    void* stream);

/*
 * ekv_shadow_reset — LogicalShadow.reset (:26-28): initialized[l][locations[r]] = 0
 * for each of n_layers flag arrays (a HOST array of device addresses).
 */
int ekv_shadow_reset(
    const uint64_t* initialized, int n_layers, int64_t capacity, const void* locations, int loc_esize, int64_t n,
    int device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EKV_KERNELS_H */
