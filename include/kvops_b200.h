/*
 * kvops_b200.h — C ABI of the B200 (sm_100a) decode-time KV hot path.
 *
 * The entry points mirror the reference's launch extension `kvops_ext._kvops`
 * (kvops/kvops_ext/kvops_ext.cpp), one C function per pybind function, with the
 * same argument order and meaning. All tensor arguments are raw device (or UVA)
 * addresses as uint64_t, owned by the caller; `stream` is a cudaStream_t as
 * uint64_t (0 = the legacy default stream of the calling thread's device).
 *
 * Return convention: KVOPS_OK (0) or a positive KVOPS_E_* code; the message of
 * the last failure on the calling thread is returned by kvops_last_error().
 * Launches are asynchronous on `stream`; device-side failures are reported as
 * errCode values in the 64-byte status slot, as in the reference.
 *
 * Status slot layout (one self-consistent choice among the reference's conflicting
 * writers and pollers, kvc_gather_rows.cpp:22-23 vs xds_ems_pool.py:238): a launch for
 * segment `my_node` with `block_dim` = B writes B 64-bit words at
 * status + my_node*64 + b*8 (b < B), each equal to (1 << 32) | errCode once every
 * row of the launch has landed. That is exactly what EmsPool.wait polls
 * (xds/xds_ems_pool.py:233-241).
 *
 * Clearing: every call zeroes the words it will publish before its launch. Words in pinned
 * host memory (kvops_alloc_status) are zeroed by the host during the call. Words in device
 * memory are zeroed on the launch stream (cudaMemsetAsync, so the clear is ordered before the
 * kernel and is captured with it), and must therefore be read in stream order:
 * kvops_poll_status reads them on the legacy default stream, which is ordered after launches
 * on the legacy stream and on blocking streams; after a launch on a non-blocking stream, order
 * the poll yourself (synchronize the stream, or wait on an event recorded after the call).
 * A slot must not be reused while an earlier launch that publishes into it may still run:
 * that launch's done word could land after the clear (the reference's EmsPool cycles 8 x N
 * slots for the same reason).
 */
#ifndef KVOPS_B200_H
#define KVOPS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVOPS_OK 0
#define KVOPS_E_NOT_INITED 1     /* "kvops not inited" (kvops_ext.cpp:131-136) */
#define KVOPS_E_ALREADY_INITED 2 /* "kvops already inited" (kvops_ext.cpp:141-143) */
#define KVOPS_E_INVALID 3        /* argument validation failed */
#define KVOPS_E_CUDA 4           /* a CUDA runtime call failed */
#define KVOPS_E_NOMEM 5          /* an allocation failed */

/* kv_poll_status results besides errCode >= 0 (kvops_ext.cpp:207,213). */
#define KVOPS_POLL_COPY_FAILED (-0x1000)
#define KVOPS_POLL_TIMEOUT (-0x2000)

/* Device-side errCode bands (kvops/kernel/kvc_common.h:24). */
#define KVOPS_ERR_SEG_NULL 0x101u  /* segment base is 0: nothing touched (0x1xx, init band) */
#define KVOPS_ERR_ROW_BASE 0x200u  /* 0x200 + (index & 0xFF) + (1 << 16): row out of the segment */
#define KVOPS_ERR_COPY_TIMEOUT 0x102u  /* kvops_sieve_import: a copy CTA stopped waiting for a walk list */

/* Largest node count of one layout (common/kv_layout.h:45, KvLayoutValidate). */
#define KVOPS_MAX_NODES 64

/* Message of the last failing call on this thread ("" if none). */
const char *kvops_last_error(void);

/* Replaces kv_init (kvops/kvops_ext/kvops_ext.cpp:139-185). Selects `device_id`.
 * The kernels are linked into this library, so `fatbin_path` is only checked to
 * name an existing file when non-empty, and `rt_lib` is ignored. */
int kvops_init(int device_id, const char *fatbin_path, const char *rt_lib);

/* Replaces kv_close (kvops_ext.cpp:360-371): frees status slots and per-device
 * bookkeeping; a later kvops_init is allowed. */
int kvops_close(void);

/* Replaces kv_alloc_status (kvops_ext.cpp:187-196): `count` zeroed 64-byte slots in
 * pinned, mapped host memory; *out_addr is the address kernels write and the
 * host polls (UVA, valid on every device). */
int kvops_alloc_status(int count, uint64_t *out_addr);

/* Replaces kv_poll_status (kvops_ext.cpp:198-218). Spins on the 64-bit word at
 * status_addr until (word >> 32) == 1 and stores (word & 0xFFFFFFFF) in *out_rc;
 * stores KVOPS_POLL_TIMEOUT after timeout_us microseconds (< 0: wait forever) and
 * KVOPS_POLL_COPY_FAILED if a device-memory word cannot be read. */
int kvops_poll_status(uint64_t status_addr, int64_t timeout_us, int64_t *out_rc);

/* Replaces kv_import_seg + kvc_gather_rows (kvops_ext.cpp:221-254,
 * kvops/kernel/kvc_gather_rows.cpp:12-96): copy every is_miss row owned by
 * `my_node` from seg_base[(layer_offset_rows + segRow) * row_bytes] to
 * hot_row_base[slot * row_bytes]. `channel` is accepted and ignored (seg_base is a
 * UVA address: own HBM, a peer GPU's HBM, or pinned host memory). block_dim must
 * be 1..8 (status words), the grid is sized for the GPU independently of it. */
int kvops_import_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                     uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                     uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                     uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                     uint64_t status, uint64_t stream, uint32_t block_dim);

/* Opt-in behaviour that the reference does not have; zero-initialised = reference. */
typedef struct KvopsRowOpts {
    /* 0: dst = hot_row_base + slot*row_bytes (reference: shared by all requests).
     * >0: dst = hot_row_base + (req_pool_idx*hot_req_stride_rows + slot)*row_bytes. */
    uint64_t hot_req_stride_rows;
    /* 0: segRow = (row/S)/N (reference, collides for S > 1).
     * 1: segRow = ((row/S)/N)*S + row%S (injective; per_layer_seg_rows must then be
     *    ceil(ceil(layer_rows/S)/N)*S). */
    uint32_t injective;
    /* kvops_sieve_import only (ignored elsewhere): how the layer-step runs. Every path gives the
     * same results; a path that does not fit the shapes falls back to SPLIT.
     * COOP: one cooperative launch; the SIEVE CTAs publish their outputs after the hand sweep and
     *   the other CTAs resident on the GPU copy the miss rows meanwhile (16-byte aligned rows).
     * FUSED: one launch; a copy warp in each SIEVE CTA moves its rows by bulk copies (device
     *   memory segments only).
     * SPLIT: the SIEVE kernel, then the gather launched as its programmatic dependent.
     * AUTO: COOP when it fits, else SPLIT. */
    uint32_t step_path;
    /* Error word (0 = none): the address (device memory, or pinned mapped host memory) of a
     * uint32 into which every launch of the call stores its first device-side errCode by
     * compare-and-swap from 0, besides (or, with status == 0, instead of) the status words. A
     * call captured into a CUDA graph publishes no status words; this word is how its replays
     * report errors. The caller reads it after the launch and clears it. */
    uint64_t err_word;
    /* kvops_sieve_import, COOP path: how many times a copy CTA polls the walk lists before it
     * stops waiting and reports KVOPS_ERR_COPY_TIMEOUT, leaving rows uncopied (0 = the default,
     * 2^22 polls with a 256 ns back-off, about one second). */
    uint32_t copy_wait_polls;
    uint32_t reserved;
} KvopsRowOpts;

#define KVOPS_STEP_AUTO 0u
#define KVOPS_STEP_FUSED 1u
#define KVOPS_STEP_SPLIT 2u
#define KVOPS_STEP_COOP 3u

/* kvops_import_seg with options (opts may be NULL). */
int kvops_import_seg_ex(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                        uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                        uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                        uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num,
                        uint32_t my_node, uint64_t status, uint64_t stream, uint32_t block_dim,
                        const KvopsRowOpts *opts);

/* All `node_num` segments of one layer in ONE launch (the per-segment loop of
 * EmsPool.batch_read, xds/xds_ems_pool.py:204-217, fused). seg_bases[s] is node
 * s's segment base. Writes the status pages of every node s, as node_num
 * separate import_seg launches would. */
int kvops_import_multi(uint32_t node_num, const uint64_t *seg_bases, uint32_t layer_offset_rows,
                       uint32_t per_layer_seg_rows, uint32_t row_bytes, uint64_t topk_indices,
                       uint64_t req_pool_indices, uint64_t req_host_base, uint64_t topk_device_slots,
                       uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base, uint32_t top_k,
                       uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                       uint32_t block_dim, const KvopsRowOpts *opts);

/* The single-layer indexed export of decode increments, kvc_scatter_rows: designed in the
 * reference with the arguments of kvc_gather_rows and the opposite data direction
 * (doc/kv_offload_design.md:394-396), its implementation later deleted (:544). For every position
 * (batch row < num_real, k < top_k) whose export_flags byte is set, with a valid token, slot and
 * pool row on node my_node, copies the hot row (hot_row_base + slot, or the per-request stride
 * of opts) to segment row segRow of layer_offset_rows -- kvops_import_seg's rules, reversed.
 * Same status words and errCodes. Positions that name the same segment row race. */
int kvops_export_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                     uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                     uint64_t topk_device_slots, uint64_t export_flags, uint64_t num_real, uint64_t hot_row_base,
                     uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                     uint64_t status, uint64_t stream, uint32_t block_dim, const KvopsRowOpts *opts);

/* Replaces kv_export_seg_alllayer + kvc_scatter_rows_alllayer (kvops_ext.cpp:256-278,
 * kvops/kernel/kvc_scatter_rows_alllayer.cpp:11-67): for every layer l and row in
 * [row_lo, row_lo+row_cnt) owned by my_node, the segment row
 * seg_base + (l*per_layer_seg_rows + segRow)*row_bytes ends up holding
 * src_layer0_base + l*src_layer_stride + row*row_bytes, with the reference's
 * last-row-wins result where its S > 1 map collides. */
int kvops_export_seg_alllayer(uint64_t channel, uint64_t seg_base, uint32_t per_layer_seg_rows, uint32_t row_bytes,
                              uint32_t row_lo, uint32_t row_cnt, uint32_t layer_num, uint64_t src_layer0_base,
                              uint64_t src_layer_stride, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                              uint64_t status, uint64_t stream, uint32_t block_dim);

/* kvops_export_seg_alllayer with options (only `injective` applies; opts may be NULL). */
int kvops_export_seg_alllayer_ex(uint64_t channel, uint64_t seg_base, uint32_t per_layer_seg_rows,
                                 uint32_t row_bytes, uint32_t row_lo, uint32_t row_cnt, uint32_t layer_num,
                                 uint64_t src_layer0_base, uint64_t src_layer_stride, uint32_t stripe_rows,
                                 uint32_t node_num, uint32_t my_node, uint64_t status, uint64_t stream,
                                 uint32_t block_dim, const KvopsRowOpts *opts);

/* Replaces kv_sieve_update + hisp_sieve_update (kvops_ext.cpp:281-336,
 * kvops/kernel/hisp_sieve_update.cpp:17-176). Same validation (padded % 16,
 * padded <= 65534, visited stride) and hash-table size derivation; the reference's
 * 176 KB UB budget is replaced by a shared-memory/global tier choice, so large hot
 * buffers (up to the uint16 slot limit) are accepted. One CTA per batch row;
 * block_dim is validated (>= 1) and otherwise unused. */
int kvops_sieve_update(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                       uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                       uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                       uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs, uint32_t pool_size, uint64_t stream,
                       uint32_t block_dim);

/* SIEVE kernel tiers (no counterpart in the reference, whose kernel has one tier and rejects
 * states over its 176 KB UB budget, kvops_ext.cpp:302-306). Every tier gives the same outputs
 * and state bytes.
 * SHARED: the phase-parallel step with the request's state in shared memory (tables up to 65536
 *   cells that fit, e.g. hot buffers up to ~8K slots).
 * LARGE: the large-table tier: the same phases with a direct token index and the table updated
 *   in global memory by run re-packing (any table; one scratch area per device, ~3 MB per SM,
 *   allocated on the first call of such a shape or by kvops_step_prepare, so launches that use
 *   it on one device must be ordered: one stream, or ordered by events).
 * ORDERED: the reference's position-ordered loop, in shared memory when the state fits, else in
 *   global memory. AUTO: SHARED when it fits, else LARGE, else ORDERED. */
#define KVOPS_TIER_AUTO 0u
#define KVOPS_TIER_SHARED 1u
#define KVOPS_TIER_LARGE 2u
#define KVOPS_TIER_ORDERED 3u

/* The tier the calling thread's later SIEVE launches use (AUTO by default); a tier that cannot
 * run a shape falls back to AUTO's choice. */
int kvops_set_sieve_tier(uint32_t tier);

/* The tier the calling thread's last SIEVE launch ran (AUTO before any). */
uint32_t kvops_last_sieve_tier(void);

/* Replaces kv_sieve_ht_init + hisp_sieve_ht_init (kvops_ext.cpp:339-358,
 * kvops/kernel/hisp_sieve_ht_init.cpp:14-60). Rebuilds the tables of
 * min(block_dim, layer_num*num_reqs) (layer, request) pairs; block_dim 0 means all. */
int kvops_sieve_ht_init(uint64_t device_buffer_tokens, uint64_t device_buffer_ht, uint64_t prefill_lens,
                        uint32_t req_start, uint32_t num_reqs, uint32_t layer_num, uint32_t pool_size,
                        uint32_t device_buffer_size, uint32_t padded_buffer_size, uint32_t ht_size,
                        uint64_t stream, uint32_t block_dim);

/* One decode layer-step in one call: kvops_sieve_update followed by kvops_import_multi over
 * the same tensors, with identical results (slots, miss flags, SIEVE state, hot rows, status
 * words, errCodes). No counterpart in the reference, whose driver issues the two calls
 * (xds/xds_decode.py:225-233). opts->step_path chooses how (KVOPS_STEP_*, default AUTO).
 * block_dim: status words per node (1..8), as in kvops_import_multi. A row copy that never
 * completes, or a request whose outputs never become ready, sets errCode KVOPS_ERR_COPY_TIMEOUT. */
int kvops_sieve_import(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                       uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                       uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                       uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs, uint32_t pool_size, uint32_t node_num,
                       const uint64_t *seg_bases, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                       uint32_t row_bytes, uint64_t req_host_base, uint64_t hot_row_base, uint32_t stripe_rows,
                       uint64_t status, uint64_t stream, uint32_t block_dim, const KvopsRowOpts *opts);

/* KVOPS_STEP_COOP, _FUSED or _SPLIT: the path the calling thread's last successful
 * kvops_sieve_import ran (KVOPS_STEP_AUTO before any). No counterpart in the reference. */
uint32_t kvops_last_step_path(void);

/* Does, without launching, the one-time setup the first kvops_sieve_import of this shape on
 * the current device would do (device bookkeeping, cooperative-step scratch, kernel limits),
 * so that later calls may be captured into a CUDA graph. No counterpart in the reference. */
int kvops_step_prepare(uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs);

/* No counterpart in the reference. kvops_import_multi for callers that cannot allocate
 * device memory (an engine whose HBM is owned by its own allocator or fixed budget, or a
 * decode loop that cannot pay for cudaMalloc/cudaFree): it calls no allocating routine.
 * Its only scratch, the launch's 8-byte completion ticket, lives in a static device array
 * of KVOPS_NOALLOC_SCRATCH_BYTES bytes held by every GPU that loads the library until exit.
 * All calls share that array (cleared on `stream` before each launch), so calls whose
 * launches overlap on the GPU race and must not be issued. The first call on a device looks
 * up the array's device address; make it before any stream capture. Launches that would
 * need more scratch than the array holds are rejected with KVOPS_E_INVALID. Like every
 * other entry point it requires kvops_init (KVOPS_E_NOT_INITED before it), and it clears
 * the status words as they do (pinned words by the host, device words on `stream`). */
#define KVOPS_NOALLOC_SCRATCH_BYTES 256
int kvops_import_multi_noalloc(uint32_t node_num, const uint64_t *seg_bases, uint32_t layer_offset_rows,
                               uint32_t per_layer_seg_rows, uint32_t row_bytes, uint64_t topk_indices,
                               uint64_t req_pool_indices, uint64_t req_host_base, uint64_t topk_device_slots,
                               uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base, uint32_t top_k,
                               uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                               uint32_t block_dim, const KvopsRowOpts *opts);

/* Pool plumbing that replaces the EMS control plane (not a reference entry point):
 * segment memory on a device (or pinned host memory with device = -1), peer access,
 * and CUDA IPC so that one process per GPU can map the other GPUs' segments. Device
 * segments are allocated in whole 2 MiB units (other GPUs read an IPC-mapped allocation of
 * any other size at under half the NVLink rate). */
int kvops_segment_alloc(int device, uint64_t bytes, uint64_t *out_addr);
int kvops_segment_free(uint64_t addr);
int kvops_enable_peer_access(int device, int peer);
int kvops_ipc_get_handle(uint64_t addr, uint8_t out_handle[64]);
int kvops_ipc_open_handle(int device, const uint8_t handle[64], uint64_t *out_addr);
int kvops_ipc_close_handle(uint64_t addr);

#ifdef __cplusplus
}
#endif

#endif /* KVOPS_B200_H */
