// kvops_internal.cuh — shared device helpers and launch-parameter blocks of the
// B200 hot path (sieve, gather, export). Host code fills the *Params structs; each
// kernel receives one by value (well under the 32 KB kernel-parameter limit).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kvops_b200.h"

namespace kvb {

constexpr int kHandStride = 16;   // int32 words per hand row (hisp_kernel_common.h:21)
constexpr int kMaxNodes = KVOPS_MAX_NODES;
constexpr uint32_t kAllNodes = 0xFFFFFFFFu;

// Knuth multiplicative hash (hisp_kernel_common.h:23-26): 32-bit wrapping product, >> 16.
__host__ __device__ __forceinline__ uint32_t ht_hash(int32_t token)
{
    return (static_cast<uint32_t>(token) * 2654435761u) >> 16;
}

// Stripe ownership (kvc_common.h:81-89). S == 0 means node 0 and identity rows.
__host__ __device__ __forceinline__ uint32_t node_of(uint32_t row, uint32_t S, uint32_t N)
{
    return S == 0 ? 0u : (row / S) % N;
}
__host__ __device__ __forceinline__ uint32_t seg_row_of(uint32_t row, uint32_t S, uint32_t N, bool injective)
{
    if (S == 0) return row;
    const uint32_t g = row / S;
    return injective ? (g / N) * S + (row - g * S) : g / N;
}

// Completion ticket: one per in-flight launch. The last CTA to arrive publishes the
// status words and resets the ticket to zero for its next user.
struct Ticket {
    unsigned int arrived;
    unsigned int err;
};

// Status publication target of one launch: pages[node] for node in [node_lo, node_hi),
// words [0, block_dim) of each 64-byte page.
struct StatusTarget {
    uint64_t *status;      // base of the slot array (nullptr: no status)
    uint32_t node_lo;
    uint32_t node_hi;
    uint32_t block_dim;
    Ticket *ticket;        // device memory, zero between launches
    uint32_t *err_word;    // caller's error word (KvopsRowOpts::err_word), nullptr: none
};

struct SieveParams {
    const int32_t *topk;        // [max_num_reqs, top_k]
    const int64_t *req_pool;    // [max_num_reqs]
    const int32_t *seq_lens;    // [max_num_reqs]
    const int32_t *prefill;     // [pool]
    int32_t *tokens;            // [pool, padded]   (layer slice)
    uint8_t *visited;           // [pool, vis_stride]
    uint16_t *ht;               // [pool, ht_size]
    int32_t *hand;              // [pool, 16]
    int32_t *out_slots;         // [max_num_reqs, top_k]
    int8_t *is_miss;            // [max_num_reqs, top_k]
    const int32_t *num_real;    // [1]
    int32_t top_k, dbs, padded, vis_stride, max_num_reqs, pool_size, ht_size;
    uint8_t *big;               // large-table tier: global scratch, big_slots slots (nullptr: tier unavailable)
    uint64_t big_slot_bytes;
    int32_t big_slots;
};

struct HtInitParams {
    const int32_t *tokens;      // [layer_num, pool, padded]
    uint16_t *ht;               // [layer_num, pool, ht_size]
    int32_t req_start, num_reqs, layer_num, pool_size, dbs, padded, ht_size;
    int32_t pairs;              // number of (layer, req) pairs to rebuild
};

struct GatherParams {
    const int32_t *topk;
    const int64_t *req_pool;
    const int64_t *host_base;
    const int32_t *slots;
    const int8_t *is_miss;
    const int32_t *num_real;         // nullptr: nothing to scan (max_num_reqs or top_k is 0)
    uint8_t *hot;
    uint64_t hot_req_stride_bytes;   // 0: reference (all requests share the hot rows)
    uint64_t layer_offset_rows;
    uint32_t plsr, row_bytes, stripe, nodes, my_node, top_k, max_num_reqs;
    uint32_t injective;
    StatusTarget st;
    const uint8_t *seg[kMaxNodes];   // per-node segment bases (only [my_node] for one segment)
};

struct ExportParams {
    const uint8_t *src0;
    uint64_t src_layer_stride;
    uint8_t *seg;
    uint32_t plsr, row_bytes, row_lo, row_cnt, layer_num, stripe, nodes, my_node;
    uint32_t injective;
    uint32_t seg_null;               // 1: segment base was 0 (report KVOPS_ERR_SEG_NULL only)
    uint64_t units_per_layer;        // destination rows written per layer
    uint64_t g_first;                // first owned stripe index (S > 0)
    StatusTarget st;
};

// Extra arguments of the layer-step kernels (sieve.cu).
// Words of one cooperative layer-step's block: epoch, arrival count, walk-list progress (layout in sieve.cu).
constexpr uint32_t kCoopBlockWords = 2048;

struct StepExtra {
    int32_t nsl;        // copy warp: sets of 32 ring slots
    uint32_t ring_off;  // copy warp: byte offset of the ring in dynamic shared memory
    uint32_t *flags;    // cooperative step: the launch's block of kCoopBlockWords words
    uint32_t epoch;     // cooperative step: set in the kernel from the block (host passes 0)
    uint32_t magic;     // copy helpers: multiply-high constant of cta_copy_rows (0: divide)
    uint2 *wl;          // cooperative step: the launch's walk lists, max_num_reqs x top_k entries
    uint32_t wait_polls;  // cooperative step: walk-list polls of a copy CTA before it gives up
};

// Publishes completion: called by thread 0 of every CTA after a __syncthreads() that
// follows the CTA's last data store. The last CTA to arrive writes
// (1<<32)|err into each status word with system-scope release, then recycles the ticket.
__device__ __forceinline__ void arrive_and_publish(const StatusTarget &st)
{
    if (st.ticket == nullptr) return;
    __threadfence();
    const unsigned int prev = atomicAdd(&st.ticket->arrived, 1u);
    if (prev != gridDim.x * gridDim.y * gridDim.z - 1) return;
    __threadfence();
    const unsigned int err = atomicAdd(&st.ticket->err, 0u);
    if (st.status != nullptr) {
        __threadfence_system();
        const unsigned long long word = (1ull << 32) | static_cast<unsigned long long>(err);
        for (uint32_t n = st.node_lo; n < st.node_hi; ++n) {
            for (uint32_t b = 0; b < st.block_dim; ++b) {
                unsigned long long *w = reinterpret_cast<unsigned long long *>(st.status) + n * 8u + b;
                asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(w), "l"(word) : "memory");
            }
        }
    }
    st.ticket->err = 0u;
    st.ticket->arrived = 0u;
    __threadfence();
}

// Records the first device-side error of a launch (the reference's early-return
// errCode, kvc_gather_rows.cpp:78-81) in its ticket (published in the status words) and in
// the caller's error word; later errors are dropped.
__device__ __forceinline__ void record_error(const StatusTarget &st, unsigned int code)
{
    if (st.ticket != nullptr) atomicCAS(&st.ticket->err, 0u, code);
    if (st.err_word != nullptr) atomicCAS_system(st.err_word, 0u, code);
}

// Records `msg` as the calling thread's last error (capi.cu) and returns `code`.
int set_last_error(int code, const char *msg);
// Whether kvops_init has run (and kvops_close has not since).
bool is_inited();
// Zeroes the status words [node_lo, node_hi) x [0, block_dim) at `status` before a launch
// publishes them: pinned host words by the host now, device words on `stream` (capi.cu).
int clear_status_words(uint64_t status, uint32_t node_lo, uint32_t node_hi, uint32_t block_dim, cudaStream_t stream);

// SIEVE tiers (KVOPS_TIER_*): the caller's choice for the calling thread, and the tier its last
// launch_sieve_update ran.
void set_sieve_tier(uint32_t tier);
uint32_t last_sieve_tier();
// Bytes of one slot of the large-table tier's scratch and the slots it needs (*slots = 0: the
// shape does not use that tier under the calling thread's choice). The kernel needs no initial
// contents in it.
uint64_t sieve_big_scratch(const SieveParams &p, int sm_count, int32_t *slots);

// Kernel launchers (defined next to their kernels).
cudaError_t launch_sieve_update(const SieveParams &p, cudaStream_t s, int sm_count);
cudaError_t launch_sieve_ht_init(const HtInitParams &p, cudaStream_t s);
cudaError_t launch_gather(const GatherParams &p, cudaStream_t s, int sm_count);
// The gather's rules in the opposite direction (kvc_scatter_rows): hot row -> segment row for
// every position whose flag (p.is_miss) is set.
cudaError_t launch_scatter(const GatherParams &p, cudaStream_t s, int sm_count);
cudaError_t launch_export(const ExportParams &p, cudaStream_t s, int sm_count);
// Fused SIEVE step + miss-row gather (one CTA per request). Sets *launched = false, launching
// nothing, when the request's state and the copy ring do not fit shared memory; the caller
// then runs launch_sieve_update and launch_gather instead.
cudaError_t launch_sieve_import(const SieveParams &p, const GatherParams &g, cudaStream_t s, bool *launched);
// The same step as one cooperative launch: the SIEVE CTAs list each request's misses in its
// walk list (wl: max_num_reqs x top_k entries) as the hand sweep makes them final, and every
// other CTA resident on the GPU copies the listed rows (progress words in `flags`, a
// zero-initialised block of kCoopBlockWords words that no other launch uses while this one
// runs). *launched = false (nothing launched) when wl is null, fewer than max(8, min_copy_ctas)
// copy CTAs fit beside the SIEVE CTAs, there are more than 252 requests, or the state does not fit.
// wait_polls: walk-list polls of a copy CTA before it reports KVOPS_ERR_COPY_TIMEOUT (0: 2^22).
// min_copy_ctas: launch only if at least this many copy CTAs (and never fewer than 8) fit.
cudaError_t launch_sieve_coop(const SieveParams &p, const GatherParams &g, uint32_t *flags, uint2 *wl,
                              uint32_t wait_polls, int32_t min_copy_ctas, cudaStream_t s, bool *launched);
// Sets up, without launching, what the first cooperative step of this shape would: the
// kernel's shared-memory limit and the cached residency (so a later call may be captured).
cudaError_t prepare_sieve_coop(const SieveParams &p);

}  // namespace kvb
