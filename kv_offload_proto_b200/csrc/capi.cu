// capi.cu — extern "C" entry points of libkvops_b200.so (declared in include/kvops_b200.h).
//
// Host-side counterpart of the reference's kvops/kvops_ext/kvops_ext.cpp: argument
// validation and derivations (htSize, status layout), module state (init/close),
// status slots in pinned mapped host memory, completion polling, and the pool
// plumbing (segments, peer access, IPC) that replaces the EMS control plane.
// Nothing here reads device memory on a launch path; launches are asynchronous.
#include <cuda_runtime.h>
#include <immintrin.h>
#include <stdint.h>
#include <sys/stat.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "kvops_internal.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string &msg)
{
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what)
{
    cudaGetLastError();  // clear a non-sticky error so the next call starts clean
    return fail(KVOPS_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

struct DeviceState {
    kvb::Ticket *ring = nullptr;  // completion tickets, zero when idle
    uint32_t ring_size = 0;
    std::atomic<uint32_t> next{0};
    int sm_count = 0;
    uint32_t *ready = nullptr;  // cooperative layer-steps: kReadyBlocks blocks of kReadyWords words
    std::atomic<uint32_t> ready_next{0};
    uint2 *wl = nullptr;         // cooperative layer-steps: kWalkListBufs walk-list buffers
    size_t wl_entries = 0;       // entries per buffer
    std::vector<uint2 *> wl_old;  // outgrown buffers (a captured graph may still name one)
    uint8_t *big = nullptr;      // large-table SIEVE tier: scratch (no initial contents needed)
    size_t big_bytes = 0;
    std::vector<uint8_t *> big_old;  // outgrown scratch (a captured graph may still name one)
};

// Words of cooperative layer-steps: launch n uses block n % kReadyBlocks, so a block is reused
// only after kReadyBlocks later launches; the kernel keeps each block's epoch itself. Launch n
// also uses walk-list buffer n % kWalkListBufs: cooperative launches fill the device, so no
// more than two consecutive ones are ever resident together.
constexpr uint32_t kReadyBlocks = 1024, kReadyWords = kvb::kCoopBlockWords, kWalkListBufs = 4;

std::mutex g_mu;
thread_local uint32_t t_last_step_path = KVOPS_STEP_AUTO;  // path the last kvops_sieve_import ran
thread_local uint32_t t_tier_choice = KVOPS_TIER_AUTO;      // kvops_set_sieve_tier of this thread
bool g_inited = false;
int g_home_device = 0;
std::vector<void *> g_status_allocs;
std::unordered_map<int, DeviceState *> g_devices;
std::unordered_map<uint64_t, int> g_segments;  // addr -> device (-1: pinned host)

constexpr uint32_t kTicketRing = 4096;

// Per-device bookkeeping for the calling thread's current device (created on first use).
int current_device_state(DeviceState **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_devices.find(dev);
    if (it != g_devices.end()) {
        *out = it->second;
        return KVOPS_OK;
    }
    DeviceState *ds = new DeviceState();
    e = cudaMalloc(&ds->ring, sizeof(kvb::Ticket) * kTicketRing);
    if (e != cudaSuccess) {
        delete ds;
        return cuda_fail(e, "cudaMalloc(ticket ring)");
    }
    e = cudaMemset(ds->ring, 0, sizeof(kvb::Ticket) * kTicketRing);
    if (e != cudaSuccess) {
        cudaFree(ds->ring);
        delete ds;
        return cuda_fail(e, "cudaMemset(ticket ring)");
    }
    ds->ring_size = kTicketRing;
    cudaDeviceGetAttribute(&ds->sm_count, cudaDevAttrMultiProcessorCount, dev);
    g_devices[dev] = ds;
    *out = ds;
    return KVOPS_OK;
}

bool is_host_memory(uint64_t addr)
{
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, reinterpret_cast<void *>(addr)) != cudaSuccess) {
        cudaGetLastError();
        return true;  // unregistered host memory
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeUnregistered;
}

// Zeroes the status words a launch will publish, before the launch, so a poller never
// sees the previous use's done word. Pinned host words are written by the host now. Device
// words are cleared on the launch stream, ordered before the kernel and captured with it
// into a CUDA graph (the reference's synchronous memset, kvops_ext.cpp:252, is neither; the
// header states how such words are then read in stream order).
int reset_status(uint64_t status, uint32_t node_lo, uint32_t node_hi, uint32_t block_dim, cudaStream_t stream)
{
    if (status == 0) return KVOPS_OK;
    if (is_host_memory(status)) {
        for (uint32_t n = node_lo; n < node_hi; ++n)
            for (uint32_t b = 0; b < block_dim; ++b)
                __atomic_store_n(reinterpret_cast<uint64_t *>(status) + n * 8u + b, 0ull, __ATOMIC_RELEASE);
        return KVOPS_OK;
    }
    for (uint32_t n = node_lo; n < node_hi; ++n) {
        cudaError_t e = cudaMemsetAsync(reinterpret_cast<void *>(status + n * 64ull), 0, block_dim * 8ull, stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(status)");
    }
    return KVOPS_OK;
}

int make_status_target(uint64_t status, uint32_t node_lo, uint32_t node_hi, uint32_t block_dim, DeviceState *ds,
                       uint64_t err_word, cudaStream_t stream, kvb::StatusTarget *st)
{
    st->status = reinterpret_cast<uint64_t *>(status);
    st->node_lo = node_lo;
    st->node_hi = node_hi;
    st->block_dim = block_dim;
    st->ticket = nullptr;
    st->err_word = reinterpret_cast<uint32_t *>(err_word);
    if (status == 0) return KVOPS_OK;
    const uint32_t i = ds->next.fetch_add(1, std::memory_order_relaxed) % ds->ring_size;
    st->ticket = ds->ring + i;
    return reset_status(status, node_lo, node_hi, block_dim, stream);
}

#define KV_REQUIRE_INIT()                                              \
    do {                                                               \
        if (!g_inited) return fail(KVOPS_E_NOT_INITED, "kvops not inited"); \
    } while (0)

int build_gather(uint32_t node_num, const uint64_t *seg_bases, uint32_t node_lo, uint32_t node_hi,
                  uint32_t my_node, uint32_t layer_offset_rows, uint32_t plsr, uint32_t row_bytes,
                  uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                  uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                  uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                  uint32_t block_dim, const KvopsRowOpts *opts, kvb::GatherParams *out, DeviceState **ds_out,
                  const char *what = "import")
{
    const std::string w(what);
    KV_REQUIRE_INIT();
    if (block_dim > 8) return fail(KVOPS_E_INVALID, w + " blockDim must be <= 8 (status slot layout)");
    if (block_dim == 0) return fail(KVOPS_E_INVALID, w + " blockDim must be >= 1");
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, w + " node_num must be in [1, 64]");
    if (my_node != kvb::kAllNodes && my_node >= node_num)
        return fail(KVOPS_E_INVALID, w + " my_node must be < node_num");
    if (row_bytes == 0) return fail(KVOPS_E_INVALID, w + " row_bytes must be > 0");
    if (max_num_reqs > 0 && top_k > 0 &&
        (topk_indices == 0 || req_pool_indices == 0 || req_host_base == 0 || topk_device_slots == 0 ||
         is_miss == 0 || num_real == 0 || hot_row_base == 0))
        return fail(KVOPS_E_INVALID, w + ": a tensor address is 0");
    const KvopsRowOpts o = opts ? *opts : KvopsRowOpts{};
    if (o.injective > 1) return fail(KVOPS_E_INVALID, w + ": injective must be 0 or 1");
    if ((o.err_word & 3) != 0) return fail(KVOPS_E_INVALID, w + ": err_word must be 4-byte aligned");
    DeviceState *ds = nullptr;
    int rc = current_device_state(&ds);
    if (rc != KVOPS_OK) return rc;

    kvb::GatherParams p{};
    p.topk = reinterpret_cast<const int32_t *>(topk_indices);
    p.req_pool = reinterpret_cast<const int64_t *>(req_pool_indices);
    p.host_base = reinterpret_cast<const int64_t *>(req_host_base);
    p.slots = reinterpret_cast<const int32_t *>(topk_device_slots);
    p.is_miss = reinterpret_cast<const int8_t *>(is_miss);
    p.num_real = reinterpret_cast<const int32_t *>(num_real);
    p.hot = reinterpret_cast<uint8_t *>(hot_row_base);
    p.hot_req_stride_bytes = o.hot_req_stride_rows * row_bytes;
    p.layer_offset_rows = layer_offset_rows;
    p.plsr = plsr;
    p.row_bytes = row_bytes;
    p.stripe = stripe_rows;
    p.nodes = node_num;
    p.my_node = my_node;
    p.top_k = top_k;
    p.max_num_reqs = max_num_reqs;
    p.injective = o.injective;
    for (uint32_t n = 0; n < node_num; ++n) p.seg[n] = reinterpret_cast<const uint8_t *>(seg_bases[n]);
    rc = make_status_target(status, node_lo, node_hi, block_dim, ds, o.err_word, reinterpret_cast<cudaStream_t>(stream),
                            &p.st);
    if (rc != KVOPS_OK) return rc;
    if (max_num_reqs == 0 || top_k == 0) p.num_real = nullptr;  // nothing to scan: still completes the status
    *out = p;
    *ds_out = ds;
    return KVOPS_OK;
}

int import_common(uint32_t node_num, const uint64_t *seg_bases, uint32_t node_lo, uint32_t node_hi,
                  uint32_t my_node, uint32_t layer_offset_rows, uint32_t plsr, uint32_t row_bytes,
                  uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                  uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                  uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                  uint32_t block_dim, const KvopsRowOpts *opts)
{
    kvb::GatherParams p{};
    DeviceState *ds = nullptr;
    int rc = build_gather(node_num, seg_bases, node_lo, node_hi, my_node, layer_offset_rows, plsr, row_bytes,
                          topk_indices, req_pool_indices, req_host_base, topk_device_slots, is_miss, num_real,
                          hot_row_base, top_k, max_num_reqs, stripe_rows, status, stream, block_dim, opts, &p, &ds);
    if (rc != KVOPS_OK) return rc;
    cudaError_t e = kvb::launch_gather(p, reinterpret_cast<cudaStream_t>(stream), ds->sm_count);
    if (e != cudaSuccess) return cuda_fail(e, "launch kvc_gather_rows");
    return KVOPS_OK;
}

int export_common(uint64_t seg_base, uint32_t plsr, uint32_t row_bytes, uint32_t row_lo, uint32_t row_cnt,
                  uint32_t layer_num, uint64_t src_layer0_base, uint64_t src_layer_stride, uint32_t stripe_rows,
                  uint32_t node_num, uint32_t my_node, uint64_t status, uint64_t stream, uint32_t block_dim,
                  const KvopsRowOpts *opts)
{
    KV_REQUIRE_INIT();
    if (block_dim > 8) return fail(KVOPS_E_INVALID, "export blockDim must be <= 8 (status slot layout)");
    if (block_dim == 0) return fail(KVOPS_E_INVALID, "export blockDim must be >= 1");
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, "export node_num must be in [1, 64]");
    if (my_node >= node_num) return fail(KVOPS_E_INVALID, "export my_node must be < node_num");
    if (row_bytes == 0) return fail(KVOPS_E_INVALID, "export row_bytes must be > 0");
    if (static_cast<uint64_t>(row_lo) + row_cnt > (1ull << 32))
        return fail(KVOPS_E_INVALID, "export row_lo + row_cnt exceeds the 32-bit row space");
    const KvopsRowOpts o = opts ? *opts : KvopsRowOpts{};
    if (o.injective > 1) return fail(KVOPS_E_INVALID, "export: injective must be 0 or 1");
    if ((o.err_word & 3) != 0) return fail(KVOPS_E_INVALID, "export: err_word must be 4-byte aligned");
    DeviceState *ds = nullptr;
    int rc = current_device_state(&ds);
    if (rc != KVOPS_OK) return rc;

    kvb::ExportParams p{};
    p.src0 = reinterpret_cast<const uint8_t *>(src_layer0_base);
    p.src_layer_stride = src_layer_stride;
    p.seg = reinterpret_cast<uint8_t *>(seg_base);
    p.plsr = plsr;
    p.row_bytes = row_bytes;
    p.row_lo = row_lo;
    p.row_cnt = row_cnt;
    p.layer_num = layer_num;
    p.stripe = stripe_rows;
    p.nodes = node_num;
    p.my_node = my_node;
    p.injective = o.injective;
    // Units (destination rows) per layer owned by my_node.
    uint64_t units = 0;
    if (row_cnt > 0 && layer_num > 0) {
        if (stripe_rows == 0) {
            units = my_node == 0 ? row_cnt : 0;
        } else {
            const uint64_t S = stripe_rows, N = node_num;
            const uint64_t lo_g = row_lo / S, hi_g = (static_cast<uint64_t>(row_lo) + row_cnt - 1) / S;
            const uint64_t g_first = lo_g + (my_node + N - lo_g % N) % N;
            const uint64_t stripes = g_first <= hi_g ? (hi_g - g_first) / N + 1 : 0;
            p.g_first = g_first;
            units = o.injective ? stripes * S : stripes;
        }
    }
    p.units_per_layer = units;
    rc = make_status_target(status, my_node, my_node + 1, block_dim, ds, o.err_word,
                            reinterpret_cast<cudaStream_t>(stream), &p.st);
    if (rc != KVOPS_OK) return rc;
    if (seg_base == 0 && units > 0) {  // null segment: init-band error, nothing touched
        p.units_per_layer = 0;
        p.seg_null = 1;
    }
    cudaError_t e = kvb::launch_export(p, reinterpret_cast<cudaStream_t>(stream), ds->sm_count);
    if (e != cudaSuccess) return cuda_fail(e, "launch kvc_scatter_rows_alllayer");
    return KVOPS_OK;
}

int attach_big_scratch(DeviceState *ds, kvb::SieveParams *p);

int build_sieve(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                       uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                       uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                       uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs, uint32_t pool_size, uint64_t stream,
                       uint32_t block_dim, kvb::SieveParams *out, DeviceState **ds_out)
{
    KV_REQUIRE_INIT();
    // Validation of kvops_ext.cpp:288-296, in the same order and with the same messages.
    if (padded_buffer_size % 16 != 0)
        return fail(KVOPS_E_INVALID, "sieve_update: padded_buffer_size must be a multiple of 16 (64-byte rows)");
    if (padded_buffer_size > 65534)
        return fail(KVOPS_E_INVALID, "sieve_update: padded_buffer_size must be <= 65534 (uint16 hash slots)");
    if (visited_stride_b % 64 != 0 || visited_stride_b < (padded_buffer_size + 7) / 8)
        return fail(KVOPS_E_INVALID, "sieve_update: visited bitmap stride must be 64B aligned and cover padded");
    // Domain checks the reference leaves to its callers (a zero block_dim divides by zero
    // there, kvops_ext.cpp:308; dbs outside [1, padded] indexes past the token row).
    if (block_dim == 0) return fail(KVOPS_E_INVALID, "sieve_update: block_dim must be >= 1");
    if (device_buffer_size == 0 || device_buffer_size > padded_buffer_size)
        return fail(KVOPS_E_INVALID, "sieve_update: device_buffer_size must be in [1, padded_buffer_size]");
    if (top_k > (1u << 24) || max_num_reqs > (1u << 24))
        return fail(KVOPS_E_INVALID, "sieve_update: top_k / max_num_reqs out of range");
    int64_t ht_size = 1024;  // kvops_ext.cpp:297-300
    while (ht_size < 2 * (static_cast<int64_t>(padded_buffer_size) + top_k)) ht_size <<= 1;
    *ds_out = nullptr;
    if (max_num_reqs == 0 || top_k == 0) return KVOPS_OK;  // nothing to do (*ds_out stays null)
    if (topk_indices == 0 || req_pool_indices == 0 || seq_lens == 0 || prefill_lens == 0 ||
        device_buffer_tokens == 0 || device_buffer_visited == 0 || device_buffer_ht == 0 || sieve_hand == 0 ||
        topk_device_slots == 0 || is_miss == 0 || num_real == 0)
        return fail(KVOPS_E_INVALID, "sieve_update: a tensor address is 0");
    DeviceState *ds = nullptr;
    int rc = current_device_state(&ds);
    if (rc != KVOPS_OK) return rc;
    kvb::SieveParams p{};
    p.topk = reinterpret_cast<const int32_t *>(topk_indices);
    p.req_pool = reinterpret_cast<const int64_t *>(req_pool_indices);
    p.seq_lens = reinterpret_cast<const int32_t *>(seq_lens);
    p.prefill = reinterpret_cast<const int32_t *>(prefill_lens);
    p.tokens = reinterpret_cast<int32_t *>(device_buffer_tokens);
    p.visited = reinterpret_cast<uint8_t *>(device_buffer_visited);
    p.ht = reinterpret_cast<uint16_t *>(device_buffer_ht);
    p.hand = reinterpret_cast<int32_t *>(sieve_hand);
    p.out_slots = reinterpret_cast<int32_t *>(topk_device_slots);
    p.is_miss = reinterpret_cast<int8_t *>(is_miss);
    p.num_real = reinterpret_cast<const int32_t *>(num_real);
    p.top_k = static_cast<int32_t>(top_k);
    p.dbs = static_cast<int32_t>(device_buffer_size);
    p.padded = static_cast<int32_t>(padded_buffer_size);
    p.vis_stride = static_cast<int32_t>(visited_stride_b);
    p.max_num_reqs = static_cast<int32_t>(max_num_reqs);
    p.pool_size = static_cast<int32_t>(pool_size);
    p.ht_size = static_cast<int32_t>(ht_size);
    (void)stream;
    rc = attach_big_scratch(ds, &p);
    if (rc != KVOPS_OK) return rc;
    *out = p;
    *ds_out = ds;
    return KVOPS_OK;
}

// Whether every row of a gather can move as 16-byte chunks (the copy helpers' width).
bool vec16_ok(const kvb::GatherParams &g)
{
    uint64_t a = g.row_bytes | reinterpret_cast<uintptr_t>(g.hot) | g.hot_req_stride_bytes;
    for (uint32_t n = 0; n < g.nodes; ++n) a |= reinterpret_cast<uintptr_t>(g.seg[n]);
    return (a & 15) == 0;
}

// Allocates (once per device) the zeroed word blocks of cooperative layer-steps.
int ensure_ready_words(DeviceState *ds)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (ds->ready != nullptr) return KVOPS_OK;
    const size_t bytes = sizeof(uint32_t) * kReadyBlocks * kReadyWords;
    cudaError_t e = cudaMalloc(&ds->ready, bytes);
    if (e != cudaSuccess) {
        ds->ready = nullptr;
        return cuda_fail(e, "cudaMalloc(cooperative step words)");
    }
    e = cudaMemset(ds->ready, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(ds->ready);
        ds->ready = nullptr;
        return cuda_fail(e, "cudaMemset(cooperative step words)");
    }
    return KVOPS_OK;
}

// Grows (once per shape, never shrinking) the walk-list buffers to `entries` entries each.
int ensure_walk_lists(DeviceState *ds, size_t entries)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (ds->wl != nullptr && ds->wl_entries >= entries) return KVOPS_OK;
    uint2 *w = nullptr;
    cudaError_t e = cudaMalloc(&w, sizeof(uint2) * entries * kWalkListBufs);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(walk lists)");
    if (ds->wl != nullptr) ds->wl_old.push_back(ds->wl);
    ds->wl = w;
    ds->wl_entries = entries;
    return KVOPS_OK;
}

// Grows (once per shape, never shrinking) the large-table tier's scratch to `bytes` (zeroed for
// tidiness only: the kernel initialises every array it reads).
int ensure_big_scratch(DeviceState *ds, size_t bytes)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (ds->big != nullptr && ds->big_bytes >= bytes) return KVOPS_OK;
    uint8_t *b = nullptr;
    cudaError_t e = cudaMalloc(&b, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(large-table SIEVE scratch)");
    e = cudaMemset(b, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(b);
        return cuda_fail(e, "cudaMemset(large-table SIEVE scratch)");
    }
    if (ds->big != nullptr) ds->big_old.push_back(ds->big);
    ds->big = b;
    ds->big_bytes = bytes;
    return KVOPS_OK;
}

// Points the launch at the large-table tier's scratch when its shape uses that tier.
int attach_big_scratch(DeviceState *ds, kvb::SieveParams *p)
{
    int32_t slots = 0;
    const uint64_t slot_bytes = kvb::sieve_big_scratch(*p, ds->sm_count, &slots);
    if (slots <= 0) return KVOPS_OK;
    const int rc = ensure_big_scratch(ds, static_cast<size_t>(slot_bytes) * slots);
    if (rc != KVOPS_OK) return rc;
    p->big = ds->big;
    p->big_slot_bytes = slot_bytes;
    p->big_slots = slots;
    return KVOPS_OK;
}

// The block of words and the walk-list buffer (max_num_reqs x top_k entries) for the next
// cooperative layer-step on this device.
int next_ready_block(DeviceState *ds, size_t wl_entries, uint32_t **words, uint2 **wl)
{
    int rc = ensure_ready_words(ds);
    if (rc != KVOPS_OK) return rc;
    rc = ensure_walk_lists(ds, wl_entries);
    if (rc != KVOPS_OK) return rc;
    const uint32_t n = ds->ready_next.fetch_add(1, std::memory_order_relaxed);
    *words = ds->ready + static_cast<size_t>(n % kReadyBlocks) * kReadyWords;
    *wl = ds->wl + static_cast<size_t>(n % kWalkListBufs) * ds->wl_entries;
    return KVOPS_OK;
}

// Whether every row copy of the fused step may be a bulk copy: 16-byte multiples and
// alignment on both sides, and every segment in device memory (own or peer HBM). *remote is
// set when a segment is on another GPU.
bool bulk_copy_ok(const kvb::GatherParams &g, bool *remote)
{
    *remote = false;
    if (g.row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(g.hot) % 16 != 0 || g.hot_req_stride_bytes % 16 != 0)
        return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    for (uint32_t n = 0; n < g.nodes; ++n) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(g.seg[n]);
        if (a == 0) continue;  // reported as KVOPS_ERR_SEG_NULL, never read
        if (a % 16 != 0) return false;
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, g.seg[n]) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (at.type != cudaMemoryTypeDevice) return false;
        if (at.device != dev) *remote = true;
    }
    return true;
}

}  // namespace

namespace kvb {
// Lets other translation units of this library report a failure through kvops_last_error().
int set_last_error(int code, const char *msg) { return fail(code, msg); }
bool is_inited()
{
    std::lock_guard<std::mutex> lk(g_mu);
    return g_inited;
}
int clear_status_words(uint64_t status, uint32_t node_lo, uint32_t node_hi, uint32_t block_dim, cudaStream_t stream)
{
    return reset_status(status, node_lo, node_hi, block_dim, stream);
}
}  // namespace kvb

extern "C" {

const char *kvops_last_error(void) { return g_last_error.c_str(); }

int kvops_init(int device_id, const char *fatbin_path, const char *rt_lib)
{
    (void)rt_lib;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (g_inited) return fail(KVOPS_E_ALREADY_INITED, "kvops already inited");
    }
    if (fatbin_path != nullptr && fatbin_path[0] != '\0') {
        struct stat sb;
        if (stat(fatbin_path, &sb) != 0)
            return fail(KVOPS_E_INVALID, std::string("kernel binary path does not exist: ") + fatbin_path);
    }
    cudaError_t e = cudaSetDevice(device_id);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    e = cudaFree(nullptr);  // create the primary context now, not inside a later capture
    if (e != cudaSuccess) return cuda_fail(e, "context init");
    std::lock_guard<std::mutex> lk(g_mu);
    g_home_device = device_id;
    g_inited = true;
    return KVOPS_OK;
}

int kvops_close(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    int cur = 0;
    cudaGetDevice(&cur);
    for (void *p : g_status_allocs) cudaFreeHost(p);
    g_status_allocs.clear();
    for (auto &kv : g_devices) {
        cudaSetDevice(kv.first);
        cudaFree(kv.second->ring);
        if (kv.second->ready) cudaFree(kv.second->ready);
        if (kv.second->wl) cudaFree(kv.second->wl);
        for (uint2 *w : kv.second->wl_old) cudaFree(w);
        if (kv.second->big) cudaFree(kv.second->big);
        for (uint8_t *b : kv.second->big_old) cudaFree(b);
        delete kv.second;
    }
    g_devices.clear();
    cudaSetDevice(cur);
    g_inited = false;
    return KVOPS_OK;
}

int kvops_alloc_status(int count, uint64_t *out_addr)
{
    KV_REQUIRE_INIT();
    if (count <= 0) return fail(KVOPS_E_INVALID, "alloc_status: count must be > 0");
    // Twice the slots asked for: EmsPool.wait polls status + s*64 for s < node_num from
    // any cursor position (xds_ems_pool.py:182-185,238), which can run past `count`.
    const size_t bytes = static_cast<size_t>(count) * 2 * 64;
    void *p = nullptr;
    cudaError_t e = cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return cuda_fail(e, "alloc status failed");
    memset(p, 0, bytes);
    void *dp = nullptr;
    e = cudaHostGetDevicePointer(&dp, p, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(p);
        return cuda_fail(e, "cudaHostGetDevicePointer(status)");
    }
    if (dp != p) {
        cudaFreeHost(p);
        return fail(KVOPS_E_CUDA, "status memory is not unified-addressed");
    }
    std::lock_guard<std::mutex> lk(g_mu);
    g_status_allocs.push_back(p);
    *out_addr = reinterpret_cast<uint64_t>(p);
    return KVOPS_OK;
}

int kvops_poll_status(uint64_t status_addr, int64_t timeout_us, int64_t *out_rc)
{
    KV_REQUIRE_INIT();
    if (status_addr == 0 || (status_addr & 7) != 0) return fail(KVOPS_E_INVALID, "poll_status: bad address");
    const bool host = is_host_memory(status_addr);
    const auto t0 = std::chrono::steady_clock::now();
    uint64_t spins = 0;
    while (true) {
        uint64_t val = 0;
        if (host) {
            val = __atomic_load_n(reinterpret_cast<const uint64_t *>(status_addr), __ATOMIC_ACQUIRE);
        } else if (cudaMemcpy(&val, reinterpret_cast<const void *>(status_addr), 8, cudaMemcpyDeviceToHost) !=
                   cudaSuccess) {
            cudaGetLastError();
            *out_rc = KVOPS_POLL_COPY_FAILED;
            return KVOPS_OK;
        }
        if ((val >> 32) == 1) {
            *out_rc = static_cast<int64_t>(val & 0xFFFFFFFFull);
            return KVOPS_OK;
        }
        if (timeout_us >= 0) {
            const auto us = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0);
            if (us.count() >= timeout_us) {
                *out_rc = KVOPS_POLL_TIMEOUT;
                return KVOPS_OK;
            }
        }
        if (++spins < 20000) {
            _mm_pause();
        } else {
            std::this_thread::yield();
        }
    }
}

int kvops_import_seg_ex(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                        uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                        uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                        uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num,
                        uint32_t my_node, uint64_t status, uint64_t stream, uint32_t block_dim,
                        const KvopsRowOpts *opts)
{
    (void)channel;
    KV_REQUIRE_INIT();
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, "import node_num must be in [1, 64]");
    if (my_node >= node_num) return fail(KVOPS_E_INVALID, "import my_node must be < node_num");
    uint64_t segs[KVOPS_MAX_NODES] = {0};
    segs[my_node] = seg_base;
    return import_common(node_num, segs, my_node, my_node + 1, my_node, layer_offset_rows, per_layer_seg_rows,
                         row_bytes, topk_indices, req_pool_indices, req_host_base, topk_device_slots, is_miss,
                         num_real, hot_row_base, top_k, max_num_reqs, stripe_rows, status, stream, block_dim, opts);
}

int kvops_export_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                     uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                     uint64_t topk_device_slots, uint64_t export_flags, uint64_t num_real, uint64_t hot_row_base,
                     uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                     uint64_t status, uint64_t stream, uint32_t block_dim, const KvopsRowOpts *opts)
{
    (void)channel;
    KV_REQUIRE_INIT();
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, "export_seg node_num must be in [1, 64]");
    if (my_node >= node_num) return fail(KVOPS_E_INVALID, "export_seg my_node must be < node_num");
    uint64_t segs[KVOPS_MAX_NODES] = {0};
    segs[my_node] = seg_base;
    kvb::GatherParams p{};
    DeviceState *ds = nullptr;
    int rc = build_gather(node_num, segs, my_node, my_node + 1, my_node, layer_offset_rows, per_layer_seg_rows,
                          row_bytes, topk_indices, req_pool_indices, req_host_base, topk_device_slots, export_flags,
                          num_real, hot_row_base, top_k, max_num_reqs, stripe_rows, status, stream, block_dim, opts,
                          &p, &ds, "export_seg");
    if (rc != KVOPS_OK) return rc;
    cudaError_t e = kvb::launch_scatter(p, reinterpret_cast<cudaStream_t>(stream), ds->sm_count);
    if (e != cudaSuccess) return cuda_fail(e, "launch kvc_scatter_rows");
    return KVOPS_OK;
}

int kvops_import_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                     uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                     uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                     uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                     uint64_t status, uint64_t stream, uint32_t block_dim)
{
    return kvops_import_seg_ex(channel, seg_base, layer_offset_rows, per_layer_seg_rows, row_bytes, topk_indices,
                               req_pool_indices, req_host_base, topk_device_slots, is_miss, num_real, hot_row_base,
                               top_k, max_num_reqs, stripe_rows, node_num, my_node, status, stream, block_dim,
                               nullptr);
}

int kvops_import_multi(uint32_t node_num, const uint64_t *seg_bases, uint32_t layer_offset_rows,
                       uint32_t per_layer_seg_rows, uint32_t row_bytes, uint64_t topk_indices,
                       uint64_t req_pool_indices, uint64_t req_host_base, uint64_t topk_device_slots,
                       uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base, uint32_t top_k,
                       uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                       uint32_t block_dim, const KvopsRowOpts *opts)
{
    KV_REQUIRE_INIT();
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, "import node_num must be in [1, 64]");
    if (seg_bases == nullptr) return fail(KVOPS_E_INVALID, "import_multi: seg_bases is NULL");
    return import_common(node_num, seg_bases, 0, node_num, kvb::kAllNodes, layer_offset_rows, per_layer_seg_rows,
                         row_bytes, topk_indices, req_pool_indices, req_host_base, topk_device_slots, is_miss,
                         num_real, hot_row_base, top_k, max_num_reqs, stripe_rows, status, stream, block_dim, opts);
}

int kvops_export_seg_alllayer_ex(uint64_t channel, uint64_t seg_base, uint32_t per_layer_seg_rows,
                                 uint32_t row_bytes, uint32_t row_lo, uint32_t row_cnt, uint32_t layer_num,
                                 uint64_t src_layer0_base, uint64_t src_layer_stride, uint32_t stripe_rows,
                                 uint32_t node_num, uint32_t my_node, uint64_t status, uint64_t stream,
                                 uint32_t block_dim, const KvopsRowOpts *opts)
{
    (void)channel;
    return export_common(seg_base, per_layer_seg_rows, row_bytes, row_lo, row_cnt, layer_num, src_layer0_base,
                         src_layer_stride, stripe_rows, node_num, my_node, status, stream, block_dim, opts);
}

int kvops_export_seg_alllayer(uint64_t channel, uint64_t seg_base, uint32_t per_layer_seg_rows, uint32_t row_bytes,
                              uint32_t row_lo, uint32_t row_cnt, uint32_t layer_num, uint64_t src_layer0_base,
                              uint64_t src_layer_stride, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                              uint64_t status, uint64_t stream, uint32_t block_dim)
{
    return kvops_export_seg_alllayer_ex(channel, seg_base, per_layer_seg_rows, row_bytes, row_lo, row_cnt, layer_num,
                                        src_layer0_base, src_layer_stride, stripe_rows, node_num, my_node, status,
                                        stream, block_dim, nullptr);
}

int kvops_sieve_update(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                       uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                       uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                       uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs, uint32_t pool_size, uint64_t stream,
                       uint32_t block_dim)
{
    kvb::SieveParams p{};
    DeviceState *ds = nullptr;
    int rc = build_sieve(topk_indices, req_pool_indices, seq_lens, prefill_lens, device_buffer_tokens,
                         device_buffer_visited, device_buffer_ht, sieve_hand, topk_device_slots, is_miss, num_real,
                         top_k, device_buffer_size, padded_buffer_size, visited_stride_b, max_num_reqs, pool_size,
                         stream, block_dim, &p, &ds);
    if (rc != KVOPS_OK || ds == nullptr) return rc;
    cudaError_t e = kvb::launch_sieve_update(p, reinterpret_cast<cudaStream_t>(stream), ds->sm_count);
    if (e != cudaSuccess) return cuda_fail(e, "launch hisp_sieve_update");
    return KVOPS_OK;
}

int kvops_sieve_import(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                       uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                       uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                       uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs, uint32_t pool_size, uint32_t node_num,
                       const uint64_t *seg_bases, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                       uint32_t row_bytes, uint64_t req_host_base, uint64_t hot_row_base, uint32_t stripe_rows,
                       uint64_t status, uint64_t stream, uint32_t block_dim, const KvopsRowOpts *opts)
{
    KV_REQUIRE_INIT();
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return fail(KVOPS_E_INVALID, "sieve_import node_num must be in [1, 64]");
    if (seg_bases == nullptr) return fail(KVOPS_E_INVALID, "sieve_import: seg_bases is NULL");
    kvb::SieveParams sp{};
    DeviceState *sds = nullptr;  // null: the SIEVE step has nothing to do
    int rc = build_sieve(topk_indices, req_pool_indices, seq_lens, prefill_lens, device_buffer_tokens,
                         device_buffer_visited, device_buffer_ht, sieve_hand, topk_device_slots, is_miss, num_real,
                         top_k, device_buffer_size, padded_buffer_size, visited_stride_b, max_num_reqs, pool_size,
                         stream, 1u, &sp, &sds);
    if (rc != KVOPS_OK) return rc;
    kvb::GatherParams gp{};
    DeviceState *ds = nullptr;
    rc = build_gather(node_num, seg_bases, 0, node_num, kvb::kAllNodes, layer_offset_rows, per_layer_seg_rows,
                      row_bytes, topk_indices, req_pool_indices, req_host_base, topk_device_slots, is_miss, num_real,
                      hot_row_base, top_k, max_num_reqs, stripe_rows, status, stream, block_dim, opts, &gp, &ds);
    if (rc != KVOPS_OK) return rc;
    const uint32_t path = opts ? opts->step_path : KVOPS_STEP_AUTO;
    if (path > KVOPS_STEP_COOP) return fail(KVOPS_E_INVALID, "sieve_import: step_path must be 0, 1, 2 or 3");
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // The one-kernel paths run the shared-memory tier; another chosen tier runs as SPLIT.
    const bool shared_tier = t_tier_choice == KVOPS_TIER_AUTO || t_tier_choice == KVOPS_TIER_SHARED;
    if (sds != nullptr && shared_tier && (path == KVOPS_STEP_AUTO || path == KVOPS_STEP_COOP) && vec16_ok(gp)) {
        uint32_t *words = nullptr;
        uint2 *wl = nullptr;
        rc = next_ready_block(sds, static_cast<size_t>(max_num_reqs) * top_k, &words, &wl);
        if (rc != KVOPS_OK) return rc;
        bool launched = false;
        // AUTO takes the cooperative step only when the copy CTAs number at least half the
        // requests; with fewer, the full-GPU gather after the SIEVE kernel moves the rows faster.
        const int32_t min_copy = path == KVOPS_STEP_AUTO ? static_cast<int32_t>(max_num_reqs / 2) : 8;
        cudaError_t e = kvb::launch_sieve_coop(sp, gp, words, wl, opts ? opts->copy_wait_polls : 0u, min_copy, st,
                                               &launched);
        if (e != cudaSuccess) return cuda_fail(e, "launch sieve_import (cooperative)");
        if (launched) {
            t_last_step_path = KVOPS_STEP_COOP;
            return KVOPS_OK;
        }
    }
    bool remote = false;
    if (sds != nullptr && shared_tier && path == KVOPS_STEP_FUSED && bulk_copy_ok(gp, &remote)) {
        bool launched = false;
        cudaError_t e = kvb::launch_sieve_import(sp, gp, st, &launched);
        if (e != cudaSuccess) return cuda_fail(e, "launch sieve_import");
        if (launched) {
            t_last_step_path = KVOPS_STEP_FUSED;
            return KVOPS_OK;
        }
    }
    t_last_step_path = KVOPS_STEP_SPLIT;
    // The same step as two kernels (state too large for the fused kernel, host or unaligned rows).
    if (sds != nullptr) {
        cudaError_t e = kvb::launch_sieve_update(sp, st, sds->sm_count);
        if (e != cudaSuccess) return cuda_fail(e, "launch hisp_sieve_update");
    }
    cudaError_t e = kvb::launch_gather(gp, st, ds->sm_count);
    if (e != cudaSuccess) return cuda_fail(e, "launch kvc_gather_rows");
    return KVOPS_OK;
}

uint32_t kvops_last_step_path(void) { return t_last_step_path; }

int kvops_set_sieve_tier(uint32_t tier)
{
    if (tier > KVOPS_TIER_ORDERED) return fail(KVOPS_E_INVALID, "set_sieve_tier: tier must be 0, 1, 2 or 3");
    t_tier_choice = tier;
    kvb::set_sieve_tier(tier);
    return KVOPS_OK;
}

uint32_t kvops_last_sieve_tier(void) { return kvb::last_sieve_tier(); }

int kvops_step_prepare(uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size,
                       uint32_t visited_stride_b, uint32_t max_num_reqs)
{
    KV_REQUIRE_INIT();
    DeviceState *ds = nullptr;
    int rc = current_device_state(&ds);
    if (rc != KVOPS_OK) return rc;
    rc = ensure_ready_words(ds);
    if (rc != KVOPS_OK) return rc;
    rc = ensure_walk_lists(ds, static_cast<size_t>(max_num_reqs) * top_k);
    if (rc != KVOPS_OK) return rc;
    int64_t ht_size = 1024;
    while (ht_size < 2 * (static_cast<int64_t>(padded_buffer_size) + top_k)) ht_size <<= 1;
    kvb::SieveParams p{};
    p.top_k = static_cast<int32_t>(top_k);
    p.dbs = static_cast<int32_t>(device_buffer_size);
    p.padded = static_cast<int32_t>(padded_buffer_size);
    p.vis_stride = static_cast<int32_t>(visited_stride_b);
    p.max_num_reqs = static_cast<int32_t>(max_num_reqs);
    p.ht_size = static_cast<int32_t>(ht_size);
    rc = attach_big_scratch(ds, &p);
    if (rc != KVOPS_OK) return rc;
    cudaError_t e = kvb::prepare_sieve_coop(p);
    if (e != cudaSuccess) return cuda_fail(e, "step_prepare");
    return KVOPS_OK;
}

int kvops_sieve_ht_init(uint64_t device_buffer_tokens, uint64_t device_buffer_ht, uint64_t prefill_lens,
                        uint32_t req_start, uint32_t num_reqs, uint32_t layer_num, uint32_t pool_size,
                        uint32_t device_buffer_size, uint32_t padded_buffer_size, uint32_t ht_size, uint64_t stream,
                        uint32_t block_dim)
{
    KV_REQUIRE_INIT();
    (void)prefill_lens;  // passed but unused by the reference kernel too (hisp_sieve_ht_init.cpp)
    if (ht_size == 0 || (ht_size & (ht_size - 1)) != 0 || ht_size > (1u << 26))
        return fail(KVOPS_E_INVALID, "sieve_ht_init: ht_size must be a power of two");
    if (device_buffer_size > padded_buffer_size)
        return fail(KVOPS_E_INVALID, "sieve_ht_init: device_buffer_size must be <= padded_buffer_size");
    if (padded_buffer_size > 65534)
        return fail(KVOPS_E_INVALID, "sieve_ht_init: padded_buffer_size must be <= 65534 (uint16 hash slots)");
    const uint64_t all = static_cast<uint64_t>(layer_num) * num_reqs;
    const uint64_t pairs = block_dim == 0 ? all : (block_dim < all ? block_dim : all);
    if (pairs == 0) return KVOPS_OK;
    if (pairs > (1u << 30)) return fail(KVOPS_E_INVALID, "sieve_ht_init: too many (layer, request) pairs");
    if (device_buffer_tokens == 0 || device_buffer_ht == 0)
        return fail(KVOPS_E_INVALID, "sieve_ht_init: a tensor address is 0");
    kvb::HtInitParams p{};
    p.tokens = reinterpret_cast<const int32_t *>(device_buffer_tokens);
    p.ht = reinterpret_cast<uint16_t *>(device_buffer_ht);
    p.req_start = static_cast<int32_t>(req_start);
    p.num_reqs = static_cast<int32_t>(num_reqs);
    p.layer_num = static_cast<int32_t>(layer_num);
    p.pool_size = static_cast<int32_t>(pool_size);
    p.dbs = static_cast<int32_t>(device_buffer_size);
    p.padded = static_cast<int32_t>(padded_buffer_size);
    p.ht_size = static_cast<int32_t>(ht_size);
    p.pairs = static_cast<int32_t>(pairs);
    cudaError_t e = kvb::launch_sieve_ht_init(p, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "launch hisp_sieve_ht_init");
    return KVOPS_OK;
}

int kvops_segment_alloc(int device, uint64_t bytes, uint64_t *out_addr)
{
    if (bytes == 0) return fail(KVOPS_E_INVALID, "segment_alloc: bytes must be > 0");
    void *p = nullptr;
    if (device < 0) {
        cudaError_t e = cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(segment)");
    } else {
        // Device segments are allocated in whole 2 MiB units. A segment is read by other GPUs
        // through CUDA IPC, and an allocation whose size is not a multiple of 2 MiB was mapped
        // there so that random row reads crossing many pages ran at under half the link rate
        // (N=4 B200, 61 per-layer regions of 201 MB: 251 GB/s per GPU against 540 GB/s with the
        // size rounded up); local reads are unaffected.
        constexpr uint64_t kUnit = 2ull << 20;
        bytes = (bytes + kUnit - 1) / kUnit * kUnit;
        int cur = 0;
        cudaGetDevice(&cur);
        cudaError_t e = cudaSetDevice(device);
        if (e == cudaSuccess) e = cudaMalloc(&p, bytes);
        cudaSetDevice(cur);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(segment)");
    }
    std::lock_guard<std::mutex> lk(g_mu);
    g_segments[reinterpret_cast<uint64_t>(p)] = device;
    *out_addr = reinterpret_cast<uint64_t>(p);
    return KVOPS_OK;
}

int kvops_segment_free(uint64_t addr)
{
    int device;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_segments.find(addr);
        if (it == g_segments.end()) return fail(KVOPS_E_INVALID, "segment_free: unknown segment");
        device = it->second;
        g_segments.erase(it);
    }
    cudaError_t e = device < 0 ? cudaFreeHost(reinterpret_cast<void *>(addr)) : cudaFree(reinterpret_cast<void *>(addr));
    if (e != cudaSuccess) return cuda_fail(e, "segment free");
    return KVOPS_OK;
}

int kvops_enable_peer_access(int device, int peer)
{
    int ok = 0;
    cudaError_t e = cudaDeviceCanAccessPeer(&ok, device, peer);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
    if (!ok) return fail(KVOPS_E_INVALID, "peer access not supported between these devices");
    int cur = 0;
    cudaGetDevice(&cur);
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        e = cudaSuccess;
    }
    cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
    return KVOPS_OK;
}

int kvops_ipc_get_handle(uint64_t addr, uint8_t out_handle[64])
{
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(addr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(out_handle, &h, 64);
    return KVOPS_OK;
}

int kvops_ipc_open_handle(int device, const uint8_t handle[64], uint64_t *out_addr)
{
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    int cur = 0;
    cudaGetDevice(&cur);
    void *p = nullptr;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    cudaSetDevice(cur);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *out_addr = reinterpret_cast<uint64_t>(p);
    return KVOPS_OK;
}

int kvops_ipc_close_handle(uint64_t addr)
{
    cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void *>(addr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
    return KVOPS_OK;
}

}  // extern "C"
