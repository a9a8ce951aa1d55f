// noalloc.cu — kvops_import_multi_noalloc: the all-segment miss-row gather of
// kvops_import_multi, for callers that cannot allocate device memory.
//
// Who needs it: a serving engine whose device memory is owned by its own allocator or a
// fixed HBM budget (every byte pre-reserved for KV pages, so a library must not take
// memory behind its back), and latency-critical decode loops that cannot pay for
// cudaMalloc/cudaFree (cudaFree synchronizes the device). The regular entry point
// allocates, on its first launch on a device, a ring of completion tickets with cudaMalloc;
// this one keeps its only scratch in the static array below instead and calls no
// allocating routine at all.
//
// Scratch: one 8-byte completion ticket (the CTA arrival count and the first errCode of
// the launch), inside a file-scope static __device__ array of KVOPS_NOALLOC_SCRATCH_BYTES
// bytes that every GPU loading this library holds until the process exits. Every call
// shares it: the ticket is cleared on the caller's stream before each launch, and calls
// whose launches overlap on the GPU (other streams, other threads) race on it and must not
// be issued. The device address of the array is looked up once per device, on the first
// call made with that device current; make that first call before any stream capture.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "kvops_internal.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KVOPS_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
std::unordered_map<int, void *> g_noalloc_ptr;  // device -> device address of g_noalloc_scratch

// Device address of the scratch array for the current device (set-up on first use).
int noalloc_scratch(void **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return kvb::set_last_error(KVOPS_E_CUDA, "import_multi_noalloc: cudaGetDevice failed");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    auto it = g_noalloc_ptr.find(dev);
    if (it != g_noalloc_ptr.end()) {
        *out = it->second;
        return KVOPS_OK;
    }
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return kvb::set_last_error(KVOPS_E_CUDA, (std::string("import_multi_noalloc: cudaGetSymbolAddress failed: ") +
                                                  cudaGetErrorString(e)).c_str());
    }
    g_noalloc_ptr[dev] = p;
    *out = p;
    return KVOPS_OK;
}

}  // namespace

extern "C" int kvops_import_multi_noalloc(uint32_t node_num, const uint64_t *seg_bases, uint32_t layer_offset_rows,
                                          uint32_t per_layer_seg_rows, uint32_t row_bytes, uint64_t topk_indices,
                                          uint64_t req_pool_indices, uint64_t req_host_base,
                                          uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                                          uint64_t hot_row_base, uint32_t top_k, uint32_t max_num_reqs,
                                          uint32_t stripe_rows, uint64_t status, uint64_t stream, uint32_t block_dim,
                                          const KvopsRowOpts *opts)
{
    using kvb::set_last_error;
    if (!kvb::is_inited()) return set_last_error(KVOPS_E_NOT_INITED, "kvops not inited");
    if (node_num == 0 || node_num > KVOPS_MAX_NODES)
        return set_last_error(KVOPS_E_INVALID, "import node_num must be in [1, 64]");
    if (seg_bases == nullptr) return set_last_error(KVOPS_E_INVALID, "import_multi: seg_bases is NULL");
    if (block_dim > 8) return set_last_error(KVOPS_E_INVALID, "import blockDim must be <= 8 (status slot layout)");
    if (block_dim == 0) return set_last_error(KVOPS_E_INVALID, "import blockDim must be >= 1");
    if (row_bytes == 0) return set_last_error(KVOPS_E_INVALID, "import row_bytes must be > 0");
    if (max_num_reqs > 0 && top_k > 0 &&
        (topk_indices == 0 || req_pool_indices == 0 || req_host_base == 0 || topk_device_slots == 0 ||
         is_miss == 0 || num_real == 0 || hot_row_base == 0))
        return set_last_error(KVOPS_E_INVALID, "import: a tensor address is 0");
    const KvopsRowOpts o = opts ? *opts : KvopsRowOpts{};
    if (o.injective > 1) return set_last_error(KVOPS_E_INVALID, "import: injective must be 0 or 1");
    if ((o.err_word & 3) != 0) return set_last_error(KVOPS_E_INVALID, "import: err_word must be 4-byte aligned");
    // The launch's scratch is one completion ticket when it publishes status words.
    const size_t need = status != 0 ? sizeof(kvb::Ticket) : 0;
    if (need > KVOPS_NOALLOC_SCRATCH_BYTES)
        return set_last_error(KVOPS_E_INVALID, "import_multi_noalloc: the launch needs more scratch than the "
                                               "static array holds (KVOPS_NOALLOC_SCRATCH_BYTES)");
    void *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc != KVOPS_OK) return rc;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

    kvb::GatherParams p{};
    p.topk = reinterpret_cast<const int32_t *>(topk_indices);
    p.req_pool = reinterpret_cast<const int64_t *>(req_pool_indices);
    p.host_base = reinterpret_cast<const int64_t *>(req_host_base);
    p.slots = reinterpret_cast<const int32_t *>(topk_device_slots);
    p.is_miss = reinterpret_cast<const int8_t *>(is_miss);
    p.num_real = (max_num_reqs == 0 || top_k == 0) ? nullptr : reinterpret_cast<const int32_t *>(num_real);
    p.hot = reinterpret_cast<uint8_t *>(hot_row_base);
    p.hot_req_stride_bytes = o.hot_req_stride_rows * row_bytes;
    p.layer_offset_rows = layer_offset_rows;
    p.plsr = per_layer_seg_rows;
    p.row_bytes = row_bytes;
    p.stripe = stripe_rows;
    p.nodes = node_num;
    p.my_node = kvb::kAllNodes;
    p.top_k = top_k;
    p.max_num_reqs = max_num_reqs;
    p.injective = o.injective;
    for (uint32_t n = 0; n < node_num; ++n) p.seg[n] = reinterpret_cast<const uint8_t *>(seg_bases[n]);
    p.st.status = reinterpret_cast<uint64_t *>(status);
    p.st.node_lo = 0;
    p.st.node_hi = node_num;
    p.st.block_dim = block_dim;
    p.st.ticket = nullptr;
    p.st.err_word = reinterpret_cast<uint32_t *>(o.err_word);
    if (status != 0) {
        // The ticket must start at zero: clear it in stream order. The status words the launch
        // will publish are cleared as every other entry point clears them.
        cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(kvb::Ticket), s);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_last_error(KVOPS_E_CUDA, "import_multi_noalloc: cudaMemsetAsync(ticket) failed");
        }
        p.st.ticket = static_cast<kvb::Ticket *>(scratch);
        rc = kvb::clear_status_words(status, 0, node_num, block_dim, s);
        if (rc != KVOPS_OK) return rc;
    }
    cudaError_t e = kvb::launch_gather(p, s, sms);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_last_error(KVOPS_E_CUDA, (std::string("launch kvc_gather_rows (no-alloc): ") +
                                             cudaGetErrorString(e)).c_str());
    }
    return KVOPS_OK;
}
