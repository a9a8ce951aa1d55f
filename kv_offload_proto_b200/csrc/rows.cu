// rows.cu — miss-row gather (kvc_gather_rows) and striped all-layer export
// (kvc_scatter_rows_alllayer) for sm_100a.
//
// Both are sparse row copies bounded by HBM / NVLink / host-link bandwidth; no tensor
// cores. A CTA owns a tile of 256 candidate rows per iteration: threads evaluate one
// position (or destination row) each, the accepted rows are appended to a shared list, and
// the whole CTA then streams the list as one flat array of 16-byte chunks with 8 loads in
// flight per thread before the matching stores. Sources may be own HBM, a peer GPU's HBM (UVA,
// NVLink/NVSwitch) or pinned host memory; every load is a plain global load.
#include <stdint.h>

#include "kvops_internal.cuh"
#include "rows_common.cuh"

namespace kvb {
namespace {

constexpr int kRowThreads = 256;
constexpr int kUnroll = 8;

// One tile = kGatherTile consecutive positions per CTA iteration: every thread evaluates one
// position (kvc_gather_rows.cpp:54-76), the accepted rows are appended to a shared list, and
// the CTA then copies the list with cta_copy_rows. The grid is sized to the GPU and loops over
// tiles, so no wave is left partly empty.
constexpr int kGatherTile = kRowThreads;

template <typename V, bool kScatter>
__global__ void __launch_bounds__(kRowThreads, 4) gather_kernel(const GatherParams p, uint32_t magic)
{
    __shared__ const uint8_t *s_src[kGatherTile];
    __shared__ uint8_t *s_dst[kGatherTile];
    __shared__ int s_n;
    // Launched as a programmatic dependent of the SIEVE step: the CTAs may start while that
    // kernel runs and wait here for its completion (and memory flush) before reading its
    // outputs. Without the launch attribute this returns at once.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    int32_t num_real = p.num_real != nullptr ? *p.num_real : 0;
    if (num_real > static_cast<int32_t>(p.max_num_reqs)) num_real = static_cast<int32_t>(p.max_num_reqs);
    const int64_t total = num_real > 0 ? static_cast<int64_t>(num_real) * p.top_k : 0;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * kGatherTile; base < total;
         base += static_cast<int64_t>(gridDim.x) * kGatherTile) {
        const int64_t end = base + kGatherTile < total ? base + kGatherTile : total;
        gather_tile<V, kUnroll, false, kScatter>(p, base, end, s_src, s_dst, &s_n, magic);
    }
    __syncthreads();
    if (threadIdx.x == 0) arrive_and_publish(p.st);
}

// Destination unit k of one layer -> (source row, segment row); false if outside the range.
// Reference map with S > 1: unit k is the k-th owned stripe and only its last row in range is
// copied, because the reference's ascending per-row writes leave exactly that row in the
// shared segment row (kvc_scatter_rows_alllayer.cpp:34-53).
__device__ __forceinline__ bool export_unit(const ExportParams &p, uint64_t k, uint32_t *src_row, uint32_t *seg_row)
{
    const uint64_t lo = p.row_lo, hi = static_cast<uint64_t>(p.row_lo) + p.row_cnt - 1;
    if (p.stripe == 0) {
        *src_row = static_cast<uint32_t>(lo + k);
        *seg_row = *src_row;
        return true;
    }
    const uint64_t S = p.stripe;
    if (!p.injective) {
        const uint64_t g = p.g_first + k * p.nodes;
        const uint64_t last = (g + 1) * S - 1;
        *src_row = static_cast<uint32_t>(last < hi ? last : hi);
        *seg_row = static_cast<uint32_t>(g / p.nodes);
        return true;
    }
    const uint64_t g = p.g_first + (k / S) * p.nodes;
    const uint64_t r = g * S + k % S;
    if (r < lo || r > hi) return false;
    *src_row = static_cast<uint32_t>(r);
    *seg_row = static_cast<uint32_t>((g / p.nodes) * S + k % S);
    return true;
}

template <typename V>
__global__ void __launch_bounds__(kRowThreads, 4) export_kernel(const ExportParams p, uint32_t magic)
{
    __shared__ const uint8_t *s_src[kGatherTile];
    __shared__ uint8_t *s_dst[kGatherTile];
    __shared__ int s_n;
    const int lane = threadIdx.x & 31;
    const uint64_t total = p.units_per_layer * p.layer_num;
    if (p.seg_null && blockIdx.x == 0 && threadIdx.x == 0) record_error(p.st, KVOPS_ERR_SEG_NULL);
    for (uint64_t base = static_cast<uint64_t>(blockIdx.x) * kGatherTile; base < total;
         base += static_cast<uint64_t>(gridDim.x) * kGatherTile) {
        if (threadIdx.x == 0) s_n = 0;
        __syncthreads();
        const uint64_t u = base + threadIdx.x;
        bool ok = false;
        const uint8_t *src = nullptr;
        uint8_t *dst = nullptr;
        if (u < total) {
            const uint64_t l = u / p.units_per_layer;
            const uint64_t k = u - l * p.units_per_layer;
            uint32_t src_row, seg_row;
            if (export_unit(p, k, &src_row, &seg_row)) {
                if (seg_row >= p.plsr) {
                    const uint64_t idx = l * p.row_cnt + (src_row - p.row_lo);
                    record_error(p.st, KVOPS_ERR_ROW_BASE + static_cast<uint32_t>(idx & 0xFFu) + (1u << 16));
                } else {
                    src = p.src0 + l * p.src_layer_stride + static_cast<uint64_t>(src_row) * p.row_bytes;
                    dst = p.seg + (l * p.plsr + seg_row) * static_cast<uint64_t>(p.row_bytes);
                    ok = true;
                }
            }
        }
        const unsigned mask = __ballot_sync(0xFFFFFFFFu, ok);
        int at = 0;
        if (lane == 0 && mask) at = atomicAdd(&s_n, __popc(mask));
        at = __shfl_sync(0xFFFFFFFFu, at, 0) + __popc(mask & ((1u << lane) - 1u));
        if (ok) {
            s_src[at] = src;
            s_dst[at] = dst;
        }
        __syncthreads();
        cta_copy_rows<V, kUnroll>(s_src, s_dst, s_n, p.row_bytes, magic);
        __syncthreads();
    }
    __syncthreads();
    if (threadIdx.x == 0) arrive_and_publish(p.st);
}

// Widest vector every row address allows: all bases and the row size share the alignment.
int vec_bytes(uint64_t addr_or, uint32_t row_bytes)
{
    const uint64_t a = addr_or | row_bytes;
    if ((a & 15) == 0) return 16;
    if ((a & 7) == 0) return 8;
    if ((a & 3) == 0) return 4;
    return 1;
}


}  // namespace

template <bool kScatter>
cudaError_t launch_rows(const GatherParams &p, cudaStream_t s, int sm_count)
{
    uint64_t addr_or = reinterpret_cast<uint64_t>(p.hot) | p.hot_req_stride_bytes;
    for (uint32_t n = 0; n < p.nodes && n < static_cast<uint32_t>(kMaxNodes); ++n)
        addr_or |= reinterpret_cast<uint64_t>(p.seg[n]);
    const uint64_t positions = static_cast<uint64_t>(p.max_num_reqs) * p.top_k;
    const uint64_t tiles = (positions + kGatherTile - 1) / kGatherTile;
    const uint64_t cap = static_cast<uint64_t>(sm_count > 0 ? sm_count : 148) * 4;
    const int grid = static_cast<int>(tiles < 1 ? 1 : (tiles < cap ? tiles : cap));
    const int vb = vec_bytes(addr_or, p.row_bytes);
    // chunk index < tile rows * chunks per row; exact multiply-high division needs i * e < 2^32
    const uint64_t cpr = p.row_bytes / vb;
    const uint32_t magic = (cpr > 0 && cpr < 65536 && kGatherTile * cpr < 65536)
                               ? static_cast<uint32_t>(((1ull << 32) + cpr - 1) / cpr) : 0u;
    // Programmatic stream serialization: the CTAs launch as soon as the previous kernel (the
    // SIEVE step, which triggers at entry) lets them, and gather_kernel waits for its completion.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kRowThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    switch (vb) {
        case 16: return cudaLaunchKernelEx(&cfg, gather_kernel<uint4, kScatter>, p, magic);
        case 8: return cudaLaunchKernelEx(&cfg, gather_kernel<uint2, kScatter>, p, magic);
        case 4: return cudaLaunchKernelEx(&cfg, gather_kernel<uint32_t, kScatter>, p, magic);
        default: return cudaLaunchKernelEx(&cfg, gather_kernel<uint8_t, kScatter>, p, magic);
    }
}

cudaError_t launch_gather(const GatherParams &p, cudaStream_t s, int sm_count)
{
    return launch_rows<false>(p, s, sm_count);
}

cudaError_t launch_scatter(const GatherParams &p, cudaStream_t s, int sm_count)
{
    return launch_rows<true>(p, s, sm_count);
}

cudaError_t launch_export(const ExportParams &p, cudaStream_t s, int sm_count)
{
    const uint64_t addr_or = reinterpret_cast<uint64_t>(p.src0) | p.src_layer_stride | reinterpret_cast<uint64_t>(p.seg);
    const uint64_t units = p.units_per_layer * p.layer_num;
    const uint64_t tiles = (units + kGatherTile - 1) / kGatherTile;
    const uint64_t cap = static_cast<uint64_t>(sm_count > 0 ? sm_count : 148) * 4;
    const int grid = static_cast<int>(tiles < 1 ? 1 : (tiles < cap ? tiles : cap));
    const int vb = vec_bytes(addr_or, p.row_bytes);
    const uint64_t cpr = p.row_bytes / vb;
    const uint32_t magic = (cpr > 0 && cpr < 65536 && kGatherTile * cpr < 65536)
                               ? static_cast<uint32_t>(((1ull << 32) + cpr - 1) / cpr) : 0u;
    switch (vb) {
        case 16: export_kernel<uint4><<<grid, kRowThreads, 0, s>>>(p, magic); break;
        case 8: export_kernel<uint2><<<grid, kRowThreads, 0, s>>>(p, magic); break;
        case 4: export_kernel<uint32_t><<<grid, kRowThreads, 0, s>>>(p, magic); break;
        default: export_kernel<uint8_t><<<grid, kRowThreads, 0, s>>>(p, magic); break;
    }
    return cudaGetLastError();
}

}  // namespace kvb
