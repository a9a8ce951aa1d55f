// rows.cu — miss-row gather (kvc_gather_rows) and striped all-layer export
// (kvc_scatter_rows_alllayer) for sm_100a.
//
// Both are sparse row copies bounded by HBM / NVLink / host-link bandwidth; no tensor
// cores. A warp owns 32 candidate rows per iteration: lanes evaluate one position (or
// destination row) each, the accepted rows are compacted with a ballot, and the warp
// then streams them as one flat array of 16-byte chunks with 8 loads in flight per
// lane before the matching stores. Sources may be own HBM, a peer GPU's HBM (UVA,
// NVLink/NVSwitch) or pinned host memory; loads are plain (no TMA, no multicast).
#include <stdint.h>

#include "kvops_internal.cuh"

namespace kvb {
namespace {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kUnroll = 8;

template <typename V>
__device__ __forceinline__ V load_stream(const V *p)
{
    return __ldcs(p);
}
template <>
__device__ __forceinline__ uint8_t load_stream<uint8_t>(const uint8_t *p)
{
    return *reinterpret_cast<const volatile uint8_t *>(p);
}

// Copies n rows (src[i] -> dst[i], i < n, n <= 32) of `row_bytes` bytes with the whole warp.
template <typename V>
__device__ __forceinline__ void warp_copy_rows(const uint8_t *const *src, uint8_t *const *dst, int n,
                                               uint32_t row_bytes, int lane)
{
    const uint32_t cpr = row_bytes / sizeof(V);  // chunks per row
    const uint32_t total = static_cast<uint32_t>(n) * cpr;
    // (r, c) = divmod(i, cpr) for i = lane, advanced by 32 per step without a division.
    uint32_t r = 0, c = static_cast<uint32_t>(lane);
    while (c >= cpr && r < static_cast<uint32_t>(n)) {
        c -= cpr;
        ++r;
    }
    for (uint32_t i0 = lane; i0 < total; i0 += 32u * kUnroll) {
        V v[kUnroll];
        uint32_t rr[kUnroll], cc[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            rr[u] = r;
            cc[u] = c;
            if (i0 + 32u * u < total) v[u] = load_stream(reinterpret_cast<const V *>(src[r]) + c);
            c += 32;
            while (c >= cpr) {
                c -= cpr;
                ++r;
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            if (i0 + 32u * u < total) reinterpret_cast<V *>(dst[rr[u]])[cc[u]] = v[u];
        }
    }
}

template <typename V>
__global__ void __launch_bounds__(kRowThreads) gather_kernel(const GatherParams p)
{
    __shared__ const uint8_t *s_src[kRowWarps][32];
    __shared__ uint8_t *s_dst[kRowWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int32_t num_real = p.num_real != nullptr ? *p.num_real : 0;
    if (num_real > static_cast<int32_t>(p.max_num_reqs)) num_real = static_cast<int32_t>(p.max_num_reqs);
    const int64_t total = num_real > 0 ? static_cast<int64_t>(num_real) * p.top_k : 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kRowWarps * 32;
    for (int64_t base = (static_cast<int64_t>(blockIdx.x) * kRowWarps + warp) * 32; base < total; base += stride) {
        const int64_t pos = base + lane;
        bool ok = false;
        const uint8_t *src = nullptr;
        uint8_t *dst = nullptr;
        if (pos < total && p.is_miss[pos] != 0) {  // kvc_gather_rows.cpp:55-57
            const int32_t t = p.topk[pos];
            const int32_t slot = p.slots[pos];
            const int64_t bid = pos / p.top_k;
            const int64_t req = p.req_pool[bid];
            if (t >= 0 && slot >= 0 && req >= 0) {  // :62-68
                const uint32_t row = static_cast<uint32_t>(p.host_base[bid] + t);
                const uint32_t node = node_of(row, p.stripe, p.nodes);
                if (p.my_node == kAllNodes || node == p.my_node) {  // :69-72
                    const uint32_t seg_row = seg_row_of(row, p.stripe, p.nodes, p.injective != 0);
                    const uint8_t *seg = node < static_cast<uint32_t>(kMaxNodes) ? p.seg[node] : nullptr;
                    if (seg == nullptr) {
                        record_error(p.st, KVOPS_ERR_SEG_NULL);
                    } else if (seg_row >= p.plsr) {  // bounds check the reference lacks
                        record_error(p.st, KVOPS_ERR_ROW_BASE + (static_cast<uint32_t>(pos) & 0xFFu) + (1u << 16));
                    } else {
                        src = seg + (p.layer_offset_rows + seg_row) * static_cast<uint64_t>(p.row_bytes);
                        dst = p.hot + static_cast<uint64_t>(req) * p.hot_req_stride_bytes +
                              static_cast<uint64_t>(slot) * p.row_bytes;  // :73-76
                        ok = true;
                    }
                }
            }
        }
        const unsigned mask = __ballot_sync(0xFFFFFFFFu, ok);
        if (ok) {
            const int idx = __popc(mask & ((1u << lane) - 1u));
            s_src[warp][idx] = src;
            s_dst[warp][idx] = dst;
        }
        __syncwarp();
        if (mask) warp_copy_rows<V>(s_src[warp], s_dst[warp], __popc(mask), p.row_bytes, lane);
        __syncwarp();
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
__global__ void __launch_bounds__(kRowThreads) export_kernel(const ExportParams p)
{
    __shared__ const uint8_t *s_src[kRowWarps][32];
    __shared__ uint8_t *s_dst[kRowWarps][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t total = p.units_per_layer * p.layer_num;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kRowWarps * 32;
    if (p.seg_null && blockIdx.x == 0 && threadIdx.x == 0) record_error(p.st, KVOPS_ERR_SEG_NULL);
    for (uint64_t base = (static_cast<uint64_t>(blockIdx.x) * kRowWarps + warp) * 32; base < total; base += stride) {
        const uint64_t u = base + lane;
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
        if (ok) {
            const int idx = __popc(mask & ((1u << lane) - 1u));
            s_src[warp][idx] = src;
            s_dst[warp][idx] = dst;
        }
        __syncwarp();
        if (mask) warp_copy_rows<V>(s_src[warp], s_dst[warp], __popc(mask), p.row_bytes, lane);
        __syncwarp();
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

int grid_for(uint64_t work_warps, int sm_count)
{
    const uint64_t want = (work_warps + kRowWarps - 1) / kRowWarps;
    const uint64_t cap = static_cast<uint64_t>(sm_count > 0 ? sm_count : 148) * (2048 / kRowThreads);
    uint64_t g = want < cap ? want : cap;
    return g < 1 ? 1 : static_cast<int>(g);
}

}  // namespace

cudaError_t launch_gather(const GatherParams &p, cudaStream_t s, int sm_count)
{
    uint64_t addr_or = reinterpret_cast<uint64_t>(p.hot) | p.hot_req_stride_bytes;
    for (uint32_t n = 0; n < p.nodes && n < static_cast<uint32_t>(kMaxNodes); ++n)
        addr_or |= reinterpret_cast<uint64_t>(p.seg[n]);
    const uint64_t positions = static_cast<uint64_t>(p.max_num_reqs) * p.top_k;
    const int grid = grid_for((positions + 31) / 32, sm_count);
    switch (vec_bytes(addr_or, p.row_bytes)) {
        case 16: gather_kernel<uint4><<<grid, kRowThreads, 0, s>>>(p); break;
        case 8: gather_kernel<uint2><<<grid, kRowThreads, 0, s>>>(p); break;
        case 4: gather_kernel<uint32_t><<<grid, kRowThreads, 0, s>>>(p); break;
        default: gather_kernel<uint8_t><<<grid, kRowThreads, 0, s>>>(p); break;
    }
    return cudaGetLastError();
}

cudaError_t launch_export(const ExportParams &p, cudaStream_t s, int sm_count)
{
    const uint64_t addr_or = reinterpret_cast<uint64_t>(p.src0) | p.src_layer_stride | reinterpret_cast<uint64_t>(p.seg);
    const uint64_t units = p.units_per_layer * p.layer_num;
    const int grid = grid_for((units + 31) / 32, sm_count);
    switch (vec_bytes(addr_or, p.row_bytes)) {
        case 16: export_kernel<uint4><<<grid, kRowThreads, 0, s>>>(p); break;
        case 8: export_kernel<uint2><<<grid, kRowThreads, 0, s>>>(p); break;
        case 4: export_kernel<uint32_t><<<grid, kRowThreads, 0, s>>>(p); break;
        default: export_kernel<uint8_t><<<grid, kRowThreads, 0, s>>>(p); break;
    }
    return cudaGetLastError();
}

}  // namespace kvb
