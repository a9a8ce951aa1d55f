// rows_common.cuh — the miss-row gather's per-position rule and CTA-wide row copy, shared by
// gather_kernel (rows.cu) and the copy helpers of the cooperative layer-step (sieve.cu).
#pragma once

#include <stdint.h>

#include "kvops_internal.cuh"

namespace kvb {

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

// Copies n rows (src[i] -> dst[i]) of `row_bytes` with threads [0, nthreads) of a group (gt:
// this thread's index in it): the rows form one flat array of V-sized chunks split evenly over
// the threads, kUnroll loads in flight per thread before the matching stores. `magic` =
// ceil(2^32 / chunks_per_row) when exact division by multiply-high is valid for every chunk
// index (host-checked), else 0.
template <typename V, int kUnroll>
__device__ __forceinline__ void group_copy_rows(const uint8_t *const *src, uint8_t *const *dst, int n,
                                                uint32_t row_bytes, uint32_t magic, uint32_t gt, uint32_t nthreads)
{
    const uint32_t cpr = row_bytes / sizeof(V);
    const uint32_t total = static_cast<uint32_t>(n) * cpr;
    for (uint32_t i0 = gt; i0 < total; i0 += nthreads * kUnroll) {
        V v[kUnroll];
        uint32_t rr[kUnroll], cc[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const uint32_t i = i0 + u * nthreads;
            const uint32_t r = magic ? __umulhi(i, magic) : i / cpr;
            rr[u] = r;
            cc[u] = i - r * cpr;
            if (i < total) v[u] = load_stream(reinterpret_cast<const V *>(src[r]) + cc[u]);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            if (i0 + u * nthreads < total) reinterpret_cast<V *>(dst[rr[u]])[cc[u]] = v[u];
        }
    }
}

// The same with the whole CTA.
template <typename V, int kUnroll>
__device__ __forceinline__ void cta_copy_rows(const uint8_t *const *src, uint8_t *const *dst, int n,
                                              uint32_t row_bytes, uint32_t magic)
{
    group_copy_rows<V, kUnroll>(src, dst, n, row_bytes, magic, threadIdx.x, blockDim.x);
}

// The gather rule for flat position `pos` (= batch row * top_k + k) of one layer
// (kvc_gather_rows.cpp:54-76) on its loaded inputs: true with the row's source and hot
// destination when the position is a miss with a valid token, slot and pool row on a selected
// node. Records KVOPS_ERR_SEG_NULL or the row band for a null segment or a row past the segment.
__device__ __forceinline__ bool gather_eval(const GatherParams &p, int64_t pos, int8_t miss, int32_t t, int32_t slot,
                                            int64_t req, int64_t base, const uint8_t **src_out, uint8_t **dst_out)
{
    if (miss == 0) return false;                     // :55-57
    if (t < 0 || slot < 0 || req < 0) return false;  // :62-68
    const uint32_t row = static_cast<uint32_t>(base + t);
    const uint32_t node = node_of(row, p.stripe, p.nodes);
    if (p.my_node != kAllNodes && node != p.my_node) return false;  // :69-72
    const uint32_t seg_row = seg_row_of(row, p.stripe, p.nodes, p.injective != 0);
    const uint8_t *seg = node < static_cast<uint32_t>(kMaxNodes) ? p.seg[node] : nullptr;
    if (seg == nullptr) {
        record_error(p.st, KVOPS_ERR_SEG_NULL);
        return false;
    }
    if (seg_row >= p.plsr) {  // bounds check the reference lacks
        record_error(p.st, KVOPS_ERR_ROW_BASE + (static_cast<uint32_t>(pos) & 0xFFu) + (1u << 16));
        return false;
    }
    *src_out = seg + (p.layer_offset_rows + seg_row) * static_cast<uint64_t>(p.row_bytes);
    *dst_out = p.hot + static_cast<uint64_t>(req) * p.hot_req_stride_bytes +
               static_cast<uint64_t>(slot) * p.row_bytes;  // :73-76
    return true;
}

// The same rule with its own loads. kFresh: the slots / miss flags were written earlier in
// the same kernel by another CTA, so they are read at L2 (ld.global.cg), never from a
// possibly stale L1 line.
template <bool kFresh>
__device__ __forceinline__ bool gather_position(const GatherParams &p, int64_t pos, const uint8_t **src_out,
                                                uint8_t **dst_out)
{
    const int8_t miss = kFresh ? __ldcg(p.is_miss + pos) : p.is_miss[pos];
    if (miss == 0) return false;
    const int64_t bid = pos / p.top_k;
    return gather_eval(p, pos, miss, p.topk[pos], kFresh ? __ldcg(p.slots + pos) : p.slots[pos], p.req_pool[bid],
                       p.host_base[bid], src_out, dst_out);
}

// Appends the accepted rows of the calling threads to a shared list (warp-aggregated).
__device__ __forceinline__ void list_append(bool ok, const uint8_t *src, uint8_t *dst, const uint8_t **s_src,
                                            uint8_t **s_dst, int *s_n)
{
    const int lane = threadIdx.x & 31;
    const unsigned mask = __ballot_sync(0xFFFFFFFFu, ok);
    int at = 0;
    if (lane == 0 && mask) at = atomicAdd(s_n, __popc(mask));
    at = __shfl_sync(0xFFFFFFFFu, at, 0) + __popc(mask & ((1u << lane) - 1u));
    if (ok) {
        s_src[at] = src;
        s_dst[at] = dst;
    }
}

// Positions [base, end) of one tile (end - base <= blockDim.x): each thread evaluates one, the
// accepted rows are appended to the shared list (warp-aggregated), and the CTA copies them.
// kScatter: the opposite direction (kvc_scatter_rows: hot row -> segment row) under the same
// rules, with p.is_miss holding the export flags. s_n must be zero on entry and is zero again
// on return; ends with a barrier.
template <typename V, int kUnroll, bool kFresh, bool kScatter = false>
__device__ __forceinline__ void gather_tile(const GatherParams &p, int64_t base, int64_t end, const uint8_t **s_src,
                                            uint8_t **s_dst, int *s_n, uint32_t magic)
{
    const int64_t pos = base + threadIdx.x;
    const uint8_t *src = nullptr;
    uint8_t *dst = nullptr;
    const bool ok = pos < end && gather_position<kFresh>(p, pos, &src, &dst);
    if (kScatter) {
        const uint8_t *hot_row = dst;
        dst = const_cast<uint8_t *>(src);
        src = hot_row;
    }
    list_append(ok, src, dst, s_src, s_dst, s_n);
    __syncthreads();
    cta_copy_rows<V, kUnroll>(s_src, s_dst, *s_n, p.row_bytes, magic);
    __syncthreads();
    if (threadIdx.x == 0) *s_n = 0;
    __syncthreads();
}

}  // namespace kvb
