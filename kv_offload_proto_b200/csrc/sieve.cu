// sieve.cu — SIEVE miss detector (hisp_sieve_update) and admission hash-table build
// (hisp_sieve_ht_init) for sm_100a.
//
// One CTA per batch row (request). The request's state — token row, visited bitmap,
// uint16 open-addressing table and hand — is staged in shared memory when it fits
// the per-CTA opt-in limit and updated in place in global memory otherwise. The
// SIEVE itself runs in the reference's strict position order
// (hisp_sieve_update.cpp:115-163), so outputs and the persisted state (including
// the hash-table bytes) are identical to the reference kernel's.
#include <stdint.h>

#include "kvops_internal.cuh"

namespace kvb {
namespace {

constexpr int kSieveThreads = 256;
constexpr uint16_t kHtEmpty = 0;

// ---- hash table on a token row (hisp_kernel_common.h:29-112) -------------------
// Every probe loop is bounded by the table size: a well-formed table (load <= 0.5)
// never reaches the bound; a corrupted one cannot hang the GPU. An entry naming a slot
// past the token row (possible only in a corrupted table) reads as token -1, which no
// probed token equals, so it is never dereferenced.

__device__ __forceinline__ int32_t tok_of(const int32_t *tok, uint16_t e, int32_t padded)
{
    const int32_t s = static_cast<int32_t>(e) - 1;
    return s < padded ? tok[s] : -1;
}

__device__ __forceinline__ int32_t ht_find(const uint16_t *ht, const int32_t *tok, int32_t token, uint32_t mask,
                                           int32_t padded)
{
    uint32_t idx = ht_hash(token) & mask;
    for (uint32_t n = 0; n <= mask; ++n) {
        const uint16_t e = ht[idx];
        if (e == kHtEmpty) return -1;
        if (tok_of(tok, e, padded) == token) return static_cast<int32_t>(e) - 1;
        idx = (idx + 1) & mask;
    }
    return -1;
}

__device__ __forceinline__ void ht_insert(uint16_t *ht, const int32_t *tok, int32_t token, int32_t slot,
                                          uint32_t mask, int32_t padded)
{
    uint32_t idx = ht_hash(token) & mask;
    for (uint32_t n = 0; n <= mask; ++n) {
        const uint16_t e = ht[idx];
        if (e == kHtEmpty) {
            ht[idx] = static_cast<uint16_t>(slot + 1);
            return;
        }
        if (tok_of(tok, e, padded) == token) return;  // first slot of a duplicate wins
        idx = (idx + 1) & mask;
    }
}

// Backward-shift deletion, Knuth 6.4 Algorithm R (hisp_kernel_common.h:64-94).
__device__ __forceinline__ void ht_erase(uint16_t *ht, const int32_t *tok, int32_t token, uint32_t mask,
                                         int32_t padded)
{
    uint32_t idx = ht_hash(token) & mask;
    uint32_t n = 0;
    for (; n <= mask; ++n) {
        const uint16_t e = ht[idx];
        if (e == kHtEmpty) return;
        if (tok_of(tok, e, padded) == token) break;
        idx = (idx + 1) & mask;
    }
    if (n > mask) return;
    int32_t j = static_cast<int32_t>(idx), i = j;
    for (n = 0; n <= mask; ++n) {
        i = static_cast<int32_t>((static_cast<uint32_t>(i) + 1) & mask);
        const uint16_t e = ht[i];
        if (e == kHtEmpty) break;
        const int32_t home = static_cast<int32_t>(ht_hash(tok_of(tok, e, padded)) & mask);
        const bool move = (j < i) ? (home <= j || home > i) : (home <= j && home > i);
        if (move) {
            ht[j] = e;
            j = i;
        }
    }
    ht[j] = kHtEmpty;
}

__device__ __forceinline__ bool vis_get(const uint8_t *v, int32_t s) { return (v[s >> 3] >> (s & 7)) & 1; }
__device__ __forceinline__ void vis_set(uint8_t *v, int32_t s) { v[s >> 3] |= static_cast<uint8_t>(1u << (s & 7)); }
__device__ __forceinline__ void vis_clr(uint8_t *v, int32_t s) { v[s >> 3] &= static_cast<uint8_t>(~(1u << (s & 7))); }

// The reference's per-request loop (hisp_sieve_update.cpp:115-163), run by one thread
// on generic pointers (shared or global). Returns the new hand; sets *dirty when the
// token row / table changed.
__device__ int32_t sieve_sequential(const int32_t *tp, int32_t K, int32_t *os, int8_t *om, int32_t *tok,
                                    uint8_t *vis, uint16_t *ht, uint32_t mask, int32_t dbs, int32_t padded,
                                    int32_t seq_len, int32_t prefill, int32_t hand, bool *dirty)
{
    bool d = false;
    for (int32_t k = 0; k < K; ++k) {
        const int32_t t = tp[k];
        if (t < 0 || t >= seq_len) {
            os[k] = -1;
            om[k] = 0;
            continue;
        }
        if (t >= prefill) {  // decode-extension slot, never evicted, never a miss
            os[k] = padded + (t - prefill);
            om[k] = 0;
            continue;
        }
        const int32_t hit = ht_find(ht, tok, t, mask, padded);
        if (hit >= 0) {
            os[k] = hit;
            om[k] = 0;
            vis_set(vis, hit);
            continue;
        }
        int32_t h = hand;
        for (int32_t n = 0; n <= dbs && vis_get(vis, h); ++n) {  // clears bits, so ends within dbs+1
            vis_clr(vis, h);
            if (++h == dbs) h = 0;
        }
        const int32_t old = tok[h];
        if (old >= 0) ht_erase(ht, tok, old, mask, padded);
        ht_insert(ht, tok, t, h, mask, padded);
        d = true;
        os[k] = h;
        om[k] = 1;
        tok[h] = t;
        vis_set(vis, h);
        hand = h + 1;
        if (hand == dbs) hand = 0;
    }
    *dirty = d;
    return hand;
}

// Cooperative copy of `bytes` bytes using the widest access both pointers allow.
__device__ __forceinline__ void coop_copy(void *dst, const void *src, size_t bytes)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
    if (((a | bytes) & 15) == 0) {
        uint4 *d = static_cast<uint4 *>(dst);
        const uint4 *s = static_cast<const uint4 *>(src);
        for (size_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
    } else if (((a | bytes) & 3) == 0) {
        uint32_t *d = static_cast<uint32_t *>(dst);
        const uint32_t *s = static_cast<const uint32_t *>(src);
        for (size_t i = threadIdx.x; i < bytes / 4; i += blockDim.x) d[i] = s[i];
    } else {
        uint8_t *d = static_cast<uint8_t *>(dst);
        const uint8_t *s = static_cast<const uint8_t *>(src);
        for (size_t i = threadIdx.x; i < bytes; i += blockDim.x) d[i] = s[i];
    }
}

__device__ __forceinline__ void fill_dummy(int32_t *os, int8_t *om, int32_t K)
{
    for (int32_t k = threadIdx.x; k < K; k += blockDim.x) {
        os[k] = -1;
        om[k] = 0;
    }
}

__host__ __device__ __forceinline__ size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared-memory layout of one request: tokens | table | visited | topk->slots | is_miss.
struct SmemLayout {
    size_t tok, ht, vis, slots, miss, total;
};

__host__ __device__ __forceinline__ SmemLayout sieve_smem_layout(int32_t padded, int32_t ht_size, int32_t vis_stride,
                                                                 int32_t K)
{
    SmemLayout L;
    L.tok = 0;
    L.ht = align_up(L.tok + 4ull * padded, 16);
    L.vis = align_up(L.ht + 2ull * ht_size, 16);
    L.slots = align_up(L.vis + static_cast<size_t>(vis_stride), 16);
    L.miss = align_up(L.slots + 4ull * K, 16);
    L.total = align_up(L.miss + static_cast<size_t>(K), 16);
    return L;
}

template <bool kStaged>
__global__ void __launch_bounds__(kSieveThreads) sieve_update_kernel(const SieveParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int32_t bid = blockIdx.x;
    const int32_t K = p.top_k;
    int32_t *g_slots = p.out_slots + static_cast<int64_t>(bid) * K;
    int8_t *g_miss = p.is_miss + static_cast<int64_t>(bid) * K;

    int32_t num_real = *p.num_real;
    if (num_real > p.max_num_reqs) num_real = p.max_num_reqs;  // hisp_sieve_update.cpp:31-34
    const int64_t req = bid < num_real ? p.req_pool[bid] : -1;
    if (bid >= num_real || req < 0 || req >= p.pool_size) {  // :72-88
        fill_dummy(g_slots, g_miss, K);
        return;
    }
    const int32_t seq_len = p.seq_lens[bid];
    const int32_t prefill = p.prefill[req];
    const int32_t *g_topk = p.topk + static_cast<int64_t>(bid) * K;
    int32_t *g_tok = p.tokens + req * p.padded;
    uint8_t *g_vis = p.visited + req * p.vis_stride;
    uint16_t *g_ht = p.ht + req * p.ht_size;
    int32_t *g_hand = p.hand + req * kHandStride;
    const uint32_t mask = static_cast<uint32_t>(p.ht_size) - 1u;

    if constexpr (kStaged) {
        const SmemLayout L = sieve_smem_layout(p.padded, p.ht_size, p.vis_stride, K);
        int32_t *s_tok = reinterpret_cast<int32_t *>(smem + L.tok);
        uint16_t *s_ht = reinterpret_cast<uint16_t *>(smem + L.ht);
        uint8_t *s_vis = reinterpret_cast<uint8_t *>(smem + L.vis);
        int32_t *s_slots = reinterpret_cast<int32_t *>(smem + L.slots);
        int8_t *s_miss = reinterpret_cast<int8_t *>(smem + L.miss);
        __shared__ int32_t s_hand;
        __shared__ bool s_dirty;
        coop_copy(s_tok, g_tok, 4ull * p.padded);
        coop_copy(s_ht, g_ht, 2ull * p.ht_size);
        coop_copy(s_vis, g_vis, p.vis_stride);
        coop_copy(s_slots, g_topk, 4ull * K);
        __syncthreads();
        if (threadIdx.x == 0) {
            int32_t hand = *g_hand;
            if (hand < 0 || hand >= p.dbs) hand = 0;  // :108-111
            bool dirty = false;
            // Positions are read from s_slots[k] before s_slots[k] is overwritten.
            s_hand = sieve_sequential(s_slots, K, s_slots, s_miss, s_tok, s_vis, s_ht, mask, p.dbs, p.padded,
                                      seq_len, prefill, hand, &dirty);
            s_dirty = dirty;
        }
        __syncthreads();
        coop_copy(g_slots, s_slots, 4ull * K);
        coop_copy(g_miss, s_miss, static_cast<size_t>(K));
        coop_copy(g_vis, s_vis, p.vis_stride);
        if (s_dirty) {  // tokens/table written back only when changed (:165-173)
            coop_copy(g_tok, s_tok, 4ull * p.padded);
            coop_copy(g_ht, s_ht, 2ull * p.ht_size);
        }
        if (threadIdx.x == 0) *g_hand = s_hand;
    } else {
        if (threadIdx.x == 0) {
            int32_t hand = *g_hand;
            if (hand < 0 || hand >= p.dbs) hand = 0;
            bool dirty = false;
            *g_hand = sieve_sequential(g_topk, K, g_slots, g_miss, g_tok, g_vis, g_ht, mask, p.dbs, p.padded,
                                       seq_len, prefill, hand, &dirty);
        }
    }
}

// Admission build (hisp_sieve_ht_init.cpp:25-58): clear, then insert slots in order.
template <bool kStaged>
__global__ void __launch_bounds__(kSieveThreads) sieve_ht_init_kernel(const HtInitParams p)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int32_t b = blockIdx.x;
    if (b >= p.pairs) return;
    const int64_t layer = b / p.num_reqs;
    const int64_t req = static_cast<int64_t>(p.req_start) + b % p.num_reqs;
    if (req < 0 || req >= p.pool_size) return;
    const int32_t *g_tok = p.tokens + (layer * p.pool_size + req) * p.padded;
    uint16_t *g_ht = p.ht + (layer * p.pool_size + req) * p.ht_size;
    const uint32_t mask = static_cast<uint32_t>(p.ht_size) - 1u;
    if constexpr (kStaged) {
        int32_t *s_tok = reinterpret_cast<int32_t *>(smem);
        uint16_t *s_ht = reinterpret_cast<uint16_t *>(smem + align_up(4ull * p.padded, 16));
        coop_copy(s_tok, g_tok, 4ull * p.padded);
        for (int32_t i = threadIdx.x; i < p.ht_size; i += blockDim.x) s_ht[i] = kHtEmpty;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int32_t s = 0; s < p.dbs; ++s) {
                const int32_t t = s_tok[s];
                if (t >= 0) ht_insert(s_ht, s_tok, t, s, mask, p.padded);
            }
        }
        __syncthreads();
        coop_copy(g_ht, s_ht, 2ull * p.ht_size);
    } else {
        for (int32_t i = threadIdx.x; i < p.ht_size; i += blockDim.x) g_ht[i] = kHtEmpty;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int32_t s = 0; s < p.dbs; ++s) {
                const int32_t t = g_tok[s];
                if (t >= 0) ht_insert(g_ht, g_tok, t, s, mask, p.padded);
            }
        }
    }
}

int max_optin_smem()
{
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

}  // namespace

cudaError_t launch_sieve_update(const SieveParams &p, cudaStream_t s, int /*sm_count*/)
{
    if (p.max_num_reqs <= 0) return cudaSuccess;
    const SmemLayout L = sieve_smem_layout(p.padded, p.ht_size, p.vis_stride, p.top_k);
    const int limit = max_optin_smem();
    if (L.total <= static_cast<size_t>(limit)) {
        cudaError_t e = cudaFuncSetAttribute(sieve_update_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(L.total));
        if (e != cudaSuccess) return e;
        sieve_update_kernel<true><<<p.max_num_reqs, kSieveThreads, L.total, s>>>(p);
    } else {
        sieve_update_kernel<false><<<p.max_num_reqs, 32, 0, s>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_sieve_ht_init(const HtInitParams &p, cudaStream_t s)
{
    if (p.pairs <= 0) return cudaSuccess;
    const size_t bytes = align_up(4ull * p.padded, 16) + 2ull * p.ht_size;
    const int limit = max_optin_smem();
    if (bytes <= static_cast<size_t>(limit)) {
        cudaError_t e = cudaFuncSetAttribute(sieve_ht_init_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(bytes));
        if (e != cudaSuccess) return e;
        sieve_ht_init_kernel<true><<<p.pairs, kSieveThreads, bytes, s>>>(p);
    } else {
        sieve_ht_init_kernel<false><<<p.pairs, kSieveThreads, 0, s>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace kvb
