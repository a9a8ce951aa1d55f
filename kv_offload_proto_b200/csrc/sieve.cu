// sieve.cu — SIEVE miss detector (hisp_sieve_update) and admission hash-table build
// (hisp_sieve_ht_init) for sm_100a.
//
// One CTA per batch row (request). The request's state — token row, visited bitmap,
// uint16 open-addressing table and hand — is staged in shared memory. The default kernel
// (sieve_fast_kernel) computes the step in parallel phases that reproduce the reference's
// strict position order (hisp_sieve_update.cpp:115-163) exactly; steps outside its
// assumptions, and states too large for shared memory, run the position-ordered loop
// itself (sieve_sequential), staged or in place in global memory. Either way the outputs
// and the persisted state (including the hash-table bytes) equal the reference kernel's.
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "kvops_internal.cuh"
#include "rows_common.cuh"

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
__device__ __forceinline__ void coop_copy_n(void *dst, const void *src, size_t bytes, unsigned tid, unsigned nt)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
    if (((a | bytes) & 15) == 0) {
        uint4 *d = static_cast<uint4 *>(dst);
        const uint4 *s = static_cast<const uint4 *>(src);
        for (size_t i = tid; i < bytes / 16; i += nt) d[i] = s[i];
    } else if (((a | bytes) & 3) == 0) {
        uint32_t *d = static_cast<uint32_t *>(dst);
        const uint32_t *s = static_cast<const uint32_t *>(src);
        for (size_t i = tid; i < bytes / 4; i += nt) d[i] = s[i];
    } else {
        uint8_t *d = static_cast<uint8_t *>(dst);
        const uint8_t *s = static_cast<const uint8_t *>(src);
        for (size_t i = tid; i < bytes; i += nt) d[i] = s[i];
    }
}

__device__ __forceinline__ void coop_copy(void *dst, const void *src, size_t bytes)
{
    coop_copy_n(dst, src, bytes, threadIdx.x, blockDim.x);
}

// Asynchronous global -> shared staging: 16-byte cp.async when both sides allow it (all
// copies of a phase stay in flight together; cp_async_wait_all() ends the phase), plain
// cooperative copies otherwise.
__device__ __forceinline__ void stage_async(void *dst_smem, const void *src, size_t bytes)
{
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst_smem) | reinterpret_cast<uintptr_t>(src);
    if (((a | bytes) & 15) != 0) {
        coop_copy(dst_smem, src, bytes);
        return;
    }
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
    const char *g = static_cast<const char *>(src);
    for (size_t i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + static_cast<uint32_t>(i * 16)),
                     "l"(g + i * 16)
                     : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
    // Lets a programmatic dependent (the gather of this layer-step) launch its CTAs now; they
    // wait for this grid's completion before reading its outputs.
    asm volatile("griddepcontrol.launch_dependents;");
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

// ==== Parallel exact path ===========================================================
//
// The same step as sieve_sequential, computed in phases instead of position order:
//  1. every position probes the step-initial table in parallel; for each hot slot the first
//     and last position that looks up its resident token are recorded (Tf, Tl); tokens that
//     are not resident are de-duplicated, their first occurrences are the initial misses;
//  2. one warp replays the hand sweep: misses are taken in position order and each one evicts
//     the next slot (from the hand) whose visited bit is clear and whose token is not looked
//     up before that miss (bit clear and Tf > miss); evicting a slot whose token is looked up
//     later turns that later lookup into a miss (Tf is queued). 32 slots are tested per ballot;
//  3. outputs, final visited bits and the new hand follow in parallel;
//  4. the table is updated in two parallel passes: the evicted tokens are deleted (each
//     affected probe run is re-packed from its first deleted cell, which is what
//     backward-shift deletion produces), then the new tokens are inserted with priority
//     = miss position (cells are claimed by 16-bit CAS; an earlier miss displaces a later
//     one). Linear probing with backward-shift deletion leaves the table exactly as if the
//     surviving keys had been inserted in order, so this equals the reference's
//     erase/insert sequence byte for byte.
// Phase 2 assumes the sweep passes no slot twice in one step, and phase 4 assumes the table
// maps each resident token to exactly its slot (true of any state these kernels or the
// reference build). A step that breaks either assumption is detected before anything is
// written back and is recomputed by the sequential path from the untouched global state.

constexpr int kFastThreads = 512;
constexpr int kHelpBatch = 256;  // numbers per walk-list batch (cooperative step)

constexpr uint16_t kNone16 = 0xFFFFu;
constexpr uint16_t kDelMark = 0xFFFFu;   // table cell: deleted entry (entries are <= 65520)
constexpr uint16_t kLeadMark = 0xFFFEu;  // table cell: first deleted entry of its probe run
constexpr uint8_t kClsNone = 0, kClsRes = 1, kClsNew = 2, kClsPending = 3, kClsPlaced = 4;

struct FastLayout {
    size_t ht, tok, topk, os, om, cls, aux, tf, evt, vini, vfin, dkey, dfirst, posl, missb, wofs, nslot, hpos, total;
    int32_t dcap;
};

__host__ __device__ __forceinline__ size_t take(size_t *o, size_t bytes)
{
    const size_t r = *o;
    *o = align_up(*o + bytes, 16);
    return r;
}

__host__ __device__ __forceinline__ FastLayout fast_layout(int32_t padded, int32_t ht_size, int32_t vis_stride,
                                                           int32_t K, int32_t dbs)
{
    FastLayout L;
    L.dcap = 1;
    while (L.dcap < 2 * K) L.dcap <<= 1;
    size_t o = 0;
    L.ht = take(&o, 2ull * ht_size);
    L.tok = take(&o, 4ull * padded);
    L.topk = take(&o, 4ull * K);
    L.os = take(&o, 4ull * K);
    L.om = take(&o, static_cast<size_t>(K));
    L.cls = take(&o, static_cast<size_t>(K));
    L.aux = take(&o, 2ull * K);
    L.tf = take(&o, 4ull * dbs);
    L.evt = take(&o, 2ull * padded);
    L.vini = take(&o, static_cast<size_t>(vis_stride));
    L.vfin = take(&o, static_cast<size_t>(vis_stride));
    // The dedup table (phase 1) and the candidate list + miss positions (phase 2) share one region.
    const size_t cl = align_up(4ull * dbs + 16, 16);  // +16: whole 16-B chunks
    const size_t dd = 8ull * L.dcap > cl + 2ull * K ? 8ull * L.dcap : cl + 2ull * K;
    L.dkey = take(&o, dd);
    L.dfirst = L.dkey + 4ull * L.dcap;
    L.posl = L.dkey + cl;
    L.missb = take(&o, 4ull * ((K + 31) / 32));
    L.wofs = take(&o, 4ull * ((dbs + 31) / 32 + 1));
    L.nslot = take(&o, 2ull * K);         // miss number -> slot (cooperative step)
    L.hpos = take(&o, 2ull * kHelpBatch);  // walk-list batch: positions
    L.total = o;
    return L;
}


// Phase 2 replays the hand sweep. Only slots whose visited bit is clear at the start of the
// step can be evicted (a set bit is cleared and skipped; with no wrap the sweep never comes
// back to it), so the walk runs over the compacted list of those candidate slots:
//  2a. all threads build the list in slot order, entries (Tf << 16) | slot;
//  2b. one warp walks it from the hand: the current miss evicts the next candidate whose
//      token is not looked up before it (Tf > miss); an evicted slot whose token is looked up
//      later queues that lookup as a miss. Each visited entry is overwritten with its
//      arrival time (the miss in progress when the sweep reaches it);
//  2c. all threads set the final visited bits of the passed slots: evicted ones are set, the
//      others were cleared on arrival and are set again iff their token is looked up after
//      it. A passed slot's arrival time is that of the next candidate at or after it.

// 2a: candidate list and per-word offsets. The offsets depend only on the step-initial bits
// (candidate_offsets: per word of slots, how many candidates precede it; *n_out the count, set
// by warp 0; no trailing barrier), the entries also on Tf (put_candidate, one slot).
__device__ __forceinline__ uint32_t candidate_bits(const uint32_t *vini, int32_t w, int32_t dbs)
{
    const int32_t rem = dbs - (w << 5);
    const uint32_t valid = rem >= 32 ? 0xFFFFFFFFu : ((1u << rem) - 1u);
    return ~vini[w] & valid;
}

__device__ void candidate_offsets(const uint32_t *vini, uint32_t *wofs, int32_t dbs, int32_t *n_out,
                                  int32_t *warp_sums)
{
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5;
    const int32_t nwords = (dbs + 31) >> 5;
    const int32_t per = (nwords + nt - 1) / nt;
    const int32_t w0 = min(tid * per, nwords), w1 = min(w0 + per, nwords);
    int32_t mine = 0;
    for (int32_t w = w0; w < w1; ++w) mine += __popc(candidate_bits(vini, w, dbs));
    // block-wide exclusive scan of `mine`
    int32_t incl = mine;
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = nt >> 5;
        int32_t v = lane < nw ? warp_sums[lane] : 0, inc = v;
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t u = __shfl_up_sync(0xFFFFFFFFu, inc, d);
            if (lane >= d) inc += u;
        }
        if (lane < nw) warp_sums[lane] = inc - v;  // exclusive warp offsets
        if (lane == nw - 1) *n_out = inc;
    }
    __syncthreads();
    int32_t at = warp_sums[wid] + incl - mine;
    for (int32_t w = w0; w < w1; ++w) {
        wofs[w] = static_cast<uint32_t>(at);
        at += __popc(candidate_bits(vini, w, dbs));
    }
}

// Slot c's entry (Tf << 16) | c at its word's offset + the candidates before it, if c is one.
__device__ __forceinline__ void put_candidate(const uint32_t *vini, const uint32_t *tf, uint32_t *cand,
                                              const uint32_t *wofs, int32_t dbs, int32_t c)
{
    const uint32_t b = candidate_bits(vini, c >> 5, dbs), below = b & ((1u << (c & 31)) - 1u);
    if ((b >> (c & 31)) & 1u) cand[wofs[c >> 5] + __popc(below)] = ((tf[c] & 0xFFFFu) << 16) | static_cast<uint32_t>(c);
}

__device__ void build_candidates(const uint32_t *vini, const uint32_t *tf, uint32_t *cand, uint32_t *wofs,
                                 int32_t dbs, int32_t *n_out, int32_t *warp_sums)
{
    candidate_offsets(vini, wofs, dbs, n_out, warp_sums);
    __syncthreads();
    for (int32_t c = threadIdx.x; c < dbs; c += blockDim.x) put_candidate(vini, tf, cand, wofs, dbs, c);
}

// 2b: the walk (one warp), 32 candidates per batch, one per lane, in sweep order from the
// hand. Misses are consumed in position order, so the m-th consumed miss is the m-th set bit
// of the final miss queue: the walk records miss numbers, and a parallel pass afterwards turns
// them into positions. One round resolves many candidates at once:
//  - the window: the queue words w0 .. w0+31, of which the first s0 misses are consumed
//    (created misses always land after the consumed ones, so s0 stays exact);
//  - each lane ranks its token's first lookup Tf among the window's unconsumed misses: t_j =
//    those before Tf (a lookup before them ranks 0; none, or one past the window, ranks all);
//  - the sweep with this queue is the recurrence k <- k + (k < t_j) over the lanes: the lane
//    is reached by unconsumed miss number k and evicted iff k < t_j; only lanes with
//    0 < t_j < 32 need k first;
//  - an evicted lane whose token is looked up later creates the miss Tf, which this queue
//    lacks. Every lane reached before the earliest such Tf (cmin) is exact, since the queue
//    is exact below cmin; those lanes, always at least the first one, are committed with
//    arrival number G + k (G: misses consumed before the round), evicted slots get evt = that
//    number, and the created misses join the queue.
// Each round commits a lane, or moves the window: past 32 fully consumed words, or up to the
// word of the next unconsumed miss (at most once per commit), which bounds the rounds.
// Returns false when the sweep would pass a slot twice (misses remain after every candidate),
// or if the bound were ever exceeded. *nvis_out: candidates visited (a prefix of sweep order).
// nslot (optional): nslot[m] = the slot evicted for miss number m; prog (optional): prog[0] =
// misses consumed so far, published after each round (numbers below it are final).
__device__ bool walk_candidates(uint32_t *cand, int32_t n, int32_t n0, uint16_t *evt, uint32_t *missb, int32_t K,
                                int32_t *last_out, int32_t *nvis_out, uint16_t *nslot, int32_t *prog)
{
    const unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const int32_t qwords = (K + 31) >> 5;
    int32_t w0 = 0, s0 = 0, G = 0, last = -1, nvis = 0;
    bool done = false;
    int32_t rounds = 2 * n + (qwords >> 5) + 4;
    // sweep position s (0 <= s < n) is candidate index (n0 + s) mod n
    auto index_of = [&](int32_t sp) { return n0 + sp >= n ? n0 + sp - n : n0 + sp; };
    uint32_t xnext = lane < n ? cand[index_of(lane)] : 0u;
    for (int32_t sb = 0; sb < n && !done; sb += 32) {
        const uint32_t xv = xnext;
        const uint32_t f = xv >> 16;
        const int32_t cnt = min(32, n - sb);
        const int32_t my = index_of(sb + lane < n ? sb + lane : 0);
        if (sb + 32 + lane < n) xnext = cand[index_of(sb + 32 + lane)];  // next batch, loaded ahead
        int cur = 0;
        while (cur < cnt) {
            if (--rounds < 0) return false;
            const uint32_t W = w0 + lane < qwords ? missb[w0 + lane] : 0u;
            const uint32_t pop = static_cast<uint32_t>(__popc(W));
            // the words' miss counts, bit-sliced over six ballots (counts are 0..32)
            uint32_t bs[6];
#pragma unroll
            for (int b = 0; b < 6; ++b) bs[b] = __ballot_sync(kAll, (pop >> b) & 1u);
            auto before = [&](uint32_t lanes) {  // misses in the words of `lanes`
                int32_t c = 0;
#pragma unroll
                for (int b = 0; b < 6; ++b) c += __popc(bs[b] & lanes) << b;
                return c;
            };
            const int32_t e_me = before((1u << lane) - 1u);  // misses in the window's words before mine
            const int32_t avail = before(kAll) - s0;
            if (avail <= 0) {  // every miss in these 32 words is consumed
                if (w0 + 32 >= qwords) {
                    done = true;
                    break;
                }
                w0 += 32;
                s0 = 0;
                continue;
            }
            if (avail < 32 && w0 + 32 < qwords) {  // move up to the word of the next unconsumed miss
                const int ls = __ffs(__ballot_sync(kAll, e_me + static_cast<int32_t>(pop) > s0)) - 1;
                if (ls > 0) {
                    s0 -= __shfl_sync(kAll, e_me, ls);
                    w0 += ls;
                    continue;
                }
            }
            const int32_t mw = min(32, avail);
            const bool live = lane >= cur && lane < cnt;
            const int32_t wf = f == kNone16 ? 32 : static_cast<int32_t>(f >> 5) - w0;
            const int src = wf < 0 ? 0 : (wf > 31 ? 31 : wf);
            const uint32_t ws = __shfl_sync(kAll, W, src);
            const int32_t es = __shfl_sync(kAll, e_me, src);
            int32_t tj = 0;
            if (live) {
                if (wf >= 32) {
                    tj = mw;
                } else if (wf >= 0) {
                    const int32_t r = es + __popc(ws & ((1u << (f & 31)) - 1u)) - s0;
                    tj = r < 0 ? 0 : (r > mw ? mw : r);
                }
            }
            // t_j = 0 always passes and t_j = mw always evicts once reached; only a lane whose
            // lookup falls inside the window needs its k_j first, taken in lane order.
            uint32_t evm = __ballot_sync(kAll, live && tj >= mw);
            uint32_t am = __ballot_sync(kAll, live && tj > 0 && tj < mw);
            while (am) {
                const int a = __ffs(am) - 1;
                am &= am - 1u;
                const int32_t ta = __shfl_sync(kAll, tj, a);
                if (__popc(evm & ((1u << a) - 1u)) < ta) evm |= 1u << a;
            }
            const int32_t myk = __popc(evm & ((1u << lane) - 1u));
            const bool reached = live && myk < mw;
            const bool ev = reached && ((evm >> lane) & 1u);
            // the earliest miss this round creates, ranked among the window's unconsumed misses
            const uint32_t cmin = __reduce_min_sync(kAll, ev && f != kNone16 ? f : 0xFFFFFFFFu);
            int32_t rc = 0x7FFFFFFF;
            if (cmin != 0xFFFFFFFFu) {
                const int32_t wc = static_cast<int32_t>(cmin >> 5) - w0;  // >= 0: cmin follows a reached miss
                const uint32_t wcs = __shfl_sync(kAll, W, wc < 32 ? wc : 0);
                const int32_t ecs = __shfl_sync(kAll, e_me, wc < 32 ? wc : 0);
                if (wc < 32) rc = ecs + __popc(wcs & ((1u << (cmin & 31)) - 1u)) - s0;
            }
            const bool com = reached && myk < rc;
            const uint32_t cm = __ballot_sync(kAll, com);
            const uint32_t em = __ballot_sync(kAll, com && ev);
            if (com) {
                const uint32_t slot = xv & 0xFFFFu;
                const uint32_t num = static_cast<uint32_t>(G + myk);
                cand[my] = (num << 16) | slot;
                if (ev) {
                    evt[slot] = static_cast<uint16_t>(num);
                    if (nslot != nullptr) nslot[num] = static_cast<uint16_t>(slot);
                    if (f != kNone16) atomicOr(&missb[f >> 5], 1u << (f & 31));  // created miss
                }
            }
            if (em) last = static_cast<int32_t>(__shfl_sync(kAll, xv, 31 - __clz(em)) & 0xFFFFu);
            const int32_t ec = __popc(em);
            G += ec;
            s0 += ec;
            if (cm == 0u) return false;  // cannot happen: the first lane is always committed
            cur = 32 - __clz(cm);
            nvis = sb + cur;
            __syncwarp();  // created misses visible before the next round reads the queue
            if (prog != nullptr && ec > 0 && lane == 0) {
                __threadfence_block();
                *reinterpret_cast<volatile int32_t *>(prog) = G;
            }
        }
    }
    if (!done) {  // every candidate was visited: unconsumed misses mean the sweep would wrap
        int32_t rem = 0;
        for (int32_t w = w0 + lane; w < qwords; w += 32) rem += __popc(missb[w]);
        for (int d = 16; d >= 1; d >>= 1) rem += __shfl_xor_sync(kAll, rem, d);
        if (rem - s0 > 0) return false;
    }
    *last_out = last;
    *nvis_out = nvis;
    return true;
}

// 2b': miss numbers -> positions. posl[m] = position of the m-th set bit of the miss queue
// (all threads; known >= 0: posl is complete already and holds `known` numbers), then every
// evicted slot's number and every visited candidate's arrival number is replaced by its
// position, and the misses' outputs are written. *nmiss: the number of misses.
// 2b'': with posl final: every evicted slot's number and every visited candidate's arrival number
// replaced by its position, and the misses' outputs written.
__device__ void resolve_outputs(const uint16_t *posl, uint16_t *evt, int32_t *os, int8_t *om, uint32_t *cand,
                                int32_t n, int32_t n0, int32_t nvis, int32_t dbs)
{
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int32_t c = tid; c < dbs; c += nt) {
        const uint16_t m = evt[c];
        if (m == kNone16) continue;
        const uint16_t pos = posl[m];
        evt[c] = pos;
        os[pos] = c;
        om[pos] = 1;
    }
    for (int32_t sp = tid; sp < nvis; sp += nt) {
        const int32_t i = n0 + sp >= n ? n0 + sp - n : n0 + sp;
        const uint32_t x = cand[i];
        cand[i] = (static_cast<uint32_t>(posl[x >> 16]) << 16) | (x & 0xFFFFu);
    }
}

__device__ void resolve_miss_numbers(const uint32_t *missb, int32_t K, uint16_t *posl, uint16_t *evt, int32_t *os,
                                     int8_t *om, uint32_t *cand, int32_t n, int32_t n0, int32_t nvis, int32_t dbs,
                                     int32_t *warp_sums, int32_t *nmiss, int32_t known)
{
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5;
    if (known >= 0) {  // posl already holds the position of every number (the listing warp's)
        if (tid == 0) *nmiss = known;
        resolve_outputs(posl, evt, os, om, cand, n, n0, nvis, dbs);
        return;
    }
    const int32_t nwords = (K + 31) >> 5;
    const int32_t per = (nwords + nt - 1) / nt;
    const int32_t w0 = min(tid * per, nwords), w1 = min(w0 + per, nwords);
    int32_t mine = 0;
    for (int32_t w = w0; w < w1; ++w) mine += __popc(missb[w]);
    int32_t incl = mine;
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = nt >> 5;
        int32_t v = lane < nw ? warp_sums[lane] : 0, inc = v;
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t u = __shfl_up_sync(0xFFFFFFFFu, inc, d);
            if (lane >= d) inc += u;
        }
        if (lane < nw) warp_sums[lane] = inc - v;
        if (lane == nw - 1) *nmiss = inc;
    }
    __syncthreads();
    int32_t at = warp_sums[wid] + incl - mine;
    for (int32_t w = w0; w < w1; ++w) {
        for (uint32_t b = missb[w]; b; b &= b - 1u) posl[at++] = static_cast<uint16_t>((w << 5) + __ffs(b) - 1);
    }
    __syncthreads();
    resolve_outputs(posl, evt, os, om, cand, n, n0, nvis, dbs);
}

// 2c: final visited bits of the slots passed: one slot per lane, one 32-slot word per warp
// (the word's bits are gathered by ballot).
__device__ void passed_bits(const uint32_t *vini, uint32_t *vfin, const uint32_t *tf, const uint16_t *evt,
                            const uint32_t *cand, const uint32_t *wofs, int32_t n, int32_t dbs, int32_t hand0,
                            int32_t last)
{
    const unsigned kAll = 0xFFFFFFFFu;
    const int32_t nwords = (dbs + 31) >> 5;
    const int32_t pend = (last - hand0 + dbs) % dbs + 1;  // slots passed, in sweep order from the hand
    const int lane = threadIdx.x & 31;
    const int32_t nwarps = static_cast<int32_t>(blockDim.x >> 5);
    for (int32_t w = static_cast<int32_t>(threadIdx.x >> 5); w < nwords; w += nwarps) {
        const int32_t c = (w << 5) + lane;
        const uint32_t ini = vini[w];
        bool in = false, bit = false;
        if (c < dbs) {
            int32_t pos = c - hand0;
            if (pos < 0) pos += dbs;
            if (pos < pend) {
                in = true;
                if (evt[c] != kNone16) {
                    bit = true;
                } else {
                    // candidates before c in slot order; the one at that index is the next at or after c
                    const int32_t q = static_cast<int32_t>(wofs[w]) + __popc(~ini & ((1u << lane) - 1u));
                    const uint32_t arr = cand[q == n ? 0 : q] >> 16;
                    const uint32_t x = tf[c];
                    bit = (x & 0xFFFFu) != kNone16 && (x >> 16) > arr;
                }
            }
        }
        const uint32_t m = __ballot_sync(kAll, in), bits = __ballot_sync(kAll, bit);
        if (lane == 0 && m) vfin[w] = (vfin[w] & ~m) | (bits & m);
    }
}

// ==== Fused step: the miss rows are copied while the table passes run ====================
//
// sieve_fast_kernel<true> adds a 17th warp. All 17 warps run phases 0-3; the outputs
// (slots, miss flags) are final there. The extra warp then copies the request's miss rows
// (kvc_gather_rows.cpp:54-76, the same position rules and error codes as gather_kernel) while
// the other 16 run phases 4-6 on named barrier 1. Rows move through a shared-memory ring by
// bulk copies: global -> shared completing on an mbarrier, then shared -> global into the
// hot row. Sources are own or peer HBM (the host checks the 16-byte alignment every bulk
// copy needs and routes other cases to the two-kernel path). Every wait is bounded.

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Waits for the phase with the given parity to complete; false after ~2^22 polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity)
{
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void *src, uint32_t bytes, uint32_t bar)
{
    asm volatile(
        "{\n\t.reg .u64 g;\n\t"
        "cvta.to.global.u64 g, %1;\n\t"
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [g], %2, [%3];\n\t}" ::"r"(dst_smem),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_store(void *dst, uint32_t src_smem, uint32_t bytes)
{
    asm volatile(
        "{\n\t.reg .u64 g;\n\t"
        "cvta.to.global.u64 g, %0;\n\t"
        "cp.async.bulk.global.shared::cta.bulk_group [g], [%1], %2;\n\t"
        "cp.async.bulk.commit_group;\n\t}" ::"l"(dst),
        "r"(src_smem), "r"(bytes)
        : "memory");
}


__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void bulk_wait_all()
{
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// The copy warp. The miss positions are listed in order, then moved in groups of 32 rows
// (one per lane) through `nset` sets of 32 ring slots: group g loads into set g % nset while
// group g - (nset - 1) is stored, so up to nset groups are in flight. One mbarrier per set,
// armed by lane 0 with the group's byte count, keeps every wait warp-uniform.
constexpr int kMaxSets = 4;

__device__ void copy_miss_rows(const GatherParams &g, int32_t bid, int64_t req, const int32_t *topk,
                               const int32_t *os, const int8_t *om, int32_t K, unsigned char *ring, uint64_t *bars,
                               uint16_t *list, int32_t nset)
{
    const unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const uint32_t rb = g.row_bytes;
    int32_t n = 0;  // miss positions, in position order (kvc_gather_rows.cpp:55-57)
    for (int32_t k0 = 0; k0 < K; k0 += 32) {
        const int32_t k = k0 + lane;
        const bool m = k < K && om[k] != 0;
        const uint32_t bal = __ballot_sync(kAll, m);
        if (m) list[n + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(k);
        n += __popc(bal);
    }
    const uint32_t ring0 = smem_u32(ring), bar0 = smem_u32(bars);
    if (lane < nset) mbar_init(bar0 + 8u * lane, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    const int64_t base = g.host_base[bid];
    const uint64_t pos0 = static_cast<uint64_t>(bid) * g.top_k;
    const int32_t ngroups = (n + 31) / 32;
    uint8_t *dsts[kMaxSets] = {nullptr, nullptr, nullptr, nullptr};  // this lane's row per set
    bool alive = true;
    for (int32_t gi = 0; gi < ngroups + nset - 1 && alive; ++gi) {
        if (gi < ngroups) {  // load group gi into set gi % nset
            const int32_t set = gi % nset;
            bulk_wait_read_all();  // the stores of the set's previous group have read it
            const int32_t i = gi * 32 + lane;
            const uint8_t *src = nullptr;
            uint8_t *dst = nullptr;
            if (i < n) {
                const int32_t k = list[i];
                const int32_t t = topk[k];
                const int32_t slot = os[k];
                if (t >= 0 && slot >= 0 && req >= 0) {  // :62-68
                    const uint32_t row = static_cast<uint32_t>(base + t);
                    const uint32_t node = node_of(row, g.stripe, g.nodes);
                    const uint32_t seg_row = seg_row_of(row, g.stripe, g.nodes, g.injective != 0);
                    const uint8_t *seg = node < static_cast<uint32_t>(kMaxNodes) ? g.seg[node] : nullptr;
                    if (seg == nullptr) {
                        record_error(g.st, KVOPS_ERR_SEG_NULL);
                    } else if (seg_row >= g.plsr) {  // bounds check the reference lacks
                        record_error(g.st, KVOPS_ERR_ROW_BASE + (static_cast<uint32_t>(pos0 + k) & 0xFFu) + (1u << 16));
                    } else {
                        src = seg + (g.layer_offset_rows + seg_row) * static_cast<uint64_t>(rb);
                        dst = g.hot + static_cast<uint64_t>(req) * g.hot_req_stride_bytes +
                              static_cast<uint64_t>(slot) * rb;  // :73-76
                    }
                }
            }
            const uint32_t bal = __ballot_sync(kAll, dst != nullptr);
            if (lane == 0) mbar_expect_tx(bar0 + 8u * set, static_cast<uint32_t>(__popc(bal)) * rb);
            __syncwarp();
            if (dst != nullptr) bulk_load(ring0 + static_cast<uint32_t>(set * 32 + lane) * rb, src, rb, bar0 + 8u * set);
#pragma unroll
            for (int q = 0; q < kMaxSets; ++q)
                if (q == set) dsts[q] = dst;
        }
        const int32_t r = gi - (nset - 1);  // store group r
        if (r >= 0) {
            const int32_t set = r % nset;
            if (!mbar_wait(bar0 + 8u * set, static_cast<uint32_t>(r / nset) & 1u)) {
                if (lane == 0) record_error(g.st, KVOPS_ERR_COPY_TIMEOUT);
                alive = false;
                break;
            }
            uint8_t *dst = nullptr;
#pragma unroll
            for (int q = 0; q < kMaxSets; ++q)
                if (q == set) dst = dsts[q];
            if (dst != nullptr) bulk_store(dst, ring0 + static_cast<uint32_t>(set * 32 + lane) * rb, rb);
        }
    }
    bulk_wait_all();
    __syncwarp();
}

// Compute-role barrier: the whole CTA, or with the copy warp split off, the 16 compute warps.
template <bool kFused>
__device__ __forceinline__ void compute_sync()
{
    if (kFused)
        asm volatile("bar.sync 1, %0;" ::"r"(kFastThreads) : "memory");
    else
        __syncthreads();
}

// compute_sync that also returns whether any compute thread passed true.
template <bool kFused>
__device__ __forceinline__ bool compute_sync_or(bool v)
{
    if (!kFused) return __syncthreads_or(v) != 0;
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(kFastThreads)
        : "memory");
    return r != 0;
}

// Warp-aggregated append: the index of this lane's item in a shared list counted by *n (all
// 32 lanes call it; lanes with want == false get an unused index).
__device__ __forceinline__ int warp_append(int32_t *n, bool want)
{
    const unsigned bal = __ballot_sync(0xFFFFFFFFu, want);
    const int lane = threadIdx.x & 31;
    int at = 0;
    if (lane == 0 && bal) at = atomicAdd(n, __popc(bal));
    return __shfl_sync(0xFFFFFFFFu, at, 0) + __popc(bal & ((1u << lane) - 1u));
}

// ---- cooperative layer-step: walk-list progress words ----

// Layout of a launch's block of kCoopBlockWords words. While a request's walk runs, its walk
// list (StepExtra::wl) receives one entry per miss number the walk has made final, and when the
// request's outputs are final the rest; word kProgBase + 2 r publishes
// (epoch << 32) | (entries << 1) | final, and copy CTAs copy the listed rows as they appear.
// The epoch itself lives on the device: every CTA reads kEpochWord at entry and uses its value
// + 1; the last CTA to finish (kArriveWord) stores that value back. A launch replayed from a
// CUDA graph therefore gets a new epoch each time without any host work.
constexpr int kArriveWord = 254, kEpochWord = 255, kMaxCoopReqs = 252;
constexpr int kProgBase = 1024;  // kMaxCoopReqs 64-bit progress words
static_assert(kProgBase + 2 * kMaxCoopReqs <= static_cast<int>(kCoopBlockWords), "block layout");
constexpr int kCoopUnroll = 12;  // 16-byte loads in flight per thread of a copy CTA

// Publishes that request r's walk list holds `entries` entries (final: no more will come).
// The caller's entry stores are fenced (gpu scope) before this.
__device__ __forceinline__ void wl_publish(const StepExtra &x, int32_t r, int32_t entries, bool final)
{
    const uint64_t v = (static_cast<uint64_t>(x.epoch) << 32) | (static_cast<uint32_t>(entries) << 1) |
                       (final ? 1u : 0u);
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(x.flags + kProgBase + 2 * r), "l"(v) : "memory");
}

// Request r's walk-list progress this epoch: (entries << 1) | final, or -1 before any.
__device__ __forceinline__ int32_t wl_probe(const StepExtra &x, int32_t r)
{
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(x.flags + kProgBase + 2 * r) : "memory");
    return static_cast<uint32_t>(v >> 32) == x.epoch ? static_cast<int32_t>(static_cast<uint32_t>(v) & 0x7FFFFFFFu) : -1;
}

// Called by thread 0 of every CTA of a cooperative step once the CTA has finished.
__device__ __forceinline__ void finish_block(const StepExtra &x)
{
    __threadfence();
    if (atomicAdd(x.flags + kArriveWord, 1u) != gridDim.x - 1) return;
    *reinterpret_cast<volatile uint32_t *>(x.flags + kArriveWord) = 0u;
    __threadfence();
    *reinterpret_cast<volatile uint32_t *>(x.flags + kEpochWord) = x.epoch;
    __threadfence();
}

// ---- cooperative step: the walk helpers ----
// While warp 0 walks, the warps of the other three SM sub-partitions (warp % 4 != 0: 12 of
// 16) copy rows; the walk warp's own sub-partition keeps its issue slots and memory queue.
constexpr int kHelpers = (kFastThreads / 32 - kFastThreads / 128) * 32;

__device__ __forceinline__ bool is_walk_helper(int tid) { return (tid >> 5) % 4 != 0; }

// This helper's index among the helper threads.
__device__ __forceinline__ int helper_index(int tid)
{
    const int w = tid >> 5;
    return (w - 1 - w / 4) * 32 + (tid & 31);
}

__device__ __forceinline__ bool helper_sync_or(bool v)
{
    uint32_t r;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 2, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
                 : "=r"(r)
                 : "r"(static_cast<uint32_t>(v)), "r"(kHelpers)
                 : "memory");
    return r != 0;
}

// Lists every position with om != 0, in position order, as entries 0.. of request bid's walk
// list; returns the count (all threads; contains barriers).
__device__ int32_t list_misses_in_order(const StepExtra &x, const int8_t *om, const int32_t *os, const int32_t *topk,
                                        int32_t K, int32_t bid, int32_t *warp_sums)
{
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5;
    const int32_t per = (K + nt - 1) / nt;
    const int32_t k0 = min(tid * per, K), k1 = min(k0 + per, K);
    int32_t mine = 0;
    for (int32_t k = k0; k < k1; ++k) mine += om[k] != 0;
    int32_t incl = mine;
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int nw = nt >> 5;
        const int32_t v = lane < nw ? warp_sums[lane] : 0;
        int32_t inc = v;
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t u = __shfl_up_sync(0xFFFFFFFFu, inc, d);
            if (lane >= d) inc += u;
        }
        if (lane < nw) warp_sums[lane] = inc - v;
        if (lane == nw - 1) warp_sums[31] = inc;
    }
    __syncthreads();
    int32_t at = warp_sums[wid] + incl - mine;
    uint2 *wl = x.wl + static_cast<int64_t>(bid) * K;
    for (int32_t k = k0; k < k1; ++k)
        if (om[k] != 0)
            wl[at++] = make_uint2(static_cast<uint32_t>(topk[k]), (static_cast<uint32_t>(k) << 16) |
                                                                   static_cast<uint32_t>(os[k]));
    const int32_t total = warp_sums[31];
    __syncthreads();
    return total;
}

// Every candidate's table entry is checked first, as phase 3 checks the evicted ones (only
// candidates are ever evicted), so the walk's decisions hold as it commits them; *verified
// reports that all passed (phase 3 then skips its check), and if any failed nothing is
// listed. Then warp 1 lists the misses the walk has numbered, in number order: numbers below
// prog[0] are final (a miss the walk creates always follows every miss consumed before it),
// each number's position being that set bit of the miss queue. Entry m of request bid's walk
// list is {token, (position << 16) | slot}; after each batch the count is published
// (wl_publish). When the walk has ended (prog[1]: 1 = completed, 2 = failed), a completed walk's
// remaining numbers are listed and the list is published as final at once (*final_out = 1):
// with every candidate verified the outputs are final when the walk completes. Returns (in warp
// 1) how many numbers were listed: exactly the misses at positions below the position of that
// number.
__device__ int32_t help_walk(const StepExtra &x, const uint32_t *cand, int32_t n, const int32_t *tok,
                             const uint16_t *ht, uint32_t mask, int32_t padded, const int32_t *topk,
                             const uint32_t *missb, const uint16_t *nslot, const int32_t *prog, int32_t K, int32_t bid,
                             uint16_t *hpos, uint16_t *posl, int *verified, int *final_out)
{
    const unsigned kAll = 0xFFFFFFFFu;
    const int htid = helper_index(threadIdx.x), lane = threadIdx.x & 31;
    bool bad = false;
    for (int32_t i = htid; i < n; i += kHelpers) {
        const int32_t c = static_cast<int32_t>(reinterpret_cast<const volatile uint32_t *>(cand)[i] & 0xFFFFu);
        const int32_t t = tok[c];
        if (t < 0) continue;
        uint32_t idx = ht_hash(t) & mask;
        int32_t found = -1;
        bool ended = false, dup = false;
        for (uint32_t q = 0; q <= mask; ++q) {
            const uint16_t e = ht[idx];
            if (e == kHtEmpty) {
                ended = true;
                break;
            }
            if (tok_of(tok, e, padded) == t) {
                if (found >= 0) {
                    dup = true;
                    break;
                }
                found = static_cast<int32_t>(e) - 1;
            }
            idx = (idx + 1) & mask;
        }
        if (found != c || dup || !ended) bad = true;
    }
    if (helper_sync_or(bad) || htid >= 32) return 0;
    if (lane == 0) *verified = 1;
    if (x.wl == nullptr) return 0;
    const int32_t qwords = (K + 31) >> 5;
    const volatile int32_t *vprog = prog;
    uint2 *wl = x.wl + static_cast<int64_t>(bid) * K;
    int32_t m0 = 0, wb = 0, nb = 0;  // cursor: first word that may hold number m0; misses before it
    for (uint32_t iter = 0; iter < (1u << 22); ++iter) {
        int32_t done = 0, gm = 0;
        if (lane == 0) {
            done = vprog[1];
            __threadfence_block();
            gm = vprog[0];
        }
        done = __shfl_sync(kAll, done, 0);
        gm = __shfl_sync(kAll, gm, 0);
        if (done == 2) break;  // the walk failed: the step falls back and relists everything
        const int32_t m1 = min(gm, m0 + kHelpBatch);
        if (m1 <= m0) {
            if (done) {  // every number is listed: the list is final
                __threadfence();
                __syncwarp();
                if (lane == 0) {
                    wl_publish(x, bid, m0, true);
                    *final_out = 1;
                }
                break;
            }
            __nanosleep(128);  // nothing new yet
            continue;
        }
        __threadfence_block();
        bool found = false;
        for (int32_t w = wb, before = nb; w < qwords;) {  // positions of numbers [m0, m1)
            const uint32_t W = w + lane < qwords ? reinterpret_cast<const volatile uint32_t *>(missb)[w + lane] : 0u;
            const int32_t pc = __popc(W);
            int32_t incl = pc;
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t v = __shfl_up_sync(kAll, incl, d);
                if (lane >= d) incl += v;
            }
            const int32_t ex = before + incl - pc;
            if (ex < m1 && ex + pc > m0) {
                int32_t num = ex;
                for (uint32_t b = W; b != 0u && num < m1; b &= b - 1u, ++num)
                    if (num >= m0) {
                        const uint16_t pos = static_cast<uint16_t>((w + lane) * 32 + __ffs(b) - 1);
                        hpos[num - m0] = pos;
                        posl[num] = pos;
                    }
            }
            const unsigned reach = __ballot_sync(kAll, before + incl >= m1);
            if (reach != 0u) {  // the word holding number m1 - 1 is where the next batch starts
                const int lr = __ffs(reach) - 1;
                nb = __shfl_sync(kAll, ex, lr);
                wb = w + lr;
                found = true;
                break;
            }
            before += __shfl_sync(kAll, incl, 31);
            w += 32;
        }
        if (!found) break;  // cannot happen: numbers below prog[0] are set bits
        __syncwarp();
        for (int32_t j = lane; j < m1 - m0; j += 32) {
            const uint32_t pos = hpos[j];
            wl[m0 + j] = make_uint2(static_cast<uint32_t>(topk[pos]), (pos << 16) | nslot[m0 + j]);
        }
        m0 = m1;
        // Once the walk has ended the next pass lists the rest and publishes the list as final.
        if (done || __shfl_sync(kAll, lane == 0 ? vprog[1] : 0, 0) != 0) continue;
        __threadfence();
        __syncwarp();
        if (lane == 0) wl_publish(x, bid, m1, false);
    }
    return m0;
}

constexpr int kCopyChunk = 64;  // walk-list entries per chunk when a request's list is shared

// Shares per request list: about four units per copy CTA (a CTA holds at most 32, one per lane
// of its polling warp), one when the copy CTAs number fewer than half the requests.
__device__ __forceinline__ int32_t copy_shares(int32_t ncopy, int32_t nr)
{
    if (2 * ncopy < nr) return 1;
    const int32_t want = (4 * ncopy + nr - 1) / nr, cap = (32 * ncopy) / nr;
    return max(1, min(want, cap));
}

// Copy CTA cidx of ncopy during the walks. The work is cut into units u = j * nr + r: share j of
// request r's walk list, nb = copy_shares(ncopy, nr) shares per request. Share j holds the
// list's chunks of kCopyChunk entries j, j + nb, ... (all of it when nb = 1), so the shares stay
// even whatever the list's final length. CTA cidx holds units cidx, cidx + ncopy, ... (at most
// 32); lane i of warp 0 polls the list of the i-th. Each round the CTA copies the published
// entries of every unit it holds, up to one entry per thread (the lanes' waiting counts are
// scanned into one flat list of rows), until every unit is final and copied.
__device__ void copy_walk_lists(const GatherParams &g, const StepExtra &x, unsigned char *smem, int32_t nr,
                                int32_t K, int32_t cidx, int32_t ncopy)
{
    __shared__ int32_t s_ur[32], s_ut0[32], s_ubase[32];
    __shared__ int32_t s_total;
    __shared__ int s_wn, s_last;
    const unsigned kAll = 0xFFFFFFFFu;
    const unsigned tid = threadIdx.x, nt = blockDim.x;
    const int lane = tid & 31;
    const uint8_t **srcl = reinterpret_cast<const uint8_t **>(smem);
    uint8_t **dstl = reinterpret_cast<uint8_t **>(smem + 8 * nt);
    if (nr <= 0 || K <= 0) return;
    const int32_t nb = copy_shares(ncopy, nr);
    const int32_t chunk = nb > 1 ? kCopyChunk : K;  // nb = 1: the whole list is one chunk
    const int64_t nunits = static_cast<int64_t>(nb) * nr;
    const int64_t u = static_cast<int64_t>(cidx) + static_cast<int64_t>(lane) * ncopy;  // lane's unit (warp 0)
    const int32_t r = static_cast<int32_t>(u % nr), share = static_cast<int32_t>(u / nr);
    if (tid == 0) s_wn = 0;
    int32_t ck = share;                  // warp 0: the lane's current chunk
    int32_t mine = ck * chunk;           // warp 0: next entry of that chunk to copy
    bool done_lane = u >= nunits;        // warp 0: the lane's unit is final and every entry taken
    bool finished = false;
    for (uint32_t iter = 0; iter < x.wait_polls && !finished; ++iter) {
        if (tid < 32) {
            int32_t avail = 0, cnt = 0;
            bool fin = false;
            if (!done_lane) {
                const int32_t pv = wl_probe(x, r);
                cnt = pv < 0 ? 0 : (pv >> 1);
                fin = pv >= 0 && (pv & 1) != 0;
                avail = max(min(cnt, (ck + 1) * chunk) - mine, 0);
                if (fin && mine >= cnt) done_lane = true;
            }
            int32_t incl = avail;  // the lanes' waiting entries, scanned in lane order
            for (int d = 1; d < 32; d <<= 1) {
                const int32_t v = __shfl_up_sync(kAll, incl, d);
                if (lane >= d) incl += v;
            }
            const int32_t excl = incl - avail;
            const int32_t take = max(0, min(avail, static_cast<int32_t>(nt) - excl));
            s_ur[lane] = r;
            s_ut0[lane] = mine;
            s_ubase[lane] = excl;
            if (take > 0) {
                mine += take;
                if (mine >= (ck + 1) * chunk) {  // chunk done: the share's next one
                    ck += nb;
                    mine = ck * chunk;
                }
                if (fin && mine >= cnt) done_lane = true;  // this round ends a final unit
            }
            // Every unit done once this round's rows (if any) are copied: no further poll.
            const bool all_done = __ballot_sync(kAll, done_lane) == kAll;
            const int32_t total = min(__shfl_sync(kAll, incl, 31), static_cast<int32_t>(nt));
            if (lane == 0) {
                s_total = total;
                s_last = all_done ? 1 : 0;
            }
        }
        __syncthreads();
        const int32_t total = s_total;
        if (s_last) finished = true;  // after this round's copy
        if (total > 0) {
            const uint8_t *src = nullptr;
            uint8_t *dst = nullptr;
            bool ok = false;
            if (static_cast<int32_t>(tid) < total) {
                // the lane whose entries hold flat index tid: the last with base <= tid (bases
                // are the exclusive scan, so any later lane starts past tid)
                int L = 0;
#pragma unroll
                for (int step = 16; step >= 1; step >>= 1)
                    if (s_ubase[L + step] <= static_cast<int32_t>(tid)) L += step;
                const int32_t rr = s_ur[L];
                const int32_t e_at = s_ut0[L] + static_cast<int32_t>(tid) - s_ubase[L];
                const uint2 e = __ldcg(x.wl + static_cast<int64_t>(rr) * K + e_at);
                const int32_t pos = static_cast<int32_t>(e.y >> 16), slot = static_cast<int32_t>(e.y & 0xFFFFu);
                ok = gather_eval(g, static_cast<int64_t>(rr) * K + pos, 1, static_cast<int32_t>(e.x), slot,
                                 g.req_pool[rr], g.host_base[rr], &src, &dst);
            }
            list_append(ok, src, dst, srcl, dstl, &s_wn);
            __syncthreads();
            cta_copy_rows<uint4, kCoopUnroll>(srcl, dstl, s_wn, g.row_bytes, x.magic);
        } else if (!finished) {
            __nanosleep(256);
        }
        __syncthreads();
        if (tid == 0) s_wn = 0;
    }
    if (tid == 0 && !finished) record_error(g.st, KVOPS_ERR_COPY_TIMEOUT);
}

// Phase 3's outputs of the non-miss positions [t, t + n, ...): a resident token's slot, unless it
// was evicted before its first lookup (that lookup became a miss; later ones hit its new slot),
// and a repeated new token hits its first lookup's slot.
__device__ __forceinline__ void hit_outputs(const uint8_t *cls, const uint16_t *aux, const uint16_t *evt,
                                            const uint32_t *tf, int32_t *os, int8_t *om, int32_t K, int t, int n)
{
    for (int32_t k = t; k < K; k += n) {
        const uint8_t c = cls[k];
        if (c == kClsRes) {
            const int32_t s0 = aux[k];
            if (evt[s0] != kNone16) {  // evicted before its first lookup, which became a miss
                const int32_t T = static_cast<int32_t>(tf[s0] & 0xFFFFu);
                if (k != T) {
                    os[k] = os[T];
                    om[k] = 0;
                }
            } else {
                os[k] = s0;
                om[k] = 0;
            }
        } else if (c == kClsNew) {
            const int32_t k0 = aux[k];
            if (k != k0) {
                os[k] = os[k0];
                om[k] = 0;
            }
        }
    }
}

// Phase 4 with threads [t, t + n) of the CTA (sync: their barrier). Every miss (posl[0..nkeys),
// in position order) took exactly one evicted slot (os), so the misses list the deletions: each
// evicted token's entry is marked deleted and its cell listed in dl (*ndel zero on entry), then
// the first deleted cell of each probe run leads its re-pack; only listed cells are visited,
// never the whole table. Touches the table, dl and *ndel only.
template <typename Sync>
__device__ void delete_evicted(const uint16_t *posl, int32_t nkeys, const int32_t *os, const uint16_t *evt,
                               const int32_t *tok, uint16_t *ht, uint32_t mask, int32_t padded, uint16_t *dl,
                               int32_t *ndel, int t, int n, Sync sync)
{
    for (int32_t j0 = 0; j0 < nkeys; j0 += n) {  // mark the evicted entries, listing their cells
        const int32_t j = j0 + t;
        bool del = false;
        uint32_t idx = 0;
        if (j < nkeys) {
            const int32_t c = os[posl[j]];
            if (evt[c] != kNone16 && tok[c] >= 0) {
                idx = ht_hash(tok[c]) & mask;
                for (uint32_t q = 0; q <= mask; ++q) {
                    if (ht[idx] == static_cast<uint16_t>(c + 1)) {
                        ht[idx] = kDelMark;
                        del = true;
                        break;
                    }
                    idx = (idx + 1) & mask;
                }
            }
        }
        const int at = warp_append(ndel, del);
        if (del) dl[at] = static_cast<uint16_t>(idx);
    }
    sync();
    const int32_t nd = *ndel;
    for (int32_t j = t; j < nd; j += n) {  // the first deleted cell of each run leads its re-pack
        const uint32_t i = dl[j];
        uint32_t q = (i - 1) & mask;
        bool lead = true;
        for (uint32_t r = 0; r <= mask; ++r) {
            const uint16_t e = ht[q];
            if (e == kHtEmpty) break;
            if (e == kDelMark || e == kLeadMark) {
                lead = false;
                break;
            }
            q = (q - 1) & mask;
        }
        if (lead) ht[i] = kLeadMark;
    }
    sync();
    for (int32_t j = t; j < nd; j += n) {
        const uint32_t i = dl[j];
        if (ht[i] != kLeadMark) continue;
        // Walk the run from its first deleted cell; every surviving entry moves to the first
        // empty cell from its home, which is never past its old cell.
        uint32_t e = i;
        for (uint32_t r = 0; r <= mask; ++r) {
            const uint16_t v = ht[e];
            if (v == kHtEmpty) break;
            ht[e] = kHtEmpty;
            if (v != kDelMark && v != kLeadMark) {
                uint32_t q = ht_hash(tok_of(tok, v, padded)) & mask;
                for (uint32_t m = 0; m <= mask && ht[q] != kHtEmpty; ++m) q = (q + 1) & mask;
                ht[q] = v;
            }
            e = (e + 1) & mask;
        }
    }
    sync();
}

constexpr int kHalf = kFastThreads / 2;  // cooperative step: phase 3 and phase 4 side by side

template <int kId>
__device__ __forceinline__ void half_sync()
{
    asm volatile("bar.sync %0, %1;" ::"n"(kId), "n"(kHalf) : "memory");
}

// kMode 0: SIEVE step only (hisp_sieve_update). 1: plus a copy warp that moves the miss rows
// during phases 4-6. 2: cooperative launch with copy helper CTAs after the SIEVE CTAs.
template <int kMode>
__global__ void __launch_bounds__(kFastThreads + (kMode == 1 ? 32 : 0), 1)
    sieve_fast_kernel(const SieveParams p, const GatherParams g, const StepExtra x0)
{
    constexpr bool kFused = kMode == 1;  // the copy warp splits off after phase 3
    // Lets a programmatic dependent (the gather of this layer-step) launch its CTAs now; they
    // wait for this grid's completion before reading its outputs.
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t s_epoch;
    StepExtra x = x0;
    // The step's epoch (one more than the last finished step's): loaded at entry. A copy CTA
    // needs it at once; a SIEVE CTA takes it once its first loads are in flight, and its other
    // threads after the staging barrier.
    uint32_t epoch_raw = 0;
    if (kMode == 2 && threadIdx.x == 0) epoch_raw = *reinterpret_cast<volatile const uint32_t *>(x0.flags + kEpochWord);
    if (kMode == 2 && static_cast<int32_t>(blockIdx.x) >= p.max_num_reqs) {  // a copy CTA
        if (threadIdx.x == 0) s_epoch = epoch_raw + 1u;
        __syncthreads();
        x.epoch = s_epoch;
        if (x.wl != nullptr) {  // the rows of every miss, listed while the walks run and at publish
            const int32_t nr = min(*p.num_real, p.max_num_reqs);
            copy_walk_lists(g, x, smem, nr, p.top_k, static_cast<int32_t>(blockIdx.x) - p.max_num_reqs,
                            static_cast<int32_t>(gridDim.x) - p.max_num_reqs);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            arrive_and_publish(g.st);
            finish_block(x);
        }
        return;
    }
    __shared__ int s_flag;     // nonzero: recompute this step with the sequential path
    __shared__ int s_any_miss;
    __shared__ int32_t s_hand;
    __shared__ bool s_dirty;
    __shared__ int32_t s_warp[32];
    __shared__ int32_t s_ncand, s_last, s_nkeys, s_ndel, s_n0, s_nvis;
    __shared__ int32_t s_prog[2];  // cooperative step: misses the walk has consumed; walk ended
    __shared__ int32_t s_hm;           // walk list: numbers listed during the walk
    __shared__ int s_hver;             // every candidate's table entry checked (phase 3 need not)
    __shared__ int s_hfinal;           // the helper published the walk list as final
    __shared__ int s_dup;              // a new token is looked up more than once
    const int32_t bid = blockIdx.x;
    const int32_t K = p.top_k, dbs = p.dbs, padded = p.padded;
    const int tid = threadIdx.x, nt = blockDim.x;
    int32_t *g_slots = p.out_slots + static_cast<int64_t>(bid) * K;
    int8_t *g_miss = p.is_miss + static_cast<int64_t>(bid) * K;

    int32_t num_real = *p.num_real;
    if (num_real > p.max_num_reqs) num_real = p.max_num_reqs;  // hisp_sieve_update.cpp:31-34
    const int64_t req = bid < num_real ? p.req_pool[bid] : -1;
    if (kMode == 2 && tid == 0) {
        s_epoch = epoch_raw + 1u;
        x.epoch = s_epoch;
    }
    if (bid >= num_real || req < 0 || req >= p.pool_size) {  // :72-88
        fill_dummy(g_slots, g_miss, K);
        if (kMode != 0) {  // no rows to copy (all miss flags 0); the CTA still completes the status
            __syncthreads();
            if (kMode == 2) {
                x.epoch = s_epoch;
                if (tid == 0 && bid < num_real) wl_publish(x, bid, 0, true);
            }
            if (tid == 0) {
                arrive_and_publish(g.st);
                if (kMode == 2) finish_block(x);
            }
        }
        return;
    }
    const int32_t seq_len = p.seq_lens[bid];
    const int32_t prefill = p.prefill[req];
    const int32_t *g_topk = p.topk + static_cast<int64_t>(bid) * K;
    int32_t *g_tok = p.tokens + req * padded;
    uint8_t *g_vis = p.visited + req * p.vis_stride;
    uint16_t *g_ht = p.ht + req * p.ht_size;
    int32_t *g_hand = p.hand + req * kHandStride;
    const uint32_t mask = static_cast<uint32_t>(p.ht_size) - 1u;

    const FastLayout L = fast_layout(padded, p.ht_size, p.vis_stride, K, dbs);
    uint16_t *s_ht = reinterpret_cast<uint16_t *>(smem + L.ht);
    int32_t *s_tok = reinterpret_cast<int32_t *>(smem + L.tok);
    int32_t *s_topk = reinterpret_cast<int32_t *>(smem + L.topk);
    int32_t *s_os = reinterpret_cast<int32_t *>(smem + L.os);
    int8_t *s_om = reinterpret_cast<int8_t *>(smem + L.om);
    uint8_t *s_cls = reinterpret_cast<uint8_t *>(smem + L.cls);
    uint16_t *s_aux = reinterpret_cast<uint16_t *>(smem + L.aux);
    uint32_t *s_tf = reinterpret_cast<uint32_t *>(smem + L.tf);  // (Tl << 16) | Tf per hot slot
    uint16_t *s_evt = reinterpret_cast<uint16_t *>(smem + L.evt);
    uint32_t *s_vini = reinterpret_cast<uint32_t *>(smem + L.vini);
    uint32_t *s_vfin = reinterpret_cast<uint32_t *>(smem + L.vfin);
    int32_t *s_dkey = reinterpret_cast<int32_t *>(smem + L.dkey);
    int32_t *s_dfirst = reinterpret_cast<int32_t *>(smem + L.dfirst);
    uint32_t *s_missb = reinterpret_cast<uint32_t *>(smem + L.missb);
    const uint32_t dmask = static_cast<uint32_t>(L.dcap) - 1u;

    // ---- phase 0: stage the request's state, clear the step arrays ----
    stage_async(s_ht, g_ht, 2ull * p.ht_size);
    stage_async(s_tok, g_tok, 4ull * padded);
    stage_async(s_topk, g_topk, 4ull * K);
    stage_async(s_vini, g_vis, p.vis_stride);
    stage_async(s_vfin, g_vis, p.vis_stride);
    for (int32_t i = tid; i < dbs; i += nt) s_tf[i] = kNone16;  // Tf = none, Tl = 0
    for (int32_t i = tid; i < padded; i += nt) s_evt[i] = kNone16;
    for (int32_t i = tid; i < L.dcap; i += nt) {
        s_dkey[i] = -1;
        s_dfirst[i] = 0x7FFFFFFF;
    }
    for (int32_t i = tid; i < (K + 31) / 32; i += nt) s_missb[i] = 0u;
    if (tid == 0) {
        int32_t hand = *g_hand;
        if (hand < 0 || hand >= dbs) hand = 0;  // :108-111
        s_hand = hand;
        s_flag = 0;
        s_any_miss = 0;
        s_prog[0] = s_prog[1] = 0;
        s_hm = 0;
        s_hver = 0;
        s_hfinal = 0;
        s_dup = 0;
        s_ndel = 0;
    }
    cp_async_wait_all();
    __syncthreads();
    if (kMode == 2) x.epoch = s_epoch;

    // The candidate list's offsets need only the step-initial bits: computed before phase 1.
    uint32_t *s_wofs = reinterpret_cast<uint32_t *>(smem + L.wofs);
    candidate_offsets(s_vini, s_wofs, dbs, &s_ncand, s_warp);

    // ---- phase 1: classify and probe every position against the step-initial table ----
    // A warp covers 32 consecutive positions, one miss-queue word, per iteration. A new token's
    // position is taken as its first lookup (the word's bits by ballot); a repeated new token
    // (seen in the de-duplication table) makes the second pass below recompute them.
    const int lane = tid & 31;
    auto classify = [&](int32_t k) -> bool {  // true: k looks up a token not in the table
        const int32_t t = s_topk[k];
        s_cls[k] = kClsNone;
        if (t < 0 || t >= seq_len) {
            s_os[k] = -1;
            s_om[k] = 0;
            return false;
        }
        if (t >= prefill) {
            s_os[k] = padded + (t - prefill);
            s_om[k] = 0;
            return false;
        }
        const int32_t s0 = ht_find(s_ht, s_tok, t, mask, padded);
        if (s0 >= 0) {
            if (s0 >= dbs) {  // a table entry outside the hot slots: not a state these kernels build
                s_flag = 1;
                return false;
            }
            s_cls[k] = kClsRes;
            s_aux[k] = static_cast<uint16_t>(s0);
            uint32_t old = s_tf[s0], assumed;
            do {
                assumed = old;
                const uint32_t f = min(assumed & 0xFFFFu, static_cast<uint32_t>(k));
                const uint32_t l = max(assumed >> 16, static_cast<uint32_t>(k));
                const uint32_t nw = (l << 16) | f;
                if (nw == assumed) break;
                old = atomicCAS(&s_tf[s0], assumed, nw);
            } while (old != assumed);
            return false;
        }
        s_cls[k] = kClsNew;
        s_aux[k] = static_cast<uint16_t>(k);
        uint32_t d = ht_hash(t) & dmask;
        for (uint32_t n = 0; n <= dmask; ++n) {
            const int32_t prev = atomicCAS(&s_dkey[d], -1, t);
            if (prev == -1 || prev == t) {
                if (prev == t) s_dup = 1;
                atomicMin(&s_dfirst[d], k);
                break;
            }
            d = (d + 1) & dmask;
        }
        return true;
    };
    for (int32_t kb = tid - lane; kb < K; kb += nt) {
        const bool fresh = kb + lane < K && classify(kb + lane);
        const uint32_t b = __ballot_sync(0xFFFFFFFFu, fresh);
        if (lane == 0) s_missb[kb >> 5] = b;
    }
    __syncthreads();
    uint32_t *s_cand = reinterpret_cast<uint32_t *>(smem + L.dkey);  // shares the dedup table's space
    if (!s_flag) {
        if (s_dup) {  // a new token looked up twice: only its first lookup is a miss
            for (int32_t kb = tid - lane; kb < K; kb += nt) {
                const int32_t k = kb + lane;
                bool first = false;
                if (k < K && s_cls[k] == kClsNew) {
                    const int32_t t = s_topk[k];
                    uint32_t d = ht_hash(t) & dmask;
                    for (uint32_t n = 0; n <= dmask && s_dkey[d] != t; ++n) d = (d + 1) & dmask;
                    const int32_t f = s_dfirst[d];
                    s_aux[k] = static_cast<uint16_t>(f);
                    first = f == k;
                }
                const uint32_t b = __ballot_sync(0xFFFFFFFFu, first);
                if (lane == 0) s_missb[kb >> 5] = b;
            }
            __syncthreads();  // the de-duplication table is read no more: the candidates may overwrite it
        }
        // Per slot: the default final bit (initial bit, or a hit this step), by ballot per word,
        // and the slot's candidate entry (phase 2a).
        for (int32_t cb = tid - lane; cb < dbs; cb += nt) {
            const int32_t c = cb + lane;
            const uint32_t b = __ballot_sync(0xFFFFFFFFu, c < dbs && (s_tf[c] & 0xFFFFu) != kNone16);
            if (lane == 0 && b != 0u) s_vfin[cb >> 5] |= b;
            if (c < dbs) put_candidate(s_vini, s_tf, s_cand, s_wofs, dbs, c);
        }
    }
    __syncthreads();

    // ---- phase 2: the hand sweep (walk over the candidate list, final bits) ----
    // Every thread reads the flag before the walk can set it; a barrier separates the two, so
    // all 15 helper warps take the same branch (their named barrier counts all of them).
    const bool walk_step = !s_flag;
    if (kMode == 2) __syncthreads();
    if (walk_step && tid < 32) {
        const int32_t n = s_ncand;
        const int32_t h0 = s_hand;
        // first candidate at or after the hand, in slot order
        int32_t n0 = static_cast<int32_t>(s_wofs[h0 >> 5]) +
                     __popc(~s_vini[h0 >> 5] & ((1u << (h0 & 31)) - 1u));
        if (n0 >= n) n0 = 0;
        int32_t last = -1, nvis = 0;
        const bool ok = walk_candidates(s_cand, n, n0, s_evt, s_missb, K, &last, &nvis,
                                        kMode == 2 ? reinterpret_cast<uint16_t *>(smem + L.nslot) : nullptr,
                                        kMode == 2 ? s_prog : nullptr);
        if (kMode == 2 && tid == 0) {  // the walk has ended: the helpers stop after their batch
            __threadfence_block();
            reinterpret_cast<volatile int32_t *>(s_prog)[1] = ok ? 1 : 2;
        }
        if (tid == 0) {
            if (!ok) s_flag = 1;
            s_last = last;
            s_any_miss = last >= 0;
            s_n0 = n0;
            s_nvis = nvis;
        }
    } else if (kMode == 2 && walk_step) {
        // Cooperative step: while one warp walks, the others list the misses the walk has numbered
        // (help_walk) for the copy CTAs, which copy them during the walk.
        if (is_walk_helper(tid)) {
            const int32_t hm = help_walk(x, s_cand, s_ncand, s_tok, s_ht, mask, padded, s_topk, s_missb,
                                         reinterpret_cast<const uint16_t *>(smem + L.nslot), s_prog, K, bid,
                                         reinterpret_cast<uint16_t *>(smem + L.hpos),
                                         reinterpret_cast<uint16_t *>(smem + L.posl), &s_hver, &s_hfinal);
            if (tid == 32) s_hm = hm;
        }
    }
    __syncthreads();
    if (!s_flag)
        resolve_miss_numbers(s_missb, K, reinterpret_cast<uint16_t *>(smem + L.posl), s_evt, s_os, s_om, s_cand,
                             s_ncand, s_n0, s_nvis, dbs, s_warp, &s_nkeys, s_hfinal ? s_hm : -1);
    __syncthreads();
    if (!s_flag && s_last >= 0) {
        passed_bits(s_vini, s_vfin, s_tf, s_evt, s_cand, s_wofs, s_ncand, dbs, s_hand, s_last);
        if (tid == 0) s_hand = s_last + 1 == dbs ? 0 : s_last + 1;
    }
    __syncthreads();

    // ---- phase 3: table check for the evicted tokens; outputs of the hits ----
    // Cooperative step with every candidate's entry checked during the walk: the outputs and
    // their publication (warps 0-7) run beside phase 4's deletions (warps 8-15), which touch
    // only the table and their own cell list.
    const bool overlap = kMode == 2 && !s_flag && s_hver && s_any_miss;
    if (!s_flag && !overlap) {
        for (int32_t c = s_hver ? dbs : tid; c < dbs; c += nt) {  // s_hver: checked during the walk
            if (s_evt[c] == kNone16) continue;
            const int32_t t = s_tok[c];
            if (t < 0) continue;
            // The first entry holding t must name slot c, and no second entry may follow.
            uint32_t idx = ht_hash(t) & mask;
            int32_t found = -1;
            bool ended = false, dup = false;
            for (uint32_t n = 0; n <= mask; ++n) {
                const uint16_t e = s_ht[idx];
                if (e == kHtEmpty) {
                    ended = true;
                    break;
                }
                if (tok_of(s_tok, e, padded) == t) {
                    if (found >= 0) {
                        dup = true;
                        break;
                    }
                    found = static_cast<int32_t>(e) - 1;
                }
                idx = (idx + 1) & mask;
            }
            if (found != c || dup || !ended) s_flag = 1;
        }
        hit_outputs(s_cls, s_aux, s_evt, s_tf, s_os, s_om, K, tid, nt);
    }
    __syncthreads();

    if (kFused && tid >= kFastThreads) {  // the copy warp
        const int32_t nsl = x.nsl;
        unsigned char *ring = smem + x.ring_off;
        uint64_t *bars = reinterpret_cast<uint64_t *>(ring + static_cast<size_t>(32 * nsl) * g.row_bytes);
        uint16_t *list = reinterpret_cast<uint16_t *>(bars + kMaxSets);
        // Outputs are final now unless the step already fell back; then copy after the
        // sequential path. (A fallback raised later, by the insert-round bound, rewrites each
        // output once with the value already there: phases 2-3 verified them.)
        const bool early = !s_flag;
        if (early) copy_miss_rows(g, bid, req, s_topk, s_os, s_om, K, ring, bars, list, nsl);
        __syncthreads();  // the compute warps have finished the step
        if (!early) copy_miss_rows(g, bid, req, s_topk, s_os, s_om, K, ring, bars, list, nsl);
        if ((tid & 31) == 0) arrive_and_publish(g.st);
        return;
    }
    const int ntc = kFused ? kFastThreads : nt;  // threads of the compute role
    const bool raised = kMode == 2 && !s_flag;
    const bool update_table = !s_flag && s_any_miss;
    const uint16_t *posl = reinterpret_cast<const uint16_t *>(smem + L.posl);  // miss positions, in order
    uint16_t *s_dl = reinterpret_cast<uint16_t *>(smem + L.dkey);  // deleted cells (candidate list no longer needed)
    const int32_t nkeys = s_nkeys;
    // Cooperative step: the outputs are final now (unless the step already fell back), so they are
    // stored, the misses not listed during the walk (numbers [s_hm, G)) complete the walk list,
    // and the list is published as final, before the table passes.
    auto publish = [&](int t, int n, auto sync) {
        coop_copy_n(g_slots, s_os, 4ull * K, t, n);
        coop_copy_n(g_miss, s_om, static_cast<size_t>(K), t, n);
        const int32_t gm = s_prog[0];
        if (x.wl != nullptr) {
            uint2 *wl = x.wl + static_cast<int64_t>(bid) * K;
            for (int32_t m = s_hm + t; m < gm; m += n) {
                const uint32_t pos = posl[m];
                wl[m] = make_uint2(static_cast<uint32_t>(s_topk[pos]), (pos << 16) | static_cast<uint32_t>(s_os[pos]));
            }
        }
        sync();
        if (t == 0 && !s_hfinal) {  // else the helper published every entry as final already
            __threadfence();  // the walk list's entries and the outputs above
            wl_publish(x, bid, x.wl != nullptr ? gm : 0, true);
        }
    };

    // ---- phase 4: delete the evicted tokens from the table, re-packing each probe run ----
    if (overlap) {
        if (tid < kHalf) {
            hit_outputs(s_cls, s_aux, s_evt, s_tf, s_os, s_om, K, tid, kHalf);
            half_sync<3>();
            publish(tid, kHalf, [] { half_sync<3>(); });
        } else {
            delete_evicted(posl, nkeys, s_os, s_evt, s_tok, s_ht, mask, padded, s_dl, &s_ndel, tid - kHalf, kHalf,
                           [] { half_sync<4>(); });
        }
        __syncthreads();
    } else {
        if (raised) publish(tid, nt, [] { __syncthreads(); });
        if (update_table)
            delete_evicted(posl, nkeys, s_os, s_evt, s_tok, s_ht, mask, padded, s_dl, &s_ndel, tid, ntc,
                           [] { compute_sync<kFused>(); });
        compute_sync<kFused>();
    }

    // ---- phase 5: insert the new tokens; an earlier miss wins a contested cell ----
    // One pass per round: a placed key first checks that it still owns its cell (a displaced
    // one moves on), a pending key then passes the cells closed to it and claims the next. The
    // round's barrier ORs the progress flags; a round without a pending or displaced key leaves
    // the table final.
    if (update_table) {
        for (int32_t j = tid; j < nkeys; j += ntc) {  // every miss starts at its token's home cell
            const int32_t m = posl[j];
            s_aux[m] = static_cast<uint16_t>(ht_hash(s_topk[m]) & mask);
            s_cls[m] = kClsPending;
        }
        compute_sync<kFused>();
        const int32_t limit = 4 * p.ht_size + 64;
        for (int32_t round = 0;; ++round) {
            bool ch = false;
            for (int32_t j = tid; j < nkeys; j += ntc) {
                const int32_t m = posl[j];
                const uint16_t entry = static_cast<uint16_t>(s_os[m] + 1);
                uint8_t cls = s_cls[m];
                uint32_t at = s_aux[m];
                if (cls == kClsPlaced && s_ht[at] != entry) {  // displaced by an earlier miss
                    cls = kClsPending;
                    at = (at + 1) & mask;
                }
                if (cls != kClsPending) continue;
                ch = true;
                // A cell held by a surviving key, or by an earlier miss, stays closed to this key
                // (an earlier miss is only ever displaced by a still earlier one, and no cell is
                // emptied here): all such cells are passed in this round.
                uint16_t e = s_ht[at];
                for (uint32_t q = 0; q <= mask && e != kHtEmpty; ++q) {
                    const int32_t es = static_cast<int32_t>(e) - 1;
                    const uint16_t te = es < padded ? s_evt[es] : kNone16;
                    if (te != kNone16 && te > m) break;  // a later miss: this key displaces it
                    at = (at + 1) & mask;
                    e = s_ht[at];
                }
                if (atomicCAS(reinterpret_cast<unsigned short *>(&s_ht[at]), e, entry) == e)
                    cls = kClsPlaced;  // an empty cell, or a later miss that now moves on
                s_cls[m] = cls;
                s_aux[m] = static_cast<uint16_t>(at);
            }
            if (!compute_sync_or<kFused>(ch)) break;
            if (round > limit) {  // cannot happen on a table at load <= 0.5; recompute if it does
                if (tid == 0) s_flag = 1;
                compute_sync<kFused>();
                break;
            }
        }
    }
    compute_sync<kFused>();

    if (!s_flag) {
        // ---- phase 6: write back ----
        for (int32_t m = tid; m < K; m += ntc)
            if ((s_missb[m >> 5] >> (m & 31)) & 1u) g_tok[s_os[m]] = s_topk[m];
        if (!raised) {
            coop_copy_n(g_slots, s_os, 4ull * K, tid, ntc);
            coop_copy_n(g_miss, s_om, static_cast<size_t>(K), tid, ntc);
        }
        coop_copy_n(g_vis, s_vfin, p.vis_stride, tid, ntc);
        if (s_any_miss) coop_copy_n(g_ht, s_ht, 2ull * p.ht_size, tid, ntc);
        if (tid == 0) *g_hand = s_hand;
        if (kFused) __syncthreads();  // meets the copy warp
        if (kMode == 2) {  // the step is written back: complete the status
            __syncthreads();
            if (tid == 0) {
                arrive_and_publish(g.st);
                finish_block(x);
            }
        }
        return;
    }

    // ---- exact sequential path from the untouched global state ----
    coop_copy_n(s_ht, g_ht, 2ull * p.ht_size, tid, ntc);
    coop_copy_n(s_tok, g_tok, 4ull * padded, tid, ntc);
    coop_copy_n(s_vfin, g_vis, p.vis_stride, tid, ntc);
    compute_sync<kFused>();
    if (tid == 0) {
        int32_t hand = *g_hand;
        if (hand < 0 || hand >= dbs) hand = 0;
        bool dirty = false;
        s_hand = sieve_sequential(s_topk, K, s_os, s_om, s_tok, reinterpret_cast<uint8_t *>(s_vfin), s_ht, mask, dbs,
                                  padded, seq_len, prefill, hand, &dirty);
        s_dirty = dirty;
    }
    compute_sync<kFused>();
    coop_copy_n(g_slots, s_os, 4ull * K, tid, ntc);
    coop_copy_n(g_miss, s_om, static_cast<size_t>(K), tid, ntc);
    coop_copy_n(g_vis, s_vfin, p.vis_stride, tid, ntc);
    if (s_dirty) {
        coop_copy_n(g_tok, s_tok, 4ull * padded, tid, ntc);
        coop_copy_n(g_ht, s_ht, 2ull * p.ht_size, tid, ntc);
    }
    if (tid == 0) *g_hand = s_hand;
    if (kFused) __syncthreads();  // meets the copy warp
    if (kMode == 2) {  // a fallback raised later rewrote the published outputs with equal values
        __syncthreads();
        if (!raised) {
            // Every miss of the sequential result, in position order, from entry 0: the entries
            // listed during the walk are an exact prefix of it (the walk is exact up to where it
            // stopped), so they are rewritten with the same values and the copy CTA, which has
            // copied some of them already, goes on from where it is.
            const int32_t n = x.wl != nullptr ? list_misses_in_order(x, s_om, s_os, s_topk, K, bid, s_warp) : 0;
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                wl_publish(x, bid, n, true);
            }
        }
        if (tid == 0) {
            arrive_and_publish(g.st);
            finish_block(x);
        }
    }
}

#include "sieve_big.cuh"

thread_local uint32_t t_tier_choice = KVOPS_TIER_AUTO;  // caller's choice (kvops_set_sieve_tier)
thread_local uint32_t t_tier_last = KVOPS_TIER_AUTO;    // tier of the last launch_sieve_update

int max_optin_smem()
{
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    return v;
}

}  // namespace

void set_sieve_tier(uint32_t tier) { t_tier_choice = tier; }
uint32_t last_sieve_tier() { return t_tier_last; }

namespace {

bool shared_tier_fits(const SieveParams &p, int limit)
{
    if (p.top_k > 65535 || p.ht_size > 65536 || p.dbs > 65535) return false;  // 16-bit bookkeeping
    return fast_layout(p.padded, p.ht_size, p.vis_stride, p.top_k, p.dbs).total <= static_cast<size_t>(limit);
}

bool large_tier_fits(const SieveParams &p, int limit)
{
    if (p.top_k > 65535 || p.dbs > 65534 || p.ht_size < 1024) return false;
    return big_layout(p.ht_size, p.vis_stride, p.top_k, p.dbs).total <= static_cast<size_t>(limit);
}

// The tier a launch of this shape runs under the calling thread's choice.
uint32_t pick_tier(const SieveParams &p, int limit, bool large_scratch)
{
    const bool shared = shared_tier_fits(p, limit);
    const bool large = large_tier_fits(p, limit) && large_scratch;
    if (t_tier_choice == KVOPS_TIER_ORDERED) return KVOPS_TIER_ORDERED;
    if (t_tier_choice == KVOPS_TIER_LARGE && large) return KVOPS_TIER_LARGE;
    if (t_tier_choice == KVOPS_TIER_SHARED && shared) return KVOPS_TIER_SHARED;
    return shared ? KVOPS_TIER_SHARED : large ? KVOPS_TIER_LARGE : KVOPS_TIER_ORDERED;
}

}  // namespace

// CTAs of the large-table tier resident per SM at this shape (0: cannot launch).
int big_ctas_per_sm(const SieveParams &p)
{
    const BigLayout B = big_layout(p.ht_size, p.vis_stride, p.top_k, p.dbs);
    if (cudaFuncSetAttribute(sieve_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(B.total)) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sieve_big_kernel, kBigThreads, B.total) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return per_sm;
}

uint64_t sieve_big_scratch(const SieveParams &p, int sm_count, int32_t *slots)
{
    *slots = 0;
    if (p.max_num_reqs <= 0 || p.top_k <= 0) return 0;
    if (pick_tier(p, max_optin_smem(), true) != KVOPS_TIER_LARGE) return 0;
    const int32_t per_sm = big_ctas_per_sm(p);
    if (per_sm <= 0) return 0;  // the tier is not used: launch_sieve_update falls back
    const int32_t resident = (sm_count > 0 ? sm_count : 148) * per_sm;
    *slots = p.max_num_reqs < resident ? p.max_num_reqs : resident;
    return big_slot(p.dbs, p.padded, p.top_k).bytes;
}

cudaError_t launch_sieve_update(const SieveParams &p, cudaStream_t s, int /*sm_count*/)
{
    if (p.max_num_reqs <= 0) return cudaSuccess;
    const int limit = max_optin_smem();
    const uint32_t tier = pick_tier(p, limit, p.big != nullptr && p.big_slots > 0);
    t_tier_last = tier;
    if (tier == KVOPS_TIER_SHARED) {
        const FastLayout F = fast_layout(p.padded, p.ht_size, p.vis_stride, p.top_k, p.dbs);
        cudaError_t e = cudaFuncSetAttribute(sieve_fast_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(F.total));
        if (e != cudaSuccess) return e;
        sieve_fast_kernel<0><<<p.max_num_reqs, kFastThreads, F.total, s>>>(p, GatherParams{}, StepExtra{});
        return cudaGetLastError();
    }
    if (tier == KVOPS_TIER_LARGE) {
        const BigLayout B = big_layout(p.ht_size, p.vis_stride, p.top_k, p.dbs);
        cudaError_t e = cudaFuncSetAttribute(sieve_big_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(B.total));
        if (e != cudaSuccess) return e;
        const int grid = p.max_num_reqs < p.big_slots ? p.max_num_reqs : p.big_slots;
        sieve_big_kernel<<<grid, kBigThreads, B.total, s>>>(p);
        return cudaGetLastError();
    }
    const SmemLayout L = sieve_smem_layout(p.padded, p.ht_size, p.vis_stride, p.top_k);
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

cudaError_t launch_sieve_import(const SieveParams &p, const GatherParams &g, cudaStream_t s, bool *launched)
{
    *launched = false;
    if (p.max_num_reqs <= 0 || p.top_k <= 0) return cudaSuccess;
    if (p.top_k > 65535 || p.ht_size > 65536 || p.dbs > 65535) return cudaSuccess;
    const FastLayout F = fast_layout(p.padded, p.ht_size, p.vis_stride, p.top_k, p.dbs);
    const size_t ring_off = align_up(F.total, 128);
    const size_t limit = static_cast<size_t>(max_optin_smem());
    for (int32_t nsl = kMaxSets; nsl >= 1; --nsl) {  // sets of 32 ring slots for the copy warp
        const size_t total = ring_off + static_cast<size_t>(32 * nsl) * g.row_bytes + 8u * kMaxSets +
                             2ull * static_cast<size_t>(p.top_k);
        if (total > limit) continue;
        cudaError_t e = cudaFuncSetAttribute(sieve_fast_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(total));
        if (e != cudaSuccess) return e;
        StepExtra x{};
        x.nsl = nsl;
        x.ring_off = static_cast<uint32_t>(ring_off);
        sieve_fast_kernel<1><<<p.max_num_reqs, kFastThreads + 32, total, s>>>(p, g, x);
        *launched = true;
        return cudaGetLastError();
    }
    return cudaSuccess;
}

// CTAs of sieve_fast_kernel<2> resident at once with `smem` bytes each (0 if it does not fit),
// cached per device and size. The kernel's shared-memory limit only ever rises (to the largest
// size used on the device), so every cached size stays launchable.
cudaError_t coop_residency(size_t smem, int *resident)
{
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> cache;
    static std::map<int, size_t> limit_set;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find({dev, smem});
    if (it != cache.end()) {
        *resident = it->second;
        return cudaSuccess;
    }
    int n = 0;
    if (smem <= static_cast<size_t>(max_optin_smem())) {
        if (smem > limit_set[dev]) {
            e = cudaFuncSetAttribute(sieve_fast_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem));
            if (e != cudaSuccess) return e;
            limit_set[dev] = smem;
        }
        int sms = 0, per_sm = 0;
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sieve_fast_kernel<2>, kFastThreads, smem);
        if (e != cudaSuccess) return e;
        n = per_sm * sms;
    }
    cache[{dev, smem}] = n;
    *resident = n;
    return cudaSuccess;
}

// Dynamic shared memory of a cooperative step: the SIEVE layout, or the copy CTAs' two row lists.
size_t coop_smem(const SieveParams &p)
{
    const FastLayout F = fast_layout(p.padded, p.ht_size, p.vis_stride, p.top_k, p.dbs);
    const size_t list = 4ull * sizeof(void *) * kFastThreads;
    return F.total > list ? F.total : list;
}

cudaError_t prepare_sieve_coop(const SieveParams &p)
{
    if (p.top_k <= 0 || p.top_k > 65535 || p.ht_size > 65536 || p.dbs > 65535) return cudaSuccess;
    int resident = 0;
    return coop_residency(coop_smem(p), &resident);
}

cudaError_t launch_sieve_coop(const SieveParams &p, const GatherParams &g, uint32_t *flags, uint2 *wl,
                              uint32_t wait_polls, int32_t min_copy_ctas, cudaStream_t s, bool *launched)
{
    *launched = false;
    if (wl == nullptr) return cudaSuccess;  // the copy CTAs move rows only through the walk lists
    if (p.max_num_reqs <= 0 || p.top_k <= 0 || p.max_num_reqs > kMaxCoopReqs) return cudaSuccess;
    if (p.top_k > 65535 || p.ht_size > 65536 || p.dbs > 65535) return cudaSuccess;
    const size_t total = coop_smem(p);
    int resident = 0;
    cudaError_t e = coop_residency(total, &resident);
    if (e != cudaSuccess) return e;
    if (resident - p.max_num_reqs < (min_copy_ctas > 8 ? min_copy_ctas : 8)) return cudaSuccess;
    StepExtra x{};
    x.flags = flags;
    x.wl = wl;
    x.wait_polls = wait_polls != 0 ? wait_polls : (1u << 22);
    const uint32_t cpr = g.row_bytes / 16;  // helpers copy 16-byte chunks (host-checked)
    x.magic = (cpr > 0 && cpr < 65536 && static_cast<uint64_t>(kFastThreads) * cpr < 65536)
                  ? static_cast<uint32_t>(((1ull << 32) + cpr - 1) / cpr) : 0u;
    void *args[] = {const_cast<SieveParams *>(&p), const_cast<GatherParams *>(&g), &x};
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(sieve_fast_kernel<2>), dim3(resident),
                                    dim3(kFastThreads), args, total, s);
    if (e != cudaSuccess) return e;
    *launched = true;
    return cudaSuccess;
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
