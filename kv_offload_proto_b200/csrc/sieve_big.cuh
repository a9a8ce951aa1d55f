// sieve_big.cuh — the large-table tier of the SIEVE step (hisp_sieve_update.cpp:115-173) for
// states that do not fit shared memory, such as the stress shape (hot buffer 65518 slots, table
// 262144 cells, 794 KB per request). Part of sieve.cu's translation unit: it reuses that file's
// phase helpers (candidate list, warp walk, miss numbering, final visited bits, hit outputs).
//
// Why a tier of its own: the reference's hash yields 16-bit homes (hisp_kernel_common.h:23-26),
// so in a table of more than 65536 cells every key lives in the first quarter, where the load
// is close to 1 and one probe run covers tens of thousands of cells. A lookup of a token that is
// not resident scans to the end of that run (~32K cells on average), and so do the erases and
// inserts, which makes both the position-ordered loop and the shared-memory phases' table passes
// far too slow. This tier never walks the table for a lookup:
//  0. the table is checked to be a well-formed linear-probing table for the token row (every
//     entry names a hot slot holding a token, each slot has exactly one entry, tokens are
//     distinct, and every entry is reachable from its home through occupied cells); then
//     ht_find(t) is, exactly, the slot whose token is t, which a direct token -> slot index
//     (tokens below kBigIdxCap) answers in one load, checked against the token row (the index
//     keeps whatever earlier requests left in it). A state that fails the check, or holds a
//     token the index cannot hold, runs the position-ordered loop in global memory instead;
//  1-3. the phases of sieve_fast_kernel (probe classification, hand sweep, outputs) with the
//     index in place of the probes and the per-slot arrays in global scratch;
//  4. the evicted tokens are deleted all at once: each probe run that holds a deleted cell is
//     re-packed from its first deleted cell, every later entry of the run moving to the first
//     empty cell from its home in cell order, which is the table backward-shift deletion leaves
//     (Knuth 6.4, Algorithm R: as if the deleted keys had never been inserted);
//  5. the new tokens are inserted in miss order, each into the first empty cell from its home
//     (the reference's interleaved erase / insert sequence ends in the same table, since every
//     erase leaves the table as if its key had never been inserted).
// "First empty cell from" is answered by a bitmap of empty cells in shared memory (32 KB for
// 262144 cells). CTAs of 256 threads (two per SM at the stress shape: the serial re-pack of one
// leaves the SM's issue slots to the other) loop over the requests; each CTA owns one slot of
// global scratch, allocated once per shape by the host (sieve_big_scratch).

constexpr int kBigThreads = 256;
constexpr uint32_t kNoCell = 0xFFFFFFFFu;
constexpr int32_t kBigIdxCap = 1 << 20;  // tokens [0, kBigIdxCap) are indexed directly

// Shared memory of one CTA (one request at a time).
struct BigLayout {
    size_t vini, vfin, topk, os, om, cls, aux, missb, posl, freeb, delb, total;
    int32_t fwords;
};

__host__ __device__ __forceinline__ BigLayout big_layout(int32_t ht_size, int32_t vis_stride, int32_t K, int32_t dbs)
{
    BigLayout L;
    L.fwords = ht_size / 32;
    size_t o = 0;
    L.vini = take(&o, static_cast<size_t>(vis_stride));
    L.vfin = take(&o, static_cast<size_t>(vis_stride));
    L.topk = take(&o, 4ull * K);
    L.os = take(&o, 4ull * K);
    L.om = take(&o, static_cast<size_t>(K));
    L.cls = take(&o, static_cast<size_t>(K));
    L.aux = take(&o, 2ull * K);
    L.missb = take(&o, 4ull * ((K + 31) / 32));
    L.posl = take(&o, 2ull * K);
    L.freeb = take(&o, 4ull * L.fwords);  // bit set: the cell is empty
    L.delb = take(&o, 4ull * L.fwords);   // phase 0: last empty cell before each word; phase 4: deleted cells
    L.total = o;
    return L;
}

// Global scratch of one CTA: the token index (no initial contents needed), the per-slot arrays, the
// de-duplication table of phase 1 (then the list of run leads of phase 4) and the word offsets
// of the candidate list.
struct BigSlot {
    size_t idx, tf, cellof, cand, evt, dkey, dfirst, wofs, bytes;
    int32_t dcap;
};

__host__ __device__ __forceinline__ BigSlot big_slot(int32_t dbs, int32_t padded, int32_t K)
{
    BigSlot S;
    S.dcap = 1;
    while (S.dcap < 2 * K) S.dcap <<= 1;
    size_t o = 0;
    S.idx = take(&o, 2ull * kBigIdxCap);
    S.tf = take(&o, 4ull * dbs);
    S.cellof = take(&o, 4ull * dbs);
    S.cand = take(&o, 4ull * dbs + 16);
    S.evt = take(&o, 2ull * padded);
    S.dkey = take(&o, 4ull * S.dcap);
    S.dfirst = take(&o, 4ull * S.dcap);
    S.wofs = take(&o, 4ull * ((dbs + 31) / 32 + 1));
    S.bytes = align_up(o, 256);
    return S;
}

// First empty cell at or after h (cyclic), by one thread over the empty-cell bitmap.
__device__ __forceinline__ uint32_t big_first_empty(const uint32_t *freeb, uint32_t h, uint32_t mask)
{
    const uint32_t nwords = (mask >> 5) + 1;
    uint32_t w = h >> 5;
    uint32_t bits = freeb[w] & (0xFFFFFFFFu << (h & 31));
    for (uint32_t n = 0; n <= nwords; ++n) {
        if (bits) return (w << 5) + static_cast<uint32_t>(__ffs(bits)) - 1u;
        w = (w + 1) & (nwords - 1);
        bits = freeb[w];
    }
    return kNoCell;
}

__device__ __forceinline__ void big_set(uint32_t *b, uint32_t c) { atomicOr(&b[c >> 5], 1u << (c & 31)); }
__device__ __forceinline__ void big_clr(uint32_t *b, uint32_t c) { atomicAnd(&b[c >> 5], ~(1u << (c & 31))); }

// Re-packs the probe run that holds `lead`, its first deleted cell (one warp): the cells from the
// lead to the run's end are taken in order; a deleted entry is dropped, every other entry moves
// to the first empty cell from its home, which is never past its own cell. Cells past the
// current one are not written yet, so each batch of 32 cells is loaded before it is walked.
__device__ void big_repack_run(uint32_t lead, uint16_t *ht, const int32_t *tok, int32_t padded, uint32_t mask,
                               uint32_t *freeb, const uint32_t *delb)
{
    const unsigned kAll = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    uint32_t e = lead;
    for (uint32_t done = 0; done <= mask; done += 32) {
        const uint32_t c = (e + static_cast<uint32_t>(lane)) & mask;
        const uint16_t v = ht[c];
        const bool del = (delb[c >> 5] >> (c & 31)) & 1u;
        const unsigned endm = __ballot_sync(kAll, v == kHtEmpty && !del);  // a deleted cell keeps its entry until here
        const int nact = endm ? __ffs(endm) - 1 : 32;
        uint32_t home = 0;
        if (lane < nact && !del) home = ht_hash(tok_of(tok, v, padded)) & mask;
        for (int l = 0; l < nact; ++l) {
            const bool dl = __shfl_sync(kAll, del, l);
            const uint32_t hl = __shfl_sync(kAll, home, l);
            const uint16_t vl = static_cast<uint16_t>(__shfl_sync(kAll, static_cast<uint32_t>(v), l));
            if (lane == 0) {
                const uint32_t cl = (e + static_cast<uint32_t>(l)) & mask;
                big_set(freeb, cl);
                if (dl) {
                    ht[cl] = kHtEmpty;
                } else {
                    const uint32_t q = big_first_empty(freeb, hl, mask);  // cl is empty: q is in [hl, cl]
                    big_clr(freeb, q);
                    if (q != cl) {
                        ht[q] = vl;
                        ht[cl] = kHtEmpty;
                    }
                }
            }
        }
        __syncwarp();
        if (nact < 32) return;
        e = (e + 32) & mask;
    }
}

// Block-wide exclusive prefix maximum of `v` over the threads in order (all threads call it).
__device__ __forceinline__ int32_t big_block_exclusive_max(int32_t v, int32_t *warp_sums, int32_t *total)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int32_t incl = v;
    for (int d = 1; d < 32; d <<= 1) {
        const int32_t u = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl = max(incl, u);
    }
    __syncthreads();
    if (lane == 31) warp_sums[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        const int32_t x = lane < nw ? warp_sums[lane] : -1;
        int32_t inc = x;
        for (int d = 1; d < 32; d <<= 1) {
            const int32_t u = __shfl_up_sync(0xFFFFFFFFu, inc, d);
            if (lane >= d) inc = max(inc, u);
        }
        const int32_t ex = __shfl_up_sync(0xFFFFFFFFu, inc, 1);
        if (lane < nw) warp_sums[lane] = lane == 0 ? -1 : ex;
        if (lane == 31) *total = inc;
    }
    __syncthreads();
    const int32_t before = warp_sums[wid];
    const int32_t ex_in_warp = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
    return max(before, lane == 0 ? -1 : ex_in_warp);
}

__global__ void __launch_bounds__(kBigThreads, 2) sieve_big_kernel(const SieveParams p)
{
    // Lets a programmatic dependent (the gather of this layer-step) launch its CTAs now; they
    // wait for this grid's completion before reading its outputs.
    asm volatile("griddepcontrol.launch_dependents;");
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int s_flag, s_any_miss;
    __shared__ int32_t s_hand, s_warp[32], s_ncand, s_last, s_nkeys, s_n0, s_nvis, s_nlead, s_lastfree;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int wid = tid >> 5, nw = nt >> 5;
    const int32_t K = p.top_k, dbs = p.dbs, padded = p.padded;
    const uint32_t mask = static_cast<uint32_t>(p.ht_size) - 1u;
    const BigLayout L = big_layout(p.ht_size, p.vis_stride, K, dbs);
    const BigSlot G = big_slot(dbs, padded, K);
    unsigned char *gs = p.big + static_cast<size_t>(blockIdx.x) * p.big_slot_bytes;
    uint16_t *g_idx = reinterpret_cast<uint16_t *>(gs + G.idx);
    uint32_t *tf = reinterpret_cast<uint32_t *>(gs + G.tf);  // (Tl << 16) | Tf per hot slot
    uint32_t *cellof = reinterpret_cast<uint32_t *>(gs + G.cellof);
    uint32_t *cand = reinterpret_cast<uint32_t *>(gs + G.cand);
    uint16_t *evt = reinterpret_cast<uint16_t *>(gs + G.evt);
    uint32_t *vini = reinterpret_cast<uint32_t *>(smem + L.vini);
    uint32_t *vfin = reinterpret_cast<uint32_t *>(smem + L.vfin);
    int32_t *s_topk = reinterpret_cast<int32_t *>(smem + L.topk);
    int32_t *s_os = reinterpret_cast<int32_t *>(smem + L.os);
    int8_t *s_om = reinterpret_cast<int8_t *>(smem + L.om);
    uint8_t *s_cls = reinterpret_cast<uint8_t *>(smem + L.cls);
    uint16_t *s_aux = reinterpret_cast<uint16_t *>(smem + L.aux);
    uint32_t *s_missb = reinterpret_cast<uint32_t *>(smem + L.missb);
    uint16_t *s_posl = reinterpret_cast<uint16_t *>(smem + L.posl);
    int32_t *s_dkey = reinterpret_cast<int32_t *>(gs + G.dkey);
    int32_t *s_dfirst = reinterpret_cast<int32_t *>(gs + G.dfirst);
    uint32_t *s_wofs = reinterpret_cast<uint32_t *>(gs + G.wofs);
    uint32_t *freeb = reinterpret_cast<uint32_t *>(smem + L.freeb);
    uint32_t *delb = reinterpret_cast<uint32_t *>(smem + L.delb);
    int32_t *runs = reinterpret_cast<int32_t *>(smem + L.delb);  // phase 0 view of delb
    uint32_t *leads = reinterpret_cast<uint32_t *>(gs + G.dkey);  // phase 4 view of dkey
    const uint32_t dmask = static_cast<uint32_t>(G.dcap) - 1u;
    const int32_t fwords = L.fwords;

    int32_t num_real = *p.num_real;
    if (num_real > p.max_num_reqs) num_real = p.max_num_reqs;  // hisp_sieve_update.cpp:31-34
    for (int32_t bid = blockIdx.x; bid < p.max_num_reqs; bid += gridDim.x) {
        int32_t *g_slots = p.out_slots + static_cast<int64_t>(bid) * K;
        int8_t *g_miss = p.is_miss + static_cast<int64_t>(bid) * K;
        const int64_t req = bid < num_real ? p.req_pool[bid] : -1;
        __syncthreads();  // the previous request is done with shared memory
        if (bid >= num_real || req < 0 || req >= p.pool_size) {  // :72-88
            fill_dummy(g_slots, g_miss, K);
            continue;
        }
        const int32_t seq_len = p.seq_lens[bid];
        const int32_t prefill = p.prefill[req];
        const int32_t *g_topk = p.topk + static_cast<int64_t>(bid) * K;
        int32_t *g_tok = p.tokens + req * padded;
        uint8_t *g_vis = p.visited + req * p.vis_stride;
        uint16_t *g_ht = p.ht + req * p.ht_size;
        int32_t *g_hand = p.hand + req * kHandStride;

        // ---- phase 0: stage, clear, empty-cell bitmap, last empty cell before each word ----
        coop_copy(s_topk, g_topk, 4ull * K);
        coop_copy(vini, g_vis, static_cast<size_t>(p.vis_stride));
        coop_copy(vfin, g_vis, static_cast<size_t>(p.vis_stride));
        for (int32_t i = tid; i < dbs; i += nt) {
            tf[i] = kNone16;
            cellof[i] = kNoCell;
        }
        for (int32_t i = tid; i < padded; i += nt) evt[i] = kNone16;
        for (int32_t i = tid; i < G.dcap; i += nt) {
            s_dkey[i] = -1;
            s_dfirst[i] = 0x7FFFFFFF;
        }
        for (int32_t i = tid; i < (K + 31) / 32; i += nt) s_missb[i] = 0u;
        const int32_t per = (fwords + nt - 1) / nt;
        const int32_t w0 = min(tid * per, fwords), w1 = min(w0 + per, fwords);
        int32_t mylast = -1;  // last empty cell of this thread's words
        for (int32_t w = w0; w < w1; ++w) {
            uint32_t bits = 0;
            for (int j = 0; j < 32; ++j) bits |= (g_ht[w * 32 + j] == kHtEmpty ? 1u : 0u) << j;
            freeb[w] = bits;
            if (bits) mylast = w * 32 + 31 - __clz(bits);
        }
        if (tid == 0) {
            int32_t hand = *g_hand;
            if (hand < 0 || hand >= dbs) hand = 0;  // :108-111
            s_hand = hand;
            s_flag = 0;
            s_any_miss = 0;
            s_nlead = 0;
        }
        int32_t before = big_block_exclusive_max(mylast, s_warp, &s_lastfree);  // (contains barriers)
        {
            const int32_t lastfree = s_lastfree;  // the table's last empty cell (-1: no empty cell)
            for (int32_t w = w0; w < w1; ++w) {  // runs[w]: last empty cell before word w, cyclic
                runs[w] = before >= 0 ? before : lastfree - p.ht_size;
                const uint32_t bits = freeb[w];
                if (bits) before = w * 32 + 31 - __clz(bits);
            }
        }
        __syncthreads();

        // ---- the table check (see the file comment); any failure runs the ordered loop ----
        bool bad = s_lastfree < 0;
        for (int32_t c = tid; c < p.ht_size && !bad; c += nt) {
            const uint16_t v = g_ht[c];
            if (v == kHtEmpty) continue;
            const int32_t s = static_cast<int32_t>(v) - 1;
            if (s >= dbs) {
                bad = true;
                break;
            }
            const int32_t t = g_tok[s];
            if (t < 0 || atomicCAS(&cellof[s], kNoCell, static_cast<uint32_t>(c)) != kNoCell) {
                bad = true;
                break;
            }
            const uint32_t home = ht_hash(t) & mask;
            const uint32_t below = freeb[c >> 5] & ((1u << (c & 31)) - 1u);
            const int32_t lf = below ? (c & ~31) + 31 - __clz(below) : runs[c >> 5];
            const uint32_t dstart = (static_cast<uint32_t>(c) - static_cast<uint32_t>(lf + 1)) & mask;
            if (((static_cast<uint32_t>(c) - home) & mask) > dstart) bad = true;  // not reachable from its home
        }
        if (__syncthreads_or(bad)) {
            if (tid == 0) s_flag = 1;
        } else {
            // The index: every token's slot (the index may hold anything beforehand; every
            // lookup below checks the slot it reads against the token row).
            for (int32_t s = tid; s < dbs && !bad; s += nt) {
                const int32_t t = g_tok[s];
                if (t < 0) continue;
                if (t >= kBigIdxCap || cellof[s] == kNoCell) {
                    bad = true;
                    break;
                }
                g_idx[t] = static_cast<uint16_t>(s + 1);
            }
            if (__syncthreads_or(bad)) {
                if (tid == 0) s_flag = 1;
            } else {
                for (int32_t s = tid; s < dbs && !bad; s += nt) {  // a token held by two slots: one store lost
                    const int32_t t = g_tok[s];
                    if (t >= 0 && g_idx[t] != static_cast<uint16_t>(s + 1)) bad = true;
                }
                if (__syncthreads_or(bad) && tid == 0) s_flag = 1;
            }
        }
        __syncthreads();

        if (!s_flag) {
            // ---- phase 1: classify every position against the step-initial state ----
            for (int32_t k = tid; k < K; k += nt) {
                const int32_t t = s_topk[k];
                s_cls[k] = kClsNone;
                if (t < 0 || t >= seq_len) {
                    s_os[k] = -1;
                    s_om[k] = 0;
                    continue;
                }
                if (t >= prefill) {
                    s_os[k] = padded + (t - prefill);
                    s_om[k] = 0;
                    continue;
                }
                // resident iff the index names a hot slot that holds t (tokens are distinct)
                int32_t s0 = t < kBigIdxCap ? static_cast<int32_t>(g_idx[t]) - 1 : -1;
                if (s0 >= dbs || (s0 >= 0 && g_tok[s0] != t)) s0 = -1;
                if (s0 >= 0) {
                    s_cls[k] = kClsRes;
                    s_aux[k] = static_cast<uint16_t>(s0);
                    uint32_t old = tf[s0], assumed;
                    do {
                        assumed = old;
                        const uint32_t f = min(assumed & 0xFFFFu, static_cast<uint32_t>(k));
                        const uint32_t l = max(assumed >> 16, static_cast<uint32_t>(k));
                        const uint32_t nwv = (l << 16) | f;
                        if (nwv == assumed) break;
                        old = atomicCAS(&tf[s0], assumed, nwv);
                    } while (old != assumed);
                } else {
                    s_cls[k] = kClsNew;
                    uint32_t d = ht_hash(t) & dmask;
                    for (uint32_t n = 0; n <= dmask; ++n) {
                        const int32_t prev = atomicCAS(&s_dkey[d], -1, t);
                        if (prev == -1 || prev == t) {
                            atomicMin(&s_dfirst[d], k);
                            break;
                        }
                        d = (d + 1) & dmask;
                    }
                }
            }
            __syncthreads();
            for (int32_t k = tid; k < K; k += nt) {
                if (s_cls[k] != kClsNew) continue;
                const int32_t t = s_topk[k];
                uint32_t d = ht_hash(t) & dmask;
                for (uint32_t n = 0; n <= dmask && s_dkey[d] != t; ++n) d = (d + 1) & dmask;
                const int32_t f = s_dfirst[d];
                s_aux[k] = static_cast<uint16_t>(f);
                if (f == k) atomicOr(&s_missb[k >> 5], 1u << (k & 31));  // first lookup of a new token
            }
            for (int32_t c = tid; c < dbs; c += nt)  // default final bit: initial bit, or a hit this step
                if ((tf[c] & 0xFFFFu) != kNone16) atomicOr(&vfin[c >> 5], 1u << (c & 31));
            __syncthreads();

            // ---- phase 2: the hand sweep ----
            build_candidates(vini, tf, cand, s_wofs, dbs, &s_ncand, s_warp);
            __syncthreads();
            if (tid < 32) {
                const int32_t n = s_ncand;
                const int32_t h0 = s_hand;
                int32_t n0 = static_cast<int32_t>(s_wofs[h0 >> 5]) + __popc(~vini[h0 >> 5] & ((1u << (h0 & 31)) - 1u));
                if (n0 >= n) n0 = 0;
                int32_t last = -1, nvis = 0;
                const bool ok = walk_candidates(cand, n, n0, evt, s_missb, K, &last, &nvis, nullptr, nullptr);
                if (tid == 0) {
                    if (!ok) s_flag = 1;
                    s_last = last;
                    s_any_miss = last >= 0;
                    s_n0 = n0;
                    s_nvis = nvis;
                }
            }
            __syncthreads();
            if (!s_flag)
                resolve_miss_numbers(s_missb, K, s_posl, evt, s_os, s_om, cand, s_ncand, s_n0, s_nvis, dbs, s_warp,
                                     &s_nkeys, -1);
            __syncthreads();
            if (!s_flag && s_last >= 0) {
                passed_bits(vini, vfin, tf, evt, cand, s_wofs, s_ncand, dbs, s_hand, s_last);
                if (tid == 0) s_hand = s_last + 1 == dbs ? 0 : s_last + 1;
            }
            __syncthreads();
        }

        if (!s_flag) {
            // ---- phase 3: outputs ----
            hit_outputs(s_cls, s_aux, evt, tf, s_os, s_om, K, tid, nt);
            __syncthreads();
            coop_copy(g_slots, s_os, 4ull * K);
            coop_copy(g_miss, s_om, static_cast<size_t>(K));
            const int32_t nkeys = s_nkeys;
            if (s_any_miss) {
                // ---- phase 4: delete the evicted tokens, re-packing each affected run ----
                for (int32_t w = tid; w < fwords; w += nt) delb[w] = 0u;
                __syncthreads();
                for (int32_t j = tid; j < nkeys; j += nt) {
                    const int32_t c = s_os[s_posl[j]];
                    if (g_tok[c] >= 0) big_set(delb, cellof[c]);
                }
                __syncthreads();
                for (int32_t j = tid; j < nkeys; j += nt) {  // leads: the nearest event below is an empty cell
                    const int32_t c = s_os[s_posl[j]];
                    if (g_tok[c] < 0) continue;
                    const uint32_t cell = cellof[c];
                    uint32_t w = cell >> 5, below = (1u << (cell & 31)) - 1u;
                    for (int32_t n = 0; n <= fwords; ++n) {
                        const uint32_t f = freeb[w] & below, d = delb[w] & below;
                        if (f | d) {
                            if ((f >> (31 - __clz(f | d))) & 1u) leads[atomicAdd(&s_nlead, 1)] = cell;
                            break;
                        }
                        w = (w - 1u) & static_cast<uint32_t>(fwords - 1);
                        below = 0xFFFFFFFFu;
                    }
                }
                __syncthreads();
                for (int32_t i = wid; i < s_nlead; i += nw)
                    big_repack_run(leads[i], g_ht, g_tok, padded, mask, freeb, delb);
                __syncthreads();
                // ---- phase 5: insert the new tokens in miss order ----
                if (tid == 0) {
                    for (int32_t j = 0; j < nkeys; ++j) {
                        const int32_t m = s_posl[j];
                        const uint32_t q = big_first_empty(freeb, ht_hash(s_topk[m]) & mask, mask);
                        if (q == kNoCell) break;  // cannot happen: a table at load <= 0.5 has empty cells
                        big_clr(freeb, q);
                        g_ht[q] = static_cast<uint16_t>(s_os[m] + 1);
                    }
                }
            }
            __syncthreads();
            // ---- phase 6: write back ----
            for (int32_t m = tid; m < K; m += nt)
                if ((s_missb[m >> 5] >> (m & 31)) & 1u) g_tok[s_os[m]] = s_topk[m];
            coop_copy(g_vis, vfin, static_cast<size_t>(p.vis_stride));
            if (tid == 0) *g_hand = s_hand;
            continue;
        }

        // ---- the position-ordered loop in global memory (a state the check refuses, a wrapped sweep) ----
        if (tid == 0) {
            int32_t hand = *g_hand;
            if (hand < 0 || hand >= dbs) hand = 0;
            bool dirty = false;
            *g_hand = sieve_sequential(g_topk, K, g_slots, g_miss, g_tok, g_vis, g_ht, mask, dbs, padded, seq_len,
                                       prefill, hand, &dirty);
        }
    }
}
