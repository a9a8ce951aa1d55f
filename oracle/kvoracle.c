/*
 * kvoracle.c — CPU restatement of the kv_offload_proto decode-time KV hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA product path
 * (kv_offload_proto_b200/csrc). Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it. Nothing shipped calls it.
 *
 * It restates the reference kernels' semantics on host memory, bit for bit,
 * including the persistent SIEVE state (token rows, visited bitmap, uint16
 * hash table, hand) and not only the slots/is_miss outputs:
 *
 *   ko_hash / ko_ht_*      kvops/kernel/hisp_kernel_common.h:23-130
 *   ko_sieve_update        kvops/kernel/hisp_sieve_update.cpp:17-176
 *   ko_sieve_ht_init       kvops/kernel/hisp_sieve_ht_init.cpp:14-60
 *   ko_gather_rows         kvops/kernel/kvc_gather_rows.cpp:12-96
 *   ko_export_alllayer     kvops/kernel/kvc_scatter_rows_alllayer.cpp:11-67
 *   ko_scatter_rows        doc/kv_offload_design.md:394-396 (gather rules, opposite direction)
 *   ko_node_of/ko_seg_row  kvops/kernel/kvc_common.h:81-89, common/kv_layout.h:26-39
 *   ko_ht_size             kvops/kvops_ext/kvops_ext.cpp:297-300
 *
 * The sieve loop is threaded over batch rows (requests are independent: each
 * owns one pool row of state) so the same code is the multi-core CPU baseline.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define KO_HAND_STRIDE 16 /* int32 words per hand row: hisp_kernel_common.h:21 */

/* Knuth multiplicative hash, 32-bit wrap then >>16: hisp_kernel_common.h:23-26 */
uint32_t ko_hash(int32_t token) { return ((uint32_t)token * 2654435761u) >> 16; }

/* Hash-table size: smallest power of two >= max(1024, 2*(padded+topK)):
 * kvops_ext.cpp:297-300 (and xds_ems_pool.py:42-47). */
int64_t ko_ht_size(int64_t padded, int64_t top_k)
{
    int64_t p = 1024;
    while (p < 2 * (padded + top_k)) p <<= 1;
    return p;
}

/* Token held by the slot an entry names; an entry past the token row (only in a corrupted
 * table) reads as -1, which no probed token equals. Same guard as the CUDA kernels. */
static inline int32_t tok_of(const int32_t *tok, uint16_t e, int32_t padded)
{
    const int32_t s = (int32_t)e - 1;
    return s < padded ? tok[s] : -1;
}

/* Probe for token; returns slot or -1: hisp_kernel_common.h:29-43. Bounded by
 * the table size so a corrupted table cannot spin forever (the reference
 * loop is unbounded; on a well-formed table at load <= 0.5 the bound is never hit). */
static int32_t ht_find(const uint16_t *ht, const int32_t *tok, int32_t token, uint32_t mask, int32_t padded)
{
    uint32_t idx = ko_hash(token) & mask;
    for (uint32_t n = 0; n <= mask; n++) {
        uint16_t e = ht[idx];
        if (e == 0) return -1;
        if (tok_of(tok, e, padded) == token) return (int32_t)e - 1;
        idx = (idx + 1) & mask;
    }
    return -1;
}

/* Insert token->slot, first (lowest-probe) entry of a duplicate token wins:
 * hisp_kernel_common.h:46-61 (and the GM-token twin at :97-112). */
static void ht_insert(uint16_t *ht, const int32_t *tok, int32_t token, int32_t slot, uint32_t mask,
                      int32_t padded)
{
    uint32_t idx = ko_hash(token) & mask;
    for (uint32_t n = 0; n <= mask; n++) {
        uint16_t e = ht[idx];
        if (e == 0) {
            ht[idx] = (uint16_t)(slot + 1);
            return;
        }
        if (tok_of(tok, e, padded) == token) return;
        idx = (idx + 1) & mask;
    }
}

/* Backward-shift deletion (Knuth 6.4 Algorithm R): hisp_kernel_common.h:64-94.
 * The move test for the entry at i with home h against the gap j is
 * (j < i) ? (h <= j || h > i) : (h <= j && h > i)   (:87). */
static void ht_erase(uint16_t *ht, const int32_t *tok, int32_t token, uint32_t mask, int32_t padded)
{
    uint32_t idx = ko_hash(token) & mask;
    uint32_t n;
    for (n = 0; n <= mask; n++) {
        uint16_t e = ht[idx];
        if (e == 0) return;
        if (tok_of(tok, e, padded) == token) break;
        idx = (idx + 1) & mask;
    }
    if (n > mask) return;
    int32_t j = (int32_t)idx, i = (int32_t)idx;
    for (n = 0; n <= mask; n++) {
        i = (int32_t)(((uint32_t)i + 1) & mask);
        uint16_t e = ht[i];
        if (e == 0) break;
        int32_t home = (int32_t)(ko_hash(tok_of(tok, e, padded)) & mask);
        int move = (j < i) ? (home <= j || home > i) : (home <= j && home > i);
        if (move) {
            ht[j] = e;
            j = i;
        }
    }
    ht[j] = 0;
}

static inline int vis_get(const uint8_t *v, int32_t s) { return (v[s >> 3] >> (s & 7)) & 1; }
static inline void vis_set(uint8_t *v, int32_t s) { v[s >> 3] = (uint8_t)(v[s >> 3] | (1u << (s & 7))); }
static inline void vis_clr(uint8_t *v, int32_t s) { v[s >> 3] = (uint8_t)(v[s >> 3] & ~(1u << (s & 7))); }

typedef struct {
    const int32_t *topk;
    const int64_t *req_pool;
    const int32_t *seq_lens;
    const int32_t *prefill_lens;
    int32_t *tokens;  /* [pool, padded] layer slice */
    uint8_t *visited; /* [pool, vis_stride] */
    uint16_t *ht;     /* [pool, ht_size] */
    int32_t *hand;    /* [pool, 16] */
    int32_t *out_slots;
    int8_t *is_miss;
    int32_t num_real, top_k, dbs, padded, vis_stride, max_num_reqs, pool_size, ht_size;
    int32_t bid_lo, bid_hi;
} SieveJob;

/* One batch row of hisp_sieve_update (hisp_sieve_update.cpp:67-173), in place on
 * the state slices. Staging into UB and writing back (:97-106, :165-173) is
 * equivalent to in-place update because each pool row is private to its request. */
static void sieve_row(const SieveJob *J, int32_t bid)
{
    const int32_t K = J->top_k;
    int32_t *os = J->out_slots + (int64_t)bid * K;
    int8_t *om = J->is_miss + (int64_t)bid * K;
    int32_t num_real = J->num_real > J->max_num_reqs ? J->max_num_reqs : J->num_real; /* :31-34 */
    if (bid >= num_real) { /* padding rows: :72-78 */
        for (int32_t k = 0; k < K; k++) { os[k] = -1; om[k] = 0; }
        return;
    }
    const int64_t req = J->req_pool[bid];
    if (req < 0 || req >= J->pool_size) { /* bad pool index: :80-88 */
        for (int32_t k = 0; k < K; k++) { os[k] = -1; om[k] = 0; }
        return;
    }
    const int32_t seq_len = J->seq_lens[bid];
    const int32_t prefill = J->prefill_lens[req];
    const int32_t *tp = J->topk + (int64_t)bid * K;
    int32_t *tok = J->tokens + req * (int64_t)J->padded;
    uint8_t *vis = J->visited + req * (int64_t)J->vis_stride;
    uint16_t *ht = J->ht + req * (int64_t)J->ht_size;
    const uint32_t mask = (uint32_t)J->ht_size - 1u;
    const int32_t dbs = J->dbs;
    int32_t hand = J->hand[req * KO_HAND_STRIDE];
    if (hand < 0 || hand >= dbs) hand = 0; /* :108-111 */

    for (int32_t k = 0; k < K; k++) { /* :115-163 */
        const int32_t t = tp[k];
        if (t < 0 || t >= seq_len) { os[k] = -1; om[k] = 0; continue; }
        if (t >= prefill) { os[k] = J->padded + (t - prefill); om[k] = 0; continue; }
        const int32_t hit = ht_find(ht, tok, t, mask, J->padded);
        if (hit >= 0) { os[k] = hit; om[k] = 0; vis_set(vis, hit); continue; }
        int32_t h = hand;
        while (vis_get(vis, h)) { /* hand sweep: :139-146 */
            vis_clr(vis, h);
            if (++h == dbs) h = 0;
        }
        const int32_t old = tok[h];
        if (old >= 0) ht_erase(ht, tok, old, mask, J->padded); /* :148-151 */
        ht_insert(ht, tok, t, h, mask, J->padded);   /* :152 (before tok[h] is updated) */
        os[k] = h;
        om[k] = 1;
        tok[h] = t;
        vis_set(vis, h);
        hand = h + 1;
        if (hand == dbs) hand = 0;
    }
    J->hand[req * KO_HAND_STRIDE] = hand; /* :165 */
}

static void *sieve_worker(void *p)
{
    const SieveJob *J = (const SieveJob *)p;
    for (int32_t b = J->bid_lo; b < J->bid_hi; b++) sieve_row(J, b);
    return NULL;
}

/* Batch SIEVE update over rows [0, max_num_reqs) of one layer's state slices.
 * Returns 0, or -1 when the arguments are out of the reference's domain. */
int ko_sieve_update(const int32_t *topk, const int64_t *req_pool, const int32_t *seq_lens,
                    const int32_t *prefill_lens, int32_t *tokens, uint8_t *visited, uint16_t *ht,
                    int32_t *hand, int32_t *out_slots, int8_t *is_miss, int32_t num_real, int32_t top_k,
                    int32_t dbs, int32_t padded, int32_t vis_stride, int32_t max_num_reqs,
                    int32_t pool_size, int32_t ht_size, int32_t nthreads)
{
    if (top_k < 0 || dbs < 1 || dbs > padded || ht_size < 1 || (ht_size & (ht_size - 1)) != 0) return -1;
    SieveJob base = {topk, req_pool, seq_lens, prefill_lens, tokens, visited, ht, hand, out_slots, is_miss,
                     num_real, top_k, dbs, padded, vis_stride, max_num_reqs, pool_size, ht_size, 0,
                     max_num_reqs};
    if (nthreads <= 1 || max_num_reqs <= 1) {
        sieve_worker(&base);
        return 0;
    }
    if (nthreads > max_num_reqs) nthreads = max_num_reqs;
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    SieveJob *jobs = (SieveJob *)malloc(sizeof(SieveJob) * (size_t)nthreads);
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = base;
        jobs[i].bid_lo = (int32_t)((int64_t)max_num_reqs * i / nthreads);
        jobs[i].bid_hi = (int32_t)((int64_t)max_num_reqs * (i + 1) / nthreads);
        pthread_create(&th[i], NULL, sieve_worker, &jobs[i]);
    }
    for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
    free(th);
    free(jobs);
    return 0;
}

/* Admission hash-table build: block b -> (layer = b / num_reqs, req = req_start + b % num_reqs);
 * clear the table, insert slots 0..dbs-1 holding a non-negative token, in slot order
 * (hisp_sieve_ht_init.cpp:25-58). Only blocks b < min(nblocks, layer_num*num_reqs) run. */
int ko_sieve_ht_init(const int32_t *tokens3d, uint16_t *ht3d, int32_t req_start, int32_t num_reqs,
                     int32_t layer_num, int32_t pool_size, int32_t dbs, int32_t padded, int32_t ht_size,
                     int32_t nblocks)
{
    if (ht_size < 1 || (ht_size & (ht_size - 1)) != 0) return -1;
    const uint32_t mask = (uint32_t)ht_size - 1u;
    int64_t total = (int64_t)layer_num * num_reqs;
    if (nblocks < total) total = nblocks;
    for (int64_t b = 0; b < total; b++) {
        const int64_t layer = b / num_reqs;
        const int64_t req = (int64_t)req_start + b % num_reqs;
        if (req < 0 || req >= pool_size) continue;
        const int32_t *tok = tokens3d + (layer * pool_size + req) * padded;
        uint16_t *ht = ht3d + (layer * pool_size + req) * ht_size;
        memset(ht, 0, sizeof(uint16_t) * (size_t)ht_size);
        for (int32_t s = 0; s < dbs; s++)
            if (tok[s] >= 0) ht_insert(ht, tok, tok[s], s, mask, padded);
    }
    return 0;
}

/* Stripe ownership: kvc_common.h:81-89 (S == 0 means node 0 / identity). */
uint32_t ko_node_of(uint32_t row, uint32_t stripe, uint32_t nodes)
{
    return stripe == 0 ? 0u : (row / stripe) % nodes;
}
uint32_t ko_seg_row(uint32_t row, uint32_t stripe, uint32_t nodes)
{
    return stripe == 0 ? row : (row / stripe) / nodes;
}
/* Injective stripe map (opt-in layout, not in the reference): keeps row % S. */
uint32_t ko_seg_row_injective(uint32_t row, uint32_t stripe, uint32_t nodes)
{
    return stripe == 0 ? row : ((row / stripe) / nodes) * stripe + row % stripe;
}

/* Host restatement of kvc_gather_rows for one segment launch (kvc_gather_rows.cpp:54-84):
 * scan [0, num_real*top_k), copy row_bytes for is_miss rows owned by my_node.
 * seg_base / hot_base are host pointers. hot_req_stride_rows > 0 selects the opt-in
 * per-request hot layout dst = hot + (req*stride + slot)*row_bytes (0 = reference).
 * injective != 0 selects the opt-in injective map. Returns the number of rows copied. */
int64_t ko_gather_rows(uint8_t *seg_base, uint32_t layer_offset_rows, uint32_t row_bytes,
                       const int32_t *topk, const int64_t *req_pool, const int64_t *host_base,
                       const int32_t *slots, const int8_t *is_miss, int32_t num_real, uint8_t *hot_base,
                       uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe, uint32_t nodes,
                       uint32_t my_node, int64_t hot_req_stride_rows, int injective)
{
    if (num_real > (int32_t)max_num_reqs) num_real = (int32_t)max_num_reqs;
    const int64_t total = (int64_t)num_real * top_k;
    int64_t queued = 0;
    for (int64_t pos = 0; pos < total; pos++) {
        if (is_miss[pos] == 0) continue;
        const int64_t bid = pos / top_k;
        const int32_t t = topk[pos];
        const int32_t slot = slots[pos];
        if (t < 0 || slot < 0) continue;
        const int64_t req = req_pool[bid];
        if (req < 0) continue;
        const uint32_t row = (uint32_t)(host_base[bid] + t);
        if (ko_node_of(row, stripe, nodes) != my_node) continue;
        const uint64_t seg_row =
            injective ? ko_seg_row_injective(row, stripe, nodes) : ko_seg_row(row, stripe, nodes);
        const uint8_t *src = seg_base + ((uint64_t)layer_offset_rows + seg_row) * row_bytes;
        const int64_t dst_row = hot_req_stride_rows > 0 ? req * hot_req_stride_rows + slot : slot;
        memcpy(hot_base + (uint64_t)dst_row * row_bytes, src, row_bytes);
        queued++;
    }
    return queued;
}

/* Host restatement of kvc_scatter_rows, the single-layer indexed export of decode
 * increments (doc/kv_offload_design.md:394-396: the arguments of kvc_gather_rows with the data
 * moving hot rows -> segment; the reference deleted its implementation, :544). The selection
 * rules are the gather's (kvc_gather_rows.cpp:54-76) with export_flags in place of is_miss. */
int64_t ko_scatter_rows(uint8_t *seg_base, uint32_t layer_offset_rows, uint32_t row_bytes,
                        const int32_t *topk, const int64_t *req_pool, const int64_t *host_base,
                        const int32_t *slots, const int8_t *export_flags, int32_t num_real,
                        const uint8_t *hot_base, uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe,
                        uint32_t nodes, uint32_t my_node, int64_t hot_req_stride_rows, int injective)
{
    if (num_real > (int32_t)max_num_reqs) num_real = (int32_t)max_num_reqs;
    const int64_t total = (int64_t)num_real * top_k;
    int64_t queued = 0;
    for (int64_t pos = 0; pos < total; pos++) {
        if (export_flags[pos] == 0) continue;
        const int64_t bid = pos / top_k;
        const int32_t t = topk[pos];
        const int32_t slot = slots[pos];
        if (t < 0 || slot < 0) continue;
        const int64_t req = req_pool[bid];
        if (req < 0) continue;
        const uint32_t row = (uint32_t)(host_base[bid] + t);
        if (ko_node_of(row, stripe, nodes) != my_node) continue;
        const uint64_t seg_row =
            injective ? ko_seg_row_injective(row, stripe, nodes) : ko_seg_row(row, stripe, nodes);
        const int64_t src_row = hot_req_stride_rows > 0 ? req * hot_req_stride_rows + slot : slot;
        memcpy(seg_base + ((uint64_t)layer_offset_rows + seg_row) * row_bytes,
               hot_base + (uint64_t)src_row * row_bytes, row_bytes);
        queued++;
    }
    return queued;
}

/* Host restatement of kvc_scatter_rows_alllayer for one segment launch
 * (kvc_scatter_rows_alllayer.cpp:34-53): layer-major, rows ascending, so under the
 * non-injective S>1 map the last row of each stripe is what the segment keeps. */
int64_t ko_export_alllayer(uint8_t *seg_base, uint32_t plsr, uint32_t row_bytes, uint32_t row_lo,
                           uint32_t row_cnt, uint32_t layer_num, const uint8_t *src_layer0,
                           uint64_t src_layer_stride, uint32_t stripe, uint32_t nodes, uint32_t my_node,
                           int injective)
{
    int64_t queued = 0;
    for (uint32_t l = 0; l < layer_num; l++) {
        const uint8_t *src_layer = src_layer0 + (uint64_t)l * src_layer_stride;
        const uint64_t seg_layer = (uint64_t)l * plsr;
        for (uint32_t row = row_lo; row < row_lo + row_cnt; row++) {
            if (ko_node_of(row, stripe, nodes) != my_node) continue;
            const uint64_t seg_row =
                injective ? ko_seg_row_injective(row, stripe, nodes) : ko_seg_row(row, stripe, nodes);
            memcpy(seg_base + (seg_layer + seg_row) * row_bytes, src_layer + (uint64_t)row * row_bytes,
                   row_bytes);
            queued++;
        }
    }
    return queued;
}

typedef struct {
    uint8_t **seg_bases;
    uint32_t layer_offset_rows, row_bytes;
    const int32_t *topk;
    const int64_t *req_pool, *host_base;
    const int32_t *slots;
    const int8_t *is_miss;
    int32_t num_real;
    uint8_t *hot_base;
    uint32_t top_k, max_num_reqs, stripe, nodes;
    int64_t hot_req_stride_rows;
    int injective;
    int64_t lo, hi, copied;
} GatherJob;

static void *gather_worker(void *p)
{
    GatherJob *J = (GatherJob *)p;
    int64_t n = 0;
    for (int64_t pos = J->lo; pos < J->hi; pos++) {
        if (J->is_miss[pos] == 0) continue;
        const int64_t bid = pos / J->top_k;
        const int32_t t = J->topk[pos], slot = J->slots[pos];
        if (t < 0 || slot < 0) continue;
        const int64_t req = J->req_pool[bid];
        if (req < 0) continue;
        const uint32_t row = (uint32_t)(J->host_base[bid] + t);
        const uint32_t node = ko_node_of(row, J->stripe, J->nodes);
        const uint64_t seg_row = J->injective ? ko_seg_row_injective(row, J->stripe, J->nodes)
                                              : ko_seg_row(row, J->stripe, J->nodes);
        const int64_t dst_row = J->hot_req_stride_rows > 0 ? req * J->hot_req_stride_rows + slot : slot;
        memcpy(J->hot_base + (uint64_t)dst_row * J->row_bytes,
               J->seg_bases[node] + ((uint64_t)J->layer_offset_rows + seg_row) * J->row_bytes, J->row_bytes);
        n++;
    }
    J->copied = n;
    return NULL;
}

/* All-segment gather in one pass, threaded over positions (the CPU baseline's gather
 * leg). Equivalent to ko_gather_rows for my_node = 0..nodes-1 when destinations do
 * not collide (per-request hot stride). Returns rows copied. */
int64_t ko_gather_all(uint8_t **seg_bases, uint32_t layer_offset_rows, uint32_t row_bytes,
                      const int32_t *topk, const int64_t *req_pool, const int64_t *host_base,
                      const int32_t *slots, const int8_t *is_miss, int32_t num_real, uint8_t *hot_base,
                      uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe, uint32_t nodes,
                      int64_t hot_req_stride_rows, int injective, int32_t nthreads)
{
    if (num_real > (int32_t)max_num_reqs) num_real = (int32_t)max_num_reqs;
    const int64_t total = (int64_t)num_real * top_k;
    if (nthreads < 1) nthreads = 1;
    GatherJob base = {seg_bases, layer_offset_rows, row_bytes, topk, req_pool, host_base, slots, is_miss,
                      num_real, hot_base, top_k, max_num_reqs, stripe, nodes, hot_req_stride_rows,
                      injective, 0, total, 0};
    if (nthreads == 1) {
        gather_worker(&base);
        return base.copied;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
    GatherJob *jobs = (GatherJob *)malloc(sizeof(GatherJob) * (size_t)nthreads);
    for (int i = 0; i < nthreads; i++) {
        jobs[i] = base;
        jobs[i].lo = total * i / nthreads;
        jobs[i].hi = total * (i + 1) / nthreads;
        pthread_create(&th[i], NULL, gather_worker, &jobs[i]);
    }
    int64_t n = 0;
    for (int i = 0; i < nthreads; i++) {
        pthread_join(th[i], NULL);
        n += jobs[i].copied;
    }
    free(th);
    free(jobs);
    return n;
}
