// kvops_pybind.cpp — the Python module `_kvops`, a drop-in for the reference's
// kvops_ext._kvops (kvops/kvops_ext/kvops_ext.cpp:373-401): same function names,
// argument names, order and defaults. Each function forwards to the C ABI in
// include/kvops_b200.h and raises RuntimeError with the library's message on failure,
// as the reference raises std::runtime_error. Only poll_status releases the GIL
// (kvops_ext.cpp:201). Opt-in behaviour the reference lacks is keyword-only.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/kvops_b200.h"

namespace py = pybind11;

namespace {

void check(int rc)
{
    if (rc != KVOPS_OK) throw std::runtime_error(kvops_last_error());
}

KvopsRowOpts row_opts(uint64_t hot_req_stride_rows, bool injective, uint64_t err_word)
{
    KvopsRowOpts o{};
    o.hot_req_stride_rows = hot_req_stride_rows;
    o.injective = injective ? 1u : 0u;
    o.err_word = err_word;
    return o;
}

void init(int device_id, const std::string &fatbin_path, const std::string &rt_lib)
{
    check(kvops_init(device_id, fatbin_path.c_str(), rt_lib.c_str()));
}

uint64_t alloc_status(int count)
{
    uint64_t addr = 0;
    check(kvops_alloc_status(count, &addr));
    return addr;
}

int64_t poll_status(uint64_t status_addr, int64_t timeout_us)
{
    int64_t rc_val = 0;
    int rc;
    {
        py::gil_scoped_release release;
        rc = kvops_poll_status(status_addr, timeout_us, &rc_val);
    }
    check(rc);
    return rc_val;
}

void import_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base, uint32_t top_k,
                uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node, uint64_t status,
                uint64_t stream, uint32_t block_dim, uint64_t hot_req_stride_rows, bool injective, uint64_t err_word)
{
    const KvopsRowOpts o = row_opts(hot_req_stride_rows, injective, err_word);
    check(kvops_import_seg_ex(channel, seg_base, layer_offset_rows, per_layer_seg_rows, row_bytes, topk_indices,
                              req_pool_indices, req_host_base, topk_device_slots, is_miss, num_real, hot_row_base,
                              top_k, max_num_reqs, stripe_rows, node_num, my_node, status, stream, block_dim, &o));
}

void import_multi(const std::vector<uint64_t> &seg_bases, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                  uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                  uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real, uint64_t hot_row_base,
                  uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint64_t status, uint64_t stream,
                  uint32_t block_dim, uint64_t hot_req_stride_rows, bool injective, uint64_t err_word)
{
    const KvopsRowOpts o = row_opts(hot_req_stride_rows, injective, err_word);
    check(kvops_import_multi(static_cast<uint32_t>(seg_bases.size()), seg_bases.data(), layer_offset_rows,
                             per_layer_seg_rows, row_bytes, topk_indices, req_pool_indices, req_host_base,
                             topk_device_slots, is_miss, num_real, hot_row_base, top_k, max_num_reqs, stripe_rows,
                             status, stream, block_dim, &o));
}

void sieve_import(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                  uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                  uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                  uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size, uint32_t visited_stride_b,
                  uint32_t max_num_reqs, uint32_t pool_size, const std::vector<uint64_t> &seg_bases,
                  uint32_t layer_offset_rows, uint32_t per_layer_seg_rows, uint32_t row_bytes, uint64_t req_host_base,
                  uint64_t hot_row_base, uint32_t stripe_rows, uint64_t status, uint64_t stream, uint32_t block_dim,
                  uint64_t hot_req_stride_rows, bool injective, const std::string &path, uint64_t err_word,
                  uint32_t copy_wait_polls)
{
    KvopsRowOpts o = row_opts(hot_req_stride_rows, injective, err_word);
    o.copy_wait_polls = copy_wait_polls;
    if (path == "auto") o.step_path = KVOPS_STEP_AUTO;
    else if (path == "fused") o.step_path = KVOPS_STEP_FUSED;
    else if (path == "split") o.step_path = KVOPS_STEP_SPLIT;
    else if (path == "coop") o.step_path = KVOPS_STEP_COOP;
    else throw std::invalid_argument("sieve_import: path must be 'auto', 'coop', 'fused' or 'split'");
    check(kvops_sieve_import(topk_indices, req_pool_indices, seq_lens, prefill_lens, device_buffer_tokens,
                             device_buffer_visited, device_buffer_ht, sieve_hand, topk_device_slots, is_miss, num_real,
                             top_k, device_buffer_size, padded_buffer_size, visited_stride_b, max_num_reqs, pool_size,
                             static_cast<uint32_t>(seg_bases.size()), seg_bases.data(), layer_offset_rows,
                             per_layer_seg_rows, row_bytes, req_host_base, hot_row_base, stripe_rows, status, stream,
                             block_dim, &o));
}

void export_seg(uint64_t channel, uint64_t seg_base, uint32_t layer_offset_rows, uint32_t per_layer_seg_rows,
                uint32_t row_bytes, uint64_t topk_indices, uint64_t req_pool_indices, uint64_t req_host_base,
                uint64_t topk_device_slots, uint64_t export_flags, uint64_t num_real, uint64_t hot_row_base,
                uint32_t top_k, uint32_t max_num_reqs, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                uint64_t status, uint64_t stream, uint32_t block_dim, uint64_t hot_req_stride_rows, bool injective,
                uint64_t err_word)
{
    const KvopsRowOpts o = row_opts(hot_req_stride_rows, injective, err_word);
    check(kvops_export_seg(channel, seg_base, layer_offset_rows, per_layer_seg_rows, row_bytes, topk_indices,
                           req_pool_indices, req_host_base, topk_device_slots, export_flags, num_real, hot_row_base,
                           top_k, max_num_reqs, stripe_rows, node_num, my_node, status, stream, block_dim, &o));
}

void export_seg_alllayer(uint64_t channel, uint64_t seg_base, uint32_t per_layer_seg_rows, uint32_t row_bytes,
                         uint32_t row_lo, uint32_t row_cnt, uint32_t layer_num, uint64_t src_layer0_base,
                         uint64_t src_layer_stride, uint32_t stripe_rows, uint32_t node_num, uint32_t my_node,
                         uint64_t status, uint64_t stream, uint32_t block_dim, bool injective, uint64_t err_word)
{
    const KvopsRowOpts o = row_opts(0, injective, err_word);
    check(kvops_export_seg_alllayer_ex(channel, seg_base, per_layer_seg_rows, row_bytes, row_lo, row_cnt, layer_num,
                                       src_layer0_base, src_layer_stride, stripe_rows, node_num, my_node, status,
                                       stream, block_dim, &o));
}

void sieve_update(uint64_t topk_indices, uint64_t req_pool_indices, uint64_t seq_lens, uint64_t prefill_lens,
                  uint64_t device_buffer_tokens, uint64_t device_buffer_visited, uint64_t device_buffer_ht,
                  uint64_t sieve_hand, uint64_t topk_device_slots, uint64_t is_miss, uint64_t num_real,
                  uint32_t top_k, uint32_t device_buffer_size, uint32_t padded_buffer_size, uint32_t visited_stride_b,
                  uint32_t max_num_reqs, uint32_t pool_size, uint64_t stream, uint32_t block_dim)
{
    check(kvops_sieve_update(topk_indices, req_pool_indices, seq_lens, prefill_lens, device_buffer_tokens,
                             device_buffer_visited, device_buffer_ht, sieve_hand, topk_device_slots, is_miss, num_real,
                             top_k, device_buffer_size, padded_buffer_size, visited_stride_b, max_num_reqs, pool_size,
                             stream, block_dim));
}

void sieve_ht_init(uint64_t device_buffer_tokens, uint64_t device_buffer_ht, uint64_t prefill_lens,
                   uint32_t req_start, uint32_t num_reqs, uint32_t layer_num, uint32_t pool_size,
                   uint32_t device_buffer_size, uint32_t padded_buffer_size, uint32_t ht_size, uint64_t stream,
                   uint32_t block_dim)
{
    check(kvops_sieve_ht_init(device_buffer_tokens, device_buffer_ht, prefill_lens, req_start, num_reqs, layer_num,
                              pool_size, device_buffer_size, padded_buffer_size, ht_size, stream, block_dim));
}

void close_module() { check(kvops_close()); }

uint64_t segment_alloc(int device, uint64_t bytes)
{
    uint64_t a = 0;
    check(kvops_segment_alloc(device, bytes, &a));
    return a;
}

py::bytes ipc_get_handle(uint64_t addr)
{
    uint8_t h[64];
    check(kvops_ipc_get_handle(addr, h));
    return py::bytes(reinterpret_cast<const char *>(h), 64);
}

uint64_t ipc_open_handle(int device, const py::bytes &handle)
{
    const std::string s = handle;
    if (s.size() != 64) throw std::runtime_error("ipc_open_handle: handle must be 64 bytes");
    uint64_t a = 0;
    check(kvops_ipc_open_handle(device, reinterpret_cast<const uint8_t *>(s.data()), &a));
    return a;
}

}  // namespace

PYBIND11_MODULE(_kvops, m)
{
    m.doc() = "B200 (sm_100a) kvops launch extension: drop-in for kvops_ext._kvops";
    m.def("init", &init, py::arg("device_id"), py::arg("fatbin_path"), py::arg("rt_lib") = "libascendcl.so");
    m.def("alloc_status", &alloc_status, py::arg("count"));
    m.def("poll_status", &poll_status, py::arg("status_addr"), py::arg("timeout_us") = -1);
    m.def("import_seg", &import_seg, py::arg("channel"), py::arg("seg_base"), py::arg("layer_offset_rows"),
          py::arg("per_layer_seg_rows"), py::arg("row_bytes"), py::arg("topk_indices"), py::arg("req_pool_indices"),
          py::arg("req_host_base"), py::arg("topk_device_slots"), py::arg("is_miss"), py::arg("num_real"),
          py::arg("hot_row_base"), py::arg("top_k"), py::arg("max_num_reqs"), py::arg("stripe_rows"),
          py::arg("node_num"), py::arg("my_node"), py::arg("status"), py::arg("stream") = 0, py::arg("block_dim") = 1,
          py::kw_only(), py::arg("hot_req_stride_rows") = 0, py::arg("injective") = false, py::arg("err_word") = 0);
    m.def("import_multi", &import_multi, py::arg("seg_bases"), py::arg("layer_offset_rows"),
          py::arg("per_layer_seg_rows"), py::arg("row_bytes"), py::arg("topk_indices"), py::arg("req_pool_indices"),
          py::arg("req_host_base"), py::arg("topk_device_slots"), py::arg("is_miss"), py::arg("num_real"),
          py::arg("hot_row_base"), py::arg("top_k"), py::arg("max_num_reqs"), py::arg("stripe_rows"),
          py::arg("status"), py::arg("stream") = 0, py::arg("block_dim") = 1, py::kw_only(),
          py::arg("hot_req_stride_rows") = 0, py::arg("injective") = false, py::arg("err_word") = 0);
    // Single-layer indexed export (kvc_scatter_rows; designed in the reference, not in its module).
    m.def("export_seg", &export_seg, py::arg("channel"), py::arg("seg_base"), py::arg("layer_offset_rows"),
          py::arg("per_layer_seg_rows"), py::arg("row_bytes"), py::arg("topk_indices"), py::arg("req_pool_indices"),
          py::arg("req_host_base"), py::arg("topk_device_slots"), py::arg("export_flags"), py::arg("num_real"),
          py::arg("hot_row_base"), py::arg("top_k"), py::arg("max_num_reqs"), py::arg("stripe_rows"),
          py::arg("node_num"), py::arg("my_node"), py::arg("status"), py::arg("stream") = 0, py::arg("block_dim") = 1,
          py::kw_only(), py::arg("hot_req_stride_rows") = 0, py::arg("injective") = false, py::arg("err_word") = 0);
    m.def("export_seg_alllayer", &export_seg_alllayer, py::arg("channel"), py::arg("seg_base"),
          py::arg("per_layer_seg_rows"), py::arg("row_bytes"), py::arg("row_lo"), py::arg("row_cnt"),
          py::arg("layer_num"), py::arg("src_layer0_base"), py::arg("src_layer_stride"), py::arg("stripe_rows"),
          py::arg("node_num"), py::arg("my_node"), py::arg("status"), py::arg("stream") = 0, py::arg("block_dim") = 1,
          py::kw_only(), py::arg("injective") = false, py::arg("err_word") = 0);
    m.def("sieve_update", &sieve_update, py::arg("topk_indices"), py::arg("req_pool_indices"), py::arg("seq_lens"),
          py::arg("prefill_lens"), py::arg("device_buffer_tokens"), py::arg("device_buffer_visited"),
          py::arg("device_buffer_ht"), py::arg("sieve_hand"), py::arg("topk_device_slots"), py::arg("is_miss"),
          py::arg("num_real"), py::arg("top_k"), py::arg("device_buffer_size"), py::arg("padded_buffer_size"),
          py::arg("visited_stride_b"), py::arg("max_num_reqs"), py::arg("pool_size"), py::arg("stream") = 0,
          py::arg("block_dim") = 8);
    // One layer-step: sieve_update then import_multi, fused when possible (not in the reference module).
    m.def("sieve_import", &sieve_import, py::arg("topk_indices"), py::arg("req_pool_indices"), py::arg("seq_lens"),
          py::arg("prefill_lens"), py::arg("device_buffer_tokens"), py::arg("device_buffer_visited"),
          py::arg("device_buffer_ht"), py::arg("sieve_hand"), py::arg("topk_device_slots"), py::arg("is_miss"),
          py::arg("num_real"), py::arg("top_k"), py::arg("device_buffer_size"), py::arg("padded_buffer_size"),
          py::arg("visited_stride_b"), py::arg("max_num_reqs"), py::arg("pool_size"), py::arg("seg_bases"),
          py::arg("layer_offset_rows"), py::arg("per_layer_seg_rows"), py::arg("row_bytes"), py::arg("req_host_base"),
          py::arg("hot_row_base"), py::arg("stripe_rows"), py::arg("status"), py::arg("stream") = 0,
          py::arg("block_dim") = 1, py::kw_only(), py::arg("hot_req_stride_rows") = 0, py::arg("injective") = false,
          py::arg("path") = "auto", py::arg("err_word") = 0, py::arg("copy_wait_polls") = 0);
    m.def("step_prepare", [](uint32_t top_k, uint32_t dbs, uint32_t padded, uint32_t vis_stride, uint32_t max_num_reqs) {
        check(kvops_step_prepare(top_k, dbs, padded, vis_stride, max_num_reqs));
    }, py::arg("top_k"), py::arg("device_buffer_size"), py::arg("padded_buffer_size"), py::arg("visited_stride_b"),
          py::arg("max_num_reqs"));
    m.def("last_step_path", []() {
        switch (kvops_last_step_path()) {
            case KVOPS_STEP_COOP: return std::string("coop");
            case KVOPS_STEP_FUSED: return std::string("fused");
            case KVOPS_STEP_SPLIT: return std::string("split");
            default: return std::string("none");
        }
    });
    // SIEVE tier of this thread's later launches, and the tier of its last one (not in the reference module).
    m.def("set_sieve_tier", [](const std::string &tier) {
        uint32_t t;
        if (tier == "auto") t = KVOPS_TIER_AUTO;
        else if (tier == "shared") t = KVOPS_TIER_SHARED;
        else if (tier == "large") t = KVOPS_TIER_LARGE;
        else if (tier == "ordered") t = KVOPS_TIER_ORDERED;
        else throw std::invalid_argument("set_sieve_tier: tier must be 'auto', 'shared', 'large' or 'ordered'");
        check(kvops_set_sieve_tier(t));
    }, py::arg("tier"));
    m.def("last_sieve_tier", []() {
        switch (kvops_last_sieve_tier()) {
            case KVOPS_TIER_SHARED: return std::string("shared");
            case KVOPS_TIER_LARGE: return std::string("large");
            case KVOPS_TIER_ORDERED: return std::string("ordered");
            default: return std::string("none");
        }
    });
    m.def("sieve_ht_init", &sieve_ht_init, py::arg("device_buffer_tokens"), py::arg("device_buffer_ht"),
          py::arg("prefill_lens"), py::arg("req_start"), py::arg("num_reqs"), py::arg("layer_num"),
          py::arg("pool_size"), py::arg("device_buffer_size"), py::arg("padded_buffer_size"), py::arg("ht_size"),
          py::arg("stream") = 0, py::arg("block_dim") = 0);
    m.def("close", &close_module);
    // Pool plumbing (replaces the EMS control plane; not in the reference module).
    m.def("segment_alloc", &segment_alloc, py::arg("device"), py::arg("bytes"));
    m.def("segment_free", [](uint64_t a) { check(kvops_segment_free(a)); }, py::arg("addr"));
    m.def("enable_peer_access", [](int d, int p) { check(kvops_enable_peer_access(d, p)); }, py::arg("device"),
          py::arg("peer"));
    m.def("ipc_get_handle", &ipc_get_handle, py::arg("addr"));
    m.def("ipc_open_handle", &ipc_open_handle, py::arg("device"), py::arg("handle"));
    m.def("ipc_close_handle", [](uint64_t a) { check(kvops_ipc_close_handle(a)); }, py::arg("addr"));
}
