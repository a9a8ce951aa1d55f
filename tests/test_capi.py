"""The drop-in boundary without a GPU: the native library loads and exports every entry
point include/kvops_b200.h declares, the `_kvops` module mirrors the reference binding's
names, argument order and defaults (kvops/kvops_ext/kvops_ext.cpp:373-401), and calls
before init fail the way the reference's do (kvops_ext.cpp:131-136). No compute calls."""
import inspect
import os
import re

import pytest

import kv_offload_proto_b200 as kp
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "kvops_b200.h")

# (name, [(arg, default-or-None)]) of the reference binding, in order.
REFERENCE_BINDING = {
    "init": [("device_id", None), ("fatbin_path", None), ("rt_lib", "'libascendcl.so'")],
    "alloc_status": [("count", None)],
    "poll_status": [("status_addr", None), ("timeout_us", "-1")],
    "import_seg": [(a, None) for a in (
        "channel", "seg_base", "layer_offset_rows", "per_layer_seg_rows", "row_bytes", "topk_indices",
        "req_pool_indices", "req_host_base", "topk_device_slots", "is_miss", "num_real", "hot_row_base", "top_k",
        "max_num_reqs", "stripe_rows", "node_num", "my_node", "status")] + [("stream", "0"), ("block_dim", "1")],
    "export_seg_alllayer": [(a, None) for a in (
        "channel", "seg_base", "per_layer_seg_rows", "row_bytes", "row_lo", "row_cnt", "layer_num",
        "src_layer0_base", "src_layer_stride", "stripe_rows", "node_num", "my_node", "status")] + [
        ("stream", "0"), ("block_dim", "1")],
    "sieve_update": [(a, None) for a in (
        "topk_indices", "req_pool_indices", "seq_lens", "prefill_lens", "device_buffer_tokens",
        "device_buffer_visited", "device_buffer_ht", "sieve_hand", "topk_device_slots", "is_miss", "num_real",
        "top_k", "device_buffer_size", "padded_buffer_size", "visited_stride_b", "max_num_reqs", "pool_size")] + [
        ("stream", "0"), ("block_dim", "8")],
    "sieve_ht_init": [(a, None) for a in (
        "device_buffer_tokens", "device_buffer_ht", "prefill_lens", "req_start", "num_reqs", "layer_num",
        "pool_size", "device_buffer_size", "padded_buffer_size", "ht_size")] + [("stream", "0"), ("block_dim", "0")],
    "close": [],
}


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(kvops_[a-z_]+)\s*\(", text)))


def test_header_declares_exactly_the_exported_set():
    assert header_symbols() == sorted(kp.C_ABI_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = kp.load_library()
    for s in header_symbols():
        assert hasattr(lib, s), s


def _signature(fn):
    # pybind11 puts "name(arg: type = default, ...) -> ret" on the first docstring line.
    line = fn.__doc__.splitlines()[0]
    args = line[line.index("(") + 1:line.rindex(")")]
    out = []
    for part in filter(None, [p.strip() for p in args.split(",")]):
        if part == "*":
            out.append(("*", None))
            continue
        name = part.split(":")[0].strip()
        default = part.split("=", 1)[1].strip() if "=" in part else None
        out.append((name, default))
    return out


@pytest.mark.parametrize("name", sorted(REFERENCE_BINDING))
def test_binding_matches_reference(name):
    mod = kp.kvops()
    sig = _signature(getattr(mod, name))
    positional = sig[:sig.index(("*", None))] if ("*", None) in sig else sig
    assert positional == REFERENCE_BINDING[name]
    for a, d in sig[len(positional) + 1:]:
        assert d is not None, "opt-in argument {} must have a default".format(a)


def test_calls_before_init_raise():
    mod = kp.install_kvops_ext()
    import kvops_ext._kvops as alias
    assert alias is mod
    with pytest.raises(RuntimeError, match="kvops not inited"):
        mod.alloc_status(8)
    with pytest.raises(RuntimeError, match="kvops not inited"):
        mod.poll_status(64, 0)
    with pytest.raises(RuntimeError, match="kvops not inited"):
        mod.sieve_update(*([0] * 17))
    with pytest.raises(RuntimeError, match="kvops not inited"):
        mod.import_seg(*([0] * 18))


def test_init_validates_binary_path():
    mod = kp.kvops()
    with pytest.raises(RuntimeError, match="does not exist"):
        mod.init(0, "/nonexistent/kvc_kernel.o")


def test_no_cpu_fallback_in_product():
    """The package never imports the oracle; its compute entry points are the native module."""
    pkg = os.path.join(ROOT, "kv_offload_proto_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f
    assert inspect.ismodule(kp.kvops())
