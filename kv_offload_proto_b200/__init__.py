"""kv_offload_proto_b200 — B200-native decode-time KV hot path of kv_offload_proto.

The product is the native library ``libkvops_b200.so`` (CUDA sm_100a kernels behind the
C ABI in ``include/kvops_b200.h``) and its Python module ``kvops_ext._kvops``, a drop-in
for the reference's launch extension (kvops/kvops_ext/kvops_ext.cpp). There is no CPU
fallback: importing the module without the built extension raises.
"""
import ctypes
import importlib
import os
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libkvops_b200.so")

__all__ = ["kvops", "load_library", "install_kvops_ext", "LIB_PATH", "C_ABI_SYMBOLS"]

# Every entry point declared in include/kvops_b200.h.
C_ABI_SYMBOLS = (
    "kvops_last_error", "kvops_init", "kvops_close", "kvops_alloc_status", "kvops_poll_status",
    "kvops_import_seg", "kvops_import_seg_ex", "kvops_import_multi", "kvops_export_seg_alllayer",
    "kvops_export_seg_alllayer_ex", "kvops_sieve_update", "kvops_sieve_ht_init", "kvops_segment_alloc",
    "kvops_segment_free", "kvops_enable_peer_access", "kvops_ipc_get_handle", "kvops_ipc_open_handle",
    "kvops_ipc_close_handle", "kvops_import_multi_noalloc", "kvops_sieve_import",
    "kvops_last_step_path", "kvops_step_prepare", "kvops_export_seg", "kvops_set_sieve_tier",
    "kvops_last_sieve_tier",
)

_lib = None


def load_library():
    """ctypes handle of libkvops_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("libkvops_b200.so is not built; run `python -m kv_offload_proto_b200._build`")
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.kvops_last_error.restype = ctypes.c_char_p
    return _lib


def kvops():
    """The `_kvops` module (raises ImportError if the extension is not built)."""
    try:
        return importlib.import_module("kv_offload_proto_b200.kvops_ext._kvops")
    except ImportError as e:
        raise ImportError("kv_offload_proto_b200: the CUDA extension _kvops is not built "
                          "(python -m kv_offload_proto_b200._build): {}".format(e)) from e


def install_kvops_ext():
    """Register this package's module under the reference's name ``kvops_ext._kvops``."""
    mod = kvops()
    pkg = importlib.import_module("kv_offload_proto_b200.kvops_ext")
    sys.modules.setdefault("kvops_ext", pkg)
    sys.modules["kvops_ext._kvops"] = mod
    return mod
