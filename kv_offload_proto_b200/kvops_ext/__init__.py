"""Drop-in for the reference's ``kvops_ext`` package (kvops/kvops_ext/__init__.py).

``from kv_offload_proto_b200.kvops_ext import _kvops`` gives the B200 launch module;
``kv_offload_proto_b200.install_kvops_ext()`` also registers it under the reference's
import name ``kvops_ext._kvops`` so that unmodified callers (xds_offload, xds_ems_pool)
bind to it.
"""
