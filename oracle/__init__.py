"""CPU checker for the kv_offload_proto hot path (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this
package. The shipped product (``kv_offload_proto_b200``) never does.
"""
from .oracle import *  # noqa: F401,F403
