"""SIEVE coordinator on CUDA: the B200 counterpart of the reference's caller
``xds.xds_offload.XdsOffloadCoordinator`` (xds/xds_offload.py:20-106).

Same constructor, attributes and methods, so code written against the reference's
coordinator runs unchanged with ``device="cuda:N"``. The per-layer SIEVE state lives in
HBM with the reference's tensor layout (xds/xds_offload.py:43-53) and every update goes
through the `_kvops` launch module (sieve_ht_init / sieve_update); nothing here runs the
SIEVE on the host.
"""
import contextlib

import torch

from . import kvops as _kvops_module

__all__ = ["XdsOffloadCoordinator", "align", "compute_ht_size"]


def align(v, a):
    """Round v up to a multiple of a (xds/xds_ems_pool.py:50-51)."""
    return (v + a - 1) // a * a


def compute_ht_size(padded_buffer_size, top_k):
    """Power of two >= max(1024, 2*(padded+topK)): load factor <= 0.5
    (xds/xds_ems_pool.py:42-47; kvops_ext.cpp:297-300)."""
    p = 1024
    while p < 2 * (padded_buffer_size + top_k):
        p <<= 1
    return p


class XdsOffloadCoordinator:
    """Per-layer SIEVE state and decode-step driver for one device."""

    _require_cuda = True  # the kernels take device addresses (a host-only test subclass may lift this)

    def __init__(self, device, layer_num, pool_size, device_buffer_size, top_k, max_num_reqs, max_context_len):
        self._k = _kvops_module()
        self.device = torch.device(device)
        if self._require_cuda and self.device.type != "cuda":
            raise ValueError("XdsOffloadCoordinator needs a CUDA device, got {}".format(device))
        self.layer_num = layer_num
        self.pool_size = pool_size
        self.device_buffer_size = device_buffer_size
        self.top_k = top_k
        self.max_num_reqs = max_num_reqs
        self.max_context_len = max_context_len
        # Derived sizes (xds_offload.py:33-37).
        self.padded_buffer_size = align(device_buffer_size, 16)
        self.visited_stride_b = align((self.padded_buffer_size + 7) // 8, 64)
        self.ht_size = compute_ht_size(self.padded_buffer_size, top_k)
        L, p, padded, dev = layer_num, pool_size, self.padded_buffer_size, self.device
        self.device_buffer_tokens = torch.full((L, p, padded), -1, dtype=torch.int32, device=dev)
        self.device_buffer_visited = torch.zeros((L, p, self.visited_stride_b), dtype=torch.uint8, device=dev)
        # int16 storage, uint16 semantics (the kernel reinterprets the bits).
        self.device_buffer_ht = torch.zeros((L, p, self.ht_size), dtype=torch.int16, device=dev)
        self.sieve_hand = torch.zeros((L, p, 16), dtype=torch.int32, device=dev)
        self.prefill_lens = torch.zeros(p, dtype=torch.int32, device=dev)
        self.req_host_base = torch.zeros(max_num_reqs, dtype=torch.int64, device=dev)
        self.top_k_device_slots = torch.zeros((max_num_reqs, top_k), dtype=torch.int32, device=dev)
        self.is_miss = torch.zeros((max_num_reqs, top_k), dtype=torch.int8, device=dev)
        self.num_real = torch.zeros(1, dtype=torch.int32, device=dev)
        self._req_pool_indices = None
        self._seq_lens = None

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream if self.device.type == "cuda" else 0

    def _on_device(self):
        return torch.cuda.device(self.device) if self.device.type == "cuda" else contextlib.nullcontext()

    def admit_request(self, req_batch_idx, req_pool_idx, prefill_len, host_base_row):
        """Identity admission: slot s holds token s for s < min(prefill, dbs), then the
        tables of every layer are rebuilt on the device (xds_offload.py:56-77)."""
        if not 0 <= req_pool_idx < self.pool_size:
            raise ValueError("req_pool_idx out of range: {}".format(req_pool_idx))
        if not 0 <= req_batch_idx < self.max_num_reqs:
            raise ValueError("req_batch_idx out of range: {}".format(req_batch_idx))
        n = min(prefill_len, self.device_buffer_size)
        with self._on_device():
            self.device_buffer_tokens[:, req_pool_idx, :] = -1
            self.device_buffer_tokens[:, req_pool_idx, :n] = torch.arange(n, dtype=torch.int32, device=self.device)
            self.device_buffer_visited[:, req_pool_idx, :].zero_()
            self.sieve_hand[:, req_pool_idx, :].zero_()
            self.prefill_lens[req_pool_idx] = prefill_len
            self.req_host_base[req_batch_idx] = host_base_row
            self._k.sieve_ht_init(self.device_buffer_tokens.data_ptr(), self.device_buffer_ht.data_ptr(),
                                  self.prefill_lens.data_ptr(), req_pool_idx, 1, self.layer_num, self.pool_size,
                                  self.device_buffer_size, self.padded_buffer_size, self.ht_size, self._stream(),
                                  self.layer_num)

    def admit_all(self, prefill_lens, host_base_rows):
        """Admit pool rows 0..n-1 (batch row r = pool row r) with one table build."""
        n = len(prefill_lens)
        pre = torch.as_tensor(prefill_lens, dtype=torch.int32, device=self.device)
        with self._on_device():
            idx = torch.arange(self.padded_buffer_size, dtype=torch.int32, device=self.device)
            lim = torch.clamp(pre, max=self.device_buffer_size)[:, None]
            rows = torch.where(idx[None, :] < lim, idx[None, :], torch.full_like(idx[None, :], -1))
            self.device_buffer_tokens[:, :n, :] = rows[None]
            self.device_buffer_visited[:, :n, :].zero_()
            self.sieve_hand[:, :n, :].zero_()
            self.prefill_lens[:n] = pre
            self.req_host_base[:n] = torch.as_tensor(host_base_rows, dtype=torch.int64, device=self.device)
            self._k.sieve_ht_init(self.device_buffer_tokens.data_ptr(), self.device_buffer_ht.data_ptr(),
                                  self.prefill_lens.data_ptr(), 0, n, self.layer_num, self.pool_size,
                                  self.device_buffer_size, self.padded_buffer_size, self.ht_size, self._stream(), 0)

    def set_batch(self, req_pool_indices, seq_lens):
        """Batch context for the next decode steps (xds_offload.py:79-87)."""
        if req_pool_indices.dtype != torch.int64:
            raise ValueError("req_pool_indices must be int64")
        if seq_lens.dtype != torch.int32:
            seq_lens = seq_lens.to(torch.int32)
        self._req_pool_indices = req_pool_indices
        self._seq_lens = seq_lens
        self.num_real[0] = req_pool_indices.shape[0]

    def sieve_update(self, layer_id, topk_indices, block_dim=8, stream=None):
        """SIEVE miss detection for one layer (xds_offload.py:90-101)."""
        if topk_indices.dtype != torch.int32:
            raise ValueError("topk_indices must be int32")
        self._k.sieve_update(topk_indices.data_ptr(), self._req_pool_indices.data_ptr(), self._seq_lens.data_ptr(),
                             self.prefill_lens.data_ptr(), self.device_buffer_tokens[layer_id].data_ptr(),
                             self.device_buffer_visited[layer_id].data_ptr(),
                             self.device_buffer_ht[layer_id].data_ptr(), self.sieve_hand[layer_id].data_ptr(),
                             self.top_k_device_slots.data_ptr(), self.is_miss.data_ptr(), self.num_real.data_ptr(),
                             self.top_k, self.device_buffer_size, self.padded_buffer_size, self.visited_stride_b,
                             self.max_num_reqs, self.pool_size, self._stream() if stream is None else stream,
                             block_dim)

    def miss_count(self):
        """Device-side miss count tensor (xds_offload.py:103-106)."""
        return self.is_miss.sum()
