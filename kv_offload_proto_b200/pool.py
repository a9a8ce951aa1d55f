"""Striped row pool on B200s: the data-path half of the reference's ``EmsPool``
(xds/xds_ems_pool.py:115-241) with the remote-DRAM segments replaced by
  * HBM of this or a peer GPU (read/written in-kernel over NVLink/NVSwitch via UVA), or
  * pinned, mapped host memory (read/written in-kernel over the host link).

Segment s holds layer-major rows ``[layer][per_layer_seg_rows][row_bytes]`` for the rows
owned by node s under the unchanged stripe map node=(row/S)%N, segRow=(row/S)/N
(kvops/kernel/kvc_common.h:81-89; common/kv_layout.h:4-9). batch_read / batch_write_alllayers
/ wait / next_status keep EmsPool's signatures; the EMS control plane (TCP master, HCOMM
channels) is replaced by local allocation, peer access, or CUDA IPC handles for segments
owned by other processes.
"""
import bisect
from typing import List, Optional, Sequence

from . import kvops as _kvops_module

__all__ = ["DevicePool", "RowAllocator", "per_layer_seg_rows", "per_layer_seg_rows_injective", "node_of",
           "seg_row_of", "device_view"]


class _CudaArray:
    """Minimal __cuda_array_interface__ wrapper of a raw UVA address (uint8, 1-D)."""

    def __init__(self, addr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False),
                                         "version": 3, "strides": None}


def device_view(addr, nbytes, device):
    """uint8 torch tensor aliasing `nbytes` of device (or mapped host) memory at `addr`,
    e.g. a segment from segment_alloc or an IPC mapping; the memory is not owned."""
    import torch
    return torch.as_tensor(_CudaArray(addr, nbytes), device=device)


def per_layer_seg_rows(layer_rows, node_num):
    """ceil(layer_rows / N) (common/kv_layout.h:19-22; xds_ems_pool.py:159)."""
    return (layer_rows + node_num - 1) // node_num


def per_layer_seg_rows_injective(layer_rows, stripe_rows, node_num):
    """Rows per layer per segment for the opt-in injective map: ceil(ceil(rows/S)/N)*S."""
    stripes = (layer_rows + stripe_rows - 1) // stripe_rows
    return (stripes + node_num - 1) // node_num * stripe_rows


def node_of(row, stripe_rows, node_num):
    return 0 if stripe_rows == 0 else (row // stripe_rows) % node_num


def seg_row_of(row, stripe_rows, node_num, injective=False):
    if stripe_rows == 0:
        return row
    g = row // stripe_rows
    return (g // node_num) * stripe_rows + row % stripe_rows if injective else g // node_num


class RowAllocator:
    """Host-side pool-row allocator with the reference's contiguity contract
    (xds/xds_ems_pool.py:54-106): a request's rows must be contiguous when that is possible,
    because the gather addresses them as req_host_base + position. alloc(n) returns the first
    free run (in row order) that holds n rows; when none does, the n lowest free rows.

    Free space is kept as two sorted parallel lists (run starts, run ends), so freeing a row
    merges it with its neighbours by bisection instead of re-sorting every run. Freeing a row
    that is already free raises ValueError (the reference would count it twice)."""

    def __init__(self, capacity: int):
        if capacity < 0:
            raise ValueError("capacity must be >= 0")
        self.capacity = capacity
        self._lo: List[int] = [0] if capacity else []  # run starts, ascending
        self._hi: List[int] = [capacity] if capacity else []  # matching exclusive ends
        self._nfree = capacity

    def alloc(self, n: int) -> List[int]:
        if n <= 0:
            raise ValueError("n must be > 0")
        if n > self._nfree:
            raise MemoryError("allocator exhausted: free={} need={}".format(self._nfree, n))
        self._nfree -= n
        for i in range(len(self._lo)):
            lo, hi = self._lo[i], self._hi[i]
            if hi - lo >= n:  # first run that fits: one contiguous block
                if hi - lo == n:
                    del self._lo[i], self._hi[i]
                else:
                    self._lo[i] = lo + n
                return list(range(lo, lo + n))
        out: List[int] = []  # fragmented: the lowest free rows, whole runs first
        while len(out) < n:
            lo, hi = self._lo[0], self._hi[0]
            take = min(hi - lo, n - len(out))
            out.extend(range(lo, lo + take))
            if take == hi - lo:
                del self._lo[0], self._hi[0]
            else:
                self._lo[0] = lo + take
        return out

    def free(self, rows: List[int]) -> None:
        rows = list(rows)
        for r in rows:
            if r < 0 or r >= self.capacity:
                raise ValueError("row out of range: {}".format(r))
        if len(set(rows)) != len(rows):
            raise ValueError("row freed twice in one call")
        for r in rows:
            if self._is_free(r):
                raise ValueError("row {} is not allocated".format(r))
        for r in sorted(rows):
            self._insert(r)
        self._nfree += len(rows)

    def _is_free(self, r: int) -> bool:
        i = bisect.bisect_right(self._lo, r) - 1
        return i >= 0 and r < self._hi[i]

    def _insert(self, r: int) -> None:
        i = bisect.bisect_right(self._lo, r)  # runs [0, i) start at or before r
        joins_left = i > 0 and self._hi[i - 1] == r
        joins_right = i < len(self._lo) and self._lo[i] == r + 1
        if joins_left and joins_right:
            self._hi[i - 1] = self._hi[i]
            del self._lo[i], self._hi[i]
        elif joins_left:
            self._hi[i - 1] = r + 1
        elif joins_right:
            self._lo[i] = r
        else:
            self._lo.insert(i, r)
            self._hi.insert(i, r + 1)

    def free_runs(self) -> List[tuple]:
        """The free rows as sorted, disjoint, non-adjacent half-open runs."""
        return list(zip(self._lo, self._hi))

    def free_rows(self) -> int:
        return self._nfree

    def used_rows(self) -> int:
        return self.capacity - self._nfree


class DevicePool:
    """Pool of `node_num` segments, each on a device id (>= 0) or pinned host memory (-1).

    segment_devices[s] places segment s. Segments are allocated here unless
    `segment_addrs` gives existing UVA addresses (e.g. opened from other processes' IPC
    handles), in which case this object does not own them.
    """

    def __init__(self, device_id: int, layer_num: int, layer_rows: int, row_bytes: int, stripe_rows: int = 1,
                 segment_devices: Sequence[int] = (0,), segment_addrs: Optional[Sequence[int]] = None,
                 injective: bool = False):
        if layer_num < 1 or layer_rows < 1 or row_bytes <= 0 or row_bytes % 128 != 0:
            raise ValueError("invalid pool dims: L={} rows={} rowBytes={}".format(layer_num, layer_rows, row_bytes))
        n = len(segment_devices) if segment_addrs is None else len(segment_addrs)
        if not 1 <= n <= 64:
            raise ValueError("node count must be in [1, 64], got {}".format(n))
        if stripe_rows < 0:
            raise ValueError("stripe_rows must be >= 0")
        self._k = _kvops_module()
        self.device_id = device_id
        self.layer_num = layer_num
        self.layer_rows = layer_rows
        self.row_bytes = row_bytes
        self.stripe_rows = stripe_rows
        self.injective = injective
        self.node_num = n
        if injective and stripe_rows > 0:
            self.per_layer_seg_rows = per_layer_seg_rows_injective(layer_rows, stripe_rows, n)
        else:
            self.per_layer_seg_rows = per_layer_seg_rows(layer_rows, n)
        self.segment_bytes = layer_num * self.per_layer_seg_rows * row_bytes
        self.channels = [0] * n  # seg_base is directly dereferenceable (UVA)
        self._owned = []
        if segment_addrs is None:
            self.segment_devices = list(segment_devices)
            self.seg_bases = []
            for d in self.segment_devices:
                if d >= 0 and d != device_id:
                    self._k.enable_peer_access(device_id, d)
                a = self._k.segment_alloc(d, self.segment_bytes)
                self._owned.append(a)
                self.seg_bases.append(a)
        else:
            self.segment_devices = list(segment_devices) if segment_devices else [-2] * n
            self.seg_bases = list(segment_addrs)
        self._status_count = 8 * n
        self._status_base = self._k.alloc_status(self._status_count)
        self._status_cursor = 0

    def next_status(self) -> int:
        """Round-robin 64-byte status slot (xds_ems_pool.py:182-185)."""
        addr = self._status_base + self._status_cursor * 64
        self._status_cursor = (self._status_cursor + 1) % self._status_count
        return addr

    def make_allocator(self) -> RowAllocator:
        return RowAllocator(self.layer_rows)

    def seg_addr(self, node, layer, row):
        """Byte address of (layer, row) inside node's segment (test/kv_layout_ref.py:19-24)."""
        sr = seg_row_of(row, self.stripe_rows, self.node_num, self.injective)
        return self.seg_bases[node] + (layer * self.per_layer_seg_rows + sr) * self.row_bytes

    def batch_read(self, layer_id, topk_indices, req_pool_indices, req_host_base, topk_device_slots, is_miss,
                   num_real, hot_row_base, max_num_reqs, top_k, stream=0, block_dim=1, *, fused=True,
                   hot_req_stride_rows=0) -> int:
        """Gather the miss rows of one layer from every segment (xds_ems_pool.py:204-217).

        fused=True issues one launch over all segments (import_multi); fused=False issues the
        reference's one import_seg launch per segment. Both publish the same status pages."""
        status = self.next_status()
        off = layer_id * self.per_layer_seg_rows
        a = [_ptr(topk_indices), _ptr(req_pool_indices), _ptr(req_host_base), _ptr(topk_device_slots),
             _ptr(is_miss), _ptr(num_real), _ptr(hot_row_base)]
        if fused:
            self._k.import_multi(self.seg_bases, off, self.per_layer_seg_rows, self.row_bytes, *a, top_k, max_num_reqs,
                                 self.stripe_rows, status, stream, block_dim, hot_req_stride_rows=hot_req_stride_rows,
                                 injective=self.injective)
        else:
            for s in range(self.node_num):
                self._k.import_seg(self.channels[s], self.seg_bases[s], off, self.per_layer_seg_rows, self.row_bytes,
                                   *a, top_k, max_num_reqs, self.stripe_rows, self.node_num, s, status, stream,
                                   block_dim, hot_req_stride_rows=hot_req_stride_rows, injective=self.injective)
        return status

    def sieve_and_read(self, coord, layer_id, topk_indices, hot_row_base, stream=0, block_dim=1, *,
                       hot_req_stride_rows=0, path="auto", publish=True, err_word=0, copy_wait_polls=0) -> int:
        """One decode layer-step in one call: `coord.sieve_update(layer_id, topk_indices)`
        followed by `batch_read` of its miss rows from every segment (the reference driver's
        pair, xds_decode.py:225-233), with identical results (kvops_sieve_import). path="auto"
        runs one kernel that copies each request's miss rows during its table update when a
        segment is on another GPU, and the two kernels (the gather launched as a programmatic
        dependent) otherwise; "coop" / "fused" / "split" force one. Returns the status address for
        `wait`, or 0 with publish=False: then no status words are written and completion is
        observed on the stream (the form a CUDA graph can replay, see graph.StepGraph).
        err_word: address (or int32 tensor) of a word that receives the first device-side
        errCode by compare-and-swap from 0 (KvopsRowOpts.err_word); copy_wait_polls: bound of a
        cooperative copy CTA's wait for a walk list (KvopsRowOpts.copy_wait_polls, 0 = default)."""
        import torch
        if topk_indices.dtype != torch.int32:
            raise ValueError("topk_indices must be int32")
        status = self.next_status() if publish else 0
        self._k.sieve_import(
            _ptr(topk_indices), _ptr(coord._req_pool_indices), _ptr(coord._seq_lens), _ptr(coord.prefill_lens),
            _ptr(coord.device_buffer_tokens[layer_id]), _ptr(coord.device_buffer_visited[layer_id]),
            _ptr(coord.device_buffer_ht[layer_id]), _ptr(coord.sieve_hand[layer_id]), _ptr(coord.top_k_device_slots),
            _ptr(coord.is_miss), _ptr(coord.num_real), coord.top_k, coord.device_buffer_size,
            coord.padded_buffer_size, coord.visited_stride_b, coord.max_num_reqs, coord.pool_size, self.seg_bases,
            layer_id * self.per_layer_seg_rows, self.per_layer_seg_rows, self.row_bytes, _ptr(coord.req_host_base),
            _ptr(hot_row_base), self.stripe_rows, status, stream, block_dim, hot_req_stride_rows=hot_req_stride_rows,
            injective=self.injective, path=path, err_word=_ptr(err_word), copy_wait_polls=copy_wait_polls)
        return status

    def batch_write(self, layer_id, topk_indices, req_pool_indices, req_host_base, topk_device_slots, export_flags,
                    num_real, hot_row_base, max_num_reqs, top_k, stream=0, block_dim=1, *, hot_req_stride_rows=0) -> int:
        """Export one layer's flagged hot rows to their pool rows (kvc_scatter_rows, the single-layer
        decode-increment export of doc/kv_offload_design.md:394-396): batch_read's arguments and
        rules in the opposite direction, one launch per segment. Returns the status address."""
        status = self.next_status()
        off = layer_id * self.per_layer_seg_rows
        a = [_ptr(topk_indices), _ptr(req_pool_indices), _ptr(req_host_base), _ptr(topk_device_slots),
             _ptr(export_flags), _ptr(num_real), _ptr(hot_row_base)]
        for s in range(self.node_num):
            self._k.export_seg(self.channels[s], self.seg_bases[s], off, self.per_layer_seg_rows, self.row_bytes, *a,
                               top_k, max_num_reqs, self.stripe_rows, self.node_num, s, status, stream, block_dim,
                               hot_req_stride_rows=hot_req_stride_rows, injective=self.injective)
        return status

    def batch_write_alllayers(self, row_lo, row_cnt, src_layer0_base, src_layer_stride, stream=0, block_dim=1) -> int:
        """Export rows [row_lo, row_lo+row_cnt) of every layer to their segments
        (xds_ems_pool.py:220-230): one launch per segment, as in the reference."""
        status = self.next_status()
        for s in range(self.node_num):
            self._k.export_seg_alllayer(self.channels[s], self.seg_bases[s], self.per_layer_seg_rows, self.row_bytes,
                                        row_lo, row_cnt, self.layer_num, _ptr(src_layer0_base), src_layer_stride,
                                        self.stripe_rows, self.node_num, s, status, stream, block_dim,
                                        injective=self.injective)
        return status

    def wait(self, status, timeout_us=60_000_000, block_dim=1) -> None:
        """Wait for every node's status words (xds_ems_pool.py:233-241)."""
        for s in range(self.node_num):
            for b in range(block_dim):
                rc = self._k.poll_status(status + s * 64 + b * 8, timeout_us)
                if rc != 0:
                    raise RuntimeError("kv op failed on node {} block {}: errCode=0x{:x}".format(
                        s, b, rc & 0xFFFFFFFF))

    def destroy(self) -> None:
        for a in self._owned:
            self._k.segment_free(a)
        self._owned = []
        self.seg_bases = []


def _ptr(x):
    if isinstance(x, int):
        return x
    dp = getattr(x, "data_ptr", None)
    if dp is None:
        raise TypeError("expect tensor or int address, got {}".format(type(x)))
    return dp()
