"""CUDA-graph capture of a decode step: every layer's layer-step (`DevicePool.sieve_and_read`)
captured once and replayed as one graph launch, which removes the per-launch gap between the
layers' kernels.

The captured calls publish no status words (there is no host work in a replay to zero them);
completion is the stream's. Device-side errCodes (a row past its segment, a null segment, a
cooperative copy that stopped waiting) go to one device error word shared by the captured
calls (KvopsRowOpts.err_word): `error()` reads it after a replay and `clear_error()` resets it. Everything a captured call reads is fixed at capture time: the
coordinator's batch tensors (`set_batch`), its state tensors and `self.topk` — so a decode loop
copies each step's top-K indices into `self.topk` (and refreshes the batch tensors in place)
before `replay()`. The reference has no counterpart (its driver issues the calls one by one,
xds/xds_decode.py:225-233).
"""
from typing import Optional, Sequence

__all__ = ["StepGraph"]


class StepGraph:
    """One decode step of `layers` layer-steps, captured on construction.

    pool, coord: a DevicePool and an XdsOffloadCoordinator with `set_batch` called.
    hot: per-layer hot-row buffers (hot[l] is passed to layer l's call).
    topk: optional int32 tensor [layers, max_num_reqs, top_k] to read; allocated if None.
    after_layer: optional callable(layer) whose CUDA work is captured right after that layer's
    call, e.g. a reduction of the layer's outputs (coord.is_miss, coord.top_k_device_slots),
    which the next layer overwrites.
    """

    def __init__(self, pool, coord, hot: Sequence, layers: Optional[int] = None, *, path: str = "auto",
                 block_dim: int = 1, hot_req_stride_rows: int = 0, topk=None, after_layer=None):
        import torch
        if coord._req_pool_indices is None:
            raise RuntimeError("StepGraph: call coord.set_batch() before capturing")
        self.layers = coord.layer_num if layers is None else int(layers)
        if topk is None:
            topk = torch.empty((self.layers, coord.max_num_reqs, coord.top_k), dtype=torch.int32, device=coord.device)
        if topk.dtype != torch.int32 or tuple(topk.shape) != (self.layers, coord.max_num_reqs, coord.top_k):
            raise ValueError("StepGraph: topk must be int32 [layers, max_num_reqs, top_k]")
        self.topk = topk
        k = pool._k
        # The first call of a shape sets up device scratch and kernel limits; do that now,
        # outside the capture.
        k.step_prepare(coord.top_k, coord.device_buffer_size, coord.padded_buffer_size, coord.visited_stride_b,
                       coord.max_num_reqs)
        self.err = torch.zeros(1, dtype=torch.int32, device=coord.device)
        self.graph = torch.cuda.CUDAGraph()
        self.stream = torch.cuda.Stream(device=coord.device)
        with torch.cuda.graph(self.graph, stream=self.stream):
            s = self.stream.cuda_stream
            for layer in range(self.layers):
                pool.sieve_and_read(coord, layer, self.topk[layer], hot[layer], s, block_dim,
                                    hot_req_stride_rows=hot_req_stride_rows, path=path, publish=False,
                                    err_word=self.err)
                if after_layer is not None:
                    after_layer(layer)
        self.path = k.last_step_path()

    def replay(self) -> None:
        """Runs the captured step on the current stream."""
        self.graph.replay()

    def error(self) -> int:
        """First errCode any replay since the last clear_error() recorded (0: none); waits for
        the replays queued on the current stream."""
        return int(self.err.item()) & 0xFFFFFFFF

    def clear_error(self) -> None:
        self.err.zero_()
