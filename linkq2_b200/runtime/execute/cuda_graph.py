"""Decode and verify CUDA-graph families with shared capture and replay.

Same scheme as ``qslab/runtime/execute/cuda_graph.py:15-75``: graphs keyed by
rows per sequence (1 = decode, M = verify) and by batch bucket, captured largest
first into one memory pool over fixed input buffers; replay clears the buffers,
copies the step's metadata in and replays the smallest covering bucket.  Padding
rows carry ``slot = -1`` (no KV write) and ``context_len = 0`` (zero output).
Under tensor parallelism every rank captures its own graphs; the all-reduces are
captured with the kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from linkq2_b200 import _lib
from linkq2_b200.runtime.model.context import reset_context, set_context


@dataclass
class GraphFamily:
    graphs: dict
    buffers: dict


def batch_buckets(max_batch: int) -> list[int]:
    return sorted({bs for bs in [1, 2, 4, 8] + list(range(16, max_batch + 1, 16)) if bs <= max_batch}
                  | {max_batch})


class CUDAGraphs:
    def __init__(self, *, max_batch, max_model_len, block_size, hidden_size, verify_rows=1,
                 device="cuda"):
        self.max_batch = min(max_batch, 512)
        self.batch_sizes = batch_buckets(self.max_batch)
        self.blocks = (max_model_len + block_size - 1) // block_size
        self.hidden_size = hidden_size
        self.verify_rows = verify_rows
        self.device = device
        self.families: dict[int, GraphFamily] = {}
        self.kernels_per_graph: dict[tuple, int] = {}
        self.pool = None
        self.stream = torch.cuda.Stream(device=device)

    @torch.inference_mode()
    def capture(self, forward):
        dev = self.device
        for rows in dict.fromkeys([1, self.verify_rows]):
            size = self.max_batch * rows
            buffers = dict(
                input_ids=torch.zeros(size, dtype=torch.int64, device=dev),
                positions=torch.zeros(size, dtype=torch.int64, device=dev),
                slot_mapping=torch.full((size,), -1, dtype=torch.int32, device=dev),
                context_lens=torch.zeros(self.max_batch, dtype=torch.int32, device=dev),
                block_tables=torch.zeros(self.max_batch, self.blocks, dtype=torch.int32, device=dev),
                outputs=torch.zeros(size, self.hidden_size, dtype=torch.float16, device=dev),
            )
            graphs = {}
            # Warm-up and capture run on one side stream: the kernels' scratch
            # buffers are cached per stream, so the eager pass creates exactly the
            # buffers the captured launches then reuse.
            stream = self.stream
            for batch in reversed(self.batch_sizes):
                count = batch * rows
                graph = torch.cuda.CUDAGraph()
                set_context(False, slot_mapping=buffers['slot_mapping'][:count],
                            context_lens=buffers['context_lens'][:batch],
                            block_tables=buffers['block_tables'][:batch], verify_m=rows)
                stream.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(stream):
                    buffers['outputs'][:count] = forward(buffers['input_ids'][:count], buffers['positions'][:count])
                torch.cuda.synchronize()
                before = _lib.launches
                with torch.cuda.graph(graph, self.pool, stream=stream):
                    buffers['outputs'][:count] = forward(buffers['input_ids'][:count],
                                                         buffers['positions'][:count])
                self.kernels_per_graph[(rows, batch)] = _lib.launches - before
                if self.pool is None:
                    self.pool = graph.pool()
                graphs[batch] = graph
                torch.cuda.synchronize()
                reset_context()
            self.families[rows] = GraphFamily(graphs, buffers)

    def release(self):
        """Destroy the captured graphs.  Under tensor parallelism they hold the NCCL
        communicator's kernels, and the graphs must be gone before the process group
        is destroyed (or the interpreter tears it down at exit), else that teardown
        can block."""
        torch.cuda.synchronize(self.device)
        for family in self.families.values():
            family.graphs.clear()
        self.families.clear()
        self.pool = None

    def stage(self, input_ids, positions, slot_mapping, context_lens, block_tables, rows=1):
        """Copy one step's metadata into the fixed buffers; returns the batch bucket."""
        b = self.families[rows].buffers
        batch = input_ids.size(0) // rows
        count = batch * rows
        b['input_ids'][:count] = input_ids
        b['positions'][:count] = positions
        b['slot_mapping'].fill_(-1)
        b['slot_mapping'][:count] = slot_mapping
        b['context_lens'].zero_()
        b['context_lens'][:batch] = context_lens
        b['block_tables'].zero_()
        b['block_tables'][:batch, :block_tables.size(1)] = block_tables
        return next(bs for bs in self.batch_sizes if bs >= batch)

    def stage_packed(self, packed: torch.Tensor, batch: int, width: int):
        """The same as ``stage`` for a decode step whose metadata arrive as one packed
        int32 device record ``[ids | positions | slots | context lens | block tables]``:
        one kernel fills the fixed buffers, padding included (``lq2_stage_decode``)."""
        b = self.families[1].buffers
        with torch.cuda.device(self.device):
            status = _lib.lib.lq2_stage_decode(
                packed.data_ptr(), b['input_ids'].data_ptr(), b['positions'].data_ptr(),
                b['slot_mapping'].data_ptr(), b['context_lens'].data_ptr(), b['block_tables'].data_ptr(),
                batch, self.max_batch, width, self.blocks, torch.cuda.current_stream().cuda_stream)
        _lib.check(status, "lq2_stage_decode")
        _lib.count()
        return next(bs for bs in self.batch_sizes if bs >= batch)

    def run_graph(self, rows, bucket):
        self.families[rows].graphs[bucket].replay()
        _lib.count(self.kernels_per_graph[(rows, bucket)])

    def replay(self, input_ids, positions, context, rows=1):
        bucket = self.stage(input_ids, positions, context.slot_mapping, context.context_lens,
                            context.block_tables, rows)
        self.run_graph(rows, bucket)
        return self.families[rows].buffers['outputs'][:input_ids.size(0)]
