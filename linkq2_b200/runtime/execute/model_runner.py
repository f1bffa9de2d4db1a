"""Model runner: KV pool allocation and binding, batch preparation from pinned
host memory, eager or CUDA-graph execution, greedy sampling.

Follows ``qslab/runtime/execute/model_runner.py``: pool shapes and dtypes of
``:146-156``, SmoothAttention / K-scale binding of ``:169-187``, decode and
verify batch preparation of ``:262-314``, prefill preparation with the
pool-resident prefix plan of ``:194-260``, execution and sampling of
``:356-403``.  With tensor parallelism each rank runs the same host code on the
same inputs and holds ``kv_heads / t`` heads of every pool tensor.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from linkq2_b200.kernels.gemlite.ops import set_constant_weights
from linkq2_b200.runtime.execute.cuda_graph import CUDAGraphs
from linkq2_b200.runtime.model.attention import LONG_PROMPT
from linkq2_b200.runtime.model.context import get_context, reset_context, set_context
from linkq2_b200.runtime.parallel import get_tp
from linkq2_b200.runtime.state import Sequence


@dataclass
class RunnerConfig:
    kvcache_block_size: int = 256        # must be a multiple of 128 for kv4 (config.py:68-70)
    num_kvcache_blocks: int = 0
    v_group: int = 64
    max_num_seqs: int = 32
    max_model_len: int = 4096
    enforce_eager: bool = True
    spec_num_drafts: int = 0             # verify graphs with M = drafts + 1 rows when > 0


class ModelRunner:
    def __init__(self, model, config: RunnerConfig, *, smooth_kv: dict | None = None, device="cuda:0"):
        if config.kvcache_block_size % 128:
            raise ValueError("kv4 needs kvcache_block_size to be a multiple of 128")
        if config.num_kvcache_blocks <= 0:
            raise ValueError("no memory available for KV blocks")
        self.model, self.config, self.device = model, config, torch.device(device)
        self.block_size = config.kvcache_block_size
        self.tp = get_tp()
        self.graph_replays = 0
        self.last_logits = None
        self.keep_logits = False          # True: every step also gathers the full logits into last_logits
        self.temperature = 0.0            # 0: greedy; a float or one value per row
        self.sample_generator = None      # torch.Generator on the device, for seeded sampling
        self._pinned = self._pinned_np = self._packed_dev = None
        self.allocate_kv_cache()
        self.load_smoothing(smooth_kv)
        # The checkpoint is loaded and nothing writes the quantized weights from here on:
        # let the linear kernels fetch them ahead of stream order (before graph capture,
        # which records the setting with each launch).
        torch.cuda.synchronize(self.device)
        set_constant_weights(True)
        self.cuda_graphs = None
        if not config.enforce_eager:
            self.cuda_graphs = CUDAGraphs(
                max_batch=config.max_num_seqs, max_model_len=config.max_model_len,
                block_size=self.block_size, hidden_size=model.config.hidden_size,
                verify_rows=config.spec_num_drafts + 1, device=self.device)
            self.cuda_graphs.capture(self._forward)

    def check_exchange(self):
        """Raise if a wait of the tensor-parallel exchange kernels has run out since the library
        was loaded (their results were invalid then).  Synchronises the device."""
        if self.tp.exchange is not None:
            self.tp.exchange.check()

    def shutdown(self):
        """Release the CUDA graphs (call on every rank before the process group is
        destroyed; harmless otherwise)."""
        if self.cuda_graphs is not None:
            self.cuda_graphs.release()
            self.cuda_graphs = None

    # ---- pool ---------------------------------------------------------------
    def allocate_kv_cache(self):
        cfg, mc = self.config, self.model.config
        hkv = mc.num_key_value_heads // self.tp.size
        d, nw, ng = mc.head_dim, mc.head_dim // 8, mc.head_dim // cfg.v_group
        slots = cfg.num_kvcache_blocks * self.block_size
        self.kv_cache = []
        for _ in range(mc.num_hidden_layers):
            kq = torch.zeros(slots, hkv, nw, dtype=torch.uint32, device=self.device)
            ks = torch.zeros(hkv, d, dtype=torch.float16, device=self.device)
            vq = torch.zeros(slots, hkv, nw, dtype=torch.uint32, device=self.device)
            vs = torch.zeros(slots, hkv, ng, dtype=torch.float16, device=self.device)
            self.kv_cache.append(((kq, ks), (vq, vs)))
        layer_id = 0
        for module in self.model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                module.k_cache, module.v_cache = self.kv_cache[layer_id]
                module.v_group, module.block_n, module.kv_cache_dtype = cfg.v_group, self.block_size, 'kv4'
                layer_id += 1

    def load_smoothing(self, ck: dict | None):
        """``{'lambda': [L, HKV, D], 'kscale': [L, HKV, D]}`` over all KV heads;
        each rank keeps its heads.  KV4 requires a calibration (config.py:64-65)."""
        if ck is None:
            raise ValueError("the KV4 cache needs a SmoothAttention / K-scale calibration")
        mc = self.model.config
        expected = (mc.num_hidden_layers, mc.num_key_value_heads, mc.head_dim)
        lam, kscale = ck["lambda"].float(), ck["kscale"].float()
        for name, tensor in (("lambda", lam), ("kscale", kscale)):
            stored = tensor.half()
            if tuple(tensor.shape) != expected or not torch.isfinite(stored).all() or (stored <= 0).any():
                raise ValueError(f"{name} must have shape {expected} and finite positive FP16 values")
        hkv = mc.num_key_value_heads // self.tp.size
        heads = slice(self.tp.rank * hkv, (self.tp.rank + 1) * hkv)
        unit = bool((lam == 1).all())
        layer_id = 0
        for module in self.model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                if not unit:
                    module.set_smooth_lambda(lam[layer_id, heads].to(self.device))
                module.k_cache[1].copy_(kscale[layer_id, heads].half())
                layer_id += 1

    # ---- batch preparation ----------------------------------------------------
    def _h2d(self, data, dtype):
        return torch.tensor(data, dtype=dtype, pin_memory=True).to(self.device, non_blocking=True)

    def prepare_block_tables(self, seqs):
        width = max(len(seq.block_table) for seq in seqs)
        return self._h2d([seq.block_table + [-1] * (width - len(seq.block_table)) for seq in seqs], torch.int32)

    def prepare_decode(self, seqs: list[Sequence]):
        input_ids = self._h2d([seq.last_token for seq in seqs], torch.int64)
        positions = self._h2d([len(seq) - 1 for seq in seqs], torch.int64)
        slot_mapping = self._h2d([seq.slot(len(seq) - 1) for seq in seqs], torch.int32)
        context_lens = self._h2d([len(seq) for seq in seqs], torch.int32)
        set_context(False, slot_mapping=slot_mapping, context_lens=context_lens,
                    block_tables=self.prepare_block_tables(seqs))
        return input_ids, positions

    def prepare_verify(self, seqs: list[Sequence], drafts: list[list[int]]):
        """M = drafts + 1 rows per sequence: [last committed token, drafts...]; row m
        is position L-1+m and reads keys [0, L+m) (model_runner.py:285-314)."""
        gamma = self.config.spec_num_drafts
        m_rows = gamma + 1
        ids, pos, slots, lens = [], [], [], []
        for seq, d in zip(seqs, drafts):
            length = len(seq)
            d = list(d)[:gamma]
            ids.extend([seq.last_token] + d + [0] * (gamma - len(d)))
            pos.extend(range(length - 1, length + gamma))
            lens.append(length)
            for m in range(m_rows):
                p = length - 1 + m
                ok = m <= len(d) and p // self.block_size < len(seq.block_table)
                slots.append(seq.slot(p) if ok else -1)
        set_context(False, slot_mapping=self._h2d(slots, torch.int32), context_lens=self._h2d(lens, torch.int32),
                    block_tables=self.prepare_block_tables(seqs), verify_m=m_rows)
        return self._h2d(ids, torch.int64), self._h2d(pos, torch.int64)

    def _prefix_rows(self) -> int:
        """Query rows per block of the KV4 prefix kernel: 16, fewer when the GQA group is wider than
        four heads (the kernel holds at most 64 rows per KV head)."""
        cfg = self.model.config
        return max(1, min(16, 64 // max(1, cfg.num_attention_heads // cfg.num_key_value_heads)))

    def prepare_prefill(self, seqs: list[Sequence], counts: list[int]):
        """Schedule ``counts[i]`` prompt tokens of each sequence after its cached prefix.  The
        prefix stays in the int4 pool: the new rows are cut into blocks for the prefix kernel
        (the reference restores the prefix to fp16 instead,
        ``qslab/runtime/execute/model_runner.py:232-263``)."""
        ids, pos, slots, cu_q, cu_k = [], [], [], [0], [0]
        plan, q_off = [], 0
        rows, block_seq, lens, first, where = [], [], [], [], []
        r = self._prefix_rows()
        for i, (seq, n) in enumerate(zip(seqs, counts)):
            start, end = seq.num_cached_tokens, seq.num_cached_tokens + n
            ids.extend(seq.token_ids[start:end])
            pos.extend(range(start, end))
            slots.extend(seq.slot(p) for p in range(start, end))
            cu_q.append(cu_q[-1] + n)
            cu_k.append(cu_k[-1] + end)
            plan.append((start, q_off, q_off + n))
            first.extend([q_off] * n)
            if start > 0:
                for b0 in range(q_off, q_off + n, r):
                    real = list(range(b0, min(b0 + r, q_off + n)))
                    where.extend(range(len(rows), len(rows) + len(real)))
                    rows.extend(real + [q_off] * (r - len(real)))
                    block_seq.append(i)
                    lens.append(start)
            else:
                where.extend([-1 if n <= LONG_PROMPT else -2] * n)
            q_off += n
        extra = dict(prefix_plan=plan, chunk_first=self._h2d(first, torch.int32),
                     chunk_prefix=self._h2d(where, torch.int32))
        tables = None
        if rows:
            tables = self.prepare_block_tables(seqs)
            extra.update(prefix_rows=self._h2d(rows, torch.int64),
                         prefix_tables=tables[self._h2d(block_seq, torch.int64)].contiguous(),
                         prefix_lens=self._h2d(lens, torch.int32))
        set_context(True, self._h2d(cu_q, torch.int32), self._h2d(cu_k, torch.int32),
                    max(counts), max(c[0] + (c[2] - c[1]) for c in plan),
                    self._h2d(slots, torch.int32), None, tables, **extra)
        return self._h2d(ids, torch.int64), self._h2d(pos, torch.int64)

    # ---- execution ------------------------------------------------------------
    def _forward(self, input_ids, positions):
        return self.model(input_ids, positions)

    @torch.inference_mode()
    def run_model(self, input_ids, positions, is_prefill, *, rows=1):
        graphs = self.cuda_graphs
        if is_prefill or graphs is None or input_ids.size(0) // rows > max(graphs.batch_sizes) \
                or rows not in graphs.families:
            return self._forward(input_ids, positions)
        self.graph_replays += 1
        return graphs.replay(input_ids, positions, get_context(), rows)

    @torch.inference_mode()
    def run(self, seqs: list[Sequence], is_prefill: bool, counts: list[int] | None = None) -> list[int]:
        """One step; returns one greedy token per sequence (for prefill: the token
        after the last scheduled position)."""
        self.tp.guard()                      # a peer that has left: stop on the host, before any launch
        graphs = self.cuda_graphs
        if not is_prefill and graphs is not None and len(seqs) <= max(graphs.batch_sizes):
            return self._finish(seqs, self._decode_packed(seqs), False, None)
        if is_prefill:
            counts = counts or [len(s) - s.num_cached_tokens for s in seqs]
            input_ids, positions = self.prepare_prefill(seqs, counts)
        else:
            input_ids, positions = self.prepare_decode(seqs)
        hidden = self.run_model(input_ids, positions, is_prefill)
        return self._finish(seqs, hidden, is_prefill, counts)

    def _graph_table_width(self, seqs, extra_tokens: int) -> int:
        """Block-table columns of a graph step: the widest table, but never more than the
        graphs were captured with (``max_model_len``); blocks a sequence holds beyond that
        cannot be addressed by a step inside the limit and are left out."""
        graphs = self.cuda_graphs
        longest = max(len(seq) for seq in seqs) + extra_tokens
        if longest > graphs.blocks * self.block_size:
            raise ValueError(f"sequence of {longest} tokens exceeds max_model_len "
                             f"({graphs.blocks * self.block_size} tokens in the captured graphs)")
        return min(max(len(seq.block_table) for seq in seqs), graphs.blocks)

    def _decode_packed(self, seqs: list[Sequence]):
        """Decode step through the graphs with one pinned record, one host-to-device copy
        and one staging kernel instead of five copies and seven staging ops."""
        graphs = self.cuda_graphs
        b = len(seqs)
        width = self._graph_table_width(seqs, 0)
        if self._pinned is None:
            cap = graphs.max_batch * (4 + graphs.blocks)
            self._pinned = torch.empty(cap, dtype=torch.int32, pin_memory=True)
            self._pinned_np = self._pinned.numpy()
            self._packed_dev = torch.empty(cap, dtype=torch.int32, device=self.device)
        rec = self._pinned_np
        rec[0:b] = [seq.last_token for seq in seqs]
        rec[b:2 * b] = [len(seq) - 1 for seq in seqs]
        rec[2 * b:3 * b] = [seq.slot(len(seq) - 1) for seq in seqs]
        rec[3 * b:4 * b] = [len(seq) for seq in seqs]
        tables = rec[4 * b:4 * b + b * width].reshape(b, width)
        for i, seq in enumerate(seqs):
            n = min(len(seq.block_table), width)
            tables[i, :n] = seq.block_table[:n]
            tables[i, n:] = -1
        n = 4 * b + b * width
        self._packed_dev[:n].copy_(self._pinned[:n], non_blocking=True)
        bucket = graphs.stage_packed(self._packed_dev, b, width)
        graphs.run_graph(1, bucket)
        self.graph_replays += 1
        return graphs.families[1].buffers['outputs'][:b]

    @torch.inference_mode()
    def run_steps(self, seqs: list[Sequence], steps: int) -> list[list[int]]:
        """``steps`` greedy decode steps in a row without a host round trip between them
        (multi-step decoding): the token ids of step i+1 are taken from step i's arg-max on
        the device, every step's positions, slots and context lengths are known in advance,
        and the tokens come back through one pinned buffer, read once at the end.  Per step
        there is still one host-to-device copy of the step's record and one device-to-host
        copy of its tokens.  Appends the tokens to the sequences and returns them per step.
        The block tables must already cover ``len(seq) + steps`` positions."""
        self.tp.guard()
        graphs = self.cuda_graphs
        b = len(seqs)
        if graphs is None or b > max(graphs.batch_sizes):
            out = []
            for _ in range(steps):
                tokens = self.run(seqs, False)
                for seq, tok in zip(seqs, tokens):
                    seq.append(tok)
                out.append(tokens)
            return out
        import numpy as np
        width = self._graph_table_width(seqs, steps - 1)
        for seq in seqs:
            if (len(seq) + steps - 1) // self.block_size >= len(seq.block_table):
                raise ValueError("run_steps needs block tables that cover every new position")
        n = 4 * b + b * width
        records = torch.empty(steps, n, dtype=torch.int32, pin_memory=True)
        rec = records.numpy()
        base = np.array([len(seq) for seq in seqs], dtype=np.int64)
        tables = np.full((b, width), -1, dtype=np.int32)
        for i, seq in enumerate(seqs):
            held = min(len(seq.block_table), width)
            tables[i, :held] = seq.block_table[:held]
        bs = self.block_size
        for i in range(steps):
            pos = base - 1 + i
            rec[i, 0:b] = [seq.last_token for seq in seqs] if i == 0 else 0
            rec[i, b:2 * b] = pos
            rec[i, 2 * b:3 * b] = tables[np.arange(b), pos // bs] * bs + pos % bs
            rec[i, 3 * b:4 * b] = base + i
            rec[i, 4 * b:] = tables.reshape(-1)
        staged = torch.empty(steps, n, dtype=torch.int32, device=self.device)
        tokens_host = torch.empty(steps, b, dtype=torch.int64, pin_memory=True)
        ids = None
        for i in range(steps):
            staged[i].copy_(records[i], non_blocking=True)
            if ids is not None:
                staged[i, :b] = ids
            bucket = graphs.stage_packed(staged[i], b, width)
            graphs.run_graph(1, bucket)
            self.graph_replays += 1
            ids = self._sample(graphs.families[1].buffers['outputs'][:b])
            tokens_host[i].copy_(ids, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        out = tokens_host.tolist()
        for row in out:
            for seq, tok in zip(seqs, row):
                seq.append(tok)
        return out

    def _finish(self, seqs, hidden, is_prefill, counts):
        if is_prefill:
            hidden = hidden[(get_context().cu_seqlens_q[1:] - 1).long()]
            for seq, n in zip(seqs, counts):
                seq.num_cached_tokens += n
        tokens = self._sample(hidden).tolist()
        reset_context()
        return tokens

    def _sample(self, hidden):
        """Token ids for the rows of ``hidden``.  Greedy rows take the arg-max, which is found
        without gathering the other tensor-parallel ranks' logits unless ``keep_logits`` asks
        for them (``last_logits``).  Rows with a temperature above 1e-6 are drawn from
        softmax(logits / temperature) by the exponential race of
        ``qslab/runtime/execute/sampler.py:8-13``: arg-max of probs / Exp(1) noise."""
        temperature = self.temperature
        if isinstance(temperature, (int, float)):
            hot = temperature > 1e-6                          # decided on the host: no device round trip per step
        else:
            hot = bool((torch.as_tensor(temperature) > 1e-6).any())
        if hot:
            self.last_logits = self.model.compute_logits(hidden)
            temps = torch.as_tensor(temperature, dtype=torch.float32, device=hidden.device)
            temps = temps.expand(hidden.shape[0]) if temps.dim() == 0 else temps
            greedy = self.last_logits.argmax(dim=-1)
            probs = torch.softmax(self.last_logits.float() / temps.clamp_min(1e-6).unsqueeze(1), dim=-1)
            noise = torch.empty_like(probs).exponential_(1, generator=self.sample_generator).clamp_min_(1e-10)
            return torch.where(temps <= 1e-6, greedy, (probs / noise).argmax(dim=-1))
        if self.keep_logits:
            self.last_logits = self.model.compute_logits(hidden)
            return self.last_logits.argmax(dim=-1)
        self.last_logits = None
        return self.model.greedy_tokens(hidden)

    @torch.inference_mode()
    def verify(self, seqs: list[Sequence], drafts: list[list[int]]) -> list[list[int]]:
        """One M-row verify forward; returns the greedy token at every row."""
        self.tp.guard()
        m_rows = self.config.spec_num_drafts + 1
        input_ids, positions = self.prepare_verify(seqs, drafts)
        hidden = self.run_model(input_ids, positions, False, rows=m_rows)
        tokens = self.model.greedy_tokens(hidden).view(len(seqs), m_rows).tolist()
        reset_context()
        return tokens


def amax_calibration(num_layers: int, num_kv_heads: int, head_dim: int, kscale: float = 0.3) -> dict:
    """Unit-lambda calibration with a constant K scale, the form the reference's
    test fixture writes (``tests/conftest.py:41-43``)."""
    return {"lambda": torch.ones(num_layers, num_kv_heads, head_dim),
            "kscale": torch.full((num_layers, num_kv_heads, head_dim), kscale)}
