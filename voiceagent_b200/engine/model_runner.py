"""Text decoder stage: KV cache, batch packing on the GPU, eager/graph dispatch, sampling.

Each step the host writes one compact int32 descriptor of the batch (per request:
start, end, block-table offset/length; then the concatenated block tables and query
token ids) into pinned memory and issues ONE host-to-device copy; the
``pack_decoder`` kernel derives positions, slot mapping, cu_seqlens and padded block
tables from it (replacing the per-token Python loops and six tensor uploads of the
reference's ``_prepare``, engine/model_runner.py:183-233).
"""

from __future__ import annotations

import numpy as np
import torch

from voiceagent_b200 import kernels as kx
from voiceagent_b200.shapes import padded_rows
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.engine.graph_runner import HOST_WORK_SECONDS_PER_STEP, GraphRunner
from voiceagent_b200.engine.request import AsrRequest
from voiceagent_b200.engine.scheduler import ModelBatch
from voiceagent_b200.layers.attention import PagedAttention
from voiceagent_b200.layers.context import AttentionContext, attention_context
from voiceagent_b200.layers.sampler import GREEDY_TEMPERATURE_EPS, Sampler
from voiceagent_b200.profiling import NULL_TIMER, TRANSFERS
from voiceagent_b200.qwen3_asr.model import Qwen3ASRForConditionalGeneration


class Staging:
    """Pinned host buffer + device buffer for one-copy uploads of int32 descriptors."""

    def __init__(self, capacity: int, device):
        self.capacity = capacity
        self.host = torch.empty(capacity, dtype=torch.int32, pin_memory=True)
        self.device_buf = torch.empty(capacity, dtype=torch.int32, device=device)
        self._host_np = self.host.numpy()

    def upload(self, parts: list[np.ndarray]) -> list[torch.Tensor]:
        sizes = [int(p.size) for p in parts]
        total = sum(sizes)
        if total > self.capacity:
            raise ValueError(f"batch descriptor of {total} ints exceeds staging capacity "
                             f"{self.capacity}")
        off = 0
        views = []
        for p, n in zip(parts, sizes):
            self._host_np[off:off + n] = p
            views.append((off, n))
            off += n
        self.device_buf[:total].copy_(self.host[:total], non_blocking=True)
        TRANSFERS["h2d"] += 4 * total
        return [self.device_buf[o:o + n] for o, n in views]


class ModelRunner:
    def __init__(self, model: Qwen3ASRForConditionalGeneration, config: EngineConfig):
        self.model = model
        self.config = config
        self.device = torch.device(config.device)
        self.block_size = config.kvcache_block_size
        self.sampler = Sampler()
        self.attention_layers = [m for m in model.modules() if isinstance(m, PagedAttention)]
        self.kv_cache: torch.Tensor | None = None
        self.num_blocks = 0
        self.graph_runner: GraphRunner | None = None
        # host work to overlap with the GPU: called with a time budget (seconds) once a
        # decoder call is queued, before the host waits for its tokens (the engine stages
        # upcoming clips' waveforms)
        self.host_work = None
        self.timer = NULL_TIMER
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        max_tables = config.max_num_seqs * (-(-config.max_model_len // self.block_size))
        self.staging = Staging(4 * config.max_num_seqs + max_tables
                               + config.max_num_batched_tokens + 64, self.device)
        self._tokens_host = torch.empty(max(config.max_num_seqs, 1) * 4, dtype=torch.int64,
                                        pin_memory=True)
        # Split-K workspace so eager decode-only batches run the same kernel as the graphs.
        heads = config.model_config.text.num_attention_heads
        ws = kx.paged_decode_workspace_size(config.max_num_seqs, config.max_model_len, heads)
        self.decode_workspace = torch.zeros(ws // 4 + 64, dtype=torch.float32, device=self.device)

    # ------------------------------------------------------------------ cache

    def kv_cache_bytes_per_block(self) -> int:
        t = self.config.model_config.text
        hd = t.head_dim or t.hidden_size // t.num_attention_heads
        return 2 * t.num_hidden_layers * self.block_size * t.num_key_value_heads * hd * 2

    def determine_num_blocks(self, reserve_bytes: int = 6 * 2**30) -> int:
        """KV blocks from the free memory after weights, minus a flat activation reserve
        (the encoder's conv slices and the widest prefill); ``num_kvcache_blocks``
        overrides."""
        if self.config.num_kvcache_blocks > 0:
            return self.config.num_kvcache_blocks
        torch.cuda.empty_cache()
        free, total = torch.cuda.mem_get_info(self.device)
        budget = free * self.config.gpu_memory_utilization - reserve_bytes
        n = int(budget) // self.kv_cache_bytes_per_block()
        if n <= 0:
            raise RuntimeError(f"no memory left for the KV cache: {free / 2**30:.1f} GiB free of "
                               f"{total / 2**30:.1f} GiB")
        return n

    def allocate_kv_cache(self, num_blocks: int) -> None:
        t = self.config.model_config.text
        hd = t.head_dim or t.hidden_size // t.num_attention_heads
        self.kv_cache = torch.zeros(2, t.num_hidden_layers, num_blocks, self.block_size,
                                    t.num_key_value_heads, hd, dtype=torch.bfloat16,
                                    device=self.device)
        for i, layer in enumerate(self.attention_layers):
            layer.k_cache = self.kv_cache[0, i]
            layer.v_cache = self.kv_cache[1, i]
        self.num_blocks = num_blocks

    def capture_graphs(self) -> None:
        if self.config.enforce_eager:
            return
        if self.kv_cache is None:
            raise RuntimeError("allocate the KV cache before capturing graphs")
        runner = GraphRunner(self.model, self.config, self.error_flag)
        runner.capture()
        self.graph_runner = runner

    # bits of the device error word (include/b200asr.h; 16 = a bounded wait gave up)
    DEVICE_ERRORS = {1: "KV slot outside the cache", 2: "block id outside the pool",
                     4: "position outside the RoPE table", 8: "length beyond its table or buffer",
                     16: "a kernel's bounded wait timed out"}

    def check_device_errors(self) -> None:
        """Raise if a kernel flagged an out-of-range index or a timed-out wait since the
        last check."""
        flag = int(self.error_flag.item())
        if flag:
            self.error_flag.zero_()
            what = "; ".join(v for k, v in self.DEVICE_ERRORS.items() if flag & k)
            raise RuntimeError(f"b200asr device check failed (flags 0x{flag:x}): {what}")

    # ------------------------------------------------------------------- step

    def _prepare(self, batch: ModelBatch):
        requests = batch.requests
        n = len(requests)
        starts = np.empty(n, np.int32)
        ends = np.empty(n, np.int32)
        tlens = np.empty(n, np.int32)
        tables: list[int] = []
        tokens: list[int] = []
        spans: list[tuple[int, torch.Tensor]] = []
        cursor = 0
        for i, r in enumerate(requests):
            s, e = r.num_computed_tokens, len(r)
            starts[i], ends[i] = s, e
            tlens[i] = len(r.block_table)
            tables.extend(r.block_table)
            tokens.extend(r.token_ids[s:e])
            span = self._audio_span(r, s, e, cursor)
            if span is not None:
                spans.append(span)
            cursor += e - s
        toffs = np.zeros(n, np.int32)
        np.cumsum(tlens[:-1], out=toffs[1:])
        total = cursor
        width = int(tlens.max())
        d_start, d_end, d_toff, d_tlen, d_tables, d_tokens = self.staging.upload(
            [starts, ends, toffs, tlens, np.asarray(tables, np.int32),
             np.asarray(tokens, np.int32)])
        dev = self.device
        rows = padded_rows(total)  # bucketed (shape-stable GEMMs); see voiceagent_b200.shapes
        out = {
            "input_ids": torch.empty(rows, dtype=torch.int64, device=dev),
            "positions": torch.empty(rows, dtype=torch.int64, device=dev),
            "slot_mapping": torch.empty(rows, dtype=torch.int32, device=dev),
            "cu_seqlens_q": torch.empty(n + 1, dtype=torch.int32, device=dev),
            "cu_seqlens_k": torch.empty(n + 1, dtype=torch.int32, device=dev),
            "max_seqlen": torch.empty(2, dtype=torch.int32, device=dev),
            "block_tables": torch.empty(n, width, dtype=torch.int32, device=dev),
            "last_token_index": torch.empty(n, dtype=torch.int64, device=dev),
        }
        kx.pack_decoder(d_start, d_end, d_toff, d_tlen, d_tables, d_tokens, total_tokens=total,
                        width=width, block_size=self.block_size, out=out)
        if rows > total:  # padding rows: token 0 at position 0, never stored (slot -1)
            out["input_ids"][total:].zero_()
            out["positions"][total:].zero_()
            out["slot_mapping"][total:].fill_(-1)
        max_q = int((ends - starts).max())
        decode_only = max_q == 1 and n <= self.config.max_num_seqs
        ctx = AttentionContext(
            cu_seqlens_q=out["cu_seqlens_q"], cu_seqlens_k=out["cu_seqlens_k"],
            max_seqlen_q=max_q,
            # decode rows use the bound the graph would bake in, so both paths pick the same
            # attention kernel (short contexts: one CTA per sequence and KV head)
            max_seqlen_k=(min(kx.DECODE_SHORT_CTX, self.config.max_model_len)
                          if int(ends.max()) <= min(kx.DECODE_SHORT_CTX, self.config.max_model_len)
                          else self.config.max_model_len) if decode_only else int(ends.max()),
            slot_mapping=out["slot_mapping"], block_tables=out["block_tables"],
            decode_only=decode_only, decode_workspace=self.decode_workspace,
            error_flag=self.error_flag)
        return out, ctx, spans

    @staticmethod
    def _audio_span(request: AsrRequest, start: int, end: int, offset: int):
        if request.audio_embeds is None:
            return None
        a0 = request.layout.audio_offset
        a1 = a0 + request.layout.audio_length
        lo, hi = max(a0, start), min(a1, end)
        if lo >= hi:
            return None
        return offset + (lo - start), request.audio_embeds[lo - a0:hi - a0]

    def can_use_graph(self, batch: ModelBatch) -> bool:
        return (self.graph_runner is not None and not batch.prefill and bool(batch.decode)
                and self.graph_runner.bucket_for(len(batch.decode)) is not None
                and all(r.sampling.temperature < GREEDY_TEMPERATURE_EPS for r in batch.decode))

    @staticmethod
    def _phase_name(batch: ModelBatch) -> str:
        if batch.prefill and batch.decode:
            return "llm_mixed"
        return "llm_prefill" if batch.prefill else "llm_decode"

    @property
    def max_decode_steps(self) -> int:
        return self.graph_runner.max_steps if self.graph_runner is not None else 1

    @torch.inference_mode()
    def run_steps(self, batch: ModelBatch, steps: int) -> list[list[int]]:
        """``steps`` CUDA-graph decode steps of a decode-only batch in one host round trip
        (its block tables already cover every position they write)."""
        if not self.can_use_graph(batch) or batch.prefill:
            raise ValueError("multi-step decode needs a graph-eligible decode-only batch")
        with self.timer.phase("llm_decode"):
            return self.graph_runner.run(batch.decode, steps, host_work=self.host_work)

    @torch.inference_mode()
    def run(self, batch: ModelBatch) -> list[int]:
        with self.timer.phase(self._phase_name(batch)):
            if self.can_use_graph(batch):
                return self.graph_runner.run(batch.decode, host_work=self.host_work)
            logits = self._forward_eager(batch)
            return self._sample(logits, batch.requests)

    def _forward_hidden(self, batch: ModelBatch):
        packed, ctx, spans = self._prepare(batch)
        with attention_context(ctx):
            embeds = self.model.embed_tokens(packed["input_ids"])
            if spans:
                self.model.scatter_audio_embeddings(embeds, spans)
            hidden = self.model(None, packed["positions"], inputs_embeds=embeds)
        return hidden, packed

    def _forward_eager(self, batch: ModelBatch) -> torch.Tensor:
        hidden, packed = self._forward_hidden(batch)
        last = packed["last_token_index"]
        n = last.numel()
        rows = padded_rows(n)
        if rows > n:  # bucketed lm_head rows; the extra rows repeat row 0 and are dropped
            last = torch.cat([last, last[:1].expand(rows - n)])
        return self.model.compute_logits(hidden.index_select(0, last))[:n]

    def _sample(self, logits: torch.Tensor, requests) -> list[int]:
        temps = [r.sampling.temperature for r in requests]
        n = len(requests)
        if max(temps) < GREEDY_TEMPERATURE_EPS:
            ids = self.sampler(logits)
        else:
            ids = self.sampler(logits, torch.tensor(temps, dtype=torch.float32, device=self.device))
        host = self._tokens_host[:n] if n <= self._tokens_host.numel() else torch.empty(
            n, dtype=torch.int64, pin_memory=True)
        host.copy_(ids, non_blocking=True)
        TRANSFERS["d2h"] += 8 * n
        if self.host_work is not None:
            self.host_work(HOST_WORK_SECONDS_PER_STEP)
        torch.cuda.current_stream().synchronize()
        return host.tolist()

    @torch.inference_mode()
    def verify(self, batch: ModelBatch, draft_lens: list[int]) -> list[list[int]]:
        """Greedy predictions for the tail of each query span (speculative verify,
        engine/model_runner.py:299-335): n draft tokens -> n + 1 predictions."""
        hidden, packed = self._forward_hidden(batch)
        cu = packed["cu_seqlens_q"].tolist()
        index, widths = [], []
        for b, nd in enumerate(draft_lens):
            s, e = cu[b], cu[b + 1]
            w = min(nd + 1, e - s)
            index.extend(range(e - w, e))
            widths.append(w)
        idx = torch.tensor(index, dtype=torch.int64, device=self.device)
        preds = self.sampler(self.model.compute_logits(hidden.index_select(0, idx))).tolist()
        out, c = [], 0
        for w in widths:
            out.append(preds[c:c + w])
            c += w
        return out
