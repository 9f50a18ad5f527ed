"""CUDA-graph decode (engine/graph_runner.py of the reference, B200 version).

One graph per batch bucket. Each graph holds the WHOLE decode step: the
``pack_decode_bucket`` kernel (building input ids, positions, slot mapping,
cu_seqlens_k and block tables from a static device descriptor), the 28-layer
decoder with the split-K paged decode attention, the final norm, the lm_head GEMM
and the greedy argmax, then advances the device descriptor by the sampled tokens
(length + 1, last token). Per call the host fills a pinned descriptor, issues one
host-to-device copy, replays ``steps`` times in a row (the blocks those steps write are
allocated beforehand) and reads back the tokens of every step with one sync.

Padding rows are encoded in the descriptor as (length 1, empty block table), which
the packer turns into the reference's padding: slot -1, key length 1, an all-zero
block-table row.

Each bucket has two graphs: one whose attention is bounded to contexts of at most
``kernels.DECODE_SHORT_CTX`` tokens (paged decode with one CTA per sequence and KV head)
and one for any length up to max_model_len (the stream-K split); a call picks the
short one when every context, including the steps it adds, fits.
"""

from __future__ import annotations

import itertools
import logging

import torch

from voiceagent_b200 import kernels as kx
from voiceagent_b200.config import EngineConfig
from voiceagent_b200.layers.context import AttentionContext, attention_context
from voiceagent_b200.profiling import TRANSFERS

logger = logging.getLogger(__name__)

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64)
# Host time a call lends to ``host_work`` per queued decode step: below a step's GPU time
# (0.9 ms for the 0.6B model at 32 rows, 1.8 ms for the 1.7B at 64), so the host is back
# at the token read-back before the replays end.
HOST_WORK_SECONDS_PER_STEP = 0.4e-3


def fill_decode_descriptor(h, m: int, requests) -> tuple[int, int]:
    """Write the rows of ``requests`` into the host descriptor ``h`` (int32, laid out as
    lengths [m] | last token ids [m] | table offsets [m] | table lengths [m] | the
    concatenated block tables) with one slice store per field. Returns (the number of
    ints used, the longest length)."""
    n = len(requests)
    lengths = [len(r.token_ids) for r in requests]
    tables = [r.block_table for r in requests]
    table_lens = [len(t) for t in tables]
    flat = list(itertools.chain.from_iterable(tables))
    h[0:n] = lengths
    h[m:m + n] = [r.token_ids[-1] for r in requests]
    h[2 * m:2 * m + n] = list(itertools.accumulate(table_lens, initial=0))[:n]
    h[3 * m:3 * m + n] = table_lens
    cursor = 4 * m + len(flat)
    h[4 * m:cursor] = flat
    return cursor, max(lengths)


class GraphRunner:
    def __init__(self, model, config: EngineConfig, error_flag: torch.Tensor | None = None,
                 buckets: tuple[int, ...] = DEFAULT_BUCKETS):
        self.model = model
        self.config = config
        self.device = torch.device(config.device)
        self.block_size = config.kvcache_block_size
        self.max_blocks = -(-config.max_model_len // self.block_size)
        self.buckets = tuple(b for b in buckets if b <= config.max_num_seqs) or (config.max_num_seqs,)
        self.max_batch = self.buckets[-1]
        self.error_flag = error_flag
        self.graphs: dict[tuple[int, bool], torch.cuda.CUDAGraph] = {}
        self.kernels_per_replay: dict[tuple[int, bool], int] = {}
        self.pool = None
        self._allocate()

    def _allocate(self) -> None:
        m, dev = self.max_batch, self.device
        self.desc_len = 4 * m + m * self.max_blocks
        self.desc = torch.zeros(self.desc_len, dtype=torch.int32, device=dev)
        self.host_desc = torch.zeros(self.desc_len, dtype=torch.int32, pin_memory=True)
        self._host_np = self.host_desc.numpy()
        self.input_ids = torch.zeros(m, dtype=torch.int64, device=dev)
        self.positions = torch.zeros(m, dtype=torch.int64, device=dev)
        self.slot_mapping = torch.full((m,), -1, dtype=torch.int32, device=dev)
        self.cu_seqlens_q = torch.arange(m + 1, dtype=torch.int32, device=dev)
        self.cu_seqlens_k = torch.zeros(m + 1, dtype=torch.int32, device=dev)
        self.block_tables = torch.zeros(m, self.max_blocks, dtype=torch.int32, device=dev)
        self.token_ids = torch.zeros(m, dtype=torch.int64, device=dev)
        self.max_steps = max(1, int(getattr(self.config, "decode_steps", 1)))
        self.host_tokens = torch.zeros(self.max_steps, m, dtype=torch.int64, pin_memory=True)
        self.hidden: dict[int, torch.Tensor] = {}
        ws_bytes = kx.paged_decode_workspace_size(m, self.config.max_model_len,
                                                  self.config.model_config.text.num_attention_heads)
        self.workspace = torch.zeros(ws_bytes // 4 + 64, dtype=torch.float32, device=dev)

    def _desc_views(self, bucket: int):
        m = self.max_batch
        d = self.desc
        return (d[0:bucket], d[m:m + bucket], d[2 * m:2 * m + bucket], d[3 * m:3 * m + bucket],
                d[4 * m:])

    def _context(self, bucket: int, short: bool) -> AttentionContext:
        max_k = min(kx.DECODE_SHORT_CTX, self.config.max_model_len) if short else self.config.max_model_len
        return AttentionContext(
            cu_seqlens_q=self.cu_seqlens_q[:bucket + 1], cu_seqlens_k=self.cu_seqlens_k[:bucket + 1],
            max_seqlen_q=1, max_seqlen_k=max_k,
            slot_mapping=self.slot_mapping[:bucket], block_tables=self.block_tables[:bucket],
            decode_only=True, decode_workspace=self.workspace, error_flag=self.error_flag)

    def _step(self, bucket: int) -> torch.Tensor:
        lens, last_ids, toff, tlen, tables = self._desc_views(bucket)
        kx.pack_decode_bucket(lens, last_ids, toff, tlen, tables, batch=bucket, bucket=bucket,
                              max_blocks=self.max_blocks, block_size=self.block_size,
                              input_ids=self.input_ids, positions=self.positions,
                              slot_mapping=self.slot_mapping, cu_seqlens_k=self.cu_seqlens_k,
                              block_tables=self.block_tables)
        hidden = self.model(self.input_ids[:bucket], self.positions[:bucket])
        logits = self.model.compute_logits(hidden)
        kx.greedy_argmax(logits, out=self.token_ids[:bucket])
        kx.advance_decode_bucket(lens, last_ids, tlen, self.token_ids[:bucket], bucket=bucket)
        return hidden

    def _fill_padding(self, start: int) -> None:
        m = self.max_batch
        h = self._host_np
        h[start:m] = 1            # lens
        h[m + start:2 * m] = 0    # last ids
        h[2 * m + start:3 * m] = 0
        h[3 * m + start:4 * m] = 0  # empty tables

    @torch.inference_mode()
    def capture(self) -> None:
        self._fill_padding(0)
        self.desc.copy_(self.host_desc)
        for bucket in reversed(self.buckets):
            for short in (False, True):
                with attention_context(self._context(bucket, short)):
                    for _ in range(2):
                        self._step(bucket)
                    torch.cuda.synchronize()
                    graph = torch.cuda.CUDAGraph()
                    before = kx.LAUNCHES["count"]
                    with torch.cuda.graph(graph, self.pool):
                        self.hidden[(bucket, short)] = self._step(bucket)
                    self.kernels_per_replay[(bucket, short)] = kx.LAUNCHES["count"] - before
                self.pool = self.pool or graph.pool()
                self.graphs[(bucket, short)] = graph
        torch.cuda.synchronize()
        logger.info("captured decode graphs for buckets %s", sorted({b for b, _ in self.graphs}))

    def uses_short_graph(self, max_len: int, steps: int = 1) -> bool:
        """Whether every context of a call (longest ``max_len`` before it, growing by one
        per step) fits the short-context attention."""
        return max_len + steps - 1 <= min(kx.DECODE_SHORT_CTX, self.config.max_model_len)

    def bucket_for(self, batch_size: int) -> int | None:
        for b in self.buckets:
            if b >= batch_size:
                return b
        return None

    @torch.inference_mode()
    def run(self, requests, steps: int = 1, host_work=None) -> list[int] | list[list[int]]:
        """Replay ``steps`` decode steps for ``requests`` (their block tables must already
        cover every position those steps write). Returns the sampled ids of the one step,
        or one list per step when ``steps > 1``. ``host_work`` (a callable taking a time
        budget in seconds) runs after the replays are queued, while the GPU executes them."""
        n = len(requests)
        bucket = self.bucket_for(n)
        if bucket is None:
            raise ValueError(f"no captured graph for a batch of {n}")
        if not 1 <= steps <= self.max_steps:
            raise ValueError(f"steps must be in [1, {self.max_steps}], got {steps}")
        cursor, max_len = fill_decode_descriptor(self._host_np, self.max_batch, requests)
        self._fill_padding(n)
        self.desc[:cursor].copy_(self.host_desc[:cursor], non_blocking=True)
        key = (bucket, self.uses_short_graph(max_len, steps))
        for k in range(steps):
            self.graphs[key].replay()
            self.host_tokens[k, :n].copy_(self.token_ids[:n], non_blocking=True)
        kx.LAUNCHES["count"] += steps * self.kernels_per_replay[key]
        TRANSFERS["h2d"] += 4 * cursor
        TRANSFERS["d2h"] += 8 * n * steps
        if host_work is not None:
            host_work(steps * HOST_WORK_SECONDS_PER_STEP)
        torch.cuda.current_stream().synchronize()
        if steps == 1:
            return self.host_tokens[0, :n].tolist()
        return self.host_tokens[:steps, :n].tolist()

    def release(self) -> None:
        self.graphs.clear()
        self.hidden.clear()
        self.pool = None

