"""Qwen3 text decoder (models/qwen3.py of the reference).

Per layer the b200asr kernels do: input / post-attention RMSNorm (the latter fused
with the residual add), per-head q/k RMSNorm + RoPE fused with the KV-cache store,
paged attention and SiLU*mul. Dense projections run on torch matmul (cuBLAS) for
prefill-sized batches. Decode-sized batches (up to 64 rows) take the fused step: the
weight-streaming ``linear_small`` kernels with each RMSNorm split across the
projections around it, q/k norm + RoPE + the KV store in qkv_proj's epilogue and
SiLU*mul in gate_up_proj's -- five launches per layer.
"""

from __future__ import annotations

import torch
from torch import nn

from voiceagent_b200 import kernels as kx
from voiceagent_b200.config import TextConfig
from voiceagent_b200.layers.attention import PagedAttention
from voiceagent_b200.layers.context import get_attention_context
from voiceagent_b200.layers.norm import RMSNorm, SiluAndMul


def project(x: torch.Tensor, layer: nn.Linear) -> torch.Tensor:
    """``layer(x)``: decode-size batches on ``linear_small``, larger ones on cuBLAS."""
    if layer.bias is None and kx.linear_small_ok(x, layer.weight):
        return kx.linear_small(x, layer.weight, error_flag=get_attention_context().error_flag)
    return layer(x)


class Qwen3Attention(nn.Module):
    def __init__(self, config: TextConfig, rope: "RopeHolder"):
        super().__init__()
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.head_dim or config.hidden_size // config.num_attention_heads
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.eps = config.rms_norm_eps
        self.qkv_proj = nn.Linear(config.hidden_size, self.q_size + 2 * self.kv_size,
                                  bias=config.attention_bias)
        self.o_proj = nn.Linear(self.q_size, config.hidden_size, bias=False)
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.rope = rope
        self.attn = PagedAttention(self.num_heads, self.head_dim, self.head_dim ** -0.5,
                                   self.num_kv_heads)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        ctx = get_attention_context()
        t = hidden_states.shape[0]
        q = torch.empty(t, self.num_heads, self.head_dim, dtype=hidden_states.dtype,
                        device=hidden_states.device)
        # q/k RMSNorm + RoPE; K and V go straight into the paged cache. Decode-size batches
        # do it in the projection's epilogue (one kernel), larger ones after cuBLAS.
        heads = dict(num_heads=self.num_heads, num_kv_heads=self.num_kv_heads,
                     head_dim=self.head_dim, q_weight=self.q_norm.weight,
                     k_weight=self.k_norm.weight, cos_sin_cache=self.rope.table, q_out=q,
                     k_cache=self.attn.k_cache, v_cache=self.attn.v_cache,
                     slot_mapping=ctx.slot_mapping, error_flag=ctx.error_flag)
        if (self.qkv_proj.bias is None and self.head_dim == 128
                and kx.linear_small_ok(hidden_states, self.qkv_proj.weight)):
            kx.linear_small_qk_rope(hidden_states, self.qkv_proj.weight, positions,
                                    qk_eps=self.eps, **heads)
        else:
            qkv = project(hidden_states, self.qkv_proj)
            kx.qk_norm_rope_store(qkv, positions, eps=self.eps, **heads)
        attn_out = self.attn(q)
        return project(attn_out.view(t, self.q_size), self.o_proj)


class Qwen3MLP(nn.Module):
    def __init__(self, config: TextConfig):
        super().__init__()
        if config.hidden_act != "silu":
            raise ValueError(f"unsupported activation: {config.hidden_act}")
        self.gate_up_proj = nn.Linear(config.hidden_size, 2 * config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)
        self.act_fn = SiluAndMul()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.gate_up_proj.weight
        if kx.linear_small_ok(x, w, silu=True):  # SiLU*mul fused into the projection
            act = kx.linear_small(x, w, silu=True, error_flag=get_attention_context().error_flag)
        else:
            act = self.act_fn(self.gate_up_proj(x))
        return project(act, self.down_proj)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, config: TextConfig, rope: "RopeHolder"):
        super().__init__()
        self.self_attn = Qwen3Attention(config, rope)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward(self, positions, hidden_states, residual):
        if residual is None:
            residual = hidden_states
            hidden_states = self.input_layernorm(hidden_states)
        else:
            hidden_states, residual = self.input_layernorm(hidden_states, residual)
        hidden_states = self.self_attn(positions, hidden_states)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual)
        return self.mlp(hidden_states), residual


class RopeHolder(nn.Module):
    """Owns the fp32 RoPE table shared by every layer (a buffer, not a parameter)."""

    def __init__(self, head_dim: int, max_position: int, base: float):
        super().__init__()
        from voiceagent_b200.layers.norm import rope_table

        self.register_buffer("table", rope_table(head_dim, max_position, base, None),
                             persistent=False)


class Qwen3Model(nn.Module):
    def __init__(self, config: TextConfig, max_position: int):
        super().__init__()
        head_dim = config.head_dim or config.hidden_size // config.num_attention_heads
        self.rope = RopeHolder(head_dim, max_position, config.rope_theta)
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(
            [Qwen3DecoderLayer(config, self.rope) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.fused_decode = True  # decode-sized batches on the fused projections
        self.l2_prefetch = False  # fused decode steps: next layer's K/V + weights into L2
        self._plain: bool | None = None  # projections without bias, bf16, contiguous

    def forward(self, input_ids, positions, inputs_embeds=None) -> torch.Tensor:
        if (input_ids is None) == (inputs_embeds is None):
            raise ValueError("pass exactly one of input_ids or inputs_embeds")
        hidden = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        if self.fused_step_ok(hidden.shape[0]):
            # the residual stream is updated in place: never the caller's tensor
            return self._forward_fused(positions, hidden if inputs_embeds is None else hidden.clone())
        residual = None
        for layer in self.layers:
            hidden, residual = layer(positions, hidden, residual)
        hidden, _ = self.norm(hidden, residual)
        return hidden

    def fused_step_ok(self, rows: int) -> bool:
        """Decode-sized batches run the fused projections (five launches per layer)."""
        if not self.fused_decode or not self.layers:
            return False
        a = self.layers[0].self_attn
        return kx.fused_decode_ok(rows, self.embed_tokens.embedding_dim,
                                  self.layers[0].mlp.down_proj.in_features, a.num_heads,
                                  a.num_kv_heads, a.head_dim) and self._plain_projections

    def _forward_fused(self, positions, residual: torch.Tensor) -> torch.Tensor:
        """The same layer stack with each RMSNorm split across the projections around it
        (kernels.linear_small_add / linear_small_norm*): qkv (norm, q/k norm, RoPE, K/V
        store) -> attention -> o_proj (+ residual) -> gate_up (norm, SiLU*mul) -> down
        (+ residual); the rows travel between them as fp32 h plus tile sums of h^2."""
        ctx = get_attention_context()
        m, hidden = residual.shape
        state = kx.NormState(m, hidden, residual.device)
        kx.rms_stats(residual, state)  # layer 0's input norm reads the embeddings
        for i, layer in enumerate(self.layers):
            attn, mlp = layer.self_attn, layer.mlp
            # optional (EngineConfig.l2_prefetch): while this layer's MLP runs, gate_up
            # requests the next layer's cached K/V and its qkv / o_proj weights into L2
            prefetch = None
            if ctx.decode_only and self.l2_prefetch and i + 1 < len(self.layers):
                nxt = self.layers[i + 1].self_attn
                prefetch = kx.l2_prefetch(
                    kv=(ctx.cu_seqlens_k, ctx.block_tables, nxt.attn.k_cache, nxt.attn.v_cache),
                    ranges=(nxt.qkv_proj.weight, nxt.o_proj.weight))
            q = torch.empty(m, attn.num_heads, attn.head_dim, dtype=residual.dtype,
                            device=residual.device)
            kx.linear_small_norm_qk_rope(
                state, layer.input_layernorm.weight, layer.input_layernorm.eps,
                attn.qkv_proj.weight, positions, num_heads=attn.num_heads,
                num_kv_heads=attn.num_kv_heads, head_dim=attn.head_dim,
                q_weight=attn.q_norm.weight, k_weight=attn.k_norm.weight, qk_eps=attn.eps,
                cos_sin_cache=attn.rope.table, q_out=q, k_cache=attn.attn.k_cache,
                v_cache=attn.attn.v_cache, slot_mapping=ctx.slot_mapping,
                error_flag=ctx.error_flag)
            o = attn.attn(q)
            kx.linear_small_add(o.view(m, attn.q_size), attn.o_proj.weight, residual, state,
                                error_flag=ctx.error_flag)
            act = kx.linear_small_norm(state, layer.post_attention_layernorm.weight,
                                       layer.post_attention_layernorm.eps,
                                       mlp.gate_up_proj.weight, silu=True, prefetch=prefetch,
                                       error_flag=ctx.error_flag)
            kx.linear_small_add(act, mlp.down_proj.weight, residual, state,
                                error_flag=ctx.error_flag)
        return kx.norm_apply(state, self.norm.weight, self.norm.eps)

    @property
    def _plain_projections(self) -> bool:
        if self._plain is None:
            self._plain = all(
                lin.bias is None and lin.weight.dtype == torch.bfloat16 and lin.weight.is_contiguous()
                for layer in self.layers
                for lin in (layer.self_attn.qkv_proj, layer.self_attn.o_proj,
                            layer.mlp.gate_up_proj, layer.mlp.down_proj))
        return self._plain
