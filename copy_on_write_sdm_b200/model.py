"""Decoder model around the packed SDM layers (the serving callers of the hot path).

Module tree and parameter names equal the reference's ``copy_on_write_sdm/model.py``
(``token_embedding``, ``position_embedding``, ``stack.attention_layers[i]``,
``stack.sdm_layers[i]``, ``stack.sdm_mlps[i]``, ``final_norm``, ``output``), so
a reference checkpoint loads with ``load_state_dict``.  Serving entry points:
``prefill`` / ``decode`` / ``admit`` (reference model.py:419-482).  The dense
"A" layer keeps a fixed-capacity K/V cache and uses PyTorch SDPA.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

import torch
import torch.nn.functional as F
from torch import nn
from torch.nn.attention import SDPBackend, sdpa_kernel

from .sdm import SparseDeltaMemory

if TYPE_CHECKING:
    from .inference import FaithfulSDMDecodeState


class ResidualMLP(nn.Module):
    """Pre-norm GELU MLP branch (reference model.py:25-45)."""

    def __init__(self, width: int, *, expansion: float = 4.0, dropout: float = 0.0) -> None:
        super().__init__()
        self.hidden = max(1, int(round(width * expansion)))
        self.norm = nn.LayerNorm(width)
        self.input = nn.Linear(width, self.hidden, bias=False)
        self.activation = nn.GELU()
        self.output = nn.Linear(self.hidden, width, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.dropout(self.output(self.activation(self.input(self.norm(tokens)))))


class CausalSelfAttention(nn.Module):
    """Multi-head causal attention with a fixed-capacity K/V cache (reference model.py:47-190)."""

    def __init__(self, width: int, heads: int, *, dropout: float = 0.0) -> None:
        super().__init__()
        if width <= 0 or heads <= 0 or width % heads:
            raise ValueError("width must be positive and divisible by heads")
        self.width, self.heads, self.head_width, self.dropout = width, heads, width // heads, dropout
        self.norm = nn.LayerNorm(width)
        self.qkv = nn.Linear(width, 3 * width, bias=False)
        self.output = nn.Linear(width, width, bias=False)

    def project_qkv(self, tokens: torch.Tensor):
        batch, time, _ = tokens.shape
        qkv = self.qkv(self.norm(tokens)).reshape(batch, time, 3, self.heads, self.head_width)
        q, k, v = (qkv[:, :, i].transpose(1, 2).contiguous() for i in range(3))
        return q, k, v

    def _sdpa(self, q, k, v, *, causal: bool, mask=None) -> torch.Tensor:
        # Flash kernels for 16-bit activations, the exact math kernel for fp32.
        if q.is_cuda:
            backend = SDPBackend.FLASH_ATTENTION if (q.dtype in (torch.float16, torch.bfloat16) and mask is None) \
                else SDPBackend.MATH
            with sdpa_kernel(backend):
                return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal)
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal)

    def _merge(self, attended: torch.Tensor) -> torch.Tensor:
        batch, _, time, _ = attended.shape
        return self.output(attended.transpose(1, 2).reshape(batch, time, self.width))

    def prefill_with_cache(self, tokens: torch.Tensor):
        q, k, v = self.project_qkv(tokens)
        return self._merge(self._sdpa(q, k, v, causal=True)), k, v

    def decode_with_cache(self, tokens: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, *,
                          position: int | torch.Tensor) -> torch.Tensor:
        """One token per request; ``position`` is shared (int) or per request ([B])."""
        if tokens.shape[1] != 1 or key_cache.shape != value_cache.shape:
            raise ValueError("dense decode cache is invalid")
        q, k, v = self.project_qkv(tokens)
        if isinstance(position, int):
            key_cache[:, :, position].copy_(k[:, :, 0])
            value_cache[:, :, position].copy_(v[:, :, 0])
            out = self._sdpa(q, key_cache[:, :, : position + 1], value_cache[:, :, : position + 1], causal=False)
            return self._merge(out)
        pos = torch.as_tensor(position, device=tokens.device, dtype=torch.int64)
        if pos.shape != (tokens.shape[0],):
            raise ValueError("dense decode positions are invalid")
        rows = torch.arange(tokens.shape[0], device=tokens.device)
        key_cache[rows, :, pos] = k[:, :, 0]
        value_cache[rows, :, pos] = v[:, :, 0]
        live = int(pos.max().item()) + 1
        hidden = torch.arange(live, device=tokens.device)[None, :] > pos[:, None]
        mask = torch.zeros(tokens.shape[0], 1, 1, live, device=tokens.device, dtype=q.dtype)
        mask.masked_fill_(hidden[:, None, None, :], float("-inf"))
        return self._merge(self._sdpa(q, key_cache[:, :, :live], value_cache[:, :, :live], causal=False, mask=mask))

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.prefill_with_cache(tokens)[0]


class DenseAttentionBlock(nn.Module):
    def __init__(self, width: int, heads: int, *, mlp_expansion: float = 4.0, dropout: float = 0.0) -> None:
        super().__init__()
        self.attention = CausalSelfAttention(width, heads, dropout=dropout)
        self.mlp = ResidualMLP(width, expansion=mlp_expansion, dropout=dropout)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        tokens = tokens + self.attention(tokens)
        return tokens + self.mlp(tokens)

    def decode_residual(self, tokens: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                        position) -> torch.Tensor:
        """One decode token through the block: ``t = tokens + attention.decode_with_cache(...)``
        then ``t + mlp(t)`` (reference inference.py:640-651).  ``position`` is an int or a
        ``[B]`` tensor.  FP32 CUDA activations in eval mode run as one
        ``cow_attention_mlp_decode`` launch, which also stores this token's K/V."""
        if self._fused_decode_ok(tokens, key_cache, value_cache):
            return self._decode_fused(tokens, key_cache, value_cache, position)
        tokens = tokens + self.attention.decode_with_cache(tokens, key_cache, value_cache, position=position)
        return tokens + self.mlp(tokens)

    def _fused_decode_ok(self, tokens, key_cache, value_cache) -> bool:
        att, mlp = self.attention, self.mlp
        if not (tokens.is_cuda and tokens.dtype == key_cache.dtype == value_cache.dtype == torch.float32):
            return False
        if self.training or tokens.ndim != 3 or tokens.shape[1] != 1:
            return False
        if not (key_cache.is_contiguous() and value_cache.is_contiguous() and key_cache.shape == value_cache.shape
                and key_cache.shape[:2] == (tokens.shape[0], att.heads) and key_cache.shape[3] == att.head_width):
            return False
        if att.qkv.bias is not None or att.output.bias is not None or mlp.input.bias is not None \
                or mlp.output.bias is not None:
            return False
        if not (att.norm.elementwise_affine and att.norm.bias is not None and mlp.norm.elementwise_affine
                and mlp.norm.bias is not None and isinstance(mlp.activation, nn.GELU)
                and mlp.activation.approximate == "none"):
            return False
        # scores for every cache slot stay in shared memory; wider blocks are faster as GEMMs
        return (att.width <= 256 and mlp.hidden <= 1024 and att.heads * key_cache.shape[2] <= 16384
                and all(p.dtype == torch.float32 for p in self._decode_params()))

    def _decode_params(self):
        att, mlp = self.attention, self.mlp
        return (att.norm.weight, att.norm.bias, att.qkv.weight, att.output.weight, mlp.norm.weight, mlp.norm.bias,
                mlp.input.weight, mlp.output.weight)

    def _decode_weights(self):
        """Transposed ([in, out]) QKV, output and MLP matrices; rebuilt only when a
        parameter was replaced or changed in place."""
        params = self._decode_params()
        key = tuple((t.data_ptr(), t._version) for t in params)
        cached = self.__dict__.get("_decode_cache")
        if cached is None or cached[0] != key:
            with torch.no_grad():
                mats = tuple(w.detach().t().contiguous() for w in (self.attention.qkv.weight,
                                                                   self.attention.output.weight,
                                                                   self.mlp.input.weight, self.mlp.output.weight))
            cached = (key, mats)
            self.__dict__["_decode_cache"] = cached
        return cached[1]

    def _decode_fused(self, tokens, key_cache, value_cache, position) -> torch.Tensor:
        from . import _lib

        att, mlp = self.attention, self.mlp
        batch = tokens.shape[0]
        if isinstance(position, int):
            if not 0 <= position < key_cache.shape[2]:
                raise ValueError("dense decode position is outside the cache")
            pos = torch.full((batch,), position, dtype=torch.int64, device=tokens.device)
        else:
            pos = torch.as_tensor(position, device=tokens.device, dtype=torch.int64).contiguous()
            if pos.shape != (batch,):
                raise ValueError("dense decode positions are invalid")
        x = tokens.contiguous()
        qkv_t, out_t, w1, w2 = self._decode_weights()
        out = torch.empty_like(x)
        _lib.check(_lib.load().cow_attention_mlp_decode(
            x.data_ptr(), pos.data_ptr(), att.norm.weight.data_ptr(), att.norm.bias.data_ptr(), float(att.norm.eps),
            qkv_t.data_ptr(), out_t.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), key_cache.shape[2],
            mlp.norm.weight.data_ptr(), mlp.norm.bias.data_ptr(), float(mlp.norm.eps), w1.data_ptr(), w2.data_ptr(),
            batch, att.width, att.heads, mlp.hidden, out.data_ptr(), _lib.stream_of(tokens.device)),
            "cow_attention_mlp_decode")
        return out


class SDMDecoderStack(nn.Module):
    """Layout string of "A" (dense attention) and "B" (SDM) physical layers (reference model.py:214-325)."""

    def __init__(self, *, layout: str, width: int, heads: int, slots: int, reads: int, writes: int,
                 memory_heads: int = 1, mlp_expansion: float = 4.0, dropout: float = 0.0) -> None:
        super().__init__()
        if not layout or any(kind not in "AB" for kind in layout):
            raise ValueError("layout must contain only A and B")
        self.layout, self.width, self.heads = layout, width, heads
        self.attention_layers = nn.ModuleDict({
            str(i): DenseAttentionBlock(width, heads, mlp_expansion=mlp_expansion, dropout=dropout)
            for i, kind in enumerate(layout) if kind == "A"})
        self.sdm_layers = nn.ModuleDict({
            str(i): SparseDeltaMemory(width, slots=slots, reads=reads, writes=writes, memory_heads=memory_heads)
            for i, kind in enumerate(layout) if kind == "B"})
        self.sdm_mlps = nn.ModuleDict({
            str(i): ResidualMLP(width, expansion=mlp_expansion, dropout=dropout)
            for i, kind in enumerate(layout) if kind == "B"})

    @torch.no_grad()
    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """Eval-only full-sequence pass (exact recurrence through the sparse prefill)."""
        if tokens.ndim != 3 or tokens.shape[-1] != self.width:
            raise ValueError(f"tokens must be [B,T,{self.width}]")
        for i, kind in enumerate(self.layout):
            if kind == "A":
                tokens = self.attention_layers[str(i)](tokens)
            else:
                tokens = tokens + self.sdm_layers[str(i)](tokens)
                tokens = tokens + self.sdm_mlps[str(i)](tokens)
        return tokens

    def prefill(self, tokens, *, capacity=None, sdm_capacity_rows=None, sdm_growth_quantum_rows=0):
        from .inference import prefill_faithful_sdm_stack

        return prefill_faithful_sdm_stack(self, tokens, capacity=capacity, sdm_capacity_rows=sdm_capacity_rows,
                                          sdm_growth_quantum_rows=sdm_growth_quantum_rows)

    def decode(self, tokens, state):
        from .inference import decode_faithful_sdm_stack

        return decode_faithful_sdm_stack(self, tokens, state)


class LanguageModel(nn.Module):
    """Embeddings + stack + tied-free vocabulary head (reference model.py:327-482)."""

    def __init__(self, *, vocab_size: int, maximum_sequence_length: int, layout: str, width: int, heads: int,
                 slots: int, reads: int, writes: int, memory_heads: int = 1, mlp_expansion: float = 4.0,
                 activation_dtype: torch.dtype = torch.bfloat16) -> None:
        super().__init__()
        self.maximum_sequence_length = maximum_sequence_length
        self.activation_dtype = activation_dtype
        self.token_embedding = nn.Embedding(vocab_size, width)
        self.position_embedding = nn.Embedding(maximum_sequence_length, width)
        self.stack = SDMDecoderStack(layout=layout, width=width, heads=heads, slots=slots, reads=reads,
                                     writes=writes, memory_heads=memory_heads, mlp_expansion=mlp_expansion)
        self.final_norm = nn.LayerNorm(width)
        self.output = nn.Linear(width, vocab_size, bias=False)

    def initialize_role_keyed(self, seed: int) -> None:
        """Seeded random initialisation (normal embeddings / head, per-layer seeded resets)."""
        base = seed * 100_000
        saved = torch.random.get_rng_state()
        try:
            for offset, weight in ((101, self.token_embedding.weight), (102, self.position_embedding.weight),
                                   (103, self.output.weight)):
                torch.manual_seed(base + offset)
                nn.init.normal_(weight, mean=0.0, std=self.stack.width ** -0.5)
            self.final_norm.reset_parameters()
            for i, kind in enumerate(self.stack.layout):
                if kind == "A":
                    block = self.stack.attention_layers[str(i)]
                    _seeded_reset(block.mlp, base + 1_000 + i)
                    _seeded_reset(block.attention, base + 2_000 + i)
                else:
                    self.stack.sdm_layers[str(i)].reset_role_keyed(base + 6_000 + i)
                    _seeded_reset(self.stack.sdm_mlps[str(i)], base + 1_000 + i)
        finally:
            torch.random.set_rng_state(saved)

    def _embed(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return (self.token_embedding(input_ids) + self.position_embedding(positions)).to(self.activation_dtype)

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        if input_ids.ndim != 2:
            raise ValueError("input_ids must be [B,T]")
        time = input_ids.shape[1]
        if time > self.maximum_sequence_length:
            raise ValueError("sequence exceeds maximum_sequence_length")
        tokens = self._embed(input_ids, torch.arange(time, device=input_ids.device)[None, :])
        return self.output(self.final_norm(self.stack(tokens)))

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor, *, capacity: int | None = None,
                sdm_capacity_rows: int | tuple[int, ...] | None = None, sdm_growth_quantum_rows: int = 0):
        if input_ids.ndim != 2 or input_ids.shape[1] <= 0:
            raise ValueError("prefill input_ids must be non-empty [B,T]")
        time = input_ids.shape[1]
        cap = self.maximum_sequence_length if capacity is None else capacity
        if time > cap or cap > self.maximum_sequence_length:
            raise ValueError("prefill capacity is invalid")
        tokens = self._embed(input_ids, torch.arange(time, device=input_ids.device)[None, :])
        tokens, state = self.stack.prefill(tokens, capacity=cap, sdm_capacity_rows=sdm_capacity_rows,
                                           sdm_growth_quantum_rows=sdm_growth_quantum_rows)
        return self.output(self.final_norm(tokens)), state

    @torch.no_grad()
    def decode(self, input_ids: torch.Tensor, state: "FaithfulSDMDecodeState") -> torch.Tensor:
        if input_ids.ndim != 2 or input_ids.shape != (state.batch, 1):
            raise ValueError(f"decode input_ids must be [{state.batch},1]")
        positions = state.current_positions()
        if bool((positions >= self.maximum_sequence_length).any()):
            raise ValueError("sequence exceeds maximum_sequence_length")
        tokens = self._embed(input_ids, positions[:, None])
        return self.output(self.final_norm(self.stack.decode(tokens, state)))

    @torch.no_grad()
    def admit(self, input_ids: torch.Tensor, state: "FaithfulSDMDecodeState", *,
              sdm_growth_quantum_rows: int | None = None) -> torch.Tensor:
        """Prefill a new cohort and admit it into the live state's pools."""
        if sdm_growth_quantum_rows is None:
            sdm_growth_quantum_rows = state.sdm_states[0].growth_quantum_rows if state.sdm_states else 0
        logits, incoming = self.prefill(input_ids, capacity=state.capacity,
                                        sdm_growth_quantum_rows=sdm_growth_quantum_rows)
        state.admit(incoming)
        return logits


def _seeded_reset(module: nn.Module, seed: int) -> None:
    saved = torch.random.get_rng_state()
    try:
        torch.manual_seed(seed)
        for child in module.modules():
            if child is not module and callable(getattr(child, "reset_parameters", None)):
                child.reset_parameters()
    finally:
        torch.random.set_rng_state(saved)
